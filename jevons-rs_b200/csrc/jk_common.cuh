// jk_common.cuh -- device helpers shared by the sm_100a kernels: the B200 weight layout, exact
// scalar decode of GGML blocks, packed-f32 arithmetic, and thin PTX wrappers for mbarriers,
// TMA, and tcgen05 (tensor memory + 5th-generation MMA).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

// Optional timeline hook for pipeline studies: a build may define JK_TRACE_POINT(kind, arg) to
// record (role, iteration, clock) events; the library's own build compiles it to nothing.
#ifndef JK_TRACE_POINT
#define JK_TRACE_POINT(kind, arg) ((void)0)
#endif

namespace jk {

// ---------------------------------------------------------------------------------------------
// Device weight layout ("B200 layout"). One matrix = [rows = experts * n, k].
//
//   Q4_K : q = the GGML 144-byte super-blocks unchanged, row-major [rows][k/256] (144 = 9 x 16 B,
//          so every block and every row starts 16-byte aligned for vector loads and TMA).
//   Q6_K : q = the first 208 bytes of each 210-byte block (ql[128] qh[64] sc[16], 13 x 16 B),
//          row-major [rows][k/256]; d = the block's f16 scale, [rows][k/256].
//   Q8_0 : q = the int8 quants as a plain row-major int8 matrix [rows][k]; d = f16 [rows][k/32].
//   Q5_0 : q = the 16 nibble bytes of each block, [rows][k/32][16]; h = the 32 high bits (u32)
//          [rows][k/32]; d = f16 [rows][k/32].
//   F16  : q = row-major FP16 [rows][k] (caller-owned view).
// Total bytes equal the GGUF bytes (nothing padded), so weight-streaming throughput and the
// roofline use the GGUF byte counts directly.
// ---------------------------------------------------------------------------------------------
enum Fmt : int { FMT_Q4K = 0, FMT_Q6K = 1, FMT_Q5_0 = 2, FMT_Q8_0 = 3, FMT_F16 = 4 };

struct WView {
    int fmt;
    const uint8_t* q;
    const uint16_t* d;
    const uint32_t* h;
    int64_t rows;       // experts * n
    int64_t n;          // rows per expert
    int64_t k;
    int64_t q_row_bytes;
};

__host__ __device__ constexpr int64_t q_row_bytes(int fmt, int64_t k) {
    return fmt == FMT_Q4K ? k / 256 * 144
         : fmt == FMT_Q6K ? k / 256 * 208
         : fmt == FMT_Q8_0 ? k
         : fmt == FMT_Q5_0 ? k / 2
         : 2 * k;
}

// Error codes written to the per-device error word (bit flags).
enum : uint32_t {
    ERR_WAIT_TIMEOUT = 1u,   // a bounded mbarrier wait ran out
    ERR_BAD_LAUNCH = 2u,     // a kernel found its launch arguments inconsistent
};

// ---------------------------------------------------------------------------------------------
// Scalar helpers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    float f;
    asm("{ .reg .f16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"((unsigned short)h16));
    return f;
}

// Byte `i` of `w` as a float 2^23 + byte (exponent byte 0x4B); subtracting 2^23 (or 2^23 + c)
// afterwards gives the byte value (minus c) exactly.
__device__ __forceinline__ float magic_byte(uint32_t w, int i) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + (uint32_t)i));
}
constexpr float MAGIC = 8388608.0f;  // 2^23

// Q4_K (scale, min) pair j (0..7) from the three header words s0,s1,s2 holding scales[0..12).
// Same bit selection as quant.rs:14-23.
__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j,
                                              uint32_t& sc, uint32_t& mn) {
    if (j < 4) {
        sc = (s0 >> (8 * j)) & 63u;
        mn = (s1 >> (8 * j)) & 63u;
    } else {
        const int jj = j - 4;
        const uint32_t a = (s0 >> (8 * jj)) & 0xFFu;   // q[j-4]
        const uint32_t b = (s1 >> (8 * jj)) & 0xFFu;   // q[j]
        const uint32_t c = (s2 >> (8 * jj)) & 0xFFu;   // q[j+4]
        sc = (c & 15u) | ((a >> 6) << 4);
        mn = (c >> 4) | ((b >> 6) << 4);
    }
}

// ---------------------------------------------------------------------------------------------
// Packed f32x2 arithmetic (sm_100): one instruction, two IEEE round-to-nearest results.
// ---------------------------------------------------------------------------------------------
union F2 {
    unsigned long long u;
    float2 f;
};
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    F2 x, y, r; x.f = a; y.f = b;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.u) : "l"(x.u), "l"(y.u));
    return r.f;
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
    F2 x, y, r; x.f = a; y.f = b;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.u) : "l"(x.u), "l"(y.u));
    return r.f;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    F2 x, y, z, r; x.f = a; y.f = b; z.f = c;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.u) : "l"(x.u), "l"(y.u), "l"(z.u));
    return r.f;
}

// Round two floats to a packed pair of 16-bit floats (RNE): lo -> bits 0..15, hi -> 16..31.
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    uint32_t r;
    if constexpr (BF16) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// 128-bit read-only load (ld.global.nc.v4). A plain intrinsic, not volatile asm, so the compiler
// may batch the loads of several iterations before their uses.
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------------------------
// mbarrier (shared::cta) with bounded waits. A wait that runs past WAIT_LIMIT_NS records
// ERR_WAIT_TIMEOUT in the error word and returns false; callers then skip their remaining work
// but still reach the kernel's final barrier so tensor memory is always released.
// ---------------------------------------------------------------------------------------------
constexpr uint64_t WAIT_LIMIT_NS = 4000000000ull;  // 4 s

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0 && globaltimer() - t0 > WAIT_LIMIT_NS) {
            atomicOr(err, ERR_WAIT_TIMEOUT);
            return false;
        }
    }
}

// The same wait with cluster-scope acquire: for barriers that the other CTA of a pair arrives on
// (its writes before a release.cluster arrive are visible after this wait).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, uint32_t* err) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((i & 63u) == 0 && globaltimer() - t0 > WAIT_LIMIT_NS) {
            atomicOr(err, ERR_WAIT_TIMEOUT);
            return false;
        }
    }
}

// For waits expected to last long (an epilogue waiting for a whole main loop): after a short spin,
// sleep between polls so the waiting warps leave their issue slots to the working warps.
__device__ __forceinline__ bool mbar_wait_sleepy(uint32_t bar, uint32_t parity, uint32_t* err) {
    for (int i = 0; i < 16; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        __nanosleep(256);
        if ((i & 15u) == 0 && globaltimer() - t0 > WAIT_LIMIT_NS) {
            atomicOr(err, ERR_WAIT_TIMEOUT);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// TMA (no multicast anywhere in this library).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch(const CUtensorMap* m) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(m) : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* m, int32_t c0, int32_t c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(dst), "l"(m), "r"(c0), "r"(c1), "r"(bar) : "memory");
}

// ---------------------------------------------------------------------------------------------
// One lane of the converged warp (elect.sync): the issuing lane of MMAs, commits and TMA copies
// whose operands the whole warp computed (warp-uniform values stay in the uniform datapath).
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile("{ .reg .pred p; elect.sync _|p, 0xffffffff; selp.u32 %0, 1, 0, p; }" : "=r"(pred));
    return pred != 0;
}

// tcgen05: tensor memory and MMA (cta_group::1).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(dst_smem), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy smem writes (the dequantizing threads) -> visible to the async proxy (MMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 or f16 inputs, f32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T: A read from tensor memory (row m of A in lane m, two
// 16-bit values per 32-bit column in k order), kind::f16.
__device__ __forceinline__ void mma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }"
        :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive on `bar` once all previously issued MMAs of this thread have completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar) : "memory");
}

// Shared-memory matrix descriptor for a K-major operand in the 128-byte swizzled canonical
// layout: 8-row x 128-byte atoms stacked along M/N every 1024 bytes (stride byte offset), the
// leading byte offset unused (1), descriptor version 1 (sm_100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu)
         | ((uint64_t)1u << 16)
         | ((uint64_t)(1024u >> 4) << 32)
         | ((uint64_t)1u << 46)
         | ((uint64_t)2u << 61);
}

// Instruction descriptor, kind::f16: f32 accumulator, A/B both bf16 (1) or both f16 (0),
// both K-major, N>>3 at bit 17, M>>4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int m, int n) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10)
         | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// 32 lanes x 32 columns of 32-bit accumulators from tensor memory: thread i of the warp gets
// lane (taddr.lane + i), columns taddr.col .. +31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 columns of 32-bit words into tensor memory: thread i writes v[0..31] to lane
// (taddr.lane + i), columns taddr.col .. +31 (asynchronous; complete after tmem_st_wait).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
           "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
           "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
           "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

}  // namespace jk
