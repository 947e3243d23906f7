// jk_q8_int8.cu -- the Q8_0 int8 tensor-core path: per-32 activation quantization and a product
// whose every Q8_0 block dot is an exact int32 tcgen05 kind::i8 MMA, scaled in f32 afterwards.
//
// The reference runs Q8_0 products on FP16 tensor cores with dequantized weights; its int8 plan
// (docs/cubecl-int8-plan.md:48-60) quantizes activations per 32 values (like llama.cpp's q8_1) so
// that a weight block and an activation block meet as an integer dot product, and applies the
// two block scales in f32. That is this path:
//
//   jk_quantize_act_q8  one warp per (row, 32-value block): amax = max |x| (warp shuffles),
//                       d = amax / 127, q = rint(x * (127 / amax)) clamped to [-127, 127]
//                       (round to nearest even, IEEE f32 operations throughout), q -> xq [m][k]
//                       int8, d -> xd [k / 32][m_pad] f32 (block-major, m_pad = m rounded up to 4,
//                       so one block's scales of 128 activation rows are one 512-byte TMA box).
//   gemm_i8_kernel      persistent, one CTA per SM, tiles of 128 weight rows x 128 activation
//                       rows. Per stage (128 k = 4 Q8_0 blocks = one 128-byte swizzle atom of
//                       int8) TMA brings the weight tile, the activation tile and the 4 x 128
//                       activation scales. The MMA warp issues ONE tcgen05.mma kind::i8 (K = 32)
//                       per Q8_0 block into its own int32 accumulator (accumulate = 0), rotating
//                       over four 128-column tensor-memory buffers, and commits each. Eight
//                       rescale warps (2 per TMEM lane quarter, 64 activation columns each) read
//                       a finished buffer with tcgen05.ld (two 32-column halves, one in flight
//                       while the other is folded in), free it, and fold it into f32 registers:
//                       acc[c] = fma(f32(dot), f32(d_w[r, b]) * d_x[c, b], acc[c])
//                       in increasing block order. The int32 dots are exact (|dot| <= 32 * 127 *
//                       127 < 2^24), so the product is bit-exact with a CPU restatement of the
//                       same f32 operations.
//
// The CUDA cores, not the tensor pipe, bound this kernel: per 32-k block every accumulator
// element costs an integer add and half a packed subtract (the int32 -> f32 conversion), half a
// packed multiply (the scale product) and half a packed FMA, 16384 elements per tile and block,
// while the MMA of that block takes ~64 tensor cycles.
#include "jk_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdio>

namespace jk {
namespace {

constexpr int I8_BW = 128;                  // weight rows per tile (MMA M)
constexpr int I8_BT = 128;                  // activation rows per tile (MMA N)
constexpr int I8_KC = 128;                  // k per stage: 4 Q8_0 blocks, one 128-byte swizzle atom
constexpr int I8_W_BYTES = I8_BW * I8_KC;   // 16 KB
constexpr int I8_X_BYTES = I8_BT * I8_KC;   // 16 KB
constexpr int I8_S_BYTES = 4 * I8_BT * 4;   // 2 KB: activation scales of the stage's 4 blocks
constexpr int I8_STAGE = I8_W_BYTES + I8_X_BYTES + I8_S_BYTES;
constexpr int I8_STAGES = 6;
constexpr int I8_NBUF = 4;                  // int32 accumulators of 128 columns: all of TMEM
constexpr int I8_RS_WARPS = 8;              // rescale warps 4..11: 2 per TMEM lane quarter
constexpr int I8_COLS = I8_BT / 2;          // activation columns per rescale warp
constexpr int I8_RS_WARP0 = 4;
constexpr int I8_THREADS = 32 * (I8_RS_WARP0 + I8_RS_WARPS);
constexpr int I8_OFF_BAR = I8_STAGES * I8_STAGE;
// full[S] | empty[S] | acc_full[4] | acc_empty[4] | drain (error path of the MMA warp)
constexpr int I8_N_BAR = 2 * I8_STAGES + 2 * I8_NBUF + 1;
constexpr int I8_OFF_TMEM = I8_OFF_BAR + 8 * I8_N_BAR;
constexpr int I8_SMEM = I8_OFF_TMEM + 16 + 1024;
static_assert(I8_STAGE % 1024 == 0, "swizzled tiles stay 1024-byte aligned");
static_assert(I8_SMEM <= 227 * 1024, "shared memory budget");

// kind::i8 instruction descriptor: s32 accumulator (2 at bit 4), A and B signed int8 (1 at bits 7
// and 10), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t idesc_i8(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p; }"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(0u) : "memory");
}

__device__ __forceinline__ void gdc_launch_i8() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void gdc_wait_i8() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// acc[C0 + c] = fma(f32(v[c]), dw * sx[C0 + c], acc[C0 + c]) for c < 32, in packed f32x2 arithmetic.
// int32 -> f32 without the conversion unit: |v| < 2^22, so the bits of 1.5 * 2^23 + v are those of
// 0x4B400000 + v and one exact subtraction leaves v.
template <int C0 = 0>
__device__ __forceinline__ void rescale32(float (&acc)[I8_COLS], const uint32_t (&v)[32], float dw, const float* sx) {
    const float2 dw2 = make_float2(dw, dw), magic = make_float2(12582912.0f, 12582912.0f);
    const float4* s4 = reinterpret_cast<const float4*>(sx + C0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 d4 = s4[q];
        const float2 sa = mul2(dw2, make_float2(d4.x, d4.y));
        const float2 sb = mul2(dw2, make_float2(d4.z, d4.w));
        const float2 fa = sub2(make_float2(__int_as_float(0x4B400000 + (int)v[4 * q]),
                                           __int_as_float(0x4B400000 + (int)v[4 * q + 1])), magic);
        const float2 fb = sub2(make_float2(__int_as_float(0x4B400000 + (int)v[4 * q + 2]),
                                           __int_as_float(0x4B400000 + (int)v[4 * q + 3])), magic);
        const float2 ra = fma2(fa, sa, make_float2(acc[C0 + 4 * q], acc[C0 + 4 * q + 1]));
        const float2 rb = fma2(fb, sb, make_float2(acc[C0 + 4 * q + 2], acc[C0 + 4 * q + 3]));
        acc[C0 + 4 * q] = ra.x;
        acc[C0 + 4 * q + 1] = ra.y;
        acc[C0 + 4 * q + 2] = rb.x;
        acc[C0 + 4 * q + 3] = rb.y;
    }
}

struct I8Sched {
    int64_t tiles, tiles_m;
    int kst;   // stages per tile
    int nblk;  // Q8_0 blocks per row (k / 32)
};

__global__ void __launch_bounds__(I8_THREADS, 1)
gemm_i8_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
               const __grid_constant__ CUtensorMap tm_s, WView w, float* __restrict__ out, int64_t m, int64_t ldo,
               I8Sched sc, uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + I8_OFF_BAR;
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (I8_STAGES + s); };
    auto acc_full = [&](int b) { return bar0 + 8u * (2 * I8_STAGES + b); };
    auto acc_empty = [&](int b) { return bar0 + 8u * (2 * I8_STAGES + I8_NBUF + b); };
    const uint32_t drain = bar0 + 8u * (2 * I8_STAGES + 2 * I8_NBUF);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + I8_OFF_TMEM);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < I8_STAGES; ++s) {
            mbar_init(full(s), 1);                    // the producer's arrival with the stage's bytes
            mbar_init(empty(s), 1 + I8_RS_WARPS);     // the MMAs' commit + every rescale warp (scales read)
        }
        for (int b = 0; b < I8_NBUF; ++b) {
            mbar_init(acc_full(b), 1);
            mbar_init(acc_empty(b), I8_RS_WARPS);
        }
        mbar_init(drain, 1);
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    gdc_launch_i8();

    const int G = gridDim.x;
    bool ok = true;
    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        gdc_wait_i8();  // the quantized activations come from the previous kernel
        if (elect_one()) {
            tma_prefetch(&tm_w);
            tma_prefetch(&tm_x);
            tma_prefetch(&tm_s);
        }
        __syncwarp();
        int it = 0;
        for (int64_t t = blockIdx.x; t < sc.tiles && ok; t += G) {
            const int32_t w0 = (int32_t)((t / sc.tiles_m) * I8_BW), m0 = (int32_t)((t % sc.tiles_m) * I8_BT);
            for (int ks = 0; ks < sc.kst && ok; ++ks, ++it) {
                const int s = it % I8_STAGES;
                if (it >= I8_STAGES) ok = __all_sync(0xFFFFFFFFu, mbar_wait(empty(s), ((it / I8_STAGES) - 1) & 1, err));
                if (!ok) break;
                if (elect_one()) {
                    const uint32_t st = sbase + (uint32_t)(s * I8_STAGE);
                    mbar_expect_tx(full(s), (uint32_t)I8_STAGE);
                    tma_load_2d(st, &tm_w, ks * I8_KC, w0, full(s));
                    tma_load_2d(st + I8_W_BYTES, &tm_x, ks * I8_KC, m0, full(s));
                    tma_load_2d(st + I8_W_BYTES + I8_X_BYTES, &tm_s, m0, ks * 4, full(s));
                }
                __syncwarp();
            }
        }
        if (!ok)  // copies in flight land before the CTA exits
            for (int i = it - I8_STAGES < 0 ? 0 : it - I8_STAGES; i < it; ++i)
                mbar_wait(full(i % I8_STAGES), (i / I8_STAGES) & 1, err);
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        constexpr uint32_t IDESC = idesc_i8(I8_BW, I8_BT);
        int it = 0, g = 0;
        bool issued = false;
        for (int64_t t = blockIdx.x; t < sc.tiles && ok; t += G) {
            for (int ks = 0; ks < sc.kst && ok; ++ks, ++it) {
                const int s = it % I8_STAGES;
                ok = __all_sync(0xFFFFFFFFu, mbar_wait(full(s), (it / I8_STAGES) & 1, err));
                if (!ok) break;
                tc_fence_after();
                const uint32_t st = sbase + (uint32_t)(s * I8_STAGE);
                const uint64_t wd = sw128_kmajor_desc(st), xd = sw128_kmajor_desc(st + I8_W_BYTES);
                const int nb = sc.nblk - 4 * ks < 4 ? sc.nblk - 4 * ks : 4;
                for (int j = 0; j < nb && ok; ++j, ++g) {
                    const int b = g % I8_NBUF;
                    if (g >= I8_NBUF) ok = __all_sync(0xFFFFFFFFu, mbar_wait(acc_empty(b), ((g / I8_NBUF) - 1) & 1, err));
                    if (!ok) break;
                    tc_fence_after();
                    if (elect_one()) {
                        // one Q8_0 block: k = 32 bytes = +2 in the descriptors' 16-byte address units
                        mma_i8(tmem + (uint32_t)(b * I8_BT), wd + 2u * j, xd + 2u * j, IDESC);
                        mma_commit(acc_full(b));
                    }
                    __syncwarp();
                    issued = true;
                }
                if (!ok) break;
                if (elect_one()) mma_commit(empty(s));  // the stage's tiles are free once its MMAs are done
                __syncwarp();
            }
        }
        if (!ok && issued) {
            // drain the MMAs issued so far before tensor memory is released
            if (elect_one()) mma_commit(drain);
            __syncwarp();
            (void)mbar_wait(drain, 0, err);
        }
    } else if (warp >= I8_RS_WARP0) {
        // ------------------------------ rescale warps ------------------------------
        // Warp 4 + i reads TMEM lanes 32 (i % 4) .. (its weight rows) and activation columns
        // 64 (i / 4) .. of every block accumulator, as two 32-column halves H0 / H1 held in vA / vB.
        // Software pipeline: the load of one half is in flight while the other half is folded in,
        // so the tensor-memory load latency and the next block's barrier wait overlap arithmetic.
        const int i = warp - I8_RS_WARP0;
        const int quarter = warp & 3;
        const int cgrp = i >> 2;
        const int row_in_tile = 32 * quarter + lane;
        const uint32_t tbase = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(I8_COLS * cgrp);
        int it = 0, g = 0;
        uint32_t vA[32], vB[32];
        for (int64_t t = blockIdx.x; t < sc.tiles && ok; t += G) {
            const int64_t wrow = (t / sc.tiles_m) * I8_BW + row_in_tile;
            const int64_t m0 = (t % sc.tiles_m) * I8_BT + I8_COLS * cgrp;
            const bool row_ok = wrow < w.rows;
            const uint16_t* dw_row = w.d + (row_ok ? wrow : 0) * (int64_t)sc.nblk;
            float acc[I8_COLS];
#pragma unroll
            for (int c = 0; c < I8_COLS; ++c) acc[c] = 0.f;
            // prologue: H0 of the tile's first block
            ok = __all_sync(0xFFFFFFFFu, mbar_wait(acc_full(g % I8_NBUF), (g / I8_NBUF) & 1, err));
            if (!ok) break;
            tc_fence_after();
            tmem_ld32(tbase + (uint32_t)((g % I8_NBUF) * I8_BT), vA);
            tmem_ld_wait();
            uint32_t dwp0 = 0, dwp1 = 0;  // the row's 4 f16 block scales of the current stage
            const float* sx = nullptr;
            for (int bl = 0; bl < sc.nblk; ++bl, ++g) {
                const int ks = bl >> 2, j = bl & 3;
                const int s = (it + ks) % I8_STAGES;
                if (j == 0) {
                    // the stage's activation scales (TMA) are visible after its full phase
                    ok = __all_sync(0xFFFFFFFFu, mbar_wait(full(s), ((it + ks) / I8_STAGES) & 1, err));
                    if (!ok) break;
                    const uint16_t* dp = dw_row + 4 * ks;
                    const int nb = sc.nblk - 4 * ks;
                    dwp0 = nb >= 2 ? __ldg(reinterpret_cast<const uint32_t*>(dp)) : (uint32_t)__ldg(dp);
                    dwp1 = nb >= 4 ? __ldg(reinterpret_cast<const uint32_t*>(dp) + 1) : nb == 3 ? (uint32_t)__ldg(dp + 2) : 0u;
                    sx = reinterpret_cast<const float*>(smem + s * I8_STAGE + I8_W_BYTES + I8_X_BYTES) + I8_COLS * cgrp;
                }
                const uint32_t b = (uint32_t)(g % I8_NBUF);
                const float dw = half_bits_to_float(((j < 2 ? dwp0 : dwp1) >> (16 * (j & 1))) & 0xFFFFu);
                const float* sxj = sx + j * I8_BT;
                tmem_ld32(tbase + b * I8_BT + 32, vB);            // H1 of this block, in flight ...
                rescale32(acc, vA, dw, sxj);                       // ... while H0 is folded in
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acc_empty(b));          // both halves are in registers
                const bool more = bl + 1 < sc.nblk;
                if (more) {
                    const int gn = g + 1;
                    ok = __all_sync(0xFFFFFFFFu, mbar_wait(acc_full(gn % I8_NBUF), (gn / I8_NBUF) & 1, err));
                    if (!ok) break;
                    tc_fence_after();
                    tmem_ld32(tbase + (uint32_t)((gn % I8_NBUF) * I8_BT), vA);  // next block's H0 ...
                }
                rescale32<32>(acc, vB, dw, sxj);                   // ... while H1 is folded in
                if (more) tmem_ld_wait();
                if (j == 3 || !more) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty(s));           // done with the stage's scales
                }
            }
            if (!ok) break;
            it += sc.kst;
            if (row_ok) {
                float* o = out + m0 * ldo + wrow;
#pragma unroll
                for (int c = 0; c < I8_COLS; ++c)
                    if (m0 + c < m) o[c * ldo] = acc[c];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// One warp per (row, 32-value block) of x.
template <typename T>
__device__ __forceinline__ float load_act(const T* x, int64_t i);
template <>
__device__ __forceinline__ float load_act<float>(const float* x, int64_t i) { return x[i]; }
template <>
__device__ __forceinline__ float load_act<__half>(const __half* x, int64_t i) { return __half2float(x[i]); }
template <>
__device__ __forceinline__ float load_act<__nv_bfloat16>(const __nv_bfloat16* x, int64_t i) {
    return __bfloat162float(x[i]);
}

template <typename T>
__global__ void __launch_bounds__(256) quantize_act_q8_kernel(const T* __restrict__ x, int64_t m, int64_t k,
                                                              int8_t* __restrict__ xq, float* __restrict__ xd,
                                                              int64_t m_pad) {
    // programmatic dependent launch: the product that follows may start its prologue at once; x
    // may come from the previous kernel, so wait for it before reading
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int64_t nblk = k / 32;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (gw >= m * nblk) return;
    const int lane = threadIdx.x & 31;
    const int64_t row = gw / nblk, b = gw % nblk;
    const int64_t i = row * k + 32 * b + lane;
    const float v = load_act<T>(x, i);
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
    float q = rintf(__fmul_rn(v, id));
    q = fminf(fmaxf(q, -127.f), 127.f);
    xq[i] = (int8_t)(int)q;
    if (lane == 0) xd[b * m_pad + row] = d;
}

}  // namespace

}  // namespace jk

using jk::fail;

extern "C" jk_status jk_quantize_act_q8(const void* x, int x_dtype, size_t m, size_t k, int8_t* xq, size_t xq_len,
                                        float* xd, size_t xd_len, void* stream) {
    if (x_dtype != JK_DTYPE_F32 && x_dtype != JK_DTYPE_F16 && x_dtype != JK_DTYPE_BF16)
        return fail(JK_ERR_INVALID, "unknown activation dtype");
    if (k == 0 || k % 32) {
        char buf[96];
        snprintf(buf, sizeof buf, "quantize_act_q8: k = %zu is not a multiple of 32", k);
        return fail(JK_ERR_SHAPE, buf);
    }
    if (m > (size_t)INT32_MAX) return fail(JK_ERR_INVALID, "m too large");
    const size_t m_pad = (m + 3) / 4 * 4;
    if (xq_len < m * k || xd_len < k / 32 * m_pad) {
        char buf[200];
        snprintf(buf, sizeof buf, "quantize_act_q8: buffers too small for m=%zu, k=%zu (xq %zu < %zu or xd %zu < %zu)", m,
                 k, xq_len, m * k, xd_len, k / 32 * m_pad);
        return fail(JK_ERR_INVALID, buf);
    }
    if (m == 0) return JK_OK;
    if (!x || !xq || !xd) return fail(JK_ERR_INVALID, "null activation or output pointer");
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    // rows m..m_pad of every block's scales: zero (the product reads them for its padded tiles)
    if (m_pad > m) {
        cudaError_t e = cudaMemset2DAsync(xd + m, m_pad * 4, 0, (m_pad - m) * 4, k / 32, cs);
        if (e != cudaSuccess) return jk::cuda_fail(e, "clear padded activation scales");
    }
    const size_t warps = m * (k / 32);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((warps * 32 + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = cs;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (x_dtype == JK_DTYPE_F32)
        e = cudaLaunchKernelEx(&cfg, jk::quantize_act_q8_kernel<float>, static_cast<const float*>(x), (int64_t)m,
                               (int64_t)k, xq, xd, (int64_t)m_pad);
    else if (x_dtype == JK_DTYPE_F16)
        e = cudaLaunchKernelEx(&cfg, jk::quantize_act_q8_kernel<__half>, static_cast<const __half*>(x), (int64_t)m,
                               (int64_t)k, xq, xd, (int64_t)m_pad);
    else
        e = cudaLaunchKernelEx(&cfg, jk::quantize_act_q8_kernel<__nv_bfloat16>, static_cast<const __nv_bfloat16*>(x),
                               (int64_t)m, (int64_t)k, xq, xd, (int64_t)m_pad);
    if (e != cudaSuccess) return jk::cuda_fail(e, "activation quantization launch");
    return jk::cuda_fail(cudaGetLastError(), "activation quantization launch");
}

extern "C" jk_status jk_matmul_q8_int8(const jk_qmatrix* w, const int8_t* xq, size_t xq_len, const float* xd,
                                       size_t xd_len, size_t m, float* out, size_t out_len, void* stream) {
    if (!w) return fail(JK_ERR_INVALID, "null matrix");
    if (w->type != JK_TYPE_Q8_0) return fail(JK_ERR_UNSUPPORTED, "the int8 product takes Q8_0 weights");
    if (m > (size_t)INT32_MAX) return fail(JK_ERR_INVALID, "m too large");
    const size_t m_pad = (m + 3) / 4 * 4;
    if (xq_len < m * w->k || xd_len < w->k / 32 * m_pad || out_len < m * w->n) {
        char buf[220];
        snprintf(buf, sizeof buf, "Q8_0 [%zux%zu, %zu]: buffers too small for m=%zu (xq %zu < %zu, xd %zu < %zu or out %zu < %zu)",
                 w->experts, w->n, w->k, m, xq_len, m * w->k, xd_len, w->k / 32 * m_pad, out_len, m * w->n);
        return fail(JK_ERR_INVALID, buf);
    }
    if (m == 0) return JK_OK;
    if (!xq || !xd || !out) return fail(JK_ERR_INVALID, "null activation or output pointer");
    if ((reinterpret_cast<uintptr_t>(xq) | reinterpret_cast<uintptr_t>(xd)) & 15)
        return fail(JK_ERR_INVALID, "quantized activations and scales must be 16-byte aligned");
    if (!w->has_tmap) return fail(JK_ERR_INVALID, "matrix has no tensor-core layout");
    jk::DeviceGuard dg(w->device);
    CUtensorMap tm_x, tm_s;
    jk_status st = jk::encode_tmap_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)w->k, (uint64_t)m,
                                      (uint64_t)w->k, jk::I8_KC, jk::I8_BT, CU_TENSOR_MAP_SWIZZLE_128B, xq);
    if (st != JK_OK) return st;
    st = jk::encode_tmap_2d(&tm_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)m_pad, (uint64_t)(w->k / 32),
                            (uint64_t)m_pad * 4, jk::I8_BT, 4, CU_TENSOR_MAP_SWIZZLE_NONE, xd);
    if (st != JK_OK) return st;
    auto kern = jk::gemm_i8_kernel;
    static int prepared[64] = {};
    if (w->device < 0 || w->device >= 64) return fail(JK_ERR_INVALID, "device index out of range");
    if (!prepared[w->device]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, jk::I8_SMEM);
        if (e != cudaSuccess) return jk::cuda_fail(e, "int8 gemm attributes");
        prepared[w->device] = 1;
    }
    jk::WView v = w->view;
    v.rows = (int64_t)w->n;  // dense products use expert 0's rows
    jk::I8Sched sc;
    sc.tiles_m = (int64_t)((m + jk::I8_BT - 1) / jk::I8_BT);
    sc.tiles = (v.rows + jk::I8_BW - 1) / jk::I8_BW * sc.tiles_m;
    sc.nblk = (int)(w->k / 32);
    sc.kst = (int)((w->k + jk::I8_KC - 1) / jk::I8_KC);
    int64_t g = jk::sm_budget(w->device);
    if (g > sc.tiles) g = sc.tiles;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)g);
    cfg.blockDim = dim3(jk::I8_THREADS);
    cfg.dynamicSmemBytes = jk::I8_SMEM;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, w->tm_w, tm_x, tm_s, v, out, (int64_t)m, (int64_t)w->n, sc,
                                       jk::device_error_word(w->device));
    if (e != cudaSuccess) return jk::cuda_fail(e, "int8 gemm launch");
    return jk::cuda_fail(cudaGetLastError(), "int8 gemm launch");
}
