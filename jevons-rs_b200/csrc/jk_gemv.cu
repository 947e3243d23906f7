// jk_gemv.cu -- small-row product out[r, c] = sum_j x[r, j] W[c, j] for m <= 16 rows
// (the reference's `gemv` kernel, crates/jevons-kernels/src/gemm.rs:397-530, and `matvec`,
// :1135-1168), written for B200 as an HBM-streaming kernel.
//
// Memory pipeline. The work item of a warp is a "row group" of 8 consecutive weight rows over one
// K segment. Lanes 0..7 copy the group's 8 row segments (and their f16 scales / high-bit words)
// from HBM into a shared-memory slot with one bulk async copy each (cp.async.bulk, completion on
// the slot's mbarrier). Every warp owns two slots, so two items per warp, 16 per CTA, are in
// flight. The first is issued at the very top of the kernel, before the kernel waits on the
// previous grid (programmatic dependent launch); the second right after the activations are
// staged, so the activation loads do not queue behind it. The launch asks for 2 CTAs per SM, so the next product's
// CTAs start streaming while this one finishes.
//
// Work split. `P` warps (1, 2, 4 or 8) share a row group, each taking a contiguous 1/P of its K
// super-block steps; their partial sums meet in shared memory and are added in part order.
// P grows until there are at least 8 warps per SM of work. CTAs walk row groups in a
// grid-stride loop.
//
// Arithmetic (per 4-lane quad = one weight row; a lane takes 64 weights per 256-weight step):
//   * weights stay integers: nibbles / bytes are masked into packed bytes and multiplied with the
//     activations by dp2a (two 16-bit x 8-bit products per instruction, exact int32 sums);
//   * each CTA stages the activation rows as int16 with one f32 scale per 32-element block
//     (round to nearest, |error| <= 2^-16 of the block's largest magnitude) in a padded,
//     bank-conflict-free per-lane layout;
//   * block scales are applied once per 16 or 32 weights in f32:
//       Q4_K  sum (d*sc*q - dmin*m) x  =  s_x * (d*sc * sum q*xq - dmin*m * sum xq)
//       Q6_K  d*sc * s_x * (sum q*xq - 32 sum xq)      Q8_0  d * s_x * sum q*xq
//       Q5_0  d * s_x * (sum q*xq - 16 sum xq)
//   * the 4 partial sums of a row meet in two xor-shuffles.
// Accuracy: the only approximation is the int16 rounding of x (relative 2^-16 of a block's
// maximum); products and sums are exact integers, scales f32. The tests bound the result by
// the f64 oracle within the library tolerance.
//
// Bounded waits: a slot wait that runs past 4 s records ERR_WAIT_TIMEOUT in the device error
// word; the warp then computes nothing more, still takes its part in the row-group barriers,
// and waits (bounded again) for its own copies in flight before the CTA exits.
#include "jk_decode.cuh"
#include "jk_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace jk {

namespace {

constexpr int WARPS = 8;
constexpr int THREADS = 32 * WARPS;
constexpr int GROUP_ROWS = 8;         // weight rows per warp item (4 lanes per row)
constexpr int SLOTS_PER_WARP = 2;
constexpr int WARP_TARGET = 1;        // K parts grow until row groups x parts >= SMs x WARPS x this
constexpr int SLOT_WORDS = 40;        // per (step, lane) activation slot, 160 bytes
// activation slot layout (words): [0,16) xq lo[32] int16 | [16,32) xq hi[32] | 32 s_lo | 33 s_hi |
//                                 34..37 sums of xq over lo[0:16), lo[16:32), hi[0:16), hi[16:32) | pad

// Per-launch geometry, computed on the host.
struct Geo {
    int k, steps, rowgroups;    // 32-bit: the host checks the matrix fits
    int P;                      // warps per row group
    int KS;                     // 256-weight steps per segment
    int qsb, dsb, hsb;          // bytes per 256 weights of q, d (f16 scales), h (Q5_0 high bits)
    int q_area, d_area, h_area; // per-row shared-memory bytes of a slot (16-byte multiples)
    int slot_bytes;
    int x_words;                // staged activation words
    int red_floats;             // partial-sum exchange floats
    int64_t d_row_bytes, h_row_bytes;
    int x_vec;                  // activations 16-byte aligned: vector loads
};

// Expert-grouped launch (matvec_grouped): blockIdx.y is the job; job j multiplies sorted rows
// [jobs[2j+2], min(+job_rows, offsets[e+1])) of expert e = jobs[2j+1] -- activation row
// sorted[s] / in_div -- by weight rows e*n.., and writes output row sorted[s]. jobs == null: dense.
struct Grp {
    const uint32_t* jobs;
    const uint32_t* offsets;
    const uint32_t* sorted;
    uint32_t in_div;
    int job_rows;
    int64_t x_rows;   // activation rows (sources past it read as zeros)
};

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void group_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ int dp2_16x8(uint32_t x2, uint32_t q4, int acc, bool hi) {
    // two int16 activations x (signed) times bytes 0,1 (lo) or 2,3 (hi) of q4 (signed bytes)
    return hi ? __dp2a_hi((int)x2, (int)q4, acc) : __dp2a_lo((int)x2, (int)q4, acc);
}

// sum over 16 weights: 4 words of packed bytes (4 weights each) times 8 words of int16 pairs, as
// two independent dp2a chains (integer sums: the split changes no bit of the result, and halves
// the dependent-instruction chain the warp waits on)
__device__ __forceinline__ int dot16(const uint32_t (&q)[4], const uint4& xa, const uint4& xb) {
    int a0 = 0, a1 = 0;
    a0 = dp2_16x8(xa.x, q[0], a0, false);
    a1 = dp2_16x8(xa.y, q[0], a1, true);
    a0 = dp2_16x8(xa.z, q[1], a0, false);
    a1 = dp2_16x8(xa.w, q[1], a1, true);
    a0 = dp2_16x8(xb.x, q[2], a0, false);
    a1 = dp2_16x8(xb.y, q[2], a1, true);
    a0 = dp2_16x8(xb.z, q[3], a0, false);
    a1 = dp2_16x8(xb.w, q[3], a1, true);
    return a0 + a1;
}

// Activation slot (step st, lane-in-row g, side h, 16-half) holding element e0 (a multiple of 16).
template <int FMT>
__device__ __forceinline__ void slot_of(int e0, int& st, int& g, int& h) {
    st = e0 >> 8;
    if constexpr (FMT == FMT_Q6K) {
        const int in_sb = (int)(e0 & 255);
        const int nh = in_sb >> 7, i = (in_sb & 127) >> 5;
        g = 2 * nh + (i & 1);
        h = i >> 1;
    } else {
        g = (int)((e0 & 255) >> 6);
        h = (int)((e0 & 63) >> 5);
    }
}

// Eight activations x[row, e0 .. e0+8) as floats.
__device__ __forceinline__ void load8(const void* x, int x_dtype, int64_t idx, bool vec, float (&v)[8]) {
    if (x_dtype == JK_DTYPE_F32) {
        const float* p = reinterpret_cast<const float*>(x) + idx;
        if (vec) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(p));
            const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = p[i];
        }
    } else {
        uint32_t u[4];
        if (vec) {
            const uint4 a = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + idx));
            u[0] = a.x; u[1] = a.y; u[2] = a.z; u[3] = a.w;
        } else {
            const uint16_t* p = reinterpret_cast<const uint16_t*>(x) + idx;
#pragma unroll
            for (int i = 0; i < 4; ++i) u[i] = (uint32_t)p[2 * i] | ((uint32_t)p[2 * i + 1] << 16);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f;
            if (x_dtype == JK_DTYPE_F16) f = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
            else f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i]));
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
}

// Stage x rows [0, MR) (rows >= mrows as zeros) into the int16 slot layout. Each thread takes
// 8-element chunks; the 4 chunks of a 32-element block sit in 4 consecutive lanes.
template <int FMT, int MR>
__device__ __forceinline__ void stage_x(const Geo& geo, const void* x, int x_dtype, int mrows, uint32_t* xs,
                                        const int64_t (&src)[MR]) {
    constexpr int U = 4;
    const int kc = geo.k / 8;                 // chunks per row
    const int chunks = (int)MR * kc;
    const int row_words = geo.steps * 4 * SLOT_WORDS;
    for (int c0 = 0; c0 < chunks; c0 += (int)THREADS * U) {
        float v[U][8];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = c0 + u * THREADS + threadIdx.x;
            const int r = MR == 1 ? 0 : c / kc;
            if (c < chunks && r < mrows && src[r] >= 0) {
                load8(x, x_dtype, src[r] * geo.k + (c - r * kc) * 8, geo.x_vec != 0, v[u]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (c0 + u * THREADS >= chunks) break;  // block-uniform: no lane of this pass has a chunk
            const int c = c0 + u * THREADS + threadIdx.x;
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[u][i]));
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
            const float s = amax / 32767.0f;
            const float inv = s > 0.f ? 1.0f / s : 0.f;
            uint32_t packed[4];
            int sum = 0;
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                const int q0 = __float2int_rn(v[u][i] * inv), q1 = __float2int_rn(v[u][i + 1] * inv);
                sum += q0 + q1;
                packed[i / 2] = ((uint32_t)q0 & 0xFFFFu) | ((uint32_t)q1 << 16);
            }
            const int sum16 = sum + __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
            if (c < chunks) {
                const int r = MR == 1 ? 0 : c / kc;
                const int e0 = (c - r * kc) * 8;
                int st;
                int g, h;
                slot_of<FMT>(e0 & ~15, st, g, h);
                const int half16 = (int)((e0 >> 4) & 1), sub8 = (int)((e0 >> 3) & 1);
                uint32_t* sl = xs + r * row_words + (st * 4 + g) * SLOT_WORDS;
                *reinterpret_cast<uint4*>(sl + 16 * h + 8 * half16 + 4 * sub8) =
                    make_uint4(packed[0], packed[1], packed[2], packed[3]);
                if (sub8 == 0) reinterpret_cast<float*>(sl)[34 + 2 * h + half16] = (float)sum16;
                if ((e0 & 31) == 0) reinterpret_cast<float*>(sl)[32 + h] = s;
            }
        }
    }
}

// GRP: the expert-grouped instantiation (job table, row gather and scatter); the dense products
// run a kernel compiled without that code.
template <int FMT, int MR, bool GRP>
__global__ void __launch_bounds__(THREADS, MR <= 2 ? 2 : 1) gemv_kernel(WView w, Geo geo, const void* __restrict__ x, int x_dtype,
                                                          int mrows, float* __restrict__ out, int64_t ldo,
                                                          uint32_t* err, Grp gp) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[WARPS * SLOTS_PER_WARP];
    uint32_t* xs = reinterpret_cast<uint32_t*>(smem);
    float* red = reinterpret_cast<float*>(smem + 4 * (size_t)geo.x_words);  // [2][WARPS][MR][8]
    uint8_t* slots = smem + 4 * (size_t)geo.x_words + 4 * (size_t)geo.red_floats;

    pdl_trigger();  // the next product may start its weight stream as soon as it fits on an SM
    JK_TRACE_POINT(1, 0);

    // activation row of each staged row, output row offset of each, first weight row
    int64_t src[MR], dst[MR];
    int64_t wrow0 = 0;
#pragma unroll
    for (int r = 0; r < MR; ++r) src[r] = dst[r] = r;
    if (GRP && gp.jobs) {
        // the job table comes from the previous grid (the grouping): wait for it first
        pdl_wait();
        const uint32_t j = blockIdx.y;
        if (j >= __ldg(gp.jobs)) return;  // CTA-uniform: past the job count
        const uint32_t e = __ldg(gp.jobs + 1 + 2 * j), s0 = __ldg(gp.jobs + 2 + 2 * j);
        const uint32_t end = __ldg(gp.offsets + e + 1);
        mrows = (int)(end < s0 + (uint32_t)gp.job_rows ? end - s0 : (uint32_t)gp.job_rows);
        if (mrows > MR) mrows = MR;
        wrow0 = (int64_t)e * w.n;
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            const int64_t a = r < mrows ? (int64_t)__ldg(gp.sorted + s0 + r) : -1;
            src[r] = a >= 0 && a / gp.in_div < gp.x_rows ? a / gp.in_div : -1;
            dst[r] = a;
        }
    }

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int P = geo.P;
    const int grp = warp / P, part = warp % P;
    const int per_iter = WARPS / P;
    const int st_lo = (int)part * geo.steps / P, st_hi = (int)(part + 1) * geo.steps / P;
    const int nseg = (int)((st_hi - st_lo + geo.KS - 1) / geo.KS);
    // Row groups are dealt to the CTAs round-robin: the j-th row group of this CTA is
    // blockIdx.x + j * gridDim.x, j = kk * per_iter + grp for iteration kk of warp group grp. Every
    // SM then holds the same number of row groups to within one whatever the grid (dealing blocks
    // of per_iter consecutive row groups left some SMs with twice the average).
    const int n_c = (int)blockIdx.x < geo.rowgroups ? (geo.rowgroups - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int first = (int)blockIdx.x + grp * (int)gridDim.x;
    const int stride = (int)gridDim.x * per_iter;
    const int kg = grp < n_c ? (n_c - 1 - grp) / per_iter + 1 : 0;
    const int items = kg * nseg;
    // all warps of the CTA run the same number of row-group iterations (group barriers)
    const int k_cta = (n_c + per_iter - 1) / per_iter;

    const uint32_t bar0 = smem_u32(&bars[warp * SLOTS_PER_WARP]);
    const uint32_t slot0 = smem_u32(slots) + (uint32_t)(warp * SLOTS_PER_WARP) * (uint32_t)geo.slot_bytes;
    if (lane == 0) {
        for (int s = 0; s < SLOTS_PER_WARP; ++s) mbar_init(bar0 + 8u * s, 1);
        mbar_fence_init();
    }
    __syncwarp();

    // Copies of item i into slot i % 2: row segment bytes of q, then the d / h words covering it
    // (rounded out to 16-byte boundaries; allocations carry the slack).
    auto issue = [&](int i) {
        const int kk = i / nseg;
        const int s = (int)(i - kk * nseg);
        const int rg = first + kk * stride;
        const int st0 = st_lo + (int)s * geo.KS;
        const int st1 = st0 + geo.KS < st_hi ? st0 + geo.KS : st_hi;
        const int e0 = st0 * 256, e1 = st1 * 256 < geo.k ? st1 * 256 : geo.k;
        const uint32_t slot = slot0 + (uint32_t)(i & 1) * (uint32_t)geo.slot_bytes;
        const uint32_t bar = bar0 + 8u * (uint32_t)(i & 1);
        uint32_t bytes = 0, qb = 0, db = 0, hb = 0;
        const uint8_t *qs = nullptr, *ds = nullptr, *hs = nullptr;
        if (lane < GROUP_ROWS) {
            const int64_t row = wrow0 + rg * GROUP_ROWS + lane;
            qs = w.q + row * w.q_row_bytes + (int64_t)e0 * geo.qsb / 256;
            qb = (uint32_t)((e1 - e0) * geo.qsb / 256);
            if (geo.dsb) {
                const uintptr_t a = reinterpret_cast<uintptr_t>(w.d) + row * geo.d_row_bytes + (int64_t)e0 * geo.dsb / 256;
                const uintptr_t b = a + (e1 - e0) * geo.dsb / 256;
                ds = reinterpret_cast<const uint8_t*>(a & ~(uintptr_t)15);
                db = (uint32_t)(((b + 15) & ~(uintptr_t)15) - (a & ~(uintptr_t)15));
            }
            if (geo.hsb) {
                const uintptr_t a = reinterpret_cast<uintptr_t>(w.h) + row * geo.h_row_bytes + (int64_t)e0 * geo.hsb / 256;
                const uintptr_t b = a + (e1 - e0) * geo.hsb / 256;
                hs = reinterpret_cast<const uint8_t*>(a & ~(uintptr_t)15);
                hb = (uint32_t)(((b + 15) & ~(uintptr_t)15) - (a & ~(uintptr_t)15));
            }
            bytes = qb + db + hb;
        }
        const uint32_t total = __reduce_add_sync(0xFFFFFFFFu, bytes);
        if (lane == 0) mbar_expect_tx(bar, total);
        __syncwarp();
        if (lane < GROUP_ROWS) {
            bulk_g2s(slot + (uint32_t)(lane * geo.q_area), qs, qb, bar);
            if (db) bulk_g2s(slot + (uint32_t)(GROUP_ROWS * geo.q_area + lane * geo.d_area), ds, db, bar);
            if (hb)
                bulk_g2s(slot + (uint32_t)(GROUP_ROWS * (geo.q_area + geo.d_area) + lane * geo.h_area), hs, hb, bar);
        }
    };

    if (items > 0) issue(0);
    JK_TRACE_POINT(2, 0);

    pdl_wait();  // activations come from the previous grid; outputs may be read by it
    JK_TRACE_POINT(3, 0);
    stage_x<FMT, MR>(geo, x, x_dtype, mrows, xs, src);
    // the second item's copies go out after the activations are read: issued before, they queued
    // ahead of the activation loads (measured 6.9 -> 6.5 us per 14.7 MB product)
    if (items > 1) issue(1);
    __syncthreads();
    JK_TRACE_POINT(4, 0);

    const int g = lane & 3;       // lane within the row
    const int rsub = lane >> 2;   // row within the group
    const int row_words = geo.steps * 4 * SLOT_WORDS;
    const bool upper = g >= 2;    // Q4_K: this lane's sub-blocks are 2g and 2g+1
    const int jj = (2 * g) & 3;
    bool ok = true;
    int i = 0;

    for (int kk = 0; kk < k_cta; ++kk) {
        const bool live = kk < kg;
        float acc[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[r] = 0.f;
        for (int s = 0; live && s < nseg; ++s, ++i) {
            if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar0 + 8u * (uint32_t)(i & 1), (uint32_t)((i >> 1) & 1), err));
            if (!ok) break;  // i stays at the item that did not arrive
            JK_TRACE_POINT(5, i);
            const uint8_t* slot = slots + (size_t)(warp * SLOTS_PER_WARP + (int)(i & 1)) * geo.slot_bytes;
            const uint8_t* qrow = slot + rsub * geo.q_area;
            const int st0 = st_lo + (int)s * geo.KS;
            const int st1 = st0 + geo.KS < st_hi ? st0 + geo.KS : st_hi;
            const int64_t row = wrow0 + (first + kk * stride) * GROUP_ROWS + rsub;
            // start of this row's d / h words inside the slot (the copy began 16-byte aligned)
            const uint8_t* drow = nullptr;
            const uint8_t* hrow = nullptr;
            if (geo.dsb) {
                const uintptr_t a = reinterpret_cast<uintptr_t>(w.d) + row * geo.d_row_bytes + st0 * geo.dsb;
                drow = slot + GROUP_ROWS * geo.q_area + rsub * geo.d_area + (a & 15);
            }
            if (geo.hsb) {
                const uintptr_t a = reinterpret_cast<uintptr_t>(w.h) + row * geo.h_row_bytes + st0 * geo.hsb;
                hrow = slot + GROUP_ROWS * (geo.q_area + geo.d_area) + rsub * geo.h_area + (a & 15);
            }
#pragma unroll 2
            for (int st = st0; st < st1; ++st) {
                const int sl = (int)(st - st0);
                const uint32_t* sl0 = xs + (st * 4 + g) * SLOT_WORDS;
                if constexpr (FMT == FMT_Q4K) {
                    const uint8_t* blk = qrow + sl * 144;
                    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
                    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g);
                    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * g);
                    const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hdr.x));
                    // scale/min of sub-blocks 2g (lo nibbles) and 2g+1 (hi nibbles), quant.rs:14-23
                    const uint32_t a0 = __byte_perm(hdr.y, 0, 0x4440 + jj), a1 = __byte_perm(hdr.y, 0, 0x4441 + jj);
                    const uint32_t b0 = __byte_perm(hdr.z, 0, 0x4440 + jj), b1 = __byte_perm(hdr.z, 0, 0x4441 + jj);
                    const uint32_t c0 = __byte_perm(hdr.w, 0, 0x4440 + jj), c1 = __byte_perm(hdr.w, 0, 0x4441 + jj);
                    const uint32_t sc0 = upper ? ((c0 & 15u) | ((a0 >> 6) << 4)) : (a0 & 63u);
                    const uint32_t mn0 = upper ? ((c0 >> 4) | ((b0 >> 6) << 4)) : (b0 & 63u);
                    const uint32_t sc1 = upper ? ((c1 & 15u) | ((a1 >> 6) << 4)) : (a1 & 63u);
                    const uint32_t mn1 = upper ? ((c1 >> 4) | ((b1 >> 6) << 4)) : (b1 & 63u);
                    const float dd0 = dm.x * (float)sc0, mm0 = dm.y * (float)mn0;
                    const float dd1 = dm.x * (float)sc1, mm1 = dm.y * (float)mn1;
                    const uint32_t lo0[4] = {qa.x & 0x0F0F0F0Fu, qa.y & 0x0F0F0F0Fu, qa.z & 0x0F0F0F0Fu, qa.w & 0x0F0F0F0Fu};
                    const uint32_t lo1[4] = {qb.x & 0x0F0F0F0Fu, qb.y & 0x0F0F0F0Fu, qb.z & 0x0F0F0F0Fu, qb.w & 0x0F0F0F0Fu};
                    const uint32_t hi0[4] = {(qa.x >> 4) & 0x0F0F0F0Fu, (qa.y >> 4) & 0x0F0F0F0Fu,
                                             (qa.z >> 4) & 0x0F0F0F0Fu, (qa.w >> 4) & 0x0F0F0F0Fu};
                    const uint32_t hi1[4] = {(qb.x >> 4) & 0x0F0F0F0Fu, (qb.y >> 4) & 0x0F0F0F0Fu,
                                             (qb.z >> 4) & 0x0F0F0F0Fu, (qb.w >> 4) & 0x0F0F0F0Fu};
#pragma unroll
                    for (int r = 0; r < MR; ++r) {
                        const uint4* xv = reinterpret_cast<const uint4*>(sl0 + r * row_words);
                        const float* xf = reinterpret_cast<const float*>(sl0 + r * row_words);
                        const int A = dot16(lo0, xv[0], xv[1]) + dot16(lo1, xv[2], xv[3]);
                        const int B = dot16(hi0, xv[4], xv[5]) + dot16(hi1, xv[6], xv[7]);
                        const float4 sm = *reinterpret_cast<const float4*>(xf + 32);  // s_lo s_hi S0 S1
                        const float2 sh = *reinterpret_cast<const float2*>(xf + 36);  // S2 S3
                        acc[r] += sm.x * (dd0 * (float)A - mm0 * (sm.z + sm.w)) + sm.y * (dd1 * (float)B - mm1 * (sh.x + sh.y));
                    }
                } else if constexpr (FMT == FMT_Q6K) {
                    // lane g: half nh = g/2, ql half hq = g%2: ql bytes 64nh + 32hq + [0,32): low
                    // nibbles -> i = hq, high -> i = hq + 2; qh bytes 32nh + [0,32) bits 2i
                    const int nh = g >> 1, hq = g & 1;
                    const uint8_t* body = qrow + sl * 208;
                    const uint4 l0 = *reinterpret_cast<const uint4*>(body + 64 * nh + 32 * hq);
                    const uint4 l1 = *reinterpret_cast<const uint4*>(body + 64 * nh + 32 * hq + 16);
                    const uint4 h0 = *reinterpret_cast<const uint4*>(body + 128 + 32 * nh);
                    const uint4 h1 = *reinterpret_cast<const uint4*>(body + 128 + 32 * nh + 16);
                    const uint2 scw = *reinterpret_cast<const uint2*>(body + 192 + 8 * nh);
                    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(drow + 2 * sl));
                    const int sh_lo = 2 * hq, sh_hi = 2 * hq + 4;
                    const uint32_t ql[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
                    const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                    uint32_t vlo[8], vhi[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        vlo[t] = (ql[t] & 0x0F0F0F0Fu) | (((qh[t] >> sh_lo) & 0x03030303u) << 4);
                        vhi[t] = ((ql[t] >> 4) & 0x0F0F0F0Fu) | (((qh[t] >> sh_hi) & 0x03030303u) << 4);
                    }
                    // scales sc[8nh + 2i + l/16]: lo (i = hq) bytes 2hq, 2hq+1; hi (i = hq+2) 2hq+4, 2hq+5
                    const uint32_t sw_lo = scw.x, sw_hi = scw.y;
                    const float s0 = d * (float)(int8_t)(sw_lo >> (16 * hq));
                    const float s1 = d * (float)(int8_t)(sw_lo >> (16 * hq + 8));
                    const float s2 = d * (float)(int8_t)(sw_hi >> (16 * hq));
                    const float s3 = d * (float)(int8_t)(sw_hi >> (16 * hq + 8));
                    const uint32_t v0[4] = {vlo[0], vlo[1], vlo[2], vlo[3]}, v1[4] = {vlo[4], vlo[5], vlo[6], vlo[7]};
                    const uint32_t v2[4] = {vhi[0], vhi[1], vhi[2], vhi[3]}, v3[4] = {vhi[4], vhi[5], vhi[6], vhi[7]};
#pragma unroll
                    for (int r = 0; r < MR; ++r) {
                        const uint4* xv = reinterpret_cast<const uint4*>(sl0 + r * row_words);
                        const float* xf = reinterpret_cast<const float*>(sl0 + r * row_words);
                        const float4 sm = *reinterpret_cast<const float4*>(xf + 32);
                        const float2 sh = *reinterpret_cast<const float2*>(xf + 36);
                        const float a0 = (float)dot16(v0, xv[0], xv[1]) - 32.f * sm.z;
                        const float a1 = (float)dot16(v1, xv[2], xv[3]) - 32.f * sm.w;
                        const float a2 = (float)dot16(v2, xv[4], xv[5]) - 32.f * sh.x;
                        const float a3 = (float)dot16(v3, xv[6], xv[7]) - 32.f * sh.y;
                        acc[r] += sm.x * (s0 * a0 + s1 * a1) + sm.y * (s2 * a2 + s3 * a3);
                    }
                } else if constexpr (FMT == FMT_Q8_0 || FMT == FMT_Q5_0) {
                    const int blk = 8 * st + 2 * g;  // this lane's two blocks
                    if (blk < geo.k / 32) {
                        const int lb = 8 * sl + 2 * g;     // block index within the segment
                        uint32_t q0[4], q1[4], q2[4], q3[4];
                        const uint16_t* dp = reinterpret_cast<const uint16_t*>(drow) + lb;
                        const float d0 = half_bits_to_float(dp[0]);
                        const float d1 = half_bits_to_float(dp[1]);
                        if constexpr (FMT == FMT_Q8_0) {
                            const uint4* qp = reinterpret_cast<const uint4*>(qrow + 32 * lb);
                            const uint4 a = qp[0], b = qp[1], c = qp[2], e = qp[3];
                            q0[0] = a.x; q0[1] = a.y; q0[2] = a.z; q0[3] = a.w;
                            q1[0] = b.x; q1[1] = b.y; q1[2] = b.z; q1[3] = b.w;
                            q2[0] = c.x; q2[1] = c.y; q2[2] = c.z; q2[3] = c.w;
                            q3[0] = e.x; q3[1] = e.y; q3[2] = e.z; q3[3] = e.w;
                        } else {
                            const uint4* qp = reinterpret_cast<const uint4*>(qrow + 16 * lb);
                            const uint4 a = qp[0], b = qp[1];
                            const uint32_t* hp = reinterpret_cast<const uint32_t*>(hrow) + lb;
                            const uint32_t hx = hp[0], hy = hp[1];
                            const uint32_t qa[4] = {a.x, a.y, a.z, a.w}, qb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                // element e (< 16): low nibble of byte e, high bit e; e + 16: high nibble, bit e+16
                                const uint32_t hA0 = hx >> (4 * t), hA1 = hx >> (16 + 4 * t);
                                const uint32_t hB0 = hy >> (4 * t), hB1 = hy >> (16 + 4 * t);
                                auto spread = [](uint32_t hbits) {
                                    return ((hbits & 1u) << 4) | ((hbits & 2u) << 11) | ((hbits & 4u) << 18) | ((hbits & 8u) << 25);
                                };
                                q0[t] = (qa[t] & 0x0F0F0F0Fu) | spread(hA0);
                                q1[t] = ((qa[t] >> 4) & 0x0F0F0F0Fu) | spread(hA1);
                                q2[t] = (qb[t] & 0x0F0F0F0Fu) | spread(hB0);
                                q3[t] = ((qb[t] >> 4) & 0x0F0F0F0Fu) | spread(hB1);
                            }
                        }
#pragma unroll
                        for (int r = 0; r < MR; ++r) {
                            const uint4* xv = reinterpret_cast<const uint4*>(sl0 + r * row_words);
                            const float* xf = reinterpret_cast<const float*>(sl0 + r * row_words);
                            const float4 sm = *reinterpret_cast<const float4*>(xf + 32);
                            const float2 sh = *reinterpret_cast<const float2*>(xf + 36);
                            float A = (float)(dot16(q0, xv[0], xv[1]) + dot16(q1, xv[2], xv[3]));
                            float B = (float)(dot16(q2, xv[4], xv[5]) + dot16(q3, xv[6], xv[7]));
                            if constexpr (FMT == FMT_Q5_0) {
                                A -= 16.f * (sm.z + sm.w);
                                B -= 16.f * (sh.x + sh.y);
                            }
                            acc[r] += d0 * sm.x * A + d1 * sm.y * B;
                        }
                    }
                } else {  // FMT_F16: f32 math on the half weights, x from the int16 slots
                    const int e0 = 256 * st + 64 * g;
                    if (e0 < geo.k) {
                        const uint8_t* p = qrow + 2 * (e0 - 256 * st0);
                        float wf[64];
#pragma unroll
                        for (int t = 0; t < 8; ++t) {
                            const uint4 a = *reinterpret_cast<const uint4*>(p + 16 * t);
                            const uint32_t ww[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[q]));
                                wf[8 * t + 2 * q] = f.x;
                                wf[8 * t + 2 * q + 1] = f.y;
                            }
                        }
#pragma unroll
                        for (int r = 0; r < MR; ++r) {
                            const uint32_t* xq = sl0 + r * row_words;
                            const float* xf = reinterpret_cast<const float*>(xq);
                            float s0 = 0.f, s1 = 0.f;
#pragma unroll
                            for (int t = 0; t < 32; ++t) {
                                const int16_t qa = (int16_t)(xq[t / 2] >> (16 * (t & 1)));
                                const int16_t qb = (int16_t)(xq[16 + t / 2] >> (16 * (t & 1)));
                                s0 += wf[t] * (float)qa;
                                s1 += wf[32 + t] * (float)qb;
                            }
                            acc[r] += xf[32] * s0 + xf[33] * s1;
                        }
                    }
                }
            }
            // the slot's bytes are consumed: hand it to the async proxy for the item two ahead
            JK_TRACE_POINT(6, i);
            __syncwarp();
            fence_proxy_async_smem();
            if (i + 2 < items) issue(i + 2);
        }
        // ---- row-group results -------------------------------------------------------------
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            float v = acc[r];
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
            acc[r] = v;
        }
        const int row = (first + kk * stride) * GROUP_ROWS + rsub;
        if (P == 1) {
            if (live && ok && g == 0) {
#pragma unroll
                for (int r = 0; r < MR; ++r)
                    if (r < mrows) out[dst[r] * ldo + row] = acc[r];
            }
        } else {
            float* rb = red + (size_t)(kk & 1) * WARPS * MR * GROUP_ROWS;
            if (g == 0) {
#pragma unroll
                for (int r = 0; r < MR; ++r) rb[(warp * MR + r) * GROUP_ROWS + rsub] = ok ? acc[r] : 0.f;
            }
            group_sync(1 + grp, 32 * P);
            if (live && part == 0 && g == 0) {
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    float v = 0.f;
                    for (int q = 0; q < P; ++q) v += rb[((warp + q) * MR + r) * GROUP_ROWS + rsub];
                    if (r < mrows) out[dst[r] * ldo + row] = v;
                }
            }
        }
    }
    JK_TRACE_POINT(7, 0);
    if (!ok) {
        // a wait gave up at item i: let this warp's copies still in flight land before exiting
        for (int j = i; j < items && j < i + SLOTS_PER_WARP; ++j)
            (void)mbar_wait(bar0 + 8u * (uint32_t)(j & 1), (uint32_t)((j >> 1) & 1), err);
    }
}

struct Cache {
    int smem_set[64];
};

// gp.jobs != null: grouped launch over `jobs_y` jobs (grid y), about `jobs_est` of them live.
template <int FMT, int MR>
jk_status launch_gemv_t(const WView& w, const void* x, int x_dtype, int mrows, float* out, int64_t ldo,
                        cudaStream_t stream, const Grp& gp = Grp{}, unsigned jobs_y = 1, int64_t jobs_est = 1) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = sm_budget(dev);
    Geo geo{};
    if (w.k > (1 << 30) || w.rows > (1 << 30) || (int64_t)MR * w.k / 8 > (1 << 30))
        return fail(JK_ERR_UNSUPPORTED, "gemv: matrix too large for 32-bit indexing");
    geo.k = (int)w.k;
    geo.steps = (int)((w.k + 255) / 256);
    geo.rowgroups = (int)((gp.jobs ? w.n : w.rows) / GROUP_ROWS);
    switch (FMT) {
    case FMT_Q4K: geo.qsb = 144; break;
    case FMT_Q6K: geo.qsb = 208; geo.dsb = 2; break;
    case FMT_Q8_0: geo.qsb = 256; geo.dsb = 16; break;
    case FMT_Q5_0: geo.qsb = 128; geo.dsb = 16; geo.hsb = 32; break;
    default: geo.qsb = 512; break;
    }
    if (FMT == FMT_Q6K) geo.d_row_bytes = w.k / 256 * 2;
    else if (FMT == FMT_Q8_0 || FMT == FMT_Q5_0) geo.d_row_bytes = w.k / 32 * 2;
    else geo.d_row_bytes = 0;
    geo.h_row_bytes = FMT == FMT_Q5_0 ? w.k / 32 * 4 : 0;
    geo.x_words = (int)(MR * geo.steps * 4 * SLOT_WORDS);
    geo.red_floats = 2 * WARPS * MR * GROUP_ROWS;
    geo.x_vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;

    // warps per row group: enough warp items for 8 warps per SM, never more parts than steps
    geo.P = 1;
    while (geo.P < WARPS && (int64_t)geo.rowgroups * jobs_est * geo.P < (int64_t)sms * WARPS * WARP_TARGET &&
           2 * geo.P <= geo.steps)
        geo.P *= 2;
    const int64_t steps_w = (geo.steps + geo.P - 1) / geo.P;

    // slot size: two CTAs per SM when the staged activations are small, else one
    const size_t fixed = 4 * (size_t)geo.x_words + 4 * (size_t)geo.red_floats;
    const size_t cta_budget = fixed <= 32 * 1024 ? 110 * 1024 : 220 * 1024;
    if (fixed + 16 * 1024 > cta_budget) return fail(JK_ERR_UNSUPPORTED, "gemv: activation rows too long for shared memory");
    const size_t slot_budget = (cta_budget - fixed) / (WARPS * SLOTS_PER_WARP);
    auto areas = [&](int ks) {
        geo.KS = ks;
        // pad so a row is an odd number of 16-byte chunks: the rows of a quarter-warp then hit
        // disjoint banks in every 128-bit load of the compute loop
        const int q16 = ks * geo.qsb / 16;
        geo.q_area = 16 * (q16 + ((q16 & 1) ? 2 : 1));
        geo.d_area = geo.dsb ? ((ks * geo.dsb + 15) / 16) * 16 + 16 : 0;
        geo.h_area = geo.hsb ? ((ks * geo.hsb + 15) / 16) * 16 + 16 : 0;
        geo.slot_bytes = GROUP_ROWS * (geo.q_area + geo.d_area + geo.h_area);
        geo.slot_bytes = (geo.slot_bytes + 127) / 128 * 128;
    };
    int ks = (int)(steps_w < 64 ? steps_w : 64);
    for (areas(ks); ks > 1 && (size_t)geo.slot_bytes > slot_budget; areas(--ks)) {}
    if ((size_t)geo.slot_bytes > slot_budget) return fail(JK_ERR_UNSUPPORTED, "gemv: one weight step exceeds its slot");
    // balance the segments of a warp's K range
    const int nseg = (int)((steps_w + ks - 1) / ks);
    areas((int)((steps_w + nseg - 1) / nseg));

    const size_t smem = fixed + (size_t)WARPS * SLOTS_PER_WARP * geo.slot_bytes;
    auto kern = gp.jobs ? gemv_kernel<FMT, MR, true> : gemv_kernel<FMT, MR, false>;
    static Cache caches[2] = {};
    Cache& cache = caches[gp.jobs ? 1 : 0];
    if (dev >= 0 && dev < 64 && !cache.smem_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        // all of L1 as shared memory, so two CTAs fit on an SM
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return cuda_fail(e, "gemv smem attribute");
        cache.smem_set[dev] = 1;
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, THREADS, smem);
    if (e != cudaSuccess) return cuda_fail(e, "gemv occupancy");
    if (per_sm < 1) return fail(JK_ERR_UNSUPPORTED, "gemv: kernel does not fit on an SM");
    // every CTA that can be resident (row groups are dealt round-robin, so a full grid balances
    // the SMs), but no more CTAs than row groups
    const int64_t want = (int64_t)geo.rowgroups;
    // grouped: the live jobs share the SMs
    const int64_t cap = ((int64_t)per_sm * sms + jobs_est - 1) / jobs_est;
    const unsigned grid = (unsigned)(want < cap ? want : cap);
    if (grid == 0) return JK_OK;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, jobs_y);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, w, geo, x, x_dtype, mrows, out, ldo, device_error_word(dev), gp);
    if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
    return cuda_fail(cudaGetLastError(), "gemv launch");
}

template <int FMT>
jk_status launch_gemv_fmt(const WView& w, const void* x, int x_dtype, size_t m, float* out, cudaStream_t stream) {
    const size_t elem = x_dtype == JK_DTYPE_F32 ? 4 : 2;
    const size_t row_bytes = (size_t)((w.k + 255) / 256) * 4 * SLOT_WORDS * 4;
    int cap = 16;  // rows of x per pass within 160 KB of staged activations
    while (cap > 1 && (size_t)cap * row_bytes > 160 * 1024) cap >>= 1;
    const int64_t ldo = w.rows;
    for (size_t r0 = 0; r0 < m;) {
        const size_t left = m - r0;
        int mr = 1;
        while ((size_t)mr < left && mr < cap) mr <<= 1;
        const int rows = (int)(left < (size_t)mr ? left : (size_t)mr);
        const void* xr = static_cast<const char*>(x) + r0 * (size_t)w.k * elem;
        float* o = out + r0 * (size_t)ldo;
        jk_status st;
        switch (mr) {
        case 1: st = launch_gemv_t<FMT, 1>(w, xr, x_dtype, rows, o, ldo, stream); break;
        case 2: st = launch_gemv_t<FMT, 2>(w, xr, x_dtype, rows, o, ldo, stream); break;
        case 4: st = launch_gemv_t<FMT, 4>(w, xr, x_dtype, rows, o, ldo, stream); break;
        case 8: st = launch_gemv_t<FMT, 8>(w, xr, x_dtype, rows, o, ldo, stream); break;
        default: st = launch_gemv_t<FMT, 16>(w, xr, x_dtype, rows, o, ldo, stream); break;
        }
        if (st != JK_OK) return st;
        r0 += (size_t)rows;
    }
    return JK_OK;
}

template <int FMT>
jk_status launch_gemv_grouped_fmt(const WView& w, const void* x, int x_dtype, const Grp& gp, size_t max_jobs,
                                  size_t rows, float* out, cudaStream_t stream) {
    const int64_t est = (int64_t)(max_jobs < rows ? max_jobs : rows);
    const unsigned y = (unsigned)max_jobs;
    const int64_t ldo = w.n;
    if (gp.job_rows <= 1) return launch_gemv_t<FMT, 1>(w, x, x_dtype, 1, out, ldo, stream, gp, y, est);
    if (gp.job_rows <= 2) return launch_gemv_t<FMT, 2>(w, x, x_dtype, 2, out, ldo, stream, gp, y, est);
    if (gp.job_rows <= 4) return launch_gemv_t<FMT, 4>(w, x, x_dtype, 4, out, ldo, stream, gp, y, est);
    if (gp.job_rows <= 8) return launch_gemv_t<FMT, 8>(w, x, x_dtype, 8, out, ldo, stream, gp, y, est);
    return launch_gemv_t<FMT, 16>(w, x, x_dtype, 16, out, ldo, stream, gp, y, est);
}

}  // namespace

jk_status launch_gemv_grouped(const WView& w, const void* x, int x_dtype, size_t x_rows, const uint32_t* sorted,
                              const uint32_t* offsets, const uint32_t* jobs, size_t max_jobs, uint32_t in_div,
                              int job_rows, size_t rows, float* out, cudaStream_t stream) {
    if (rows == 0 || max_jobs == 0) return JK_OK;
    if (w.n % GROUP_ROWS) return fail(JK_ERR_SHAPE, "gemv: rows must be a multiple of 8");
    if (max_jobs > 65535) return fail(JK_ERR_UNSUPPORTED, "grouped gemv: more than 65535 jobs");
    if (job_rows < 1 || job_rows > JK_GEMV_ROWS) return fail(JK_ERR_INVALID, "grouped gemv: job rows out of range");
    // 16 staged rows must fit the activation budget the dense path allows
    const size_t row_bytes = (size_t)((w.k + 255) / 256) * 4 * SLOT_WORDS * 4;
    int mr = 1;
    while (mr < job_rows) mr <<= 1;
    if ((size_t)mr * row_bytes > 160 * 1024) return fail(JK_ERR_UNSUPPORTED, "grouped gemv: rows too long for the job tile");
    Grp gp{jobs, offsets, sorted, in_div, job_rows, (int64_t)x_rows};
    switch (w.fmt) {
    case FMT_Q4K: return launch_gemv_grouped_fmt<FMT_Q4K>(w, x, x_dtype, gp, max_jobs, rows, out, stream);
    case FMT_Q6K: return launch_gemv_grouped_fmt<FMT_Q6K>(w, x, x_dtype, gp, max_jobs, rows, out, stream);
    case FMT_Q8_0: return launch_gemv_grouped_fmt<FMT_Q8_0>(w, x, x_dtype, gp, max_jobs, rows, out, stream);
    case FMT_Q5_0: return launch_gemv_grouped_fmt<FMT_Q5_0>(w, x, x_dtype, gp, max_jobs, rows, out, stream);
    default: return launch_gemv_grouped_fmt<FMT_F16>(w, x, x_dtype, gp, max_jobs, rows, out, stream);
    }
}

jk_status launch_gemv(const WView& w, const void* x, int x_dtype, size_t m, float* out, cudaStream_t stream) {
    if (m == 0) return JK_OK;
    if (w.rows % GROUP_ROWS) return fail(JK_ERR_SHAPE, "gemv: rows must be a multiple of 8");
    switch (w.fmt) {
    case FMT_Q4K: return launch_gemv_fmt<FMT_Q4K>(w, x, x_dtype, m, out, stream);
    case FMT_Q6K: return launch_gemv_fmt<FMT_Q6K>(w, x, x_dtype, m, out, stream);
    case FMT_Q8_0: return launch_gemv_fmt<FMT_Q8_0>(w, x, x_dtype, m, out, stream);
    case FMT_Q5_0: return launch_gemv_fmt<FMT_Q5_0>(w, x, x_dtype, m, out, stream);
    default: return launch_gemv_fmt<FMT_F16>(w, x, x_dtype, m, out, stream);
    }
}

}  // namespace jk
