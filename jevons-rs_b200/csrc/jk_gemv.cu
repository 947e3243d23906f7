// jk_gemv.cu -- small-row product out[r, c] = sum_j x[r, j] W[c, j] for m <= 16 rows
// (the reference's `gemv` kernel, crates/jevons-kernels/src/gemm.rs:397-530, and `matvec`,
// :1135-1168), written for B200 as an HBM-streaming kernel.
//
// Layout of the work:
//   * a group of 8 lanes owns one weight row (output column); a warp covers 4 rows, a CTA of
//     8 warps 32 rows, CTAs stride over the rows;
//   * a "unit" is 32 weights (one 16-byte Q4_K qs chunk, one Q8_0/Q5_0 block, half of a Q6_K
//     64-weight group); lane g of a group walks units g, g+8, g+16, ... so the 8 lanes read 8
//     adjacent units: 128 contiguous bytes per row per step, 128-bit loads through the
//     read-only path (ld.global.nc.v4);
//   * the x rows are staged once per CTA in shared memory as f32 (and, for Q4_K, per-16 sums
//     of x), and read as warp-broadcast 128-bit loads (the 4 row groups of a warp read the same
//     addresses);
//   * weights are decoded in registers with integer byte tricks (no int->float conversion),
//     scale factors are applied once per 16 weights (sum_j (s q_j - m) x_j = s sum q_j x_j -
//     m sum x_j), products accumulate in f32 with packed fma.rn.f32x2;
//   * the 8 partial sums of a row meet with three xor-shuffles.
// Rounding: every product q_j x_j and every sum is f32; the result differs from the reference's
// f32 evaluation order only by f32 rounding (checked against the f64 oracle within tolerance).
#include "jk_decode.cuh"
#include "jk_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace jk {

namespace {

constexpr int GEMV_THREADS = 256;
constexpr int ROWS_PER_CTA = GEMV_THREADS / 8;  // 32

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// 16 products of 4 packed words' bytes (already reduced to small unsigned values v, then value
// = v - bias) with 16 consecutive x values; returns sum (v - bias) * x in f32.
template <int BIAS>
__device__ __forceinline__ float dot16(const uint32_t (&wv)[4], const float* __restrict__ xp) {
    float2 acc = f2(0.f, 0.f);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const float4 x4 = *reinterpret_cast<const float4*>(xp + 4 * t);
        const float q0 = magic_byte(wv[t], 0) - (MAGIC + (float)BIAS);
        const float q1 = magic_byte(wv[t], 1) - (MAGIC + (float)BIAS);
        const float q2 = magic_byte(wv[t], 2) - (MAGIC + (float)BIAS);
        const float q3 = magic_byte(wv[t], 3) - (MAGIC + (float)BIAS);
        acc = fma2(f2(q0, q1), f2(x4.x, x4.y), acc);
        acc = fma2(f2(q2, q3), f2(x4.z, x4.w), acc);
    }
    return acc.x + acc.y;
}

template <int FMT, int MR>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(WView w, const void* __restrict__ x, int x_dtype,
                                                            int mrows, float* __restrict__ out, int64_t ldo) {
    extern __shared__ __align__(16) float xs[];  // [MR][K] then (Q4_K) xsum [MR][K/16]
    const int64_t K = w.k;
    float* xsum = xs + MR * K;

    // Stage x rows [0, mrows) as f32 (rows mrows..MR-1 zero).
    for (int64_t i = threadIdx.x; i < MR * K; i += GEMV_THREADS) {
        const int r = (int)(i / K);
        float v = 0.f;
        if (r < mrows) {
            if (x_dtype == JK_DTYPE_F32) v = reinterpret_cast<const float*>(x)[i];
            else if (x_dtype == JK_DTYPE_F16) v = __half2float(reinterpret_cast<const __half*>(x)[i]);
            else v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
        }
        xs[i] = v;
    }
    __syncthreads();
    if constexpr (FMT == FMT_Q4K) {
        for (int64_t g = threadIdx.x; g < MR * K / 16; g += GEMV_THREADS) {
            const float* p = xs + 16 * g;
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) s += p[i];
            xsum[g] = s;
        }
        __syncthreads();
    }

    const int lane = threadIdx.x & 31;
    const int g = lane & 7;
    const int rsub = threadIdx.x >> 3;  // row within the CTA's 32
    const int64_t units = K / 32;

    for (int64_t row0 = (int64_t)blockIdx.x * ROWS_PER_CTA; row0 < w.rows; row0 += (int64_t)gridDim.x * ROWS_PER_CTA) {
        const int64_t row = row0 + rsub;
        const bool valid = row < w.rows;
        const int64_t rr = valid ? row : 0;
        const uint8_t* rq = w.q + rr * w.q_row_bytes;
        float acc[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[r] = 0.f;

#pragma unroll 4
        for (int64_t u = g; u < units; u += 8) {
            if constexpr (FMT == FMT_Q4K) {
                const int64_t b = u >> 3;
                const int c = (int)(u & 7);
                const uint8_t* blk = rq + b * 144;
                const uint4 hdr = ldg_nc_v4(blk);
                const uint4 qv = ldg_nc_v4(blk + 16 + 16 * c);
                const int p = c >> 1;
                const float d = half_bits_to_float(hdr.x & 0xFFFFu);
                const float dmin = half_bits_to_float(hdr.x >> 16);
                uint32_t s0, m0, s1, m1;
                q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * p, s0, m0);
                q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * p + 1, s1, m1);
                const float dd_lo = d * (float)s0, mm_lo = dmin * (float)m0;
                const float dd_hi = d * (float)s1, mm_hi = dmin * (float)m1;
                const uint32_t wl[4] = {qv.x & 0x0F0F0F0Fu, qv.y & 0x0F0F0F0Fu, qv.z & 0x0F0F0F0Fu, qv.w & 0x0F0F0F0Fu};
                const uint32_t wh[4] = {(qv.x >> 4) & 0x0F0F0F0Fu, (qv.y >> 4) & 0x0F0F0F0Fu,
                                        (qv.z >> 4) & 0x0F0F0F0Fu, (qv.w >> 4) & 0x0F0F0F0Fu};
                const int64_t e_lo = 256 * b + 64 * p + 16 * (c & 1);
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    const float* xr = xs + r * K;
                    const float s_lo = dot16<0>(wl, xr + e_lo);
                    const float s_hi = dot16<0>(wh, xr + e_lo + 32);
                    const float* xsr = xsum + r * (K / 16);
                    acc[r] += (dd_lo * s_lo - mm_lo * xsr[e_lo / 16]) + (dd_hi * s_hi - mm_hi * xsr[e_lo / 16 + 2]);
                }
            } else if constexpr (FMT == FMT_Q6K) {
                // unit u: super-block b, c8 = u % 8: half nh = c8/4, ql chunk c = c8%4 (bytes
                // 64nh + 16c ..): low nibbles -> i_lo = c/2, high -> i_lo + 2; l0 = 16 (c%2).
                const int64_t b = u >> 3;
                const int c8 = (int)(u & 7);
                const int nh = c8 >> 2, c = c8 & 3;
                const int i_lo = c >> 1, l0 = 16 * (c & 1);
                const uint8_t* body = rq + b * 208;
                const uint4 ql = ldg_nc_v4(body + 64 * nh + 16 * c);
                const uint4 qh = ldg_nc_v4(body + 128 + 32 * nh + l0);
                const uint32_t sw0 = __ldg(reinterpret_cast<const uint32_t*>(body + 192 + 8 * nh));
                const uint32_t sw1 = __ldg(reinterpret_cast<const uint32_t*>(body + 192 + 8 * nh + 4));
                const float d = half_bits_to_float(__ldg(w.d + rr * (K / 256) + b));
                // scale bytes: sc[8nh + 2i + l0/16] for i = i_lo and i_lo + 2
                const int si_lo = 2 * i_lo + (l0 >> 4), si_hi = si_lo + 4;
                const int sc_lo = (int)(int8_t)(((si_lo < 4 ? sw0 : sw1) >> (8 * (si_lo & 3))) & 0xFFu);
                const int sc_hi = (int)(int8_t)((sw1 >> (8 * (si_hi & 3))) & 0xFFu);
                const float f_lo = d * (float)sc_lo, f_hi = d * (float)sc_hi;
                const uint32_t qlw[4] = {ql.x, ql.y, ql.z, ql.w};
                const uint32_t qhw[4] = {qh.x, qh.y, qh.z, qh.w};
                uint32_t v_lo[4], v_hi[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    v_lo[t] = (qlw[t] & 0x0F0F0F0Fu) | (((qhw[t] >> (2 * i_lo)) & 0x03030303u) << 4);
                    v_hi[t] = ((qlw[t] >> 4) & 0x0F0F0F0Fu) | (((qhw[t] >> (2 * i_lo + 4)) & 0x03030303u) << 4);
                }
                const int64_t e_lo = 256 * b + 128 * nh + 32 * i_lo + l0;
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    const float* xr = xs + r * K;
                    acc[r] += f_lo * dot16<32>(v_lo, xr + e_lo) + f_hi * dot16<32>(v_hi, xr + e_lo + 64);
                }
            } else if constexpr (FMT == FMT_Q8_0) {
                const uint4 a = ldg_nc_v4(rq + 32 * u);
                const uint4 bq = ldg_nc_v4(rq + 32 * u + 16);
                const float d = half_bits_to_float(__ldg(w.d + rr * (K / 32) + u));
                const uint32_t v0[4] = {a.x ^ 0x80808080u, a.y ^ 0x80808080u, a.z ^ 0x80808080u, a.w ^ 0x80808080u};
                const uint32_t v1[4] = {bq.x ^ 0x80808080u, bq.y ^ 0x80808080u, bq.z ^ 0x80808080u, bq.w ^ 0x80808080u};
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    const float* xr = xs + r * K + 32 * u;
                    acc[r] += d * (dot16<128>(v0, xr) + dot16<128>(v1, xr + 16));
                }
            } else if constexpr (FMT == FMT_Q5_0) {
                const uint4 qs = ldg_nc_v4(rq + 16 * u);
                const uint32_t qh = __ldg(w.h + rr * (K / 32) + u);
                const float d = half_bits_to_float(__ldg(w.d + rr * (K / 32) + u));
                const uint32_t qsw[4] = {qs.x, qs.y, qs.z, qs.w};
                uint32_t v0[4], v1[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint32_t h0 = qh >> (4 * t), h1 = qh >> (16 + 4 * t);
                    v0[t] = (qsw[t] & 0x0F0F0F0Fu) | ((h0 & 1u) << 4) | ((h0 & 2u) << 11) | ((h0 & 4u) << 18) | ((h0 & 8u) << 25);
                    v1[t] = ((qsw[t] >> 4) & 0x0F0F0F0Fu) | ((h1 & 1u) << 4) | ((h1 & 2u) << 11) | ((h1 & 4u) << 18) | ((h1 & 8u) << 25);
                }
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    const float* xr = xs + r * K + 32 * u;
                    acc[r] += d * (dot16<16>(v0, xr) + dot16<16>(v1, xr + 16));
                }
            } else {  // FMT_F16
                const uint8_t* p = rq + 64 * u;
                float wf[32];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint4 a = ldg_nc_v4(p + 16 * t);
                    const uint32_t ww[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        wf[8 * t + 2 * i] = half_bits_to_float(ww[i] & 0xFFFFu);
                        wf[8 * t + 2 * i + 1] = half_bits_to_float(ww[i] >> 16);
                    }
                }
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    const float* xr = xs + r * K + 32 * u;
                    float2 a2 = f2(0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < 32; i += 2) a2 = fma2(f2(wf[i], wf[i + 1]), f2(xr[i], xr[i + 1]), a2);
                    acc[r] += a2.x + a2.y;
                }
            }
        }
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            float v = acc[r];
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 4);
            acc[r] = v;
        }
        if (valid && g == 0) {
#pragma unroll
            for (int r = 0; r < MR; ++r)
                if (r < mrows) out[r * ldo + row] = acc[r];
        }
    }
}

template <int FMT, int MR>
jk_status launch_gemv_t(const WView& w, const void* x, int x_dtype, int mrows, float* out, int64_t ldo,
                        cudaStream_t stream) {
    const size_t smem = sizeof(float) * (size_t)MR * (size_t)w.k * (FMT == FMT_Q4K ? 17 : 16) / 16;
    auto kern = gemv_kernel<FMT, MR>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "gemv smem attribute");
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t tiles = (w.rows + ROWS_PER_CTA - 1) / ROWS_PER_CTA;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, GEMV_THREADS, smem);
    if (per_sm < 1) per_sm = 1;
    const int64_t cap = (int64_t)sm_count(dev) * per_sm;
    const unsigned grid = (unsigned)(tiles < cap ? tiles : cap);
    kern<<<grid, GEMV_THREADS, smem, stream>>>(w, x, x_dtype, mrows, out, ldo);
    return cuda_fail(cudaGetLastError(), "gemv launch");
}

template <int FMT>
jk_status launch_gemv_fmt(const WView& w, const void* x, int x_dtype, size_t m, float* out, cudaStream_t stream) {
    // Rows of x per pass so the staged f32 copy stays within 96 KB of shared memory.
    const size_t elem = x_dtype == JK_DTYPE_F32 ? 4 : 2;
    int cap = 16;
    while (cap > 1 && (size_t)cap * (size_t)w.k * 4 * 17 / 16 > 96 * 1024) cap >>= 1;
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

}  // namespace

jk_status launch_gemv(const WView& w, const void* x, int x_dtype, size_t m, float* out, cudaStream_t stream) {
    if (m == 0) return JK_OK;
    switch (w.fmt) {
    case FMT_Q4K: return launch_gemv_fmt<FMT_Q4K>(w, x, x_dtype, m, out, stream);
    case FMT_Q6K: return launch_gemv_fmt<FMT_Q6K>(w, x, x_dtype, m, out, stream);
    case FMT_Q8_0: return launch_gemv_fmt<FMT_Q8_0>(w, x, x_dtype, m, out, stream);
    case FMT_Q5_0: return launch_gemv_fmt<FMT_Q5_0>(w, x, x_dtype, m, out, stream);
    default: return launch_gemv_fmt<FMT_F16>(w, x, x_dtype, m, out, stream);
    }
}

}  // namespace jk
