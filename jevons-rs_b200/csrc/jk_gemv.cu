// jk_gemv.cu -- small-row product out[r, c] = sum_j x[r, j] W[c, j] for m <= 16 rows
// (the reference's `gemv` kernel, crates/jevons-kernels/src/gemm.rs:397-530, and `matvec`,
// :1135-1168), written for B200 as an HBM-streaming kernel.
//
// Work layout:
//   * one CTA per SM (16 warps); a warp task is 8 weight rows, tasks are dealt round-robin over
//     the CTAs so every SM streams the same number of rows;
//   * 4 lanes per weight row; per step a lane takes 64 weights of its row -- one Q4_K pair
//     (header + 32 qs bytes), half of a Q6_K half-block, or two Q8_0 / Q5_0 blocks -- with
//     128-bit loads through the read-only path; the 4 lanes of a row read one whole 256-weight
//     group, the 8 rows of a warp 8 of them;
//   * weights stay integers: nibbles / bytes are masked into packed bytes and multiplied with the
//     activations by dp2a (two 16-bit x 8-bit products per instruction, exact int32 sums). For this
//     each CTA stages the activation rows once as int16 with one f32 scale per 32-element block
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
#include "jk_decode.cuh"
#include "jk_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace jk {

namespace {

constexpr int WARPS = 16;
constexpr int THREADS = 32 * WARPS;
constexpr int ROWS_PER_TASK = 8;      // 4 lanes per row
constexpr int SLOT_WORDS = 40;        // per (step, lane) activation slot, 160 bytes
// slot layout (words): [0,16) xq lo[32] int16 | [16,32) xq hi[32] | 32 s_lo | 33 s_hi |
//                      34..37 sums of xq over lo[0:16), lo[16:32), hi[0:16), hi[16:32) | pad

// Element offset (within the row) of the first of the 32 "lo" (h = 0) or "hi" (h = 1) activations
// a lane uses at step `st`, lane-in-row `g`.
template <int FMT>
__device__ __forceinline__ int64_t slot_elem(int64_t st, int g, int h) {
    if constexpr (FMT == FMT_Q4K) return 256 * st + 64 * g + 32 * h;
    else if constexpr (FMT == FMT_Q6K) return 256 * st + 128 * (g >> 1) + 32 * (g & 1) + 64 * h;
    else return 256 * st + 64 * g + 32 * h;  // Q8_0 / Q5_0 / F16: blocks 8 st + 2 g + h
}

__device__ __forceinline__ int dp2_16x8(uint32_t x2, uint32_t q4, int acc, bool hi) {
    // two int16 activations x (signed) times bytes 0,1 (lo) or 2,3 (hi) of q4 (signed bytes)
    return hi ? __dp2a_hi((int)x2, (int)q4, acc) : __dp2a_lo((int)x2, (int)q4, acc);
}

// sum over 16 weights: 4 words of packed bytes (4 weights each) times 8 words of int16 pairs
__device__ __forceinline__ int dot16(const uint32_t (&q)[4], const uint4& xa, const uint4& xb) {
    int acc = 0;
    acc = dp2_16x8(xa.x, q[0], acc, false);
    acc = dp2_16x8(xa.y, q[0], acc, true);
    acc = dp2_16x8(xa.z, q[1], acc, false);
    acc = dp2_16x8(xa.w, q[1], acc, true);
    acc = dp2_16x8(xb.x, q[2], acc, false);
    acc = dp2_16x8(xb.y, q[2], acc, true);
    acc = dp2_16x8(xb.z, q[3], acc, false);
    acc = dp2_16x8(xb.w, q[3], acc, true);
    return acc;
}

template <int FMT, int MR>
__global__ void __launch_bounds__(THREADS, 1) gemv_kernel(WView w, const void* __restrict__ x, int x_dtype,
                                                          int mrows, float* __restrict__ out, int64_t ldo) {
    extern __shared__ __align__(16) uint32_t slots[];  // [MR][steps][4][SLOT_WORDS]
    __shared__ float blk_scale[MR][64];                 // per 32-block scales of one staging pass
    const int64_t K = w.k;
    const int64_t steps = (K + 255) / 256;
    const int64_t row_slots = steps * 4 * SLOT_WORDS;

    // ---- stage x: int16 with per-32 scales, in the lane-slot order of this format -------------
    for (int r = 0; r < MR; ++r) {
        const bool live = r < mrows;
        for (int64_t b0 = 0; b0 < K / 32; b0 += 64) {
            // scales of blocks b0 .. b0+63: one warp per block
            for (int bb = threadIdx.x >> 5; bb < 64; bb += WARPS) {
                const int64_t blk = b0 + bb;
                float amax = 0.f;
                if (live && blk < K / 32) {
                    const int64_t e = blk * 32 + (threadIdx.x & 31);
                    float v;
                    if (x_dtype == JK_DTYPE_F32) v = reinterpret_cast<const float*>(x)[r * K + e];
                    else if (x_dtype == JK_DTYPE_F16) v = __half2float(reinterpret_cast<const __half*>(x)[r * K + e]);
                    else v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[r * K + e]);
                    amax = fabsf(v);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
                if ((threadIdx.x & 31) == 0) blk_scale[r][bb] = amax / 32767.0f;
            }
            __syncthreads();
            // each thread quantizes one 16-element half of a slot side
            const int64_t bend = (b0 + 64 < K / 32 ? b0 + 64 : K / 32);
            for (int64_t q = threadIdx.x; q < (bend - b0) * 2; q += THREADS) {
                const int64_t blk = b0 + q / 2;
                const int half16 = (int)(q & 1);
                const int64_t e0 = blk * 32 + 16 * half16;
                // which slot (step, lane g, side h) holds element e0
                int64_t st;
                int g, h;
                if constexpr (FMT == FMT_Q6K) {
                    const int64_t in_sb = e0 & 255;
                    st = e0 >> 8;
                    const int nh = (int)(in_sb >> 7), i = (int)((in_sb & 127) >> 5);
                    g = 2 * nh + (i & 1);
                    h = i >> 1;
                } else {
                    st = e0 >> 8;
                    g = (int)((e0 & 255) >> 6);
                    h = (int)((e0 & 63) >> 5);
                }
                const float s = blk_scale[r][q / 2];
                const float inv = s > 0.f ? 1.0f / s : 0.f;
                uint32_t* sl = slots + r * row_slots + (st * 4 + g) * SLOT_WORDS;
                int sum = 0;
                uint32_t packed[8];
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    float v0 = 0.f, v1 = 0.f;
                    if (live) {
                        const int64_t e = r * K + e0 + i;
                        if (x_dtype == JK_DTYPE_F32) {
                            v0 = reinterpret_cast<const float*>(x)[e];
                            v1 = reinterpret_cast<const float*>(x)[e + 1];
                        } else if (x_dtype == JK_DTYPE_F16) {
                            v0 = __half2float(reinterpret_cast<const __half*>(x)[e]);
                            v1 = __half2float(reinterpret_cast<const __half*>(x)[e + 1]);
                        } else {
                            v0 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[e]);
                            v1 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[e + 1]);
                        }
                    }
                    const int q0 = __float2int_rn(v0 * inv), q1 = __float2int_rn(v1 * inv);
                    sum += q0 + q1;
                    packed[i / 2] = ((uint32_t)q0 & 0xFFFFu) | ((uint32_t)q1 << 16);
                }
                uint4* dst = reinterpret_cast<uint4*>(sl + 16 * h + 8 * half16);
                dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                if (half16 == 0) reinterpret_cast<float*>(sl)[32 + h] = s;
                reinterpret_cast<float*>(sl)[34 + 2 * h + half16] = (float)sum;
            }
            __syncthreads();
        }
    }

    // ---- stream the weight rows --------------------------------------------------------------
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int g = lane & 3;       // lane within the row
    const int rsub = lane >> 2;   // row within the task
    const int64_t tasks = (w.rows + ROWS_PER_TASK - 1) / ROWS_PER_TASK;
    // Q4_K: this lane's sub-blocks are 2g and 2g+1 for every super-block (lane-constant)
    const bool upper = g >= 2;
    const int jj = (2 * g) & 3;

    for (int64_t t = blockIdx.x + (int64_t)gridDim.x * warp; t < tasks; t += (int64_t)gridDim.x * WARPS) {
        const int64_t row = t * ROWS_PER_TASK + rsub;
        const bool valid = row < w.rows;
        const int64_t rr = valid ? row : 0;
        const uint8_t* rq = w.q + rr * w.q_row_bytes;
        float acc[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[r] = 0.f;

#pragma unroll 2
        for (int64_t st = 0; st < steps; ++st) {
            const uint32_t* sl0 = slots + (st * 4 + g) * SLOT_WORDS;
            if constexpr (FMT == FMT_Q4K) {
                const uint8_t* blk = rq + st * 144;
                const uint4 hdr = ldg_nc_v4(blk);
                const uint4 qa = ldg_nc_v4(blk + 16 + 32 * g);
                const uint4 qb = ldg_nc_v4(blk + 32 + 32 * g);
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
                    const uint4* xs = reinterpret_cast<const uint4*>(sl0 + r * row_slots);
                    const float* xf = reinterpret_cast<const float*>(sl0 + r * row_slots);
                    const int A = dot16(lo0, xs[0], xs[1]) + dot16(lo1, xs[2], xs[3]);
                    const int B = dot16(hi0, xs[4], xs[5]) + dot16(hi1, xs[6], xs[7]);
                    const float4 sm = *reinterpret_cast<const float4*>(xf + 32);  // s_lo s_hi S0 S1
                    const float2 sh = *reinterpret_cast<const float2*>(xf + 36);  // S2 S3
                    acc[r] += sm.x * (dd0 * (float)A - mm0 * (sm.z + sm.w)) + sm.y * (dd1 * (float)B - mm1 * (sh.x + sh.y));
                }
            } else if constexpr (FMT == FMT_Q6K) {
                // lane g: half nh = g/2, ql half hq = g%2: ql bytes 64nh + 32hq + [0,32): low
                // nibbles -> i = hq, high -> i = hq + 2; qh bytes 32nh + [0,32) bits 2i
                const int nh = g >> 1, hq = g & 1;
                const uint8_t* body = rq + st * 208;
                const uint4 l0 = ldg_nc_v4(body + 64 * nh + 32 * hq);
                const uint4 l1 = ldg_nc_v4(body + 64 * nh + 32 * hq + 16);
                const uint4 h0 = ldg_nc_v4(body + 128 + 32 * nh);
                const uint4 h1 = ldg_nc_v4(body + 128 + 32 * nh + 16);
                const uint2 scw = __ldg(reinterpret_cast<const uint2*>(body + 192 + 8 * nh));
                const float d = half_bits_to_float(__ldg(w.d + rr * (K / 256) + st));
                const int sh_lo = 2 * hq, sh_hi = 2 * hq + 4;
                const uint32_t ql[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
                const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                uint32_t vlo[8], vhi[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    vlo[i] = (ql[i] & 0x0F0F0F0Fu) | (((qh[i] >> sh_lo) & 0x03030303u) << 4);
                    vhi[i] = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> sh_hi) & 0x03030303u) << 4);
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
                    const uint4* xs = reinterpret_cast<const uint4*>(sl0 + r * row_slots);
                    const float* xf = reinterpret_cast<const float*>(sl0 + r * row_slots);
                    const float4 sm = *reinterpret_cast<const float4*>(xf + 32);
                    const float2 sh = *reinterpret_cast<const float2*>(xf + 36);
                    const float a0 = (float)dot16(v0, xs[0], xs[1]) - 32.f * sm.z;
                    const float a1 = (float)dot16(v1, xs[2], xs[3]) - 32.f * sm.w;
                    const float a2 = (float)dot16(v2, xs[4], xs[5]) - 32.f * sh.x;
                    const float a3 = (float)dot16(v3, xs[6], xs[7]) - 32.f * sh.y;
                    acc[r] += sm.x * (s0 * a0 + s1 * a1) + sm.y * (s2 * a2 + s3 * a3);
                }
            } else if constexpr (FMT == FMT_Q8_0 || FMT == FMT_Q5_0) {
                const int64_t blk = 8 * st + 2 * g;  // this lane's two blocks
                if (blk < K / 32) {
                    uint32_t q0[4], q1[4], q2[4], q3[4];
                    float d0, d1;
                    const uint32_t dw = __ldg(reinterpret_cast<const uint32_t*>(w.d + rr * (K / 32) + blk));
                    d0 = half_bits_to_float(dw & 0xFFFFu);
                    d1 = half_bits_to_float(dw >> 16);
                    if constexpr (FMT == FMT_Q8_0) {
                        const uint4 a = ldg_nc_v4(rq + 32 * blk), b = ldg_nc_v4(rq + 32 * blk + 16);
                        const uint4 c = ldg_nc_v4(rq + 32 * blk + 32), e = ldg_nc_v4(rq + 32 * blk + 48);
                        q0[0] = a.x; q0[1] = a.y; q0[2] = a.z; q0[3] = a.w;
                        q1[0] = b.x; q1[1] = b.y; q1[2] = b.z; q1[3] = b.w;
                        q2[0] = c.x; q2[1] = c.y; q2[2] = c.z; q2[3] = c.w;
                        q3[0] = e.x; q3[1] = e.y; q3[2] = e.z; q3[3] = e.w;
                    } else {
                        const uint4 a = ldg_nc_v4(rq + 16 * blk), b = ldg_nc_v4(rq + 16 * blk + 16);
                        const uint2 hh = __ldg(reinterpret_cast<const uint2*>(w.h + rr * (K / 32) + blk));
                        const uint32_t qa[4] = {a.x, a.y, a.z, a.w}, qb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            // element e (< 16): low nibble of byte e, high bit e; e + 16: high nibble, bit e+16
                            const uint32_t hA0 = hh.x >> (4 * t), hA1 = hh.x >> (16 + 4 * t);
                            const uint32_t hB0 = hh.y >> (4 * t), hB1 = hh.y >> (16 + 4 * t);
                            auto spread = [](uint32_t hb) {
                                return ((hb & 1u) << 4) | ((hb & 2u) << 11) | ((hb & 4u) << 18) | ((hb & 8u) << 25);
                            };
                            q0[t] = (qa[t] & 0x0F0F0F0Fu) | spread(hA0);
                            q1[t] = ((qa[t] >> 4) & 0x0F0F0F0Fu) | spread(hA1);
                            q2[t] = (qb[t] & 0x0F0F0F0Fu) | spread(hB0);
                            q3[t] = ((qb[t] >> 4) & 0x0F0F0F0Fu) | spread(hB1);
                        }
                    }
#pragma unroll
                    for (int r = 0; r < MR; ++r) {
                        const uint4* xs = reinterpret_cast<const uint4*>(sl0 + r * row_slots);
                        const float* xf = reinterpret_cast<const float*>(sl0 + r * row_slots);
                        const float4 sm = *reinterpret_cast<const float4*>(xf + 32);
                        const float2 sh = *reinterpret_cast<const float2*>(xf + 36);
                        float A = (float)(dot16(q0, xs[0], xs[1]) + dot16(q1, xs[2], xs[3]));
                        float B = (float)(dot16(q2, xs[4], xs[5]) + dot16(q3, xs[6], xs[7]));
                        if constexpr (FMT == FMT_Q5_0) {
                            A -= 16.f * (sm.z + sm.w);
                            B -= 16.f * (sh.x + sh.y);
                        }
                        acc[r] += d0 * sm.x * A + d1 * sm.y * B;
                    }
                }
            } else {  // FMT_F16: f32 math on the dequantized-free weights, x from the int16 slots
                const int64_t e0 = 256 * st + 64 * g;
                if (e0 < K) {
                    const uint8_t* p = rq + 2 * e0;
                    float wf[64];
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        const uint4 a = ldg_nc_v4(p + 16 * t);
                        const uint32_t ww[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[i]));
                            wf[8 * t + 2 * i] = f.x;
                            wf[8 * t + 2 * i + 1] = f.y;
                        }
                    }
#pragma unroll
                    for (int r = 0; r < MR; ++r) {
                        const uint32_t* xq = sl0 + r * row_slots;
                        const float* xf = reinterpret_cast<const float*>(xq);
                        float s0 = 0.f, s1 = 0.f;
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const int16_t qa = (int16_t)(xq[i / 2] >> (16 * (i & 1)));
                            const int16_t qb = (int16_t)(xq[16 + i / 2] >> (16 * (i & 1)));
                            s0 += wf[i] * (float)qa;
                            s1 += wf[32 + i] * (float)qb;
                        }
                        acc[r] += xf[32] * s0 + xf[33] * s1;
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            float v = acc[r];
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
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
    const int64_t steps = (w.k + 255) / 256;
    const size_t smem = sizeof(uint32_t) * (size_t)MR * (size_t)steps * 4 * SLOT_WORDS;
    auto kern = gemv_kernel<FMT, MR>;
    int dev = 0;
    cudaGetDevice(&dev);
    static int attr_set[64] = {};  // per (instantiation, device): shared-memory opt-in done
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return cuda_fail(e, "gemv smem attribute");
        attr_set[dev] = 1;
    }
    const int64_t tasks = (w.rows + ROWS_PER_TASK - 1) / ROWS_PER_TASK;
    const int64_t grid = tasks < sm_count(dev) ? tasks : sm_count(dev);
    kern<<<(unsigned)grid, THREADS, smem, stream>>>(w, x, x_dtype, mrows, out, ldo);
    return cuda_fail(cudaGetLastError(), "gemv launch");
}

template <int FMT>
jk_status launch_gemv_fmt(const WView& w, const void* x, int x_dtype, size_t m, float* out, cudaStream_t stream) {
    const size_t elem = x_dtype == JK_DTYPE_F32 ? 4 : 2;
    const size_t row_bytes = (size_t)((w.k + 255) / 256) * 4 * SLOT_WORDS * 4;
    int cap = 16;  // rows of x per pass within 192 KB of staged activations
    while (cap > 1 && (size_t)cap * row_bytes > 192 * 1024) cap >>= 1;
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
