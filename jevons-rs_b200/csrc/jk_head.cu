// jk_head.cu -- operators on a Q6_K token-embedding table (the model's tied input embedding and
// output projection, a jk_qmatrix of type Q6_K with rows = vocabulary and k = model dimension d):
//
//   jk_embed_q6k          embedding rows (+ canvas RMS norm, + attention-input norm)
//                         ops::embed / embed_q6k     crates/jevons-gemma4-diffusion/src/gpu/ops.rs:921-954, 223-291
//   jk_pick_logits        soft-capped logits of selected (row, token) pairs
//                         ops::pick / pick_logits    ops.rs:1133-1157, 590-635
//   jk_q6k_transpose_f16  dequantized, transposed FP16 copy [d, vocab] of the table
//                         ops::q6k_transposed_f16 / q6k_transpose   ops.rs:732-749, 672-715
//   jk_softcap            in-place cap * tanh(x / cap) of f32 logits
//                         ops::softcap_logits / softcap             ops.rs:1159-1168, 751-760
//
// Every kernel decodes Q6_K eight consecutive weights ("an octet") at a time from the B200 row
// layout (per row and super-block: a 208-byte body ql[128] qh[64] sc[16] in `q`, the f16 scale
// in `d`). The decoded values are the exact f32 products (d*sc)*(q-32) of quant.rs:50-58, so the
// embedding rows before normalisation and the transposed table are bit-exact with the reference;
// the reductions (RMS, dot products) are f32 sums in a different order than the reference's and
// are compared within a tolerance.
#include "jk_decode.cuh"
#include "jk_internal.h"

#include <cuda_fp16.h>

#include <cmath>
#include <cstdio>

namespace jk {
namespace {

constexpr int Q6K_BODY = 208;

// Octet o (0..31) of a Q6_K super-block: elements 8o .. 8o+7. Element 128 nh + 32 i + l has
//   q = ((ql[64 nh + 32 (i%2) + l] >> 4 (i/2)) & 15) | (((qh[32 nh + l] >> 2 i) & 3) << 4)
//   w = (d * sc[8 nh + 2 i + l/16]) * (q - 32)
// and 8o = 128 nh + 32 i + l0 gives nh = o/16, i = (o/4)%4, l0 = 8 (o%4); the eight elements
// share one scale byte (l0/16 is fixed across them). `body` is 16-byte aligned.
__device__ __forceinline__ void q6k_octet(const uint8_t* __restrict__ body, float d, int o, float (&v)[8]) {
    const int nh = o >> 4, i = (o >> 2) & 3, l0 = 8 * (o & 3);
    const uint2 ql = __ldg(reinterpret_cast<const uint2*>(body + 64 * nh + 32 * (i & 1) + l0));
    const uint2 qh = __ldg(reinterpret_cast<const uint2*>(body + 128 + 32 * nh + l0));
    const int sc = (int)(int8_t)__ldg(body + 192 + 8 * nh + 2 * i + (l0 >> 4));
    const float dsc = __fmul_rn(d, (float)sc);  // exact: 11-bit times 8-bit significand
    const int ls = 4 * (i >> 1), hs = 2 * i;
    const uint32_t q0 = ((ql.x >> ls) & 0x0F0F0F0Fu) | (((qh.x >> hs) & 0x03030303u) << 4);
    const uint32_t q1 = ((ql.y >> ls) & 0x0F0F0F0Fu) | (((qh.y >> hs) & 0x03030303u) << 4);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        // (2^23 + q) - (2^23 + 32) = q - 32 exactly; the product with dsc is exact too.
        v[e] = __fmul_rn(dsc, __fsub_rn(magic_byte(q0, e), MAGIC + 32.0f));
        v[4 + e] = __fmul_rn(dsc, __fsub_rn(magic_byte(q1, e), MAGIC + 32.0f));
    }
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Sum over the block, the same value in every thread; `red` holds one float per warp. Safe to
// call repeatedly (the leading barrier keeps a previous call's readers ahead of new writes).
__device__ __forceinline__ float block_sum(float s, float* red) {
#pragma unroll
    for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, off);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float t = 0.0f;
    const int warps = blockDim.x >> 5;
    for (int w = 0; w < warps; ++w) t += red[w];
    return t;
}

// Embedding rows: one CTA per token row, one octet per thread and OCT octets per thread.
// out[row] = E[token] * sqrt(d); rows >= first_canvas add cond[row - first_canvas] (if given)
// and are RMS-normalised without weight; x_attn[row] = f16(out * inv_rms(out) * w_attn).
// A token id outside the table sets ERR_BAD_LAUNCH and its row is computed from zeros.
template <int OCT>
__global__ void __launch_bounds__(1024) embed_q6k_kernel(WView t, const uint32_t* __restrict__ tokens,
                                                         const float* __restrict__ w_attn,
                                                         const float* __restrict__ cond, uint32_t first_canvas,
                                                         float eps, float embed_scale, float* __restrict__ out,
                                                         __half* __restrict__ x_attn, uint32_t* err) {
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    const int d = (int)t.k;
    const int octs = d >> 3;
    const uint32_t tok = __ldg(tokens + row);
    const bool bad = tok >= (uint64_t)t.rows;
    if (bad && threadIdx.x == 0) atomicOr(err, ERR_BAD_LAUNCH);
    const uint8_t* trow = t.q + (int64_t)(bad ? 0 : tok) * t.q_row_bytes;
    const uint16_t* drow = t.d + (int64_t)(bad ? 0 : tok) * (d >> 8);

    float v[OCT][8];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < OCT; ++j) {
        const int o = threadIdx.x + j * blockDim.x;
        if (o < octs && !bad) {
            q6k_octet(trow + (o >> 5) * Q6K_BODY, half_bits_to_float(__ldg(drow + (o >> 5))), o & 31, v[j]);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[j][e] = __fmul_rn(v[j][e], embed_scale);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[j][e] = 0.0f;
        }
    }
    const float inv_d = 1.0f / (float)d;
    if (row >= first_canvas) {
        if (cond) {
            const float* cr = cond + (row - first_canvas) * (int64_t)d;
#pragma unroll
            for (int j = 0; j < OCT; ++j) {
                const int o = threadIdx.x + j * blockDim.x;
                if (o < octs) {
                    const float4 a = __ldg(reinterpret_cast<const float4*>(cr + 8 * o));
                    const float4 b = __ldg(reinterpret_cast<const float4*>(cr + 8 * o + 4));
                    v[j][0] += a.x; v[j][1] += a.y; v[j][2] += a.z; v[j][3] += a.w;
                    v[j][4] += b.x; v[j][5] += b.y; v[j][6] += b.z; v[j][7] += b.w;
                }
            }
        }
#pragma unroll
        for (int j = 0; j < OCT; ++j)
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = fmaf(v[j][e], v[j][e], ss);
        const float r = 1.0f / sqrtf(block_sum(ss, red) * inv_d + eps);
        ss = 0.0f;
#pragma unroll
        for (int j = 0; j < OCT; ++j)
#pragma unroll
            for (int e = 0; e < 8; ++e) v[j][e] = __fmul_rn(v[j][e], r);
    }
#pragma unroll
    for (int j = 0; j < OCT; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[j][e], v[j][e], ss);
    const float r = 1.0f / sqrtf(block_sum(ss, red) * inv_d + eps);
#pragma unroll
    for (int j = 0; j < OCT; ++j) {
        const int o = threadIdx.x + j * blockDim.x;
        if (o >= octs) continue;
        float* orow = out + row * (int64_t)d + 8 * o;
        reinterpret_cast<float4*>(orow)[0] = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
        reinterpret_cast<float4*>(orow)[1] = make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
        const float4 wa = __ldg(reinterpret_cast<const float4*>(w_attn + 8 * o));
        const float4 wb = __ldg(reinterpret_cast<const float4*>(w_attn + 8 * o + 4));
        const float w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        uint32_t h[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
            h[e] = pack_half2(__fmul_rn(__fmul_rn(v[j][2 * e], r), w8[2 * e]),
                              __fmul_rn(__fmul_rn(v[j][2 * e + 1], r), w8[2 * e + 1]));
        *reinterpret_cast<uint4*>(x_attn + row * (int64_t)d + 8 * o) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// Candidate logits: one warp per (row, token) pair, 8 pairs per CTA. Lane l takes octets
// l, l + 32, ... so each warp step covers one super-block of the token's table row.
// A pair with row >= x_rows or token outside the table sets ERR_BAD_LAUNCH and writes NaN.
constexpr int PICK_WARPS = 8;

__global__ void __launch_bounds__(32 * PICK_WARPS) pick_logits_kernel(WView t, const __half* __restrict__ x,
                                                                      uint32_t x_rows,
                                                                      const uint32_t* __restrict__ pairs,
                                                                      uint32_t count, float cap,
                                                                      float* __restrict__ out, uint32_t* err) {
    const uint32_t p = blockIdx.x * PICK_WARPS + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (p >= count) return;
    const uint32_t row = __ldg(pairs + 2 * (size_t)p), tok = __ldg(pairs + 2 * (size_t)p + 1);
    if (row >= x_rows || tok >= (uint64_t)t.rows) {
        if (lane == 0) {
            atomicOr(err, ERR_BAD_LAUNCH);
            out[p] = __int_as_float(0x7FC00000);
        }
        return;
    }
    const int d = (int)t.k;
    const int sbs = d >> 8;
    const uint8_t* trow = t.q + (int64_t)tok * t.q_row_bytes;
    const uint16_t* drow = t.d + (int64_t)tok * sbs;
    const __half* xr = x + (int64_t)row * d;
    float acc = 0.0f;
#pragma unroll 4
    for (int sb = 0; sb < sbs; ++sb) {
        float w[8];
        q6k_octet(trow + sb * Q6K_BODY, half_bits_to_float(__ldg(drow + sb)), lane, w);
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(xr + 256 * sb + 8 * lane));
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xw[e]));
            acc = fmaf(w[2 * e], xf.x, acc);
            acc = fmaf(w[2 * e + 1], xf.y, acc);
        }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off);
    if (lane == 0) out[p] = cap * tanhf(acc / cap);
}

// Dequantized transpose: one CTA per (64 table rows, one super-block column of 256 values).
// Phase 1: warp w decodes table rows w, w+8, ... (lane = octet) into a 64 x 256 f16 tile in
// shared memory, storing row r's 16-byte chunk c at chunk position c ^ ((r / 8) % 8). Phase 2:
// each thread takes a column pair (c, c+1) and 8 consecutive rows 8a..8a+7, reads 8 words
// (the swizzle makes a warp's 32 reads hit 32 distinct banks), and writes two 16-byte runs of
// the output rows c and c+1; a warp writes four 128-byte output row segments per step.
constexpr int TR_ROWS = 64;

// Six CTAs per SM and all eight rows' loads of a warp issued before any decode: the kernel is
// bound by load latency (long-scoreboard stalls) at fewer bytes in flight. blockIdx.x is the
// super-block column, so the CTAs resident together read whole table rows.
__global__ void __launch_bounds__(256, 6) q6k_transpose_kernel(WView t, __half* __restrict__ out) {
    __shared__ __align__(16) uint8_t tile[TR_ROWS * 512];
    const int64_t r0 = (int64_t)blockIdx.y * TR_ROWS;
    const int sb = blockIdx.x;
    const int64_t vocab = t.rows;
    const int sbs = (int)(t.k >> 8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < TR_ROWS / 8; ++i) {
        const int r = warp + 8 * i;
        const int64_t row = r0 + r;
        float v[8];
        q6k_octet(t.q + row * t.q_row_bytes + sb * Q6K_BODY, half_bits_to_float(__ldg(t.d + row * sbs + sb)), lane, v);
        const uint4 h = make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]), pack_half2(v[4], v[5]),
                                   pack_half2(v[6], v[7]));
        *reinterpret_cast<uint4*>(tile + r * 512 + ((lane ^ ((r >> 3) & 7)) << 4)) = h;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int u = threadIdx.x + 256 * j;
        const int a = u & 7;           // rows 8a .. 8a+7 of the tile
        const int c = 2 * (u >> 3);    // columns c, c+1 of the super-block
        uint32_t wd[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int r = 8 * a + e;
            wd[e] = *reinterpret_cast<const uint32_t*>(tile + r * 512 + ((((c >> 3) ^ a) & 31) << 4) + ((c & 7) >> 1) * 4);
        }
        const uint4 lo = make_uint4(__byte_perm(wd[0], wd[1], 0x5410), __byte_perm(wd[2], wd[3], 0x5410),
                                    __byte_perm(wd[4], wd[5], 0x5410), __byte_perm(wd[6], wd[7], 0x5410));
        const uint4 hi = make_uint4(__byte_perm(wd[0], wd[1], 0x7632), __byte_perm(wd[2], wd[3], 0x7632),
                                    __byte_perm(wd[4], wd[5], 0x7632), __byte_perm(wd[6], wd[7], 0x7632));
        __half* o0 = out + ((int64_t)sb * 256 + c) * vocab + r0 + 8 * a;
        *reinterpret_cast<uint4*>(o0) = lo;
        *reinterpret_cast<uint4*>(o0 + vocab) = hi;
    }
}

// In-place soft capping, four values per thread (grid-stride).
__global__ void __launch_bounds__(256) softcap_kernel(float* __restrict__ x, size_t n, float cap) {
    const size_t quads = n / 4;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < quads; i += stride) {
        float4 v = reinterpret_cast<float4*>(x)[i];
        v.x = cap * tanhf(v.x / cap);
        v.y = cap * tanhf(v.y / cap);
        v.z = cap * tanhf(v.z / cap);
        v.w = cap * tanhf(v.w / cap);
        reinterpret_cast<float4*>(x)[i] = v;
    }
    const size_t tail = 4 * quads + (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (tail < n) x[tail] = cap * tanhf(x[tail] / cap);
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

jk_status check_table(const jk_qmatrix* table, const char* op) {
    if (!table) return fail(JK_ERR_INVALID, std::string(op) + ": null table");
    if (table->type != JK_TYPE_Q6_K) return fail(JK_ERR_UNSUPPORTED, std::string(op) + ": the table must be Q6_K");
    return JK_OK;
}

jk_status launched(const char* what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? JK_OK : cuda_fail(e, what);
}

}  // namespace
}  // namespace jk

using jk::DeviceGuard;
using jk::fail;

extern "C" jk_status jk_embed_q6k(const jk_qmatrix* table, const uint32_t* tokens_dev, size_t rows,
                                  const float* w_attn_dev, const float* cond_dev, size_t first_canvas, float eps,
                                  float* out_dev, void* x_attn_f16_dev, void* stream) {
    if (jk_status st = jk::check_table(table, "embed_q6k")) return st;
    const size_t d = table->k;
    if (d / 8 > 2048) return fail(JK_ERR_SHAPE, "embed_q6k: model dimension above 16384");
    if (rows == 0) return JK_OK;
    if (rows > (size_t)INT32_MAX) return fail(JK_ERR_INVALID, "embed_q6k: too many rows");
    if (!tokens_dev || !w_attn_dev || !out_dev || !x_attn_f16_dev)
        return fail(JK_ERR_INVALID, "embed_q6k: null buffer");
    if (!jk::aligned16(w_attn_dev) || !jk::aligned16(out_dev) || !jk::aligned16(x_attn_f16_dev) ||
        (cond_dev && !jk::aligned16(cond_dev)))
        return fail(JK_ERR_INVALID, "embed_q6k: w_attn, cond, out and x_attn must be 16-byte aligned");
    const int octs = (int)(d / 8);
    const int oct = octs > 1024 ? 2 : 1;
    const int threads = ((octs + oct - 1) / oct + 31) / 32 * 32;
    const float scale = std::sqrt((float)d);  // sqrt(d as f32), correctly rounded as in the reference
    const uint32_t fc = first_canvas > rows ? (uint32_t)rows : (uint32_t)first_canvas;
    DeviceGuard g(table->device);
    auto s = static_cast<cudaStream_t>(stream);
    uint32_t* err = jk::device_error_word(table->device);
    if (oct == 1)
        jk::embed_q6k_kernel<1><<<(unsigned)rows, threads, 0, s>>>(table->view, tokens_dev, w_attn_dev, cond_dev, fc,
                                                                  eps, scale, out_dev,
                                                                  static_cast<__half*>(x_attn_f16_dev), err);
    else
        jk::embed_q6k_kernel<2><<<(unsigned)rows, threads, 0, s>>>(table->view, tokens_dev, w_attn_dev, cond_dev, fc,
                                                                  eps, scale, out_dev,
                                                                  static_cast<__half*>(x_attn_f16_dev), err);
    return jk::launched("embed_q6k launch");
}

extern "C" jk_status jk_pick_logits(const jk_qmatrix* table, const void* x_f16_dev, size_t x_rows,
                                    const uint32_t* pairs_dev, size_t count, float softcap, float* out_dev,
                                    void* stream) {
    if (jk_status st = jk::check_table(table, "pick_logits")) return st;
    if (count == 0) return JK_OK;
    if (count > (size_t)UINT32_MAX / 2 || x_rows > (size_t)UINT32_MAX)
        return fail(JK_ERR_INVALID, "pick_logits: too many pairs or rows");
    if (!x_f16_dev || !pairs_dev || !out_dev) return fail(JK_ERR_INVALID, "pick_logits: null buffer");
    if (!jk::aligned16(x_f16_dev)) return fail(JK_ERR_INVALID, "pick_logits: x must be 16-byte aligned");
    DeviceGuard g(table->device);
    const unsigned blocks = (unsigned)((count + jk::PICK_WARPS - 1) / jk::PICK_WARPS);
    jk::pick_logits_kernel<<<blocks, 32 * jk::PICK_WARPS, 0, static_cast<cudaStream_t>(stream)>>>(
        table->view, static_cast<const __half*>(x_f16_dev), (uint32_t)x_rows, pairs_dev, (uint32_t)count, softcap,
        out_dev, jk::device_error_word(table->device));
    return jk::launched("pick_logits launch");
}

extern "C" jk_status jk_q6k_transpose_f16(const jk_qmatrix* table, void* out_f16_dev, size_t out_len, void* stream) {
    if (jk_status st = jk::check_table(table, "q6k_transpose")) return st;
    const size_t vocab = table->experts * table->n, d = table->k;
    if (vocab % jk::TR_ROWS != 0) {
        char buf[160];
        snprintf(buf, sizeof buf, "q6k_transpose: %zu table rows are not a multiple of 64", vocab);
        return fail(JK_ERR_SHAPE, buf);
    }
    if (out_len != vocab * d) return fail(JK_ERR_INVALID, "q6k_transpose: output must hold rows * d values");
    if (vocab == 0) return JK_OK;
    if (!out_f16_dev || !jk::aligned16(out_f16_dev))
        return fail(JK_ERR_INVALID, "q6k_transpose: output must be a 16-byte aligned device buffer");
    if (vocab / jk::TR_ROWS > 65535 || d / 256 > (size_t)INT32_MAX)
        return fail(JK_ERR_SHAPE, "q6k_transpose: table above 4194240 rows");
    DeviceGuard g(table->device);
    const dim3 grid((unsigned)(d / 256), (unsigned)(vocab / jk::TR_ROWS));
    jk::q6k_transpose_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(table->view,
                                                                                static_cast<__half*>(out_f16_dev));
    return jk::launched("q6k_transpose launch");
}

extern "C" jk_status jk_softcap(float* x_dev, size_t len, float cap, void* stream) {
    if (len == 0) return JK_OK;
    if (!x_dev || !jk::aligned16(x_dev)) return fail(JK_ERR_INVALID, "softcap: x must be a 16-byte aligned device buffer");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(JK_ERR_CUDA, "softcap: no current device");
    const size_t quads = (len + 3) / 4;
    const size_t cap_blocks = (size_t)jk::sm_count(dev) * 8;
    const size_t want = (quads + 255) / 256;
    const unsigned blocks = (unsigned)(want < cap_blocks ? want : cap_blocks);
    jk::softcap_kernel<<<blocks ? blocks : 1, 256, 0, static_cast<cudaStream_t>(stream)>>>(x_dev, len, cap);
    return jk::launched("softcap launch");
}
