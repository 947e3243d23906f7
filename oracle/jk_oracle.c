/*
 * jk_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's GGML block arithmetic, used as the checker for the
 * CUDA path. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load this library; the product (libjk.so) never links or calls it.
 *
 * What it restates (paths are within the reference project zojeda/jevons-rs):
 *   - TensorType::block()             crates/jevons-formats/src/gguf.rs:134-145
 *   - q4k_scale_min                   crates/jevons-formats/src/quant.rs:14-23
 *   - dequant_q4k / q6k / q5_0 / q8_0 crates/jevons-formats/src/quant.rs:25-80
 *   - dequantize (size checks)        crates/jevons-formats/src/quant.rs:83-101
 *   - pack / packed_words (SoA)       crates/jevons-formats/src/quant.rs:103-193
 *   - the f64 product the GPU tests compare against:
 *       want[r,c] = sum_j f64(x[r,j]) * f64(dequant(W)[c,j])
 *     crates/jevons-gemma4-diffusion/src/gpu/tests.rs:445-452
 *
 * Arithmetic order matters for bit-exactness: the reference evaluates
 *   Q4_K: (d*sc)*q - (dmin*m)   as an f32 multiply, then an f32 subtract (no FMA),
 *   Q6_K: (d*sc)*q              left to right in f32,
 *   Q5_0 / Q8_0: d*q            in f32.
 * This file is compiled with -ffp-contract=off so the C compiler keeps those roundings.
 *
 * f16 -> f32 follows IEEE 754 binary16 exactly (the reference uses crate `half` 2.7.1,
 * whose conversion is exact), so any correct conversion matches.
 *
 * Parity pin: the known-answer tests of crates/jevons-formats/src/quant.rs:199-237 are
 * replayed against this file by tests/test_oracle.py (fixtures in tests/golden/).
 *
 * The Q8_0 int8 path (jk_quantize_act_q8 / jk_matmul_q8_int8) has no counterpart that runs in
 * the reference: its docs/cubecl-int8-plan.md:48-60 plans per-32 activation quantization with
 * integer block dots and f32 block scales (llama.cpp's q8_1 scheme, not present here). The
 * build's own definition of it is restated below (jko_quantize_act_q8, jko_matmul_q8_int8):
 * parity of that path is pinned to this restatement only.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stddef.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* GGML type ids, as TensorType::from_id (gguf.rs:123-131). */
enum { T_F32 = 0, T_F16 = 1, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4K = 12, T_Q6K = 14 };

/* (elements per block, bytes per block); 0 on unsupported (gguf.rs:134-145). */
int jko_block(int kind, uint64_t *elems, uint64_t *bytes) {
    switch (kind) {
    case T_F32: *elems = 1; *bytes = 4; return 1;
    case T_F16: *elems = 1; *bytes = 2; return 1;
    case T_Q4K: *elems = 256; *bytes = 144; return 1;
    case T_Q5_0: *elems = 32; *bytes = 22; return 1;
    case T_Q6K: *elems = 256; *bytes = 210; return 1;
    case T_Q8_0: *elems = 32; *bytes = 34; return 1;
    default: *elems = 0; *bytes = 0; return 0;
    }
}

/* IEEE binary16 -> binary32, exact. */
float jko_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400));
            man &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float half_at(const uint8_t *p) { return jko_half_to_float((uint16_t)(p[0] | (p[1] << 8))); }

/* quant.rs:14-23 */
void jko_q4k_scale_min(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 15) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* quant.rs:25-41 */
static void dequant_q4k(const uint8_t *b, float *out) {
    const float d = half_at(b), dmin = half_at(b + 2);
    const uint8_t *scales = b + 4, *qs = b + 16;
    for (int pair = 0; pair < 4; pair++) {
        uint8_t s0, m0, s1, m1;
        jko_q4k_scale_min(2 * pair, scales, &s0, &m0);
        jko_q4k_scale_min(2 * pair + 1, scales, &s1, &m1);
        const float d0 = d * (float)s0, n0 = dmin * (float)m0;
        const float d1 = d * (float)s1, n1 = dmin * (float)m1;
        for (int l = 0; l < 32; l++) {
            const uint8_t q = qs[pair * 32 + l];
            out[pair * 64 + l] = d0 * (float)(q & 15) - n0;
            out[pair * 64 + 32 + l] = d1 * (float)(q >> 4) - n1;
        }
    }
}

/* quant.rs:43-61 */
static void dequant_q6k(const uint8_t *b, float *out) {
    const float d = half_at(b + 208);
    for (int n = 0; n < 2; n++) {
        const uint8_t *ql = b + 64 * n, *qh = b + 128 + 32 * n, *sc = b + 192 + 8 * n;
        float *o = out + 128 * n;
        for (int l = 0; l < 32; l++) {
            const int is = l / 16;
            const int q1 = ((ql[l] & 15) | ((qh[l] & 3) << 4)) - 32;
            const int q2 = ((ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            o[l] = d * (float)(int8_t)sc[is] * (float)q1;
            o[l + 32] = d * (float)(int8_t)sc[is + 2] * (float)q2;
            o[l + 64] = d * (float)(int8_t)sc[is + 4] * (float)q3;
            o[l + 96] = d * (float)(int8_t)sc[is + 6] * (float)q4;
        }
    }
}

/* quant.rs:63-73 */
static void dequant_q5_0(const uint8_t *b, float *out) {
    const float d = half_at(b);
    const uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
    const uint8_t *qs = b + 6;
    for (int j = 0; j < 16; j++) {
        const uint32_t h0 = ((qh >> j) << 4) & 0x10;
        const uint32_t h1 = (qh >> (j + 12)) & 0x10;
        out[j] = d * (float)((int32_t)((qs[j] & 15) | h0) - 16);
        out[j + 16] = d * (float)((int32_t)((qs[j] >> 4) | h1) - 16);
    }
}

/* quant.rs:75-80 */
static void dequant_q8_0(const uint8_t *b, float *out) {
    const float d = half_at(b);
    for (int i = 0; i < 32; i++) out[i] = d * (float)(int8_t)b[2 + i];
}

/* quant.rs:83-101. Returns 0 on success, 1 unsupported type, 2 size mismatch. */
int jko_dequantize(int kind, const uint8_t *bytes, size_t len, float *out, size_t out_len) {
    uint64_t be, bb;
    if (!jko_block(kind, &be, &bb)) return 1;
    if (len % bb != 0 || out_len != len / bb * be) return 2;
    const size_t blocks = len / bb;
#pragma omp parallel for schedule(static) if (blocks > 4096)
    for (size_t i = 0; i < blocks; i++) {
        const uint8_t *src = bytes + i * bb;
        float *dst = out + i * be;
        switch (kind) {
        case T_F32: memcpy(dst, src, 4); break;
        case T_F16: dst[0] = half_at(src); break;
        case T_Q4K: dequant_q4k(src, dst); break;
        case T_Q6K: dequant_q6k(src, dst); break;
        case T_Q5_0: dequant_q5_0(src, dst); break;
        case T_Q8_0: dequant_q8_0(src, dst); break;
        }
    }
    return 0;
}

/* quant.rs:128-136: words per block of (q, h, s, d). */
void jko_packed_words(int kind, size_t w[4]) {
    w[0] = w[1] = w[2] = w[3] = 0;
    switch (kind) {
    case T_Q4K: w[0] = 36; break;
    case T_Q6K: w[0] = 32; w[1] = 16; w[2] = 4; w[3] = 1; break;
    case T_Q5_0: w[0] = 4; w[1] = 1; w[3] = 1; break;
    case T_Q8_0: w[0] = 8; w[3] = 1; break;
    }
}

static uint32_t le32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* quant.rs:156-193. Region sizes follow jko_packed_words. Returns 0 ok, 1 unsupported,
 * 2 not a whole number of blocks. */
int jko_pack(int kind, const uint8_t *bytes, size_t len, uint32_t *q, uint32_t *h, uint32_t *s, float *d) {
    uint64_t be, bb;
    if (!jko_block(kind, &be, &bb)) return 1;
    if (kind != T_Q4K && kind != T_Q6K && kind != T_Q5_0 && kind != T_Q8_0) return 1;
    if (len % bb != 0) return 2;
    const size_t blocks = len / bb;
    for (size_t i = 0; i < blocks; i++) {
        const uint8_t *b = bytes + i * bb;
        switch (kind) {
        case T_Q4K:
            for (int w = 0; w < 36; w++) q[i * 36 + w] = le32(b + 4 * w);
            break;
        case T_Q6K:
            for (int w = 0; w < 32; w++) q[i * 32 + w] = le32(b + 4 * w);
            for (int w = 0; w < 16; w++) h[i * 16 + w] = le32(b + 128 + 4 * w);
            for (int w = 0; w < 4; w++) s[i * 4 + w] = le32(b + 192 + 4 * w);
            d[i] = half_at(b + 208);
            break;
        case T_Q5_0:
            d[i] = half_at(b);
            h[i] = le32(b + 2);
            for (int w = 0; w < 4; w++) q[i * 4 + w] = le32(b + 6 + 4 * w);
            break;
        case T_Q8_0:
            d[i] = half_at(b);
            for (int w = 0; w < 8; w++) q[i * 8 + w] = le32(b + 2 + 4 * w);
            break;
        }
    }
    return 0;
}

/* f64 product of the GPU tests (tests.rs:445-452): out[r*n + c] = sum_j x[r*k+j] * w[c*k+j],
 * with x already rounded to the activation dtype and w already dequantized. */
void jko_matmul_f64(const float *x, size_t m, size_t k, const float *w, size_t n, double *out) {
#pragma omp parallel for collapse(2) schedule(static)
    for (size_t r = 0; r < m; r++) {
        for (size_t c = 0; c < n; c++) {
            const float *xr = x + r * k, *wc = w + c * k;
            double acc = 0.0;
            for (size_t j = 0; j < k; j++) acc += (double)xr[j] * (double)wc[j];
            out[r * n + c] = acc;
        }
    }
}

/* Row norms |x_r| (f64), used by the output tolerance max|err| <= 1e-3 |x_r| |w_c|. */
void jko_row_norms(const float *a, size_t rows, size_t k, double *out) {
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; r++) {
        double s = 0.0;
        for (size_t j = 0; j < k; j++) s += (double)a[r * k + j] * (double)a[r * k + j];
        out[r] = sqrt(s);
    }
}

/* CPU baseline kernel: fused dequant + dot over raw GGML rows, f32 accumulation, one output
 * column per iteration, OpenMP over columns. This is the reference's CPU arithmetic
 * (quant.rs dequant feeding an f32 product) arranged so nothing is materialised:
 * out[r*n + c] = sum_j x[r*k + j] * dequant(W)[c, j]. Returns 0 ok, nonzero on bad type. */
int jko_gemv_fused(int kind, const uint8_t *raw, size_t n, size_t k, const float *x, size_t m, float *out, int threads) {
    uint64_t be, bb;
    if (!jko_block(kind, &be, &bb)) return 1;
    if (k % be != 0 || m == 0 || m > 64) return 2;
    const size_t nb = k / be, row_bytes = nb * bb;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel
    {
        float wbuf[256];
        float acc[64];
#pragma omp for schedule(static)
        for (size_t c = 0; c < n; c++) {
            for (size_t r = 0; r < m; r++) acc[r] = 0.0f;
            const uint8_t *row = raw + c * row_bytes;
            for (size_t b = 0; b < nb; b++) {
                const uint8_t *blk = row + b * bb;
                switch (kind) {
                case T_Q4K: dequant_q4k(blk, wbuf); break;
                case T_Q6K: dequant_q6k(blk, wbuf); break;
                case T_Q5_0: dequant_q5_0(blk, wbuf); break;
                case T_Q8_0: dequant_q8_0(blk, wbuf); break;
                case T_F16: wbuf[0] = half_at(blk); break;
                case T_F32: memcpy(wbuf, blk, 4); break;
                }
                for (size_t r = 0; r < m; r++) {
                    const float *xr = x + r * k + b * be;
                    if (be >= 8) {
                        /* eight independent partial sums so the loop vectorises */
                        float s8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                        for (size_t j = 0; j < be; j += 8)
                            for (int v = 0; v < 8; v++) s8[v] += wbuf[j + v] * xr[j + v];
                        acc[r] += ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
                    } else {
                        acc[r] += wbuf[0] * xr[0];
                    }
                }
            }
            for (size_t r = 0; r < m; r++) out[r * n + c] = acc[r];
        }
    }
    return 0;
}

int jko_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---------------------------------------------------------------------------------------------
 * Q8_0 int8 path. Activation quantization per (row, 32-value block):
 *   amax = max |x|, d = amax / 127, q = rint(x * (127 / amax)) clamped to [-127, 127]
 * (IEEE f32 division and multiplication, rint = round to nearest even; amax = 0 gives q = 0,
 * d = 0). q -> xq[row * k + j]; d -> xd[(j / 32) * m_pad + row] (block-major scales).
 * --------------------------------------------------------------------------------------------- */
void jko_quantize_act_q8(const float *x, size_t m, size_t k, int8_t *xq, float *xd, size_t m_pad) {
    const size_t nblk = k / 32;
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < m; ++r) {
        for (size_t b = 0; b < nblk; ++b) {
            const float *v = x + r * k + 32 * b;
            float amax = 0.0f;
            for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
            const float d = amax / 127.0f;
            const float id = amax > 0.0f ? 127.0f / amax : 0.0f;
            for (int j = 0; j < 32; ++j) {
                float q = rintf(v[j] * id);
                q = fminf(fmaxf(q, -127.0f), 127.0f);
                xq[r * k + 32 * b + j] = (int8_t)q;
            }
            xd[b * m_pad + r] = d;
        }
    }
}

/* The int8 product over raw GGML Q8_0 rows W [n][k/32][34 bytes]:
 *   dot = sum_j q_w[c, 32b + j] * q_x[r, 32b + j]            (exact int32)
 *   s   = f32(d_w[c, b]) * d_x[r, b]                          (f32 multiply)
 *   acc = fmaf(f32(dot), s, acc)   for b = 0, 1, ... in order (one f32 rounding per block)
 * out[r * n + c] = acc. Also returns the int32 block dots when dots != NULL:
 * dots[(r * n + c) * nblk + b]. */
void jko_matmul_q8_int8(const uint8_t *raw, size_t n, size_t k, const int8_t *xq, const float *xd, size_t m,
                        size_t m_pad, float *out, int32_t *dots) {
    const size_t nblk = k / 32;
#pragma omp parallel for schedule(dynamic, 4)
    for (size_t c = 0; c < n; ++c) {
        const uint8_t *row = raw + c * nblk * 34;
        for (size_t r = 0; r < m; ++r) {
            float acc = 0.0f;
            for (size_t b = 0; b < nblk; ++b) {
                const uint8_t *blk = row + b * 34;
                const int8_t *qx = xq + r * k + 32 * b;
                int32_t dot = 0;
                for (int j = 0; j < 32; ++j) dot += (int32_t)(int8_t)blk[2 + j] * (int32_t)qx[j];
                if (dots) dots[(r * n + c) * nblk + b] = dot;
                const float s = half_at(blk) * xd[b * m_pad + r];
                acc = fmaf((float)dot, s, acc);
            }
            out[r * n + c] = acc;
        }
    }
}
