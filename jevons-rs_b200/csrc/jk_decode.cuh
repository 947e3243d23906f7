// jk_decode.cuh -- exact decode of GGML blocks in the B200 layout, one "k-block" of 64 weights
// of one row at a time, delivered as 8 chunks of 8 consecutive f32 values.
//
// The f32 values are bit-identical to the reference CPU dequantization
// (crates/jevons-formats/src/quant.rs:25-80), which evaluates
//   Q4_K  w = (d*sc)*q - (dmin*m)          quant.rs:33-38
//   Q6_K  w = (d*sc)*(q-32)                quant.rs:50-58 (left-to-right evaluation)
//   Q8_0  w = d*q                          quant.rs:75-80
//   Q5_0  w = d*(q-16)                     quant.rs:63-73
// with separately rounded f32 operations. Every product there is exact in f32: d is an f16
// (11 significant bits), sc <= 63 (6 bits), m <= 63, q <= 15 (Q4_K), |sc| <= 128 and |q-32| <= 32
// (Q6_K), |q| <= 128 (Q8_0), |q-16| <= 16 (Q5_0), so no product needs more than 24 significant
// bits. The only rounding in the reference is Q4_K's final subtraction, so
//   (d*sc)*q - dmin*m == fma(d*sc, q, -(dmin*m))      bit for bit,
// and the other formats are exact products. The code below uses those forms (packed .f32x2
// where two values share a scale). Integers become floats through the exponent trick
// as_float(0x4B000000 | byte) - 2^23 (exact), so no int->float conversion instruction is needed.
//
// A k-block j covers k-elements [64 j, 64 j + 64) of a 256-element super-block (K-quants) or two
// consecutive 32-element blocks (Q8_0, Q5_0). Chunk c holds elements 8c .. 8c+7 of the k-block.
#pragma once

#include "jk_common.cuh"

namespace jk {

// ---------------------------------------------------------------------------------------------
// Q4_K: `blk` points at the row's 144-byte super-block (smem or global, 16-byte aligned).
// ---------------------------------------------------------------------------------------------
struct Q4KBlock {
    uint32_t qs[8];   // the 32 qs bytes of pair j
    float dd_lo, mm_lo, dd_hi, mm_hi;

    __device__ __forceinline__ void load(const uint8_t* blk, int j) {
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint4 a = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j);
        const uint4 b = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j + 16);
        qs[0] = a.x; qs[1] = a.y; qs[2] = a.z; qs[3] = a.w;
        qs[4] = b.x; qs[5] = b.y; qs[6] = b.z; qs[7] = b.w;
        const float d = half_bits_to_float(hdr.x & 0xFFFFu);
        const float dmin = half_bits_to_float(hdr.x >> 16);
        uint32_t s0, m0, s1, m1;
        q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * j, s0, m0);
        q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * j + 1, s1, m1);
        dd_lo = __fmul_rn(d, (float)s0);
        mm_lo = __fmul_rn(dmin, (float)m0);
        dd_hi = __fmul_rn(d, (float)s1);
        mm_hi = __fmul_rn(dmin, (float)m1);
    }
    // chunk c < 4: low nibbles of qs bytes 8c..8c+7 (elements 8c..); c >= 4: high nibbles of
    // bytes 8(c-4).. (elements 32 + 8(c-4)..).
    __device__ __forceinline__ void chunk(int c, float (&v)[8]) const {
        const bool hi = c >= 4;
        const int w0 = 2 * (c & 3);
        const float dd = hi ? dd_hi : dd_lo, mm = hi ? mm_hi : mm_lo;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const uint32_t w = hi ? ((qs[w0 + t] >> 4) & 0x0F0F0F0Fu) : (qs[w0 + t] & 0x0F0F0F0Fu);
#pragma unroll
            for (int i = 0; i < 4; i += 2) {
                const float2 q = sub2(make_float2(magic_byte(w, i), magic_byte(w, i + 1)), make_float2(MAGIC, MAGIC));
                const float2 r = fma2(make_float2(dd, dd), q, make_float2(-mm, -mm));
                v[4 * t + i] = r.x;
                v[4 * t + i + 1] = r.y;
            }
        }
    }
};

// ---------------------------------------------------------------------------------------------
// Q6_K: `body` points at the row's 208-byte super-block body (ql[128] qh[64] sc[16]); d is the
// block's f16 scale already converted.
//   element 128 nh + 32 i + l (i = 0..3, l = 0..31):
//     q = ((ql[64 nh + 32 (i%2) + l] >> 4 (i/2)) & 15) | (((qh[32 nh + l] >> 2i) & 3) << 4)
//     w = (d * sc[8 nh + 2 i + l/16]) * (q - 32)
// K-block j: nh = j/2 and i in {2(j%2), 2(j%2)+1}; chunk c: i = 2(j%2) + c/4, l = 8(c%4)..+8.
// ---------------------------------------------------------------------------------------------
struct Q6KBlock {
    uint32_t ql[16];  // ql bytes 64 nh .. 64 nh + 64
    uint32_t qh[8];   // qh bytes 32 nh .. 32 nh + 32
    float s[4];       // d*sc for (i0 + c/4, (c%4)/2), indexed 2 (c/4) + (c%4)/2
    int nib;          // 0 or 4: low or high nibbles of ql

    __device__ __forceinline__ void load(const uint8_t* body, float d, int j) {
        const int nh = j >> 1;
        const int odd = j & 1;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint4 a = *reinterpret_cast<const uint4*>(body + 64 * nh + 16 * t);
            ql[4 * t] = a.x; ql[4 * t + 1] = a.y; ql[4 * t + 2] = a.z; ql[4 * t + 3] = a.w;
        }
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const uint4 a = *reinterpret_cast<const uint4*>(body + 128 + 32 * nh + 16 * t);
            qh[4 * t] = a.x; qh[4 * t + 1] = a.y; qh[4 * t + 2] = a.z; qh[4 * t + 3] = a.w;
        }
        // sc bytes 8 nh + 4 odd + {0,1,2,3}: one 32-bit word (4-byte aligned)
        const uint32_t sw = *reinterpret_cast<const uint32_t*>(body + 192 + 8 * nh + 4 * odd);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int sc = (int)(int8_t)((sw >> (8 * t)) & 0xFFu);
            s[t] = __fmul_rn(d, (float)sc);
        }
        nib = 4 * odd;
    }
    __device__ __forceinline__ void chunk(int c, float (&v)[8]) const {
        const int i1 = c >> 2;                 // i - i0
        const int hshift = nib + 2 * i1;       // 2 i = 4 (j%2) + 2 (c/4)
        const float sc = s[2 * i1 + ((c & 3) >> 1)];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const uint32_t wl = (ql[2 * c + t] >> nib) & 0x0F0F0F0Fu;
            const uint32_t wh = ((qh[2 * (c & 3) + t] >> hshift) & 0x03030303u) << 4;
            const uint32_t q = wl | wh;
#pragma unroll
            for (int i = 0; i < 4; i += 2) {
                const float2 qf = sub2(make_float2(magic_byte(q, i), magic_byte(q, i + 1)),
                                       make_float2(MAGIC + 32.0f, MAGIC + 32.0f));
                const float2 r = mul2(make_float2(sc, sc), qf);
                v[4 * t + i] = r.x;
                v[4 * t + i + 1] = r.y;
            }
        }
    }
};

// ---------------------------------------------------------------------------------------------
// Q8_0: 64 int8 quants (two blocks) and their two scales.
// ---------------------------------------------------------------------------------------------
struct Q80Block {
    uint32_t q[16];
    float d0, d1;

    __device__ __forceinline__ void load(const uint8_t* q64, float d0_, float d1_) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint4 a = *reinterpret_cast<const uint4*>(q64 + 16 * t);
            q[4 * t] = a.x; q[4 * t + 1] = a.y; q[4 * t + 2] = a.z; q[4 * t + 3] = a.w;
        }
        d0 = d0_;
        d1 = d1_;
    }
    // Load from a 128-byte-swizzled smem row: logical 16-byte chunk u of the row lives at
    // physical chunk u ^ (row & 7). `row128` points at the row's 128-byte line, `u0` is the first
    // logical chunk of this k-block (0 or 4).
    __device__ __forceinline__ void load_sw(const uint8_t* row128, int u0, int row, float d0_, float d1_) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint4 a = *reinterpret_cast<const uint4*>(row128 + 16 * ((u0 + t) ^ (row & 7)));
            q[4 * t] = a.x; q[4 * t + 1] = a.y; q[4 * t + 2] = a.z; q[4 * t + 3] = a.w;
        }
        d0 = d0_;
        d1 = d1_;
    }
    __device__ __forceinline__ void chunk(int c, float (&v)[8]) const {
        const float d = c < 4 ? d0 : d1;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const uint32_t w = q[2 * c + t] ^ 0x80808080u;  // signed byte -> byte + 128
#pragma unroll
            for (int i = 0; i < 4; i += 2) {
                const float2 qf = sub2(make_float2(magic_byte(w, i), magic_byte(w, i + 1)),
                                       make_float2(MAGIC + 128.0f, MAGIC + 128.0f));
                const float2 r = mul2(make_float2(d, d), qf);
                v[4 * t + i] = r.x;
                v[4 * t + i + 1] = r.y;
            }
        }
    }
};

// ---------------------------------------------------------------------------------------------
// Q5_0: two blocks; per block 16 nibble bytes (byte e: low nibble = element e, high = e + 16),
// 32 high bits (bit e -> element e), f16 scale.
// ---------------------------------------------------------------------------------------------
struct Q50Block {
    uint32_t qs[8];
    uint32_t qh[2];
    float d[2];

    __device__ __forceinline__ void load(const uint8_t* qs32, const uint32_t* qh2, float d0, float d1) {
        load_words(*reinterpret_cast<const uint4*>(qs32), *reinterpret_cast<const uint4*>(qs32 + 16), qh2[0], qh2[1],
                   d0, d1);
    }
    // a, b: the two blocks' 16 nibble bytes; h0, h1: their high-bit words.
    __device__ __forceinline__ void load_words(uint4 a, uint4 b, uint32_t h0, uint32_t h1, float d0, float d1) {
        qs[0] = a.x; qs[1] = a.y; qs[2] = a.z; qs[3] = a.w;
        qs[4] = b.x; qs[5] = b.y; qs[6] = b.z; qs[7] = b.w;
        qh[0] = h0;
        qh[1] = h1;
        d[0] = d0;
        d[1] = d1;
    }
    __device__ __forceinline__ void chunk(int c, float (&v)[8]) const {
        const int b = c >> 2;             // block
        const int e0 = 8 * (c & 3);       // first element within the block
        const bool hi = e0 >= 16;
        const float dd = d[b];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int byte0 = (e0 & 15) + 4 * t;
            uint32_t w = qs[4 * b + (byte0 >> 2)];
            w = hi ? ((w >> 4) & 0x0F0F0F0Fu) : (w & 0x0F0F0F0Fu);
            // high bits of elements e0 + 4t .. +3 into bit 4 of each byte
            const uint32_t hb = qh[b] >> (e0 + 4 * t);
            const uint32_t hbytes = ((hb & 1u) << 4) | ((hb & 2u) << 11) | ((hb & 4u) << 18) | ((hb & 8u) << 25);
            w |= hbytes;
#pragma unroll
            for (int i = 0; i < 4; i += 2) {
                const float2 qf = sub2(make_float2(magic_byte(w, i), magic_byte(w, i + 1)),
                                       make_float2(MAGIC + 16.0f, MAGIC + 16.0f));
                const float2 r = mul2(make_float2(dd, dd), qf);
                v[4 * t + i] = r.x;
                v[4 * t + i + 1] = r.y;
            }
        }
    }
};

}  // namespace jk
