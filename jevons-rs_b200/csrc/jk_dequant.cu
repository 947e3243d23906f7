// jk_dequant.cu -- whole-matrix device dequantization to f32 (bit-exact with the reference CPU
// code, crates/jevons-formats/src/quant.rs:83-101) and the activation conversion kernel.
//
// One thread decodes one k-block (64 weights) of one row with the same jk_decode.cuh routines
// the tensor-core kernel's dequantizing warps use, so the bit-exact test of this kernel pins
// the f32 values those warps round to bf16/f16.
#include "jk_decode.cuh"
#include "jk_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace jk {

template <int FMT>
__global__ void __launch_bounds__(256) dequant_kernel(WView w, float* __restrict__ out) {
    const int64_t kbs = w.k / 64;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= w.rows * kbs) return;
    const int64_t row = idx / kbs;
    const int64_t kb = idx % kbs;
    const uint8_t* rq = w.q + row * w.q_row_bytes;
    float* o = out + row * w.k + kb * 64;
    float v[8];
    if constexpr (FMT == FMT_Q4K) {
        Q4KBlock b;
        b.load(rq + (kb / 4) * 144, (int)(kb % 4));
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            b.chunk(c, v);
            reinterpret_cast<float4*>(o + 8 * c)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(o + 8 * c)[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
    } else if constexpr (FMT == FMT_Q6K) {
        Q6KBlock b;
        const float d = half_bits_to_float(w.d[row * (w.k / 256) + kb / 4]);
        b.load(rq + (kb / 4) * 208, d, (int)(kb % 4));
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            b.chunk(c, v);
            reinterpret_cast<float4*>(o + 8 * c)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(o + 8 * c)[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
    } else if constexpr (FMT == FMT_Q8_0) {
        Q80Block b;
        const uint16_t* dr = w.d + row * (w.k / 32) + 2 * kb;
        b.load(rq + kb * 64, half_bits_to_float(dr[0]), half_bits_to_float(dr[1]));
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            b.chunk(c, v);
            reinterpret_cast<float4*>(o + 8 * c)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(o + 8 * c)[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
    } else if constexpr (FMT == FMT_Q5_0) {
        Q50Block b;
        const uint16_t* dr = w.d + row * (w.k / 32) + 2 * kb;
        b.load(rq + kb * 32, w.h + row * (w.k / 32) + 2 * kb, half_bits_to_float(dr[0]),
               half_bits_to_float(dr[1]));
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            b.chunk(c, v);
            reinterpret_cast<float4*>(o + 8 * c)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(o + 8 * c)[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
    } else {  // FMT_F16
        const __half* src = reinterpret_cast<const __half*>(rq) + kb * 64;
#pragma unroll 8
        for (int i = 0; i < 64; ++i) o[i] = __half2float(src[i]);
    }
}

jk_status launch_dequant(const WView& w, float* out, cudaStream_t stream) {
    const int64_t total = w.rows * (w.k / 64);
    if (total == 0) return JK_OK;
    const dim3 grid((unsigned)((total + 255) / 256));
    switch (w.fmt) {
    case FMT_Q4K: dequant_kernel<FMT_Q4K><<<grid, 256, 0, stream>>>(w, out); break;
    case FMT_Q6K: dequant_kernel<FMT_Q6K><<<grid, 256, 0, stream>>>(w, out); break;
    case FMT_Q8_0: dequant_kernel<FMT_Q8_0><<<grid, 256, 0, stream>>>(w, out); break;
    case FMT_Q5_0: dequant_kernel<FMT_Q5_0><<<grid, 256, 0, stream>>>(w, out); break;
    default: dequant_kernel<FMT_F16><<<grid, 256, 0, stream>>>(w, out); break;
    }
    return cuda_fail(cudaGetLastError(), "dequantize launch");
}

// f32 or f16 activations -> bf16 (round to nearest even), 8 elements per thread when aligned.
__global__ void __launch_bounds__(256) to_bf16_kernel(const void* __restrict__ x, int dtype, size_t count,
                                                      __nv_bfloat16* __restrict__ out) {
    const size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x);
    const size_t base = i * 8;
    if (base >= count) return;
    const size_t end = base + 8 < count ? base + 8 : count;
    for (size_t j = base; j < end; ++j) {
        float f = dtype == JK_DTYPE_F32 ? reinterpret_cast<const float*>(x)[j]
                                        : __half2float(reinterpret_cast<const __half*>(x)[j]);
        out[j] = __float2bfloat16_rn(f);
    }
}

jk_status launch_convert_to_bf16(const void* x, int x_dtype, size_t count, void* out, cudaStream_t stream) {
    if (count == 0) return JK_OK;
    const size_t threads = (count + 7) / 8;
    to_bf16_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(x, x_dtype, count,
                                                                         reinterpret_cast<__nv_bfloat16*>(out));
    return cuda_fail(cudaGetLastError(), "activation conversion launch");
}

}  // namespace jk
