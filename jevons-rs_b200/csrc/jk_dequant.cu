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

// f32 or f16 activations -> bf16 (round to nearest even), 8 elements per thread: one or two
// 16-byte loads and one 16-byte store when the buffers are 16-byte aligned and the count a multiple
// of 8 (every activation matrix here: k % 64 == 0), element by element otherwise.
// Launched with programmatic dependent launch: the kernel lets the product that follows start its
// prologue at once and waits for the previous kernel (which may have written x) before reading.
__global__ void __launch_bounds__(256) to_bf16_kernel(const void* __restrict__ x, int dtype, size_t count,
                                                      __nv_bfloat16* __restrict__ out, int vec) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x);
    const size_t base = i * 8;
    if (base >= count) return;
    if (vec) {
        float f[8];
        if (dtype == JK_DTYPE_F32) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(x) + 2 * i);
            const float4 b = __ldg(reinterpret_cast<const float4*>(x) + 2 * i + 1);
            f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
        } else {
            const uint4 a = __ldg(reinterpret_cast<const uint4*>(x) + i);
            const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&u[j]));
                f[2 * j] = h.x;
                f[2 * j + 1] = h.y;
            }
        }
        uint4 o;
        o.x = pack2<true>(f[0], f[1]);
        o.y = pack2<true>(f[2], f[3]);
        o.z = pack2<true>(f[4], f[5]);
        o.w = pack2<true>(f[6], f[7]);
        reinterpret_cast<uint4*>(out)[i] = o;
        return;
    }
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
    const int vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0 && count % 8 == 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((threads + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, to_bf16_kernel, x, x_dtype, count, reinterpret_cast<__nv_bfloat16*>(out), vec);
    if (e != cudaSuccess) return cuda_fail(e, "activation conversion launch");
    return cuda_fail(cudaGetLastError(), "activation conversion launch");
}

}  // namespace jk
