// jk_linear.cu -- jevons_burn::kernels::f16_linear_scaled (crates/jevons-burn/src/kernels.rs:116-129)
// on the FP16 tensor-core product.
//
// The reference divides every row of x whose largest magnitude exceeds F16_ROW_LIMIT = 16384 by
// s = max|x_r| / 16384 (f32 division, clamped below at exactly 1), casts to FP16, runs f16_linear
// and multiplies the row's outputs back by s. Here:
//   rowscale_f16_kernel  one CTA per row: the row maximum (warp shuffles + one word per warp),
//                        s_r, and f16(x / s_r) with IEEE division and round-to-nearest-even, as
//                        the reference's f32 division and FP16 cast;
//   the FP16 product     jk_matmul_plan over an FP16 view of the weights (the f16_linear plan);
//   rowmul_kernel        out[r, :] *= s_r in f32 (rows with s_r == 1 are unchanged bit for bit).
#include "jk_internal.h"

#include <cuda_fp16.h>

#include <cstdio>

namespace jk {
namespace {

constexpr float F16_ROW_LIMIT = 16384.0f;  // kernels.rs:105

__global__ void __launch_bounds__(256) rowscale_f16_kernel(const float* __restrict__ x, int64_t k,
                                                           __half* __restrict__ xh, float* __restrict__ scale) {
    const float* xr = x + (int64_t)blockIdx.x * k;
    float amax = 0.f;
    for (int64_t j = threadIdx.x; j < k; j += blockDim.x) amax = fmaxf(amax, fabsf(xr[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    __shared__ float part[8];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = amax;
    __syncthreads();
    float m = part[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, part[i]);
    const float s = fmaxf(__fdiv_rn(m, F16_ROW_LIMIT), 1.0f);
    if (threadIdx.x == 0) scale[blockIdx.x] = s;
    __half* hr = xh + (int64_t)blockIdx.x * k;
    for (int64_t j = threadIdx.x; j < k; j += blockDim.x) hr[j] = __float2half_rn(__fdiv_rn(xr[j], s));
}

__global__ void __launch_bounds__(256) rowmul_kernel(float* __restrict__ out, int64_t total, int64_t n,
                                                     const float* __restrict__ scale) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __fmul_rn(out[i], scale[i / n]);
}

}  // namespace
}  // namespace jk

using jk::fail;

extern "C" jk_status jk_f16_linear_scaled(const float* x_f32, size_t m, size_t k, const void* w_f16, size_t n,
                                          float* out, jk_split_scratch* scratch, void* stream) {
    if (k % 64 || n % 64 || k == 0 || n == 0) {
        char buf[96];
        snprintf(buf, sizeof buf, "F16 [%zu, %zu] has an unsupported shape", n, k);
        return fail(JK_ERR_SHAPE, buf);
    }
    if (m == 0) return JK_OK;
    if (!x_f32 || !w_f16 || !out) return fail(JK_ERR_INVALID, "null activation, weight or output pointer");
    if (!scratch) return fail(JK_ERR_INVALID, "f16_linear_scaled needs a scratch for the scaled FP16 rows");
    if (m > (size_t)INT32_MAX) return fail(JK_ERR_INVALID, "m too large");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return jk::cuda_fail(e, "cudaGetDevice");
    if (scratch->device != dev) return fail(JK_ERR_INVALID, "scratch belongs to another device");
    // The scratch's first bytes are the stream-K flag words other products expect to find zero:
    // the FP16 rows and the row scales go after them.
    const size_t flags = jk::stream_k_flag_bytes(dev);
    const size_t xh_bytes = (m * k * 2 + 255) / 256 * 256;
    void* sbuf = nullptr;
    jk_status st = jk::scratch_reserve(scratch, flags + xh_bytes + m * 4, &sbuf);
    if (st != JK_OK) return st;
    __half* xh = reinterpret_cast<__half*>(static_cast<char*>(sbuf) + flags);
    float* scale = reinterpret_cast<float*>(static_cast<char*>(sbuf) + flags + xh_bytes);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    jk::rowscale_f16_kernel<<<(unsigned)m, 256, 0, cs>>>(x_f32, (int64_t)k, xh, scale);
    e = cudaGetLastError();
    if (e != cudaSuccess) return jk::cuda_fail(e, "row scale launch");
    st = jk_f16_linear(xh, m, k, w_f16, n, out, stream);
    if (st != JK_OK) return st;
    const size_t total = m * n, blocks = (total + 255) / 256;
    jk::rowmul_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, cs>>>(out, (int64_t)total, (int64_t)n, scale);
    return jk::cuda_fail(cudaGetLastError(), "row rescale launch");
}
