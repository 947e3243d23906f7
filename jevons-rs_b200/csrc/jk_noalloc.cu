// jk_noalloc.cu -- the allocation-free stream-K product (jk_matmul_splitk_noalloc).
//
// Some callers cannot allocate device memory at the time they run a product: code that runs
// under an allocator or pool it does not control (a framework that owns every cudaMalloc on the
// device, so a library allocation would bypass its accounting or fail under its memory cap), and
// latency-critical paths where a cudaMalloc -- which synchronises the device -- is not
// acceptable. For them this entry point runs the split-K (stream-K) tensor-core product with its
// scratch in a fixed buffer that the library itself declares below; it calls no cudaMalloc,
// cudaFree or allocating routine. Its first call on a device looks up the buffer's device address
// (cudaGetSymbolAddress, no allocation): make that first call before any stream capture.
//
// The buffer is a file-scope __device__ array: every GPU that loads libjk.so holds
// JK_NOALLOC_SCRATCH_BYTES (20 MiB) of device memory for it until the process exits. Its layout:
// 4096 bytes of flag words (one per CTA), then one BT x 128 f32 partial tile per CTA. All calls
// on a device share it, so two calls that may run at the same time on the GPU (different
// streams without ordering between them) race on it; callers must order them (same stream, or
// events). The flag words must start at zero: each call clears them on its stream before the
// kernel; the partial tiles are fully written before they are read, so they need no clearing.
#include "jk_internal.h"

#include <cstdio>
#include <mutex>

namespace {

constexpr size_t FLAG_BYTES = 4096;  // flag words for up to 1024 CTAs

static __device__ __align__(256) unsigned char g_jk_noalloc_scratch[JK_NOALLOC_SCRATCH_BYTES];

// Device address of g_jk_noalloc_scratch on `device`, looked up once per device with that device
// current. In host code the array's name is only a handle for the runtime, never an address.
jk_status scratch_address(int device, unsigned char** out) {
    static std::mutex mu;
    static unsigned char* addr[64] = {};
    if (device < 0 || device >= 64) return jk::fail(JK_ERR_INVALID, "device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[device]) {
        int prev = -1;
        cudaGetDevice(&prev);
        if (prev != device) {
            cudaError_t e = cudaSetDevice(device);
            if (e != cudaSuccess) return jk::cuda_fail(e, "cudaSetDevice");
        }
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_jk_noalloc_scratch);
        if (prev != device && prev >= 0) cudaSetDevice(prev);
        if (e != cudaSuccess || !p) return jk::cuda_fail(e == cudaSuccess ? cudaErrorInvalidSymbol : e,
                                                         "allocation-free scratch address (cudaGetSymbolAddress)");
        addr[device] = static_cast<unsigned char*>(p);
    }
    *out = addr[device];
    return JK_OK;
}

}  // namespace

extern "C" jk_status jk_matmul_splitk_noalloc(const jk_qmatrix* w, const void* x, int x_dtype, size_t x_len,
                                              size_t m, float* out, size_t out_len, int bm, void* stream) {
    if (!w) return jk::fail(JK_ERR_INVALID, "null matrix");
    if (bm != 32 && bm != 64 && bm != 128 && bm != 256)
        return jk::fail(JK_ERR_INVALID, "bm must be 32, 64, 128 or 256");
    if (x_dtype != JK_DTYPE_BF16 && x_dtype != JK_DTYPE_F16)
        return jk::fail(JK_ERR_UNSUPPORTED,
                        "the allocation-free product takes bf16 or f16 activations (f32 would need a conversion buffer)");
    if (w->type == JK_TYPE_F16 && x_dtype != JK_DTYPE_F16)
        return jk::fail(JK_ERR_UNSUPPORTED, "FP16 weights need FP16 activations");
    // m is bounded first so that m * k and m * n below cannot wrap around
    if (m > (size_t)INT32_MAX) return jk::fail(JK_ERR_INVALID, "m too large");
    if (x_len < m * w->k || out_len < m * w->n) {
        char buf[160];
        snprintf(buf, sizeof buf, "buffers too small for m=%zu (x %zu < %zu or out %zu < %zu)", m, x_len, m * w->k,
                 out_len, m * w->n);
        return jk::fail(JK_ERR_INVALID, buf);
    }
    if (m == 0) return JK_OK;
    if (!x || !out) return jk::fail(JK_ERR_INVALID, "null activation or output pointer");
    if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return jk::fail(JK_ERR_INVALID, "activations must be 16-byte aligned");

    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != w->device) {
        cudaError_t e = cudaSetDevice(w->device);
        if (e != cudaSuccess) return jk::cuda_fail(e, "cudaSetDevice");
    }
    unsigned char* base = nullptr;
    jk_status st = scratch_address(w->device, &base);
    if (st == JK_OK) {
        cudaStream_t cs = static_cast<cudaStream_t>(stream);
        const int max_ctas = (int)((JK_NOALLOC_SCRATCH_BYTES - FLAG_BYTES) / ((size_t)bm * 128 * 4));
        const int cap = max_ctas < (int)(FLAG_BYTES / 4) ? max_ctas : (int)(FLAG_BYTES / 4);
        cudaError_t e = cudaMemsetAsync(base, 0, FLAG_BYTES, cs);  // flags start at zero
        if (e != cudaSuccess) {
            st = jk::cuda_fail(e, "clearing the allocation-free scratch flags");
        } else {
            jk_qmatrix dense = *w;
            dense.view.rows = (int64_t)w->n;  // dense products use expert 0's rows
            st = jk::launch_gemm_stream_k_fixed(&dense, x, x_dtype == JK_DTYPE_BF16, m, out, bm,
                                                reinterpret_cast<uint32_t*>(base),
                                                reinterpret_cast<float*>(base + FLAG_BYTES), cap,
                                                JK_NOALLOC_SCRATCH_BYTES, cs);
        }
    }
    if (prev != w->device && prev >= 0) cudaSetDevice(prev);
    return st;
}
