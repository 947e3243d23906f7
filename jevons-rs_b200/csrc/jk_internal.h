// jk_internal.h -- host-side declarations shared by the library's translation units.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/jk.h"
#include "jk_common.cuh"

struct jk_qmatrix {
    int type;            // GGML type id (jk_tensor_type)
    int device;
    size_t n, k, experts;
    jk::WView view;      // device pointers + shape
    void* q_alloc;       // owned allocations (null for views)
    void* d_alloc;
    void* h_alloc;
    size_t device_bytes;
    bool has_tmap;       // tm_w valid
    CUtensorMap tm_w;    // TMA descriptor of the raw weight tiles used by the tensor-core kernel
};

struct jk_split_scratch {
    int device;
    void* buf;
    size_t bytes;
};

namespace jk {

// Makes `dev` the current device for the scope and restores the previous one.
struct DeviceGuard {
    int prev = -1;
    bool changed = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) changed = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (changed) cudaSetDevice(prev);
    }
};

// Thread-local error message; returns `st` for convenient `return fail(...)`.
jk_status fail(jk_status st, const std::string& msg);
jk_status cuda_fail(cudaError_t e, const char* what);

// Per-device error word (a __device__ variable; no allocation).
uint32_t* device_error_word(int device);

// Grows a split scratch to at least `bytes` (cudaMalloc + zeroing on growth, which synchronise the
// device) and returns its base; the first stream_k_flag_bytes() stay zero between products.
jk_status scratch_reserve(jk_split_scratch* s, size_t bytes, void** out);

// Multiprocessor count of `device` (cached).
int sm_count(int device);
// SMs the products may occupy on `device`: sm_count, or the jk_set_max_ctas cap when smaller.
int sm_budget(int device);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link needed).
jk_status encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, uint64_t dim0, uint64_t dim1,
                         uint64_t stride1_bytes, uint32_t box0, uint32_t box1,
                         CUtensorMapSwizzle swizzle, const void* base);

// Kernel launchers (defined next to their kernels). All asynchronous on `stream`.
jk_status launch_dequant(const WView& w, float* out, cudaStream_t stream);
jk_status launch_gemv(const WView& w, const void* x, int x_dtype, size_t m, float* out,
                      cudaStream_t stream);
// Weight tensor map for the tensor-core kernel (stored in the qmatrix at creation).
jk_status make_weight_tmap(const WView& w, CUtensorMap* map);
// Tensor-core GEMM: bt = activation-row tile (32/64/128/256); x is bf16 or f16 [m][k].
// stream_k selects the stream-K schedule (K split across CTAs, partials combined in-kernel in
// fixed k order), which needs `workspace` of stream_k_workspace_bytes() whose first
// stream_k_flag_bytes() are zero; otherwise whole tiles per CTA (row invariant).
size_t stream_k_flag_bytes(int device);
size_t stream_k_workspace_bytes(int device, int bt);
jk_status launch_gemm(const jk_qmatrix* w, const void* x, bool x_bf16, size_t m, float* out, int bt, bool pair,
                      bool stream_k, void* workspace, size_t workspace_bytes, cudaStream_t stream);
jk_status launch_gemm_stream_k_fixed(const jk_qmatrix* w, const void* x, bool x_bf16, size_t m, float* out, int bt,
                                     uint32_t* flags, float* partials, int max_ctas, size_t capacity_bytes,
                                     cudaStream_t stream);
jk_status launch_convert_to_bf16(const void* x, int x_dtype, size_t count, void* out,
                                 cudaStream_t stream);

// Expert-grouped products. The grouped GEMM runs whole tiles over (weight tile, job) pairs:
// x_sorted holds the activation rows in expert-sorted order ([rows][k], bf16 or f16), job j covers
// sorted rows [jobs[2j+2], min(+job_rows, offsets[e+1])) of expert e = jobs[2j+1] with weight rows
// e*n.., and sorted row s is written to out row sorted[s] ([*, n] f32). Jobs at or past jobs[0]
// are skipped on the device.
jk_status launch_gemm_grouped(const jk_qmatrix* w, const void* x_sorted, bool x_bf16, size_t rows,
                              const uint32_t* sorted, const uint32_t* offsets, const uint32_t* jobs, size_t max_jobs,
                              int job_rows, float* out, int bt, bool pair, cudaStream_t stream);
// Deterministic grouping of `assignments` expert ids (one CTA); experts <= GROUP_MAX_EXPERTS.
constexpr size_t GROUP_MAX_EXPERTS = 1024;
jk_status launch_group_experts(const uint32_t* ids, size_t assignments, size_t experts, int bm, size_t max_jobs,
                               uint32_t* sorted, uint32_t* offsets, uint32_t* jobs, uint32_t* err,
                               cudaStream_t stream);
// Grouped small-row product: the GEMV over jobs of <= job_rows (<= 16) rows, grid y = max_jobs;
// activation rows are read in place (x[sorted[s] / in_div], x_rows of them).
jk_status launch_gemv_grouped(const WView& w, const void* x, int x_dtype, size_t x_rows, const uint32_t* sorted,
                              const uint32_t* offsets, const uint32_t* jobs, size_t max_jobs, uint32_t in_div,
                              int job_rows, size_t rows, float* out, cudaStream_t stream);
// out[s] = x[sorted[s] / in_div] converted to bf16 (out_bf16) or f16; rows past x_rows become 0.
jk_status launch_gather_rows(const void* x, int x_dtype, size_t x_rows, size_t k, const uint32_t* sorted,
                             size_t rows, uint32_t in_div, void* out, bool out_bf16, cudaStream_t stream);

}  // namespace jk
