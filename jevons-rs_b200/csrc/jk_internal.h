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

// Thread-local error message; returns `st` for convenient `return fail(...)`.
jk_status fail(jk_status st, const std::string& msg);
jk_status cuda_fail(cudaError_t e, const char* what);

// Per-device error word (a __device__ variable; no allocation).
uint32_t* device_error_word(int device);

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

}  // namespace jk
