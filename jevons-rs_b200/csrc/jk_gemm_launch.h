// jk_gemm_launch.h -- the interface between the tensor-core product's host code
// (jk_gemm_sm100.cu: tensor maps, workspaces, argument checks) and its kernel instantiations, one
// translation unit per weight format (jk_gemm_fmt_*.cu, all built from jk_gemm_sm100.cuh), so the
// several hundred kernel variants compile in parallel.
#pragma once

#include "jk_internal.h"

#include <cudaTypedefs.h>

namespace jk {
namespace tc {

constexpr int BW = 128;  // weight rows per tile (MMA M)
constexpr int KB = 64;   // k-block: one 128-byte swizzle atom of 16-bit values

struct LaunchArgs {
    const jk_qmatrix* wq;
    const CUtensorMap* tm_x;  // box rows BT (BT / 2 for pair launches)
    bool pair;                // clusters of 2 CTAs (cta_group::2) for quantized weights at BT >= 128
    float* out;
    int64_t m, ldo;
    bool stream_k;
    float* ws_part;
    uint32_t* ws_flag;
    int grid_cap;  // 0 = SM count x occupancy
    cudaStream_t stream;
    // expert-grouped product (whole tiles): m = sorted activation rows, ldo = n_exp
    const uint32_t* jobs = nullptr;
    const uint32_t* offsets = nullptr;
    const uint32_t* sorted = nullptr;
    int64_t n_exp = 0, max_jobs = 0;
    int job_rows = 0;
};

// One launcher per weight format (bt: activation rows per tile; bf16: activation type, else f16).
jk_status launch_q4k(const LaunchArgs& a, int bt, bool bf16);
jk_status launch_q6k(const LaunchArgs& a, int bt, bool bf16);
jk_status launch_q8_0(const LaunchArgs& a, int bt, bool bf16);
jk_status launch_q5_0(const LaunchArgs& a, int bt, bool bf16);
jk_status launch_f16(const LaunchArgs& a, int bt, bool bf16);

}  // namespace tc
}  // namespace jk
