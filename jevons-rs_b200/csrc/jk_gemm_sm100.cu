// jk_gemm_sm100.cu -- host side of the tensor-core product out[r, c] = sum_j x[r, j] W[c, j] on
// sm_100a (the reference's `gemm` kernel with `matmul_split` / `reduce_splits`,
// crates/jevons-kernels/src/gemm.rs:532-815 and :1205-1269): weight and activation tensor maps,
// the stream-K workspace, and the dispatch to the per-format kernel units (jk_gemm_fmt_*.cu; the
// kernels themselves are in jk_gemm_sm100.cuh).
#include "jk_gemm_launch.h"

#include <cstdio>

namespace jk {

using tc::BW;
using tc::KB;
using tc::LaunchArgs;

namespace {

jk_status launch_tc_fmt(const LaunchArgs& a, int bt, bool bf16) {
    switch (a.wq->view.fmt) {
    case FMT_Q4K: return tc::launch_q4k(a, bt, bf16);
    case FMT_Q6K: return tc::launch_q6k(a, bt, bf16);
    case FMT_Q8_0: return tc::launch_q8_0(a, bt, bf16);
    case FMT_Q5_0: return tc::launch_q5_0(a, bt, bf16);
    default: return tc::launch_f16(a, bt, bf16);
    }
}

}  // namespace

jk_status make_weight_tmap(const WView& w, CUtensorMap* map) {
    const uint64_t rows = (uint64_t)w.rows;
    switch (w.fmt) {
    case FMT_Q4K:
        return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, (uint64_t)(w.k / 256) * 36, rows,
                              (uint64_t)w.q_row_bytes, 36, BW, CU_TENSOR_MAP_SWIZZLE_NONE, w.q);
    case FMT_Q6K:
        return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, (uint64_t)(w.k / 256) * 52, rows,
                              (uint64_t)w.q_row_bytes, 52, BW, CU_TENSOR_MAP_SWIZZLE_NONE, w.q);
    case FMT_Q8_0:
        return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)w.k, rows, (uint64_t)w.q_row_bytes,
                              128, BW, CU_TENSOR_MAP_SWIZZLE_128B, w.q);
    case FMT_Q5_0:
        return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(w.k / 2), rows,
                              (uint64_t)w.q_row_bytes, 128, BW, CU_TENSOR_MAP_SWIZZLE_128B, w.q);
    default:
        return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)w.k, rows, (uint64_t)w.q_row_bytes,
                              KB, BW, CU_TENSOR_MAP_SWIZZLE_128B, w.q);
    }
}

// Stream-K workspace layout: first one u32 flag per CTA (at most 2 CTAs per SM), padded to 256
// bytes -- at a fixed offset so the flags are the same words whatever the tile shape, and zero
// between launches (the kernel leaves them zero) -- then one BT x 128 f32 partial tile per CTA.
size_t stream_k_flag_bytes(int device) {
    return ((size_t)sm_count(device) * 2 * 4 + 255) / 256 * 256;
}

size_t stream_k_workspace_bytes(int device, int bt) {
    return stream_k_flag_bytes(device) + (size_t)sm_count(device) * 2 * (size_t)bt * BW * 4;
}

jk_status launch_gemm(const jk_qmatrix* w, const void* x, bool x_bf16, size_t m, float* out, int bt, bool pair_tile, bool stream_k,
                      void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (m == 0) return JK_OK;
    if (!w->has_tmap) return fail(JK_ERR_INVALID, "matrix has no tensor-core layout");
    // 256-row tiles on CTA pairs (each SM loads half the activation tile); see the plan's bn
    const bool pair = pair_tile && w->view.fmt != FMT_F16 && bt >= 128;
    CUtensorMap tm_x;
    jk_status st = encode_tmap_2d(&tm_x, x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                  (uint64_t)w->k, (uint64_t)m, (uint64_t)w->k * 2, KB, (uint32_t)(pair ? bt / 2 : bt),
                                  CU_TENSOR_MAP_SWIZZLE_128B, x);
    if (st != JK_OK) return st;
    LaunchArgs a{};
    a.wq = w;
    a.tm_x = &tm_x;
    a.pair = pair;
    a.out = out;
    a.m = (int64_t)m;
    a.ldo = w->view.rows;
    a.stream = stream;
    a.stream_k = stream_k;
    if (stream_k) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (!workspace || workspace_bytes < stream_k_workspace_bytes(dev, bt))
            return fail(JK_ERR_INVALID, "stream-K workspace too small");
        a.ws_flag = static_cast<uint32_t*>(workspace);
        a.ws_part = reinterpret_cast<float*>(static_cast<char*>(workspace) + stream_k_flag_bytes(dev));
        a.grid_cap = sm_count(dev) * 2;
    }
    return launch_tc_fmt(a, bt, x_bf16);
}

jk_status launch_gemm_grouped(const jk_qmatrix* w, const void* x_sorted, bool x_bf16, size_t rows,
                              const uint32_t* sorted, const uint32_t* offsets, const uint32_t* jobs, size_t max_jobs,
                              int job_rows, float* out, int bt, bool pair_tile, cudaStream_t stream) {
    if (rows == 0 || max_jobs == 0) return JK_OK;
    if (!w->has_tmap) return fail(JK_ERR_INVALID, "matrix has no tensor-core layout");
    if (job_rows < 1 || job_rows > bt) return fail(JK_ERR_INVALID, "grouped product: job rows exceed the row tile");
    const bool pair = pair_tile && w->view.fmt != FMT_F16 && bt >= 128;
    CUtensorMap tm_x;
    jk_status st = encode_tmap_2d(&tm_x, x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                  (uint64_t)w->k, (uint64_t)rows, (uint64_t)w->k * 2, KB,
                                  (uint32_t)(pair ? bt / 2 : bt), CU_TENSOR_MAP_SWIZZLE_128B, x_sorted);
    if (st != JK_OK) return st;
    LaunchArgs a{};
    a.wq = w;
    a.tm_x = &tm_x;
    a.pair = pair;
    a.out = out;
    a.m = (int64_t)rows;
    a.ldo = (int64_t)w->n;
    a.stream = stream;
    a.jobs = jobs;
    a.offsets = offsets;
    a.sorted = sorted;
    a.n_exp = (int64_t)w->n;
    a.max_jobs = (int64_t)max_jobs;
    a.job_rows = job_rows;
    return launch_tc_fmt(a, bt, x_bf16);
}

// Stream-K launch on a workspace of fixed capacity provided by the caller: flag words at `flags`
// (zero on entry), partial tiles at `partials`, room for `max_ctas` partial tiles. Fails with
// JK_ERR_SHAPE, launching nothing, if the grid this device runs needs more partial tiles.
jk_status launch_gemm_stream_k_fixed(const jk_qmatrix* w, const void* x, bool x_bf16, size_t m, float* out, int bt,
                                     uint32_t* flags, float* partials, int max_ctas, size_t capacity_bytes,
                                     cudaStream_t stream) {
    if (m == 0) return JK_OK;
    if (!w->has_tmap) return fail(JK_ERR_INVALID, "matrix has no tensor-core layout");
    int dev = 0;
    cudaGetDevice(&dev);
    // the grid the stream-K schedule uses: one CTA per SM (every instantiation runs one per SM),
    // never more CTAs than (tile, k-block) iterations
    const int64_t tiles = ((w->view.rows + BW - 1) / BW) * (((int64_t)m + bt - 1) / bt);
    int64_t g = sm_budget(dev);
    if (g > tiles * (w->k / KB)) g = tiles * (w->k / KB);
    if (g > max_ctas) {
        char buf[200];
        snprintf(buf, sizeof buf,
                 "stream-K product with bm=%d on this device needs %lld partial tiles (%lld bytes of scratch); "
                 "the allocation-free buffer holds %zu bytes",
                 bt, (long long)g, (long long)(g * bt * BW * 4), capacity_bytes);
        return fail(JK_ERR_SHAPE, buf);
    }
    CUtensorMap tm_x;
    jk_status st = encode_tmap_2d(&tm_x, x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                  (uint64_t)w->k, (uint64_t)m, (uint64_t)w->k * 2, KB, (uint32_t)bt,
                                  CU_TENSOR_MAP_SWIZZLE_128B, x);
    if (st != JK_OK) return st;
    LaunchArgs a{};
    a.wq = w;
    a.tm_x = &tm_x;
    a.out = out;
    a.m = (int64_t)m;
    a.ldo = w->view.rows;
    a.stream = stream;
    a.stream_k = true;
    a.ws_flag = flags;
    a.ws_part = partials;
    a.grid_cap = (int)g;
    return launch_tc_fmt(a, bt, x_bf16);
}

}  // namespace jk
