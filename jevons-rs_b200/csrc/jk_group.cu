// jk_group.cu -- expert grouping of routed rows and the row gather that feeds the grouped product.
//
// Grouping follows the reference's `group` kernel contract
// (crates/jevons-gemma4-diffusion/src/gpu/ops.rs:523-585): for `assignments` route ids (each an
// expert index), write
//   sorted[experts-sorted position] = assignment index, stable (ascending index within an expert),
//   offsets[e] = first sorted position of expert e, offsets[experts] = total,
//   jobs[0] = job count, then (expert, first sorted position) per job of at most `bm` rows,
//   experts in ascending order and each expert's jobs in ascending position.
// The reference runs one workgroup with one thread per expert, each thread scanning every id. Here
// one CTA of 1024 threads splits the ids into 32 contiguous warp segments: each warp counts its
// segment per expert (warp match, one leader per distinct expert), a scan over (expert, warp) turns
// the counts into base positions, and a second pass scatters each id to its base plus its rank
// among equal ids earlier in the same 32-id chunk. The order is the reference's: fully determined
// by the ids, independent of scheduling.
#include "jk_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace jk {

namespace {

constexpr int GROUP_THREADS = 1024;
constexpr int GROUP_WARPS = GROUP_THREADS / 32;

// Exclusive block-wide prefix sum of one value per thread (all GROUP_THREADS threads call it).
__device__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_sums, uint32_t& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl += t;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        uint32_t s = warp_sums[lane];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, s, d);
            if (lane >= d) s += t;
        }
        warp_sums[lane] = s;  // inclusive over warps
    }
    __syncthreads();
    const uint32_t before = warp == 0 ? 0u : warp_sums[warp - 1];
    total = warp_sums[GROUP_WARPS - 1];
    __syncthreads();  // warp_sums is reused by the next scan
    return before + incl - v;
}

// Shared memory: cnt[GROUP_WARPS][experts] (per-warp counts, then per-warp base positions).
__global__ void __launch_bounds__(GROUP_THREADS, 1)
group_experts_kernel(const uint32_t* __restrict__ ids, uint32_t assignments, uint32_t experts, uint32_t bm,
                     uint32_t max_jobs, uint32_t* __restrict__ sorted, uint32_t* __restrict__ offsets,
                     uint32_t* __restrict__ jobs, uint32_t* __restrict__ err) {
    extern __shared__ uint32_t cnt[];
    __shared__ uint32_t warp_sums[GROUP_WARPS];
    __shared__ uint32_t bad;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t lt_mask = (1u << lane) - 1u;
    for (uint32_t i = threadIdx.x; i < GROUP_WARPS * experts; i += GROUP_THREADS) cnt[i] = 0u;
    if (threadIdx.x == 0) bad = 0u;
    __syncthreads();

    // warp segments: contiguous, whole 32-id chunks
    const uint32_t seg = ((assignments + GROUP_WARPS - 1) / GROUP_WARPS + 31u) & ~31u;
    const uint32_t s_lo = (uint32_t)warp * seg < assignments ? (uint32_t)warp * seg : assignments;
    const uint32_t s_hi = s_lo + seg < assignments ? s_lo + seg : assignments;
    uint32_t* my = cnt + (size_t)warp * experts;

    // pass 1: per-warp counts (one leader per distinct expert of a chunk adds the group size)
    for (uint32_t base = s_lo; base < s_hi; base += 32) {
        const uint32_t a = base + (uint32_t)lane;
        const uint32_t e = a < s_hi ? __ldg(ids + a) : 0xFFFFFFFFu;
        const uint32_t peers = __match_any_sync(0xFFFFFFFFu, e);
        if (a < s_hi && e >= experts) bad = 1u;
        if (e < experts && (peers & lt_mask) == 0u) my[e] += (uint32_t)__popc(peers);
        __syncwarp();
    }
    __syncthreads();

    // expert totals, then positions and jobs (experts <= GROUP_THREADS: one thread per expert)
    const uint32_t e = threadIdx.x;
    uint32_t total_e = 0;
    if (e < experts)
        for (int w = 0; w < GROUP_WARPS; ++w) total_e += cnt[(size_t)w * experts + e];
    uint32_t total_rows = 0, total_jobs = 0;
    const uint32_t start = block_exclusive_scan(e < experts ? total_e : 0u, warp_sums, total_rows);
    const uint32_t tiles = (total_e + bm - 1) / bm;
    const uint32_t job0 = block_exclusive_scan(e < experts ? tiles : 0u, warp_sums, total_jobs);
    if (e < experts) {
        uint32_t run = start;
        for (int w = 0; w < GROUP_WARPS; ++w) {  // per-warp counts -> per-warp base positions
            const uint32_t c = cnt[(size_t)w * experts + e];
            cnt[(size_t)w * experts + e] = run;
            run += c;
        }
        offsets[e] = start;
        for (uint32_t t = 0; t < tiles && job0 + t < max_jobs; ++t) {
            jobs[1 + 2 * (size_t)(job0 + t)] = e;
            jobs[2 + 2 * (size_t)(job0 + t)] = start + t * bm;
        }
    }
    if (threadIdx.x == 0) {
        offsets[experts] = total_rows;
        jobs[0] = total_jobs < max_jobs ? total_jobs : max_jobs;
        if (bad || total_jobs > max_jobs) atomicOr(err, ERR_BAD_LAUNCH);
    }
    __syncthreads();

    // pass 2: stable scatter, rank among equal ids earlier in the chunk
    for (uint32_t base = s_lo; base < s_hi; base += 32) {
        const uint32_t a = base + (uint32_t)lane;
        const uint32_t ea = a < s_hi ? __ldg(ids + a) : 0xFFFFFFFFu;
        const uint32_t peers = __match_any_sync(0xFFFFFFFFu, ea);
        if (ea < experts) sorted[my[ea] + (uint32_t)__popc(peers & lt_mask)] = a;
        __syncwarp();
        if (ea < experts && (peers & lt_mask) == 0u) my[ea] += (uint32_t)__popc(peers);
        __syncwarp();
    }
}

// x_sorted[s, :] = x[sorted[s] / in_div, :] in the product's operand type. Rows whose source lies
// past the activation rows (routes the grouping rejected) are written as zeros.
template <typename Out>
__device__ __forceinline__ Out to_out(float f);
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float f) { return __float2bfloat16_rn(f); }
template <>
__device__ __forceinline__ __half to_out<__half>(float f) { return __float2half_rn(f); }

template <typename In, typename Out, bool VEC>
__global__ void __launch_bounds__(256) gather_rows_kernel(const In* __restrict__ x, size_t x_rows, size_t k,
                                                          const uint32_t* __restrict__ sorted, uint32_t rows,
                                                          uint32_t in_div, Out* __restrict__ out) {
    const uint32_t s = blockIdx.x;
    const size_t c8 = ((size_t)blockIdx.y * blockDim.x + threadIdx.x) * 8;
    if (s >= rows || c8 >= k) return;
    const size_t src = __ldg(sorted + s) / in_div;
    Out* o = out + (size_t)s * k + c8;
    if (src >= x_rows) {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = to_out<Out>(0.0f);
        return;
    }
    const In* i = x + src * k + c8;
    if constexpr (VEC && sizeof(In) == sizeof(Out)) {  // same 16-bit type: one 16-byte copy
        *reinterpret_cast<uint4*>(o) = __ldg(reinterpret_cast<const uint4*>(i));
    } else {
        Out v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float f;
            if constexpr (sizeof(In) == 4) f = i[j];
            else if constexpr (std::is_same<In, __half>::value) f = __half2float(i[j]);
            else f = __bfloat162float(i[j]);
            v[j] = to_out<Out>(f);
        }
        if constexpr (VEC) *reinterpret_cast<uint4*>(o) = *reinterpret_cast<const uint4*>(v);
        else
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = v[j];
    }
}

template <typename In, typename Out>
jk_status gather_t(const void* x, size_t x_rows, size_t k, const uint32_t* sorted, size_t rows, uint32_t in_div,
                   void* out, cudaStream_t stream) {
    const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0 &&
                     (k * sizeof(In)) % 16 == 0;
    const dim3 grid((unsigned)rows, (unsigned)((k / 8 + 255) / 256));
    if (vec)
        gather_rows_kernel<In, Out, true><<<grid, 256, 0, stream>>>(static_cast<const In*>(x), x_rows, k, sorted,
                                                                    (uint32_t)rows, in_div, static_cast<Out*>(out));
    else
        gather_rows_kernel<In, Out, false><<<grid, 256, 0, stream>>>(static_cast<const In*>(x), x_rows, k, sorted,
                                                                     (uint32_t)rows, in_div, static_cast<Out*>(out));
    return cuda_fail(cudaGetLastError(), "row gather launch");
}

}  // namespace

size_t group_smem_bytes(size_t experts) { return (size_t)GROUP_WARPS * experts * 4; }

jk_status launch_group_experts(const uint32_t* ids, size_t assignments, size_t experts, int bm, size_t max_jobs,
                               uint32_t* sorted, uint32_t* offsets, uint32_t* jobs, uint32_t* err,
                               cudaStream_t stream) {
    const size_t smem = group_smem_bytes(experts);
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(group_experts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)group_smem_bytes(GROUP_MAX_EXPERTS));
        if (e != cudaSuccess) return cuda_fail(e, "grouping kernel attributes");
        configured[dev] = true;
    }
    group_experts_kernel<<<1, GROUP_THREADS, smem, stream>>>(ids, (uint32_t)assignments, (uint32_t)experts,
                                                             (uint32_t)bm, (uint32_t)max_jobs, sorted, offsets,
                                                             jobs, err);
    return cuda_fail(cudaGetLastError(), "grouping launch");
}

jk_status launch_gather_rows(const void* x, int x_dtype, size_t x_rows, size_t k, const uint32_t* sorted,
                             size_t rows, uint32_t in_div, void* out, bool out_bf16, cudaStream_t stream) {
    if (rows == 0) return JK_OK;
    switch (x_dtype) {
    case JK_DTYPE_F32:
        return out_bf16 ? gather_t<float, __nv_bfloat16>(x, x_rows, k, sorted, rows, in_div, out, stream)
                        : gather_t<float, __half>(x, x_rows, k, sorted, rows, in_div, out, stream);
    case JK_DTYPE_F16:
        return out_bf16 ? gather_t<__half, __nv_bfloat16>(x, x_rows, k, sorted, rows, in_div, out, stream)
                        : gather_t<__half, __half>(x, x_rows, k, sorted, rows, in_div, out, stream);
    default:
        return out_bf16 ? gather_t<__nv_bfloat16, __nv_bfloat16>(x, x_rows, k, sorted, rows, in_div, out, stream)
                        : gather_t<__nv_bfloat16, __half>(x, x_rows, k, sorted, rows, in_div, out, stream);
    }
}

}  // namespace jk
