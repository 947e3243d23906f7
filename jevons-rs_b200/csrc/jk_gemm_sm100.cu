// jk_gemm_sm100.cu -- tensor-core product out[r, c] = sum_j x[r, j] W[c, j] on sm_100a
// (the reference's `gemm` kernel + `matmul_split`/`reduce_splits`,
// crates/jevons-kernels/src/gemm.rs:532-815 and :1205-1269), designed for Blackwell:
//
//   * Roles are swapped relative to the usual activation-major GEMM: the 5th-generation MMA's
//     M side (128 TMEM lanes) carries 128 WEIGHT rows and its N side carries BT activation rows
//     (BT = 32..256), so a 32-row canvas product still fills whole MMAs and the f32 accumulator
//     tile sits in tensor memory as [weight row][activation row].
//   * Warp roles (192 threads, one output tile per CTA):
//       warp 0      TMA producer: activation tiles (bf16/f16, 128-byte swizzled) and raw
//                   quantized weight tiles (one 256-wide super-block of 128 rows per stage);
//       warp 1      allocates tensor memory; lane 0 issues tcgen05.mma (4 x K=16 per 64-wide
//                   k-block) and commits each stage back to the producers;
//       warps 2..5  dequantize: thread t decodes row t's k-block from the raw stage with the
//                   exact f32 arithmetic of the reference (jk_decode.cuh), rounds to bf16/f16
//                   and stores it into the 128-byte-swizzled K-major operand tile; after the
//                   last k-block the same warps drain the accumulators (tcgen05.ld) and store
//                   f32 outputs, 128 contiguous bytes per warp store.
//   * Pipelines: S operand stages guarded by mbarriers (full_b: TMA bytes landed; full_a:
//     4 dequant warps done; empty: the MMAs reading the stage completed), 2 raw weight stages
//     (raw_full / raw_empty). Every wait is bounded (4 s); a wait that runs out records an error
//     code in the per-device error word and the CTA skips its remaining work, drains its
//     in-flight copies and MMAs, and frees its tensor memory.
//   * FP16 weights (the Burn-facing f16_linear path) skip dequantization: the producer loads the
//     weight tile straight into the swizzled operand stage.
//   * Split-K (grid.z = splits) partitions the 64-wide k-blocks like gemm.rs:573-576 and writes
//     partial tiles to a scratch buffer, reduced in fixed split order by reduce_splits_kernel.
//     With splits == 1 each output element's accumulation order is the same for every BT and m
//     (row invariance, gemm.rs:1090-1091).
//   * No TMA multicast anywhere.
#include "jk_decode.cuh"
#include "jk_internal.h"

#include <cudaTypedefs.h>

namespace jk {

namespace {

constexpr int BW = 128;           // weight rows per tile (MMA M)
constexpr int KB = 64;            // k-block (one 128-byte swizzle atom of 16-bit values)
constexpr int THREADS = 192;
constexpr int A_STAGE_BYTES = BW * KB * 2;  // 16 KB

template <int FMT>
struct RawTile {
    // bytes of one raw weight stage (one 256-wide super-block of 128 rows)
    static constexpr int bytes = FMT == FMT_Q4K ? BW * 144
                               : FMT == FMT_Q6K ? BW * 208
                               : FMT == FMT_Q8_0 ? BW * 256
                               : FMT == FMT_Q5_0 ? BW * 128
                               : 0;
};

template <int BT>
struct Stages {
    static constexpr int S = BT >= 256 ? 3 : 4;
};

template <int FMT, int BT>
struct Smem {
    static constexpr int S = Stages<BT>::S;
    static constexpr int B_STAGE = BT * 128;
    static constexpr int off_b = 0;
    static constexpr int off_a = off_b + S * B_STAGE;
    static constexpr int off_raw = off_a + S * A_STAGE_BYTES;
    static constexpr int raw_bytes = RawTile<FMT>::bytes;
    static constexpr int off_bar = off_raw + 2 * raw_bytes;
    static constexpr int n_bar = 3 * S + 5;
    static constexpr int off_tmem = off_bar + 8 * n_bar;
    static constexpr int total = off_tmem + 16 + 1024;  // + alignment slack
};

__global__ void __launch_bounds__(256) reduce_splits_kernel(const float* __restrict__ part, float* __restrict__ out,
                                                            int64_t len, int splits) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= len) return;
    float s = 0.f;
    for (int z = 0; z < splits; ++z) s += part[(int64_t)z * len + i];
    out[i] = s;
}

template <int FMT, bool BF16, int BT>
__global__ void __launch_bounds__(THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, WView w,
               float* __restrict__ out, int64_t m, int64_t ldo, int64_t part_stride, int kb_total, int splits,
               uint32_t* err) {
    using L = Smem<FMT, BT>;
    constexpr int S = L::S;
    constexpr bool QUANT = FMT != FMT_F16;
    constexpr uint32_t TMEM_COLS = BT < 32 ? 32 : BT;
    constexpr uint32_t IDESC = idesc_f16(BF16, BW, BT);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::off_bar;
    auto full_b = [&](int s) { return bar0 + 8u * s; };
    auto full_a = [&](int s) { return bar0 + 8u * (S + s); };
    auto empty = [&](int s) { return bar0 + 8u * (2 * S + s); };
    auto raw_full = [&](int r) { return bar0 + 8u * (3 * S + r); };
    auto raw_empty = [&](int r) { return bar0 + 8u * (3 * S + 2 + r); };
    const uint32_t acc_full = bar0 + 8u * (3 * S + 4);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::off_tmem);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const int64_t n0 = (int64_t)blockIdx.x * BW;   // first weight row of the tile
    const int64_t m0 = (int64_t)blockIdx.y * BT;   // first activation row
    const int z = blockIdx.z;
    const int kb_begin = (int)((int64_t)z * kb_total / splits);
    const int kb_end = (int)((int64_t)(z + 1) * kb_total / splits);
    const int nkb = kb_end - kb_begin;
    const int sb_begin = kb_begin / 4;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full_b(s), 1);
            mbar_init(full_a(s), 4);
            mbar_init(empty(s), 1);
        }
        for (int r = 0; r < 2; ++r) {
            mbar_init(raw_full(r), 1);
            mbar_init(raw_empty(r), 4);
        }
        mbar_init(acc_full, 1);
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    bool ok = nkb > 0;

    if (warp == 0) {
        if (lane == 0 && ok) {
            // ---------------- producer ----------------
            tma_prefetch(&tm_x);
            if (QUANT || FMT == FMT_F16) tma_prefetch(&tm_w);
            int last_raw = -1;
            int issued = 0;      // operand stages whose copies were issued
            int raw_issued = 0;  // raw weight stages whose copies were issued
            for (int it = 0; it < nkb && ok; ++it) {
                const int kb = kb_begin + it;
                const int s = it % S;
                if constexpr (QUANT) {
                    const int sb = kb >> 2;
                    if (sb != last_raw) {
                        const int r = sb - sb_begin;
                        const int slot = r & 1;
                        if (r >= 2) ok = mbar_wait(raw_empty(slot), ((r >> 1) - 1) & 1, err);
                        if (!ok) break;
                        const uint32_t dst = sbase + L::off_raw + slot * L::raw_bytes;
                        mbar_expect_tx(raw_full(slot), L::raw_bytes);
                        if constexpr (FMT == FMT_Q4K) {
                            tma_load_2d(dst, &tm_w, sb * 36, (int32_t)n0, raw_full(slot));
                        } else if constexpr (FMT == FMT_Q6K) {
                            tma_load_2d(dst, &tm_w, sb * 52, (int32_t)n0, raw_full(slot));
                        } else if constexpr (FMT == FMT_Q8_0) {
                            tma_load_2d(dst, &tm_w, sb * 256, (int32_t)n0, raw_full(slot));
                            tma_load_2d(dst + BW * 128, &tm_w, sb * 256 + 128, (int32_t)n0, raw_full(slot));
                        } else {  // Q5_0
                            tma_load_2d(dst, &tm_w, sb * 128, (int32_t)n0, raw_full(slot));
                        }
                        last_raw = sb;
                        raw_issued = r + 1;
                    }
                }
                if (it >= S) ok = mbar_wait(empty(s), ((it / S) - 1) & 1, err);
                if (!ok) break;
                const uint32_t b_dst = sbase + L::off_b + s * L::B_STAGE;
                if constexpr (FMT == FMT_F16) {
                    mbar_expect_tx(full_b(s), L::B_STAGE + A_STAGE_BYTES);
                    tma_load_2d(sbase + L::off_a + s * A_STAGE_BYTES, &tm_w, kb * KB, (int32_t)n0, full_b(s));
                } else {
                    mbar_expect_tx(full_b(s), L::B_STAGE);
                }
                tma_load_2d(b_dst, &tm_x, kb * KB, (int32_t)m0, full_b(s));
                issued = it + 1;
            }
            // Error path: wait (bounded) until the copies issued last have landed before leaving,
            // so no copy writes this CTA's shared memory after it exits.
            if (!ok) {
                for (int it = issued - S < 0 ? 0 : issued - S; it < issued; ++it)
                    mbar_wait(full_b(it % S), (it / S) & 1, err);
                for (int r = raw_issued - 2 < 0 ? 0 : raw_issued - 2; r < raw_issued; ++r)
                    mbar_wait(raw_full(r & 1), (r >> 1) & 1, err);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            if (ok) {
                for (int it = 0; it < nkb; ++it) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    ok = mbar_wait(full_b(s), ph, err);
                    if (ok && QUANT) ok = mbar_wait(full_a(s), ph, err);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t ad = sw128_kmajor_desc(sbase + L::off_a + s * A_STAGE_BYTES);
                    const uint64_t bd = sw128_kmajor_desc(sbase + L::off_b + s * L::B_STAGE);
#pragma unroll
                    for (int k = 0; k < KB / 16; ++k) {
                        // +32 bytes per K=16 step inside the 128-byte swizzle atom (>>4 => +2)
                        mma_f16(tmem, ad + 2u * k, bd + 2u * k, IDESC, (it > 0 || k > 0) ? 1u : 0u);
                    }
                    mma_commit(empty(s));
                }
            }
            // Signals the epilogue (and, on the error path, lets this thread drain its MMAs).
            mma_commit(acc_full);
            if (!ok) mbar_wait(acc_full, 0, err);
        }
    } else {
        // ---------------- dequantizers, then epilogue ----------------
        const int t = threadIdx.x - 64;      // 0..127: weight row within the tile
        const int quarter = warp & 3;        // TMEM lane quarter this warp may access
        if constexpr (QUANT) {
            const int64_t row = n0 + t;
            const bool row_ok = row < w.rows;
            const int64_t rr = row_ok ? row : 0;
            for (int it = 0; it < nkb && ok; ++it) {
                const int kb = kb_begin + it;
                const int s = it % S;
                const int sb = kb >> 2;
                const int r = sb - sb_begin;
                const int slot = r & 1;
                ok = mbar_wait(raw_full(slot), (r >> 1) & 1, err);
                if (ok && it >= S) ok = mbar_wait(empty(s), ((it / S) - 1) & 1, err);
                ok = __all_sync(0xFFFFFFFFu, ok);  // keep the warp converged on every path
                if (!ok) break;
                const uint8_t* raw = smem + L::off_raw + slot * L::raw_bytes;
                uint8_t* arow = smem + L::off_a + s * A_STAGE_BYTES + t * 128;
                const int j = kb & 3;
                float v[8];
                auto store_chunk = [&](int c) {
                    const float (&vv)[8] = v;
                    uint4 pk;
                    pk.x = pack2<BF16>(vv[0], vv[1]);
                    pk.y = pack2<BF16>(vv[2], vv[3]);
                    pk.z = pack2<BF16>(vv[4], vv[5]);
                    pk.w = pack2<BF16>(vv[6], vv[7]);
                    *reinterpret_cast<uint4*>(arow + 16 * (c ^ (t & 7))) = pk;
                };
                if constexpr (FMT == FMT_Q4K) {
                    Q4KBlock b;
                    b.load(raw + t * 144, j);
#pragma unroll
                    for (int c = 0; c < 8; ++c) { b.chunk(c, v); store_chunk(c); }
                } else if constexpr (FMT == FMT_Q6K) {
                    Q6KBlock b;
                    const float d = row_ok ? half_bits_to_float(__ldg(w.d + rr * (w.k / 256) + sb)) : 0.f;
                    b.load(raw + t * 208, d, j);
#pragma unroll
                    for (int c = 0; c < 8; ++c) { b.chunk(c, v); store_chunk(c); }
                } else if constexpr (FMT == FMT_Q8_0) {
                    Q80Block b;
                    float d0 = 0.f, d1 = 0.f;
                    if (row_ok) {
                        const uint32_t dw = __ldg(reinterpret_cast<const uint32_t*>(w.d + rr * (w.k / 32) + 2 * kb));
                        d0 = half_bits_to_float(dw & 0xFFFFu);
                        d1 = half_bits_to_float(dw >> 16);
                    }
                    // k-block j of the super-block: 128-byte swizzled half (j/2), chunks 4(j%2)..
                    b.load_sw(raw + (j >> 1) * (BW * 128) + t * 128, 4 * (j & 1), t, d0, d1);
#pragma unroll
                    for (int c = 0; c < 8; ++c) { b.chunk(c, v); store_chunk(c); }
                } else {  // Q5_0
                    Q50Block b;
                    float d0 = 0.f, d1 = 0.f;
                    uint32_t qh2[2] = {0u, 0u};
                    if (row_ok) {
                        const uint32_t dw = __ldg(reinterpret_cast<const uint32_t*>(w.d + rr * (w.k / 32) + 2 * kb));
                        d0 = half_bits_to_float(dw & 0xFFFFu);
                        d1 = half_bits_to_float(dw >> 16);
                        qh2[0] = __ldg(w.h + rr * (w.k / 32) + 2 * kb);
                        qh2[1] = __ldg(w.h + rr * (w.k / 32) + 2 * kb + 1);
                    }
                    // 128-byte swizzled row of the super-block; k-block j = chunks 2j, 2j+1
                    uint8_t tmp[32];
                    const uint8_t* rowp = raw + t * 128;
                    *reinterpret_cast<uint4*>(tmp) = *reinterpret_cast<const uint4*>(rowp + 16 * ((2 * j) ^ (t & 7)));
                    *reinterpret_cast<uint4*>(tmp + 16) = *reinterpret_cast<const uint4*>(rowp + 16 * ((2 * j + 1) ^ (t & 7)));
                    b.load(tmp, qh2, d0, d1);
#pragma unroll
                    for (int c = 0; c < 8; ++c) { b.chunk(c, v); store_chunk(c); }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(full_a(s));
                    if (j == 3 || it == nkb - 1) mbar_arrive(raw_empty(slot));
                }
            }
        }
        // ---------------- epilogue ----------------
        if (nkb > 0) {
            const bool acc_ok = __all_sync(0xFFFFFFFFu, mbar_wait(acc_full, 0, err) && ok);
            tc_fence_after();
            if (acc_ok) {
                const int64_t wrow = n0 + 32 * quarter + lane;
                float* obase = out + (int64_t)z * part_stride;
#pragma unroll 1
                for (int cc = 0; cc < BT / 32; ++cc) {
                    uint32_t v[32];
                    tmem_ld32(tmem + ((uint32_t)(32 * quarter) << 16) + 32u * cc, v);
                    tmem_ld_wait();
                    if (wrow < w.rows) {
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) {
                            const int64_t mr = m0 + 32 * cc + jj;
                            if (mr < m) obase[mr * ldo + wrow] = __uint_as_float(v[jj]);
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <int FMT, bool BF16, int BT>
jk_status launch_tc(const jk_qmatrix* wq, const CUtensorMap& tm_x, float* out, int64_t m, int64_t ldo,
                    int64_t part_stride, int splits, cudaStream_t stream) {
    using L = Smem<FMT, BT>;
    auto kern = gemm_tc_kernel<FMT, BF16, BT>;
    static int attr_device_mask = 0;  // devices on which the smem attribute is set (set once each)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 31 || !(attr_device_mask & (1 << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::total);
        if (e != cudaSuccess) return cuda_fail(e, "gemm smem attribute");
        if (dev < 31) attr_device_mask |= 1 << dev;
    }
    const WView& w = wq->view;
    const int kb_total = (int)(w.k / KB);
    dim3 grid((unsigned)((w.rows + BW - 1) / BW), (unsigned)((m + BT - 1) / BT), (unsigned)splits);
    kern<<<grid, THREADS, L::total, stream>>>(tm_x, wq->tm_w, w, out, m, ldo, part_stride, kb_total, splits,
                                              device_error_word(wq->device));
    return cuda_fail(cudaGetLastError(), "gemm launch");
}

template <int FMT, bool BF16>
jk_status launch_tc_bt(const jk_qmatrix* wq, const CUtensorMap& tm_x, float* out, int64_t m, int64_t ldo,
                       int64_t part_stride, int splits, int bt, cudaStream_t stream) {
    switch (bt) {
    case 32: return launch_tc<FMT, BF16, 32>(wq, tm_x, out, m, ldo, part_stride, splits, stream);
    case 64: return launch_tc<FMT, BF16, 64>(wq, tm_x, out, m, ldo, part_stride, splits, stream);
    case 128: return launch_tc<FMT, BF16, 128>(wq, tm_x, out, m, ldo, part_stride, splits, stream);
    default: return launch_tc<FMT, BF16, 256>(wq, tm_x, out, m, ldo, part_stride, splits, stream);
    }
}

template <bool BF16>
jk_status launch_tc_fmt(const jk_qmatrix* wq, const CUtensorMap& tm_x, float* out, int64_t m, int64_t ldo,
                        int64_t part_stride, int splits, int bt, cudaStream_t stream) {
    switch (wq->view.fmt) {
    case FMT_Q4K: return launch_tc_bt<FMT_Q4K, BF16>(wq, tm_x, out, m, ldo, part_stride, splits, bt, stream);
    case FMT_Q6K: return launch_tc_bt<FMT_Q6K, BF16>(wq, tm_x, out, m, ldo, part_stride, splits, bt, stream);
    case FMT_Q8_0: return launch_tc_bt<FMT_Q8_0, BF16>(wq, tm_x, out, m, ldo, part_stride, splits, bt, stream);
    case FMT_Q5_0: return launch_tc_bt<FMT_Q5_0, BF16>(wq, tm_x, out, m, ldo, part_stride, splits, bt, stream);
    default: return launch_tc_bt<FMT_F16, BF16>(wq, tm_x, out, m, ldo, part_stride, splits, bt, stream);
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

jk_status launch_gemm(const jk_qmatrix* w, const void* x, bool x_bf16, size_t m, float* out, int bt, int splits,
                      float* part, cudaStream_t stream) {
    if (m == 0) return JK_OK;
    if (!w->has_tmap) return fail(JK_ERR_INVALID, "matrix has no tensor-core layout");
    CUtensorMap tm_x;
    jk_status st = encode_tmap_2d(&tm_x, x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                  (uint64_t)w->k, (uint64_t)m, (uint64_t)w->k * 2, KB, (uint32_t)bt,
                                  CU_TENSOR_MAP_SWIZZLE_128B, x);
    if (st != JK_OK) return st;
    const int64_t ldo = w->view.rows;
    const int64_t len = (int64_t)m * ldo;
    float* target = splits > 1 ? part : out;
    st = x_bf16 ? launch_tc_fmt<true>(w, tm_x, target, (int64_t)m, ldo, len, splits, bt, stream)
                : launch_tc_fmt<false>(w, tm_x, target, (int64_t)m, ldo, len, splits, bt, stream);
    if (st != JK_OK) return st;
    if (splits > 1) {
        reduce_splits_kernel<<<(unsigned)((len + 255) / 256), 256, 0, stream>>>(part, out, len, splits);
        return cuda_fail(cudaGetLastError(), "reduce_splits launch");
    }
    return JK_OK;
}

}  // namespace jk
