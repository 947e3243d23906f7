/*
 * jk.h -- C ABI of the B200 (sm_100a) GGML quantized matmul.
 *
 * This is the drop-in boundary for the quantized matmul path of zojeda/jevons-rs: the GGML
 * block types of `jevons-formats` and the matmul entry points of `jevons-kernels` and
 * `jevons-burn`. Each declaration names the reference item it replaces (paths are within the
 * reference project). Only plain pointers, sizes and integer codes cross this boundary.
 *
 * Conventions (mirroring the reference):
 *   - Weights W are [experts * n, k] in GGML order: row c holds output column c, and k is the
 *     contiguous row length (crates/jevons-formats/src/gguf.rs:148-156).
 *   - Activations x are row-major [m, k]; outputs are row-major f32 [m, n]:
 *       out[r, c] = sum_j x[r, j] * W[c, j]       (crates/jevons-kernels/src/gemm.rs:1)
 *   - Device pointers (x, out, scratch) are caller-owned, as the reference's `Buf`s are.
 *   - Launches are asynchronous on `stream` (a cudaStream_t; NULL = legacy default stream);
 *     nothing here synchronises except jk_qmatrix_* creation, jk_gpu_sync and jk_device_error.
 *   - Every function returns a jk_status. On failure jk_last_error() returns a thread-local
 *     message naming the tensor type and shape, like the reference's `Err(String)` values and
 *     launcher assertions (gemm.rs:840-886, 1137, 1218). Nothing aborts or throws across the ABI.
 */
#ifndef JK_H
#define JK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define JK_ABI_VERSION 1

typedef enum jk_status {
    JK_OK = 0,
    JK_ERR_INVALID = 1,     /* null pointer, bad enum value, buffer too small */
    JK_ERR_UNSUPPORTED = 2, /* tensor type without a GPU layout, device not sm_100 */
    JK_ERR_SHAPE = 3,       /* n, k, experts or byte counts that do not fit the type */
    JK_ERR_CUDA = 4,        /* a CUDA runtime call failed (message carries cudaGetErrorString) */
    JK_ERR_NCCL = 5,        /* an NCCL call failed */
    JK_ERR_TIMEOUT = 6,     /* a bounded device-side wait ran out (see jk_device_error) */
} jk_status;

/* GGML type ids, as TensorType::from_id (crates/jevons-formats/src/gguf.rs:110-132). */
typedef enum jk_tensor_type {
    JK_TYPE_F32 = 0,
    JK_TYPE_F16 = 1,
    JK_TYPE_Q5_0 = 6,
    JK_TYPE_Q8_0 = 8,
    JK_TYPE_Q4_K = 12,
    JK_TYPE_Q6_K = 14,
} jk_tensor_type;

/* Activation element types accepted by the matmul entry points. The reference takes FP16 only
 * (gemm.rs:3); bf16 and f32 are additions for the B200 path. */
typedef enum jk_dtype {
    JK_DTYPE_F32 = 0,
    JK_DTYPE_F16 = 1,
    JK_DTYPE_BF16 = 2,
} jk_dtype;

/* ---- errors / library ------------------------------------------------------------------ */

/* Thread-local message of the last failing call on this thread ("" if none). */
const char *jk_last_error(void);
int jk_abi_version(void);

/* ---- block formats (host) ---------------------------------------------------------------- */

/* TensorType::block (gguf.rs:134-145): elements and bytes per block. JK_ERR_UNSUPPORTED for an
 * unknown id. */
jk_status jk_tensor_type_block(int type, uint64_t *elements, uint64_t *bytes);

/* quant::q4k_scale_min (crates/jevons-formats/src/quant.rs:14-23): 6-bit (scale, min) pair j
 * (0..8) from the 12 packed scale bytes of a Q4_K super-block. */
jk_status jk_q4k_scale_min(int j, const uint8_t scales[12], uint8_t *scale, uint8_t *min);

/* quant::packed_words (quant.rs:128-136): words per block of the reference's SoA regions
 * (q, h, s, d). All zero for types without a GPU layout. */
jk_status jk_packed_words(int type, size_t words[4]);

/* quant::pack (quant.rs:156-193): repacks raw GGML blocks into the reference's SoA regions.
 * Region capacities are checked against blocks * jk_packed_words; d is f32. Pass NULL for an
 * empty region. */
jk_status jk_pack(int type, const void *ggml_bytes, size_t len,
                  uint32_t *q, size_t q_words, uint32_t *h, size_t h_words,
                  uint32_t *s, size_t s_words, float *d, size_t d_words);

/* quant::dequantize (quant.rs:83-101), on the host: decodes `len` bytes of whole blocks of `type`
 * (F32, F16, Q4_K, Q6_K, Q5_0, Q8_0) into out[out_len] f32, bit-exact with the reference (the same
 * f32 operations in the same order). JK_ERR_UNSUPPORTED "unsupported tensor type" for other ids;
 * JK_ERR_SHAPE "dequantization size mismatch" unless len is a whole number of blocks and out_len
 * is exactly blocks * elements per block. The device counterpart is jk_qmatrix_dequantize. */
jk_status jk_dequantize(int type, const void *bytes, size_t len, float *out, size_t out_len);

/* ---- device ------------------------------------------------------------------------------- */

/* Gpu::new (crates/jevons-kernels/src/lib.rs:181-191): checks that `device` exists and is a
 * Blackwell sm_100 part, and makes it current on this thread. */
jk_status jk_gpu_init(int device);

/* Gpu::sync (lib.rs:300-302): waits for all work queued on `stream`. */
jk_status jk_gpu_sync(void *stream);

/* Reads and clears the device-side error word of `device` (bounded waits that ran out record
 * a code there instead of hanging). Synchronises the device. *code = 0 when clean. */
jk_status jk_device_error(int device, uint32_t *code);

/* Caps the number of multiprocessors the products on `device` may occupy (0 = all of them, the
 * default). A caller that runs communication kernels (NCCL) alongside the products, as the
 * column-sharded multi-GPU layout does, leaves SMs free for them with this so both overlap.
 * Launches made after the call use the new cap. No counterpart in the reference (one device). */
jk_status jk_set_max_ctas(int device, int max_sms);
/* The cap set by jk_set_max_ctas (0 = none) and the device's SM count. */
jk_status jk_get_max_ctas(int device, int *max_sms, int *sm_total);

/* ---- quantized weight matrices -------------------------------------------------------------- */

typedef struct jk_qmatrix jk_qmatrix;

/* QMatrix::upload (gemm.rs:832-854): validates and repacks raw GGML bytes of a
 * [experts * n, k] matrix into the B200 layout and copies them to `device`.
 * Errors: JK_ERR_SHAPE "<type> [<experts>x<n>, <k>] has the wrong byte count" /
 * "... has an unsupported shape" (n % 64, k % 64, k % block), JK_ERR_UNSUPPORTED for types
 * without a GPU layout. */
jk_status jk_qmatrix_upload(int device, int type, size_t n, size_t k, size_t experts,
                            const void *ggml_bytes, size_t len, jk_qmatrix **out);

/* QMatrix::from_packed (gemm.rs:856-899): same, from the reference's SoA regions (jk_pack). */
jk_status jk_qmatrix_from_packed(int device, int type, size_t n, size_t k, size_t experts,
                                 const uint32_t *q, size_t q_words, const uint32_t *h, size_t h_words,
                                 const uint32_t *s, size_t s_words, const float *d, size_t d_words,
                                 jk_qmatrix **out);

/* QMatrix::f16_view / from_f16_words (gemm.rs:906-948): views caller-owned row-major FP16
 * weights [n, k] on `device` without copying (n % 64, k % 64). The view never frees them. */
jk_status jk_qmatrix_f16_view(int device, size_t n, size_t k, const void *f16_weights_dev,
                              jk_qmatrix **out);

/* Frees a matrix (no-op for NULL). Frees device memory only if the matrix owns it. */
void jk_qmatrix_destroy(jk_qmatrix *w);

/* Fields of QMatrix (gemm.rs:818-829) and QMatrix::bytes (:950-952): the device bytes held. */
jk_status jk_qmatrix_info(const jk_qmatrix *w, int *type, size_t *n, size_t *k, size_t *experts,
                          size_t *device_bytes);

/* Device dequantization of the whole matrix to f32 [experts * n, k], using the same decode
 * routines as the matmul kernels. Bit-exact with quant::dequantize (quant.rs:83-101). */
jk_status jk_qmatrix_dequantize(const jk_qmatrix *w, float *out_dev, size_t out_len, void *stream);

/* ---- launch plans ---------------------------------------------------------------------------- */

/* Plan (gemm.rs:973-1016). bm == 0 selects the small-row kernel (m <= JK_GEMV_ROWS).
 * Otherwise bm is the activation-row tile of the tensor-core kernel (MMA N: 32, 64, 96, 128 or
 * 256), bn the weight-row tile and splits the split-K factor (1..16). bn = 128 runs one CTA per
 * tile (MMA M = 128); bn = 256 (block-quantized weights, bm >= 128) runs each tile on a pair of
 * CTAs with one M = 256 MMA (tcgen05 cta_group::2), each CTA dequantizing 128 rows and loading
 * half the activation rows. Plans with bm > 0 and splits == 1 are row invariant: every output row
 * is accumulated in the same order whatever m, bm or bn is (gemm.rs:1090-1091). */
typedef struct jk_plan {
    int32_t bm;
    int32_t bn;
    int32_t splits;
} jk_plan;

#define JK_GEMV_ROWS 16 /* GEMV_ROWS (gemm.rs:1019) */

/* Plan::heuristic (gemm.rs:989-1004); `sms` is the multiprocessor count to fill (the
 * reference's groups_target; 0 = the device's own count). Unless row_invariant, block-quantized
 * weights get the row tile (32/64/96/128) and schedule (whole tiles or stream-K) that a cost model
 * of this kernel's measured main-loop rates and waves of tiles over the SMs predicts fastest. */
jk_status jk_plan_heuristic(const jk_qmatrix *w, size_t m, int row_invariant, int sms, jk_plan *out);

/* Plan::valid_for (gemm.rs:1006-1015): 1 if `plan` can run `w` at `m` rows, else 0. */
int jk_plan_valid_for(const jk_plan *plan, const jk_qmatrix *w, size_t m);

/* ---- split-K scratch ------------------------------------------------------------------------ */

/* SplitScratch (gemm.rs:1040-1065): device scratch for split-K partial sums and activation
 * conversion, grown on demand with cudaMalloc (the growth synchronises the device). One
 * scratch must not be used by two launches that may run at the same time. */
typedef struct jk_split_scratch jk_split_scratch;
jk_status jk_split_scratch_create(int device, jk_split_scratch **out);
void jk_split_scratch_destroy(jk_split_scratch *s);

/* ---- products -------------------------------------------------------------------------------- */

/* matmul_plan (gemm.rs:1092-1119): out[m, n] = x[m, k] . W^T with an explicit plan.
 * x_len / out_len are element counts of the caller's buffers (checked like gemm.rs:1137,1218).
 * `scratch` may be NULL when plan.splits == 1 and x is bf16 or f16. */
jk_status jk_matmul_plan(const jk_qmatrix *w, const void *x, int x_dtype, size_t x_len, size_t m,
                         float *out, size_t out_len, jk_split_scratch *scratch, jk_plan plan,
                         void *stream);

/* matmul (gemm.rs:1069-1088): matmul_plan with Plan::heuristic(w, m, false, sms). */
jk_status jk_matmul(const jk_qmatrix *w, const void *x, int x_dtype, size_t x_len, size_t m,
                    float *out, size_t out_len, jk_split_scratch *scratch, void *stream);

/* matvec (gemm.rs:1135-1168): the small-row kernel, m <= JK_GEMV_ROWS. */
jk_status jk_matvec(const jk_qmatrix *w, const void *x, int x_dtype, size_t x_len, size_t m,
                    float *out, size_t out_len, void *stream);

/* matmul_tiled (gemm.rs:1121-1133): matmul_plan with splits = 1. */
jk_status jk_matmul_tiled(const jk_qmatrix *w, const void *x, int x_dtype, size_t x_len, size_t m,
                          float *out, size_t out_len, int bm, int bn, void *stream);

/* jevons_burn::kernels::f16_linear / GemmOps::f16_matmul (crates/jevons-burn/src/kernels.rs:
 * 47-114): out[m, n] f32 = x[m, k] (FP16, dense row-major) . W[n, k]^T (FP16) with the fixed
 * row-invariant plan of kernels.rs:16-31. */
jk_status jk_f16_linear(const void *x_f16, size_t m, size_t k, const void *w_f16, size_t n,
                        float *out, void *stream);

/* jevons_burn::kernels::f16_linear_scaled (kernels.rs:116-129): jk_f16_linear for f32 activations
 * of any magnitude. Row r of x is divided by s_r = max(max_j |x[r, j]| / 16384, 1) (f32 division)
 * and cast to FP16, the FP16 product runs, and out[r, :] is multiplied back by s_r (rows with
 * s_r == 1 give exactly jk_f16_linear of the FP16-cast row). The FP16 rows and scales live in
 * `scratch` (required; grown like jk_matmul_plan's). */
jk_status jk_f16_linear_scaled(const float *x_f32, size_t m, size_t k, const void *w_f16, size_t n,
                               float *out, jk_split_scratch *scratch, void *stream);

/* ---- Q8_0 int8 path ----------------------------------------------------------------------------
 * The int8 plan of the reference (docs/cubecl-int8-plan.md:48-60; it has no implementation there):
 * activations are quantized per 32 values so that every Q8_0 weight block meets an activation
 * block as an exact int32 dot product (one tcgen05 kind::i8 MMA with K = 32 per block), and the
 * two block scales are applied in f32 afterwards. */

/* Per-32 activation quantization of x [m, k] (f32, f16 or bf16; k % 32 == 0): for each row r and
 * block b, amax = max |x[r, 32b..32b+31]|, d = amax / 127 and q = rint(x * (127 / amax)) clamped
 * to [-127, 127] (IEEE f32, round to nearest even; an all-zero block gives d = 0, q = 0).
 * xq: int8 [m, k] (xq_len >= m * k); xd: f32 scales, block-major [k / 32][m_pad] with m_pad = m
 * rounded up to a multiple of 4 (xd_len >= k / 32 * m_pad; the padding rows are set to 0).
 * Deterministic; asynchronous on `stream`. */
jk_status jk_quantize_act_q8(const void *x, int x_dtype, size_t m, size_t k, int8_t *xq, size_t xq_len,
                             float *xd, size_t xd_len, void *stream);

/* The Q8_0 product on int8 tensor cores: out[r, c] = sum over blocks b, in increasing order, of
 *   f32(dot_b) * (f32(d_w[c, b]) * xd[b][r])   accumulated with one fused multiply-add per block,
 * where dot_b = sum_j q_w[c, 32b + j] * xq[r, 32b + j] is exact in int32. w must be Q8_0 (expert 0's
 * rows for a multi-expert matrix); xq / xd as written by jk_quantize_act_q8 for the same m and
 * k (16-byte aligned); out f32 [m, n]. JK_ERR_UNSUPPORTED for other weight types. */
jk_status jk_matmul_q8_int8(const jk_qmatrix *w, const int8_t *xq, size_t xq_len, const float *xd,
                            size_t xd_len, size_t m, float *out, size_t out_len, void *stream);

/* ---- expert-grouped products ----------------------------------------------------------------- */

/* Groups (gemm.rs:955-966): a device-side grouping of routed rows by expert, as written by
 * jk_group_experts. Job j covers sorted positions [jobs[2j+2], min(jobs[2j+2] + tile,
 * offsets[e+1])) of expert e = jobs[2j+1] (jobs[0] = job count), where tile is the row tile the
 * jobs were built with; position s reads activation row sorted[s] / in_div and writes output row
 * sorted[s] (gemm.rs:9-11). */
typedef struct jk_groups {
    const uint32_t *sorted;  /* [rows] assignment index of each sorted position (the reference's ids) */
    const uint32_t *offsets; /* [experts + 1] first sorted position of each expert, then the total */
    const uint32_t *jobs;    /* [1 + 2 * max_jobs] job count, then (expert, first position) pairs */
    size_t max_jobs;         /* upper bound on the job count: the grid's job dimension */
    uint32_t in_div;         /* activation row = assignment / in_div (top_k for per-token inputs) */
    size_t rows;             /* output rows (assignments) */
} jk_groups;

/* The job bound jk_group_experts needs room for: ceil(assignments / bm) + min(experts,
 * assignments). The reference's callers size jobs as ceil(a / bm) + experts
 * (crates/jevons-gemma4-diffusion/src/model.rs:593), which is never smaller. 0 if bm < 1. */
size_t jk_group_max_jobs(size_t assignments, size_t experts, int bm);

/* group_routes (crates/jevons-gemma4-diffusion/src/gpu/ops.rs:1100-1128, kernel `group`
 * :523-585): deterministic grouping of `assignments` expert ids (device u32, each < experts) on
 * `stream`. Writes sorted[assignments] (assignment indices ordered by expert, ascending within
 * an expert), offsets[experts + 1] and jobs (jobs[0] = count, then (expert, start) pairs for tiles
 * of bm rows, experts ascending). jobs_len (elements) must hold 1 + 2 * jk_group_max_jobs(...).
 * experts <= 1024. An id >= experts is left out of every group (offsets[experts] then counts
 * fewer rows and the products never write those rows) and sets an error bit that
 * jk_device_error reports. */
jk_status jk_group_experts(int device, const uint32_t *ids, size_t assignments, size_t experts, int bm,
                           uint32_t *sorted, uint32_t *offsets, uint32_t *jobs, size_t jobs_len, void *stream);

/* matmul_grouped (gemm.rs:1271-1321): out[sorted[s], :] = x[sorted[s] / in_div, :] . W_e^T for
 * every sorted position s of expert e, W_e = rows [e * n, (e + 1) * n) of the matrix, on the
 * tensor cores. The jobs must have been built with tiles of bm rows. bm/bn as in jk_plan; splits
 * (1..16, k / 64 >= splits) is accepted for plan compatibility, and every split count gives the
 * whole-K result of splits = 1 (jobs are read on the device, so the product always runs whole
 * tiles and stays row invariant). x: x_len / k activation rows (f32, f16 or bf16); the activation
 * rows are gathered into `scratch` (required) in sorted order first. out_len >= rows * n. */
jk_status jk_matmul_grouped(const jk_qmatrix *w, const void *x, int x_dtype, size_t x_len, const jk_groups *g,
                            float *out, size_t out_len, int bm, int bn, int splits, jk_split_scratch *scratch,
                            void *stream);

/* matvec_grouped (gemm.rs:1170-1200): the grouped product on the small-row kernel, for jobs built
 * with tiles of mr <= JK_GEMV_ROWS rows. Reads activation rows in place (no scratch). */
jk_status jk_matvec_grouped(const jk_qmatrix *w, const void *x, int x_dtype, size_t x_len, const jk_groups *g,
                            float *out, size_t out_len, int mr, void *stream);

/* ---- column-sharded product across GPUs ---------------------------------------------------------
 * The multi-GPU layout of the large-N projections (the vocabulary head, the FFN up projection):
 * no counterpart in the reference, which runs on one device. Rank r of `world` (one process or
 * thread per GPU, world <= 8) holds its shard w_shard = weight rows [r n_r, (r + 1) n_r) of the
 * full [world n_r, k] matrix, and every rank ends with the whole f32 output in a rank-major buffer
 * [world][m][n_r]: rank p's output columns are rows [p m, (p + 1) m) of it. */

/* Device memory another process can map: cudaMalloc of `bytes` (zeroed) on `device` and its
 * 64-byte CUDA IPC handle. Free with jk_ipc_free. */
jk_status jk_ipc_alloc(int device, size_t bytes, void **dev_ptr, uint8_t handle[64]);
jk_status jk_ipc_free(int device, void *dev_ptr);
/* Maps another process's jk_ipc_alloc buffer on `device` (peer access enabled); unmap with
 * jk_ipc_close. */
jk_status jk_ipc_open(int device, const uint8_t handle[64], void **dev_ptr);
jk_status jk_ipc_close(int device, void *dev_ptr);

/* out_peers[p] (p < world): rank p's gathered output buffer [world][m][n_r] f32 as mapped in this
 * process (this rank's own at p == rank); flags_peers[p]: rank p's `world` u32 flag words.
 * The product of x [m, k] with the shard (jk_matmul's heuristic plan) is computed in `chunks`
 * row chunks (1..16, multiples of 32 rows) into this rank's block of its own buffer; each finished
 * chunk is pushed into every peer's buffer by the copy engines (one copy stream per peer, inside
 * the library) while the next chunk's product runs, so the exchange takes no SMs from the product.
 * The copy streams carry copies only (a kernel there would wait for an SM the products hold). With
 * 4 or more row chunks the last quarter of them is pushed to the peers by a copy kernel on `stream`
 * once the products are done (the copy engines are still busy with the earlier chunks then, and the
 * SMs are free). With
 * wait != 0 the call ends with jk_allgather_wait: the gathered output is complete on `stream`
 * after it. With wait == 0 the call returns with its copies still running beside `stream` (the
 * next product can overlap them): this rank's block of out_peers[rank] must then stay untouched
 * until the caller's next jk_allgather_wait, which covers every copy issued since the previous
 * wait (for example once after several layers, each with its own output buffers). All ranks make
 * the same calls and waits in the same order. A result stays valid until the next call on any
 * rank that writes the same buffers. */
jk_status jk_sharded_matmul_allgather(const jk_qmatrix *w_shard, const void *x, int x_dtype, size_t x_len,
                                      size_t m, int rank, int world, float *const *out_peers,
                                      uint32_t *const *flags_peers, int chunks, int wait,
                                      jk_split_scratch *scratch, void *stream);
/* Ends an exchange: after all copies this rank issued since its previous wait, adds one to
 * flags_peers[p][rank] in every peer p (a system-scope reduction ordered after those copies),
 * joins the copy streams into `stream`, and waits on `stream` (one warp) until every peer's counter
 * in this rank's flags has reached flags[rank] + 1, then advances flags[rank] (this rank's count of
 * waits). The counters live on the device, so a captured CUDA graph that replays calls and waits
 * stays in step with the peers. Bounded (2 s): a peer that never signals sets ERR_WAIT_TIMEOUT,
 * read with jk_device_error. Inside a CUDA graph capture, call it after at least one product of
 * the same capture. */
jk_status jk_allgather_wait(int device, uint32_t *const *flags_peers, int world, int rank, void *stream);

/* ---- allocation-free product ----------------------------------------------------------------- */

/* Size of the device buffer libjk.so declares for jk_matmul_splitk_noalloc (per GPU, held from
 * library load until process exit). */
#define JK_NOALLOC_SCRATCH_BYTES (20u * 1024u * 1024u)

/* No counterpart in the reference: an addition for callers that cannot allocate device memory
 * while they run a product -- code under a framework that owns every device allocation (a
 * cudaMalloc from the library would escape its accounting or exceed its cap), or paths where the
 * device synchronisation of a cudaMalloc is not acceptable.
 * Computes the same product as jk_matmul_plan with plan {bm, 128, splits > 1} (the stream-K
 * schedule), with its scratch in a fixed buffer inside the library instead of a jk_split_scratch;
 * it calls no cudaMalloc, cudaFree or allocating routine. Activations must be bf16 or f16
 * (JK_ERR_UNSUPPORTED for f32). Limit: the schedule runs one CTA per SM and needs a bm x 128 f32
 * partial tile per CTA, bm * 512 bytes each; if that exceeds JK_NOALLOC_SCRATCH_BYTES minus 4096
 * bytes of flag words (never on a 148-SM B200) the call fails with JK_ERR_SHAPE and launches
 * nothing. The first call on a device looks up the buffer's device address (cudaGetSymbolAddress,
 * no allocation); make that first call outside any stream capture. All calls on a device share
 * the buffer: calls that can overlap on the GPU race -- order them on one stream. */
jk_status jk_matmul_splitk_noalloc(const jk_qmatrix *w, const void *x, int x_dtype, size_t x_len, size_t m,
                                   float *out, size_t out_len, int bm, void *stream);

/* ---- Q6_K embedding-table ("head") operators --------------------------------------------------
 * `table` is a Q6_K matrix [vocab, d] (experts * n rows, k = d): the model's token embedding and
 * tied output projection. The reference passes the same data as the packed word regions of
 * ops::Q6kTable (crates/jevons-gemma4-diffusion/src/gpu/ops.rs:912-919, model.rs:181-184); here
 * it is a jk_qmatrix (jk_qmatrix_upload / jk_qmatrix_from_packed of type JK_TYPE_Q6_K). All device
 * pointers; all calls asynchronous on `stream`. Errors: JK_ERR_UNSUPPORTED for a table that is
 * not Q6_K; JK_ERR_INVALID for null or misaligned buffers. Ids outside the table or rows outside
 * x are found on the device: they set an error bit (2) that jk_device_error reports, instead of
 * being read out of bounds. */

/* ops::embed (ops.rs:921-954; kernel embed_q6k :223-291). For t < rows:
 *   out[t]    = E[tokens[t]] * sqrt(d)                                      f32 [rows, d]
 *   rows t >= first_canvas then add cond[t - first_canvas] (f32 [rows - first_canvas, d]) when
 *   cond_dev is not NULL and are RMS-normalised without weight:  out[t] *= 1/sqrt(mean(out[t]^2) + eps)
 *   x_attn[t] = f16(out[t] * 1/sqrt(mean(out[t]^2) + eps) * w_attn)        f16 [rows, d]
 * The pre-normalisation values are bit-exact with the reference (exact decode, one rounding by
 * sqrt(d)). d <= 16384 (JK_ERR_SHAPE above). w_attn, cond, out, x_attn 16-byte aligned. A token
 * id >= vocab computes its row from zeros. */
jk_status jk_embed_q6k(const jk_qmatrix *table, const uint32_t *tokens_dev, size_t rows, const float *w_attn_dev,
                       const float *cond_dev, size_t first_canvas, float eps, float *out_dev, void *x_attn_f16_dev,
                       void *stream);

/* ops::pick (ops.rs:1133-1157; kernel pick_logits :590-635): for p < count, with
 * (row, token) = (pairs[2p], pairs[2p+1]):  out[p] = softcap * tanh(dot(x[row], E[token]) / softcap)
 * x is f16 [x_rows, d] (16-byte aligned), out f32 [count]. A pair outside x or the table writes
 * NaN. */
jk_status jk_pick_logits(const jk_qmatrix *table, const void *x_f16_dev, size_t x_rows, const uint32_t *pairs_dev,
                         size_t count, float softcap, float *out_dev, void *stream);

/* ops::q6k_transposed_f16 (ops.rs:732-749; kernel q6k_transpose :672-715): the dequantized table
 * transposed to f16 [d, vocab] (out_len = vocab * d values, 16-byte aligned), bit-exact with
 * f16(quant::dequantize) transposed. vocab % 64 == 0 (JK_ERR_SHAPE otherwise), as the reference
 * asserts. */
jk_status jk_q6k_transpose_f16(const jk_qmatrix *table, void *out_f16_dev, size_t out_len, void *stream);

/* ops::softcap_logits (ops.rs:1159-1168; kernel softcap :751-760): x[i] = cap * tanh(x[i] / cap)
 * in place for i < len, on the current device (x 16-byte aligned). With jk_matmul over the table
 * this is the reference's full-vocabulary head (model.rs:1192-1205). */
jk_status jk_softcap(float *x_dev, size_t len, float cap, void *stream);

/* ---- GGUF reader and weight loader --------------------------------------------------------------
 * Gguf (crates/jevons-formats/src/gguf.rs:164-391), host only. Errors are JK_ERR_INVALID with the
 * reference's texts: "Invalid GGUF file: <why>", "I/O error reading the model: <why>",
 * "Missing GGUF metadata key <key>", "Missing tensor <name>". */

typedef struct jk_gguf jk_gguf;

/* TensorInfo (gguf.rs:148-156). dims in GGML order (dims[0] = contiguous row length), unused dims
 * 1; offset is absolute in the file; bytes = 0 for types without a block size. `name` is valid
 * until jk_gguf_close. */
typedef struct jk_gguf_tensor_info {
    const char *name;
    uint32_t n_dims;
    uint64_t dims[4];
    int32_t type;
    uint64_t offset;
    uint64_t bytes;
} jk_gguf_tensor_info;

/* Gguf::open (gguf.rs:234-324): parses and validates the header (magic, version 2 or 3, at most
 * 2^20 tensors and keys, metadata of the 13 GGUF kinds without nested arrays, strings <= 2^24
 * bytes of UTF-8, arrays <= 2^26 values, general.alignment a power of two (default 32), 1..4 dims,
 * block-aligned rows, every tensor aligned and inside the file, no duplicate keys or names). */
jk_status jk_gguf_open(const char *path, jk_gguf **out);
void jk_gguf_close(jk_gguf *g);
size_t jk_gguf_tensor_count(const jk_gguf *g);
size_t jk_gguf_metadata_count(const jk_gguf *g);
/* Tensor i in file order / Gguf::tensor (gguf.rs:345-350) by name. */
jk_status jk_gguf_tensor_at(const jk_gguf *g, size_t i, jk_gguf_tensor_info *out);
jk_status jk_gguf_tensor(const jk_gguf *g, const char *name, jk_gguf_tensor_info *out);
/* Gguf::read_range (gguf.rs:365-372; Gguf::read with start 0, len = bytes): raw bytes of a tensor
 * of a supported type ("tensor <name> has unsupported type Other(<id>)" otherwise). */
jk_status jk_gguf_read(const jk_gguf *g, const char *name, uint64_t start, uint64_t len, void *dst);
/* Gguf::read_f32 (gguf.rs:374-391): an F32 tensor's values (dst holds bytes / 4 floats). */
jk_status jk_gguf_read_f32(const jk_gguf *g, const char *name, float *dst, size_t dst_len);

/* Metadata. kind: the GGUF value type (0 u8 .. 12 f64; 8 string, 9 array); for arrays elem_kind
 * and len (values), for strings len (bytes), else len 1. The getters read the value at `key`, or
 * element `index` of the array at `key` when index >= 0, with Value::as_u64 / as_i64 / as_f64 /
 * as_bool / as_str semantics (gguf.rs:53-105; Gguf::u64 / f32, :332-343). Strings stay valid until
 * jk_gguf_close. */
jk_status jk_gguf_value_kind(const jk_gguf *g, const char *key, int *kind, int *elem_kind, size_t *len);
jk_status jk_gguf_u64(const jk_gguf *g, const char *key, int64_t index, uint64_t *out);
jk_status jk_gguf_i64(const jk_gguf *g, const char *key, int64_t index, int64_t *out);
jk_status jk_gguf_f32(const jk_gguf *g, const char *key, int64_t index, float *out);
jk_status jk_gguf_bool(const jk_gguf *g, const char *key, int64_t index, int *out);
jk_status jk_gguf_str(const jk_gguf *g, const char *key, int64_t index, const char **out, size_t *len);

/* The model load path for one weight: reads the tensor's raw GGML blocks and uploads them with
 * jk_qmatrix_upload as [experts * n, k] with k = dims[0], n = dims[1], experts = dims[2] * dims[3]
 * (the reference's per-layer and expert tensors). */
jk_status jk_qmatrix_from_gguf(int device, const jk_gguf *g, const char *name, jk_qmatrix **out);

/* ---- measured launch plans ---------------------------------------------------------------------
 * Tuner (crates/jevons-gemma4-diffusion/src/gpu/tune.rs): plans for the dense products timed on
 * the device, keyed by (type, n, k, row bucket, row invariance), stored in a text file keyed by a
 * device profile (name, SM count, compute capability, shared memory, L2, library ABI). A tuner is
 * used from one thread at a time for tuning; lookups are thread safe. */

typedef struct jk_tuner jk_tuner;

/* bucket (tune.rs:74-76): plans measured at m = bucket serve every m in (bucket/2, bucket];
 * the next power of two, at least 4. */
size_t jk_tune_bucket(size_t m);

/* pick (tune.rs:548-562): the fastest of `count` timed plans, unless `baseline` (the heuristic)
 * is among them and within 5% of it -- then the baseline, so noise changes nothing. */
jk_status jk_tune_pick(const double *times, const jk_plan *plans, size_t count, jk_plan baseline, jk_plan *out);

/* Tuner::new (tune.rs:139-155): a plan table for `device`. `path` (NULL = memory only) is the file
 * jk_tuner_save writes; with `load` != 0 its entries are read first when its profile line matches
 * this device and library (otherwise the file is ignored, as the reference does). */
jk_status jk_tuner_create(int device, const char *path, int load, jk_tuner **out);
void jk_tuner_destroy(jk_tuner *t);
/* Number of stored plans. */
size_t jk_tuner_size(const jk_tuner *t);

/* Tuner::dense (tune.rs:162-175): the stored plan for w's type and shape and bucket(m) if it is
 * valid for m (and has no split-K when row_invariant), else jk_plan_heuristic(w, m, row_invariant). */
jk_status jk_tuner_plan(const jk_tuner *t, const jk_qmatrix *w, size_t m, int row_invariant, jk_plan *out);

/* Tuner::tune_dense (tune.rs:231-269): times the candidate plans (bm 32..256 no taller than
 * needed, bn 128/256, splits 1/2/4/8 unless row_invariant; the GEMV plan for m <= JK_GEMV_ROWS)
 * at m = bucket(m) rows, running the product over all `count` matrices (same type and shape;
 * pass enough of them to exceed the L2 cache, so weights stream from HBM as in a forward pass),
 * and stores the pick. x / out hold bucket(m) rows (contents overwritten); scratch as for
 * jk_matmul_plan. Timing: CUDA events on `stream`, best of 3 batches of >= 2 ms. Synchronises
 * the stream. *chosen (may be NULL) receives the stored plan. */
jk_status jk_tuner_tune(jk_tuner *t, const jk_qmatrix *const *ws, size_t count, size_t m, int row_invariant,
                        const void *x, int x_dtype, size_t x_len, float *out, size_t out_len,
                        jk_split_scratch *scratch, void *stream, jk_plan *chosen);

/* Tuner::grouped (tune.rs:177-192): the stored grouped tile {bm, bn, 1} for w (type, n, k, experts)
 * and bucket(rows) when n is a multiple of its bn, else the default {32, 128, 1}. */
jk_status jk_tuner_group_plan(const jk_tuner *t, const jk_qmatrix *w, size_t rows, jk_plan *out);

/* Tuner::tune_grouped (tune.rs:271-346): for m tokens routed top_k ways, groups the first
 * a = bucket(m) * top_k ids of `ids` (device, < experts) for each candidate tile (bm 32/64/128/256
 * x bn 128/256) with jk_group_experts into sorted / offsets / jobs (jobs_len as for that call at
 * bm 32), times jk_matmul_grouped over the `count` expert matrices (x: a rows, one per route) and
 * stores the pick against the default {32, 128}. Synchronises the stream. */
jk_status jk_tuner_tune_grouped(jk_tuner *t, const jk_qmatrix *const *ws, size_t count, size_t m, size_t top_k,
                                const uint32_t *ids, size_t ids_len, const void *x, int x_dtype, size_t x_len,
                                float *out, size_t out_len, uint32_t *sorted, uint32_t *offsets, uint32_t *jobs,
                                size_t jobs_len, jk_split_scratch *scratch, void *stream, jk_plan *chosen);

/* Tuner::save (tune.rs:412-446): writes the profile line, one "dense <type> <n> <k> <bucket>
 * <row_invariant> <bm> <bn> <splits>" line per dense plan and one "grouped <type> <n> <k> <experts>
 * <bucket> <bm> <bn>" line per grouped plan to path (through path.tmp and a rename). */
jk_status jk_tuner_save(const jk_tuner *t);

#ifdef __cplusplus
}
#endif

#endif /* JK_H */
