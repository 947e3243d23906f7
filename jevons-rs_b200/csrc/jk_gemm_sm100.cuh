// jk_gemm_sm100.cuh -- the tensor-core product's kernels, out[r, c] = sum_j x[r, j] W[c, j] on
// sm_100a (the reference's `gemm` kernel with `matmul_split` / `reduce_splits`,
// crates/jevons-kernels/src/gemm.rs:532-815 and :1205-1269), designed for Blackwell. Included by
// one translation unit per weight format (jk_gemm_fmt_*.cu); the host side is jk_gemm_sm100.cu.
//
// * Roles swapped: the MMA's M side (128 TMEM lanes) carries 128 WEIGHT rows and its N side
//   carries BT activation rows (BT = 32..256), so a 32-row canvas product still issues full
//   MMAs; the f32 accumulator tile sits in tensor memory as [weight row][activation row].
// * Persistent CTAs, one per SM. The work is (tile, 64-wide k-block) iterations. Three schedules,
//   each compiled as its own kernel (template argument MODE):
//     0  dense, whole tiles (row-invariant plans, splits == 1): CTA c takes tiles c, c+G, ... --
//        every output's accumulation order is the same for any m and any BT;
//     1  dense, stream-K (splits > 1): CTA c takes the contiguous iteration range
//        [c*T/G, (c+1)*T/G) of all T = tiles * k-blocks iterations, so all SMs get equal work
//        whatever the tile count. A tile split between CTAs is finished by the CTA holding its
//        first k-block (the owner); the others (contributors) store f32 partial tiles to the
//        split scratch and raise a flag; the owner adds them in increasing k order
//        (deterministic for a given shape) and clears the flags for the next launch;
//     2  expert-grouped, whole tiles (the job table of jk_group.cu on the device).
// * Warp-specialised roles (the layouts are described at Smem and the role constants below):
//   activation TMA producer, MMA issuer (tcgen05.mma kind::f16, one elected lane), raw-weight TMA
//   producer, four epilogue warps (tcgen05.ld of a finished accumulator, f32 stores, stream-K
//   handshakes) and groups of four dequantizer warps that decode the raw super-blocks with the
//   reference's exact arithmetic (jk_decode.cuh) into tensor memory (TMEM A stages) or into
//   128-byte-swizzled K-major shared-memory tiles. The epilogue of tile i overlaps the MMAs of
//   tile i+1 (double-buffered accumulators).
// * Every mbarrier / flag wait is bounded (4 s): on expiry the error word records
//   ERR_WAIT_TIMEOUT, the CTA stops issuing work, drains what it issued and frees TMEM.
// * FP16 weights (the Burn-facing f16_linear path) skip dequantization: the producer TMA-loads the
//   weight tile straight into the swizzled operand stage.
// * No TMA multicast anywhere.
#pragma once

#include "jk_decode.cuh"
#include "jk_gemm_launch.h"

#include <cstdio>

namespace jk {
namespace tc {

constexpr int A_STAGE_BYTES = BW * KB * 2;
// Warp roles. Warp w is scheduled on SM sub-partition w % 4. The MMA issuer (warp 1) shares its
// sub-partition only with light roles (an epilogue warp, the raw-weight producer, an idle warp):
// the dequantizers' large unrolled loops would otherwise keep evicting the issuer's short loop
// from that sub-partition's instruction cache and stall every MMA issue.
//   w: 0 producer | 1 MMA | 4..7 epilogue (TMEM lane quarters 0..3) | 9 raw producer | 13 idle
//      dequantizers 2, 3, 8, 10 (group 0) and 11, 12, 14, 15 (group 1)
//
// When the dequantized weights go to tensor memory instead (TMEM_A below), a warp may only write
// the TMEM lanes of its own sub-partition (lanes 32 (w % 4) ..), so dequantizer slot s (rows
// 32 (s % 4) ..) sits on warp 8 + s; such CTAs have 20 warps and three dequantizer groups (the
// decoding, not the MMA, bounds their main loop):
//   w: 0 producer | 1 MMA | 2 raw producer | 3 idle | 4..7 epilogue
//      dequantizers 8..11 (group 0), 12..15 (group 1), 16..19 (group 2)
// (with 128-row activation tiles only two tensor-memory stages fit, and such CTAs keep 16 warps
// and two groups: see Smem::DQ_GROUPS)
// k-blocks per MMA-issue batch (one round of barrier waits and commits per batch)
#ifndef JK_MMA_BATCH
constexpr int MMA_BATCH = 1;
#else
constexpr int MMA_BATCH = JK_MMA_BATCH;
#endif
constexpr int PRODUCER_WARP = 0, MMA_WARP = 1, EPI_WARP0 = 4, EPI_WARPS = 4, DQ_WARPS = 8;
constexpr int EPI_THREADS = 32 * EPI_WARPS;  // 128: 1 per weight row
template <bool TMEM_A>
constexpr int RAW_WARP = TMEM_A ? 2 : 9;
template <bool TMEM_A>
__device__ __forceinline__ int dq_slot(int warp) {  // position among the dequantizer warps, or -1
    if constexpr (TMEM_A) {
        return warp >= 8 ? warp - 8 : -1;  // slot s on warp 8 + s: (8 + s) % 4 == s % 4
    } else {
        constexpr unsigned long long tbl = 0x76F543F2FFFF10FFull;  // nibble w: slot, F = none
        const int v = (int)((tbl >> (4 * warp)) & 15u);
        return v == 15 ? -1 : v;
    }
}

template <int FMT>
struct RawTile {
    static constexpr int bytes = FMT == FMT_Q4K ? BW * 144
                               : FMT == FMT_Q6K ? BW * 208
                               : FMT == FMT_Q8_0 ? BW * 256
                               : FMT == FMT_Q5_0 ? BW * 128
                               : 0;
};

constexpr int SMEM_LIMIT = 227 * 1024;

// The fewest tensor-memory weight stages a tile configuration keeps two accumulator buffers for.
#ifndef JK_MIN_TMEM_STAGES
#define JK_MIN_TMEM_STAGES 2
#endif

// Stage counts. Quantized weights use three rings: SX activation tiles (TMA), SA dequantized weight
// tiles, R raw super-blocks (TMA). The activation ring is decoupled from the weight ring so that
// several activation tiles are in flight (their L2 latency is the longest in the loop) while the
// dequantizers fill a few weight tiles just ahead of the MMA. FP16 weights come by TMA with their
// activation tile, so for them SX == SA (one coupled ring).
struct Rings {
    int sx, sa, r;
};
constexpr int SMEM_BUDGET = SMEM_LIMIT - 2048;  // barriers, TMEM holder, 1 KB alignment slack
constexpr Rings pick_rings(int b_stage, int raw_bytes) {
    constexpr Rings prio[] = {{8, 4, 4}, {6, 4, 4}, {6, 4, 3}, {6, 3, 3}, {5, 4, 3}, {5, 3, 3}, {4, 4, 3},
                              {4, 3, 3}, {4, 3, 2}, {4, 2, 3}, {4, 2, 2}, {3, 3, 2}, {3, 2, 2}, {2, 2, 2}};
    if (raw_bytes == 0) {
        for (int s = 6; s >= 2; --s)
            if (s * (b_stage + A_STAGE_BYTES) <= SMEM_BUDGET) return Rings{s, s, 1};
        return Rings{2, 2, 1};
    }
    for (const Rings& c : prio)
        if (c.sx * b_stage + c.sa * A_STAGE_BYTES + c.r * raw_bytes <= SMEM_BUDGET) return c;
    return Rings{2, 2, 2};
}

// Rings when the dequantized weight stages live in tensor memory: one ring of `s` stages (each
// stage's activation atoms in shared memory, its dequantized weights in tensor memory), at most
// `max_stages` (the tensor memory left by the accumulators), and the raw-weight ring.
constexpr Rings pick_rings_tmem(int b_stage, int raw_bytes, int max_stages) {
    for (int s = max_stages < 8 ? max_stages : 8; s >= 2; --s)
        for (int r = 8; r >= 3; --r)
            if (s * b_stage + r * raw_bytes <= SMEM_BUDGET && (r >= s / 2 || r >= 4)) return Rings{s, s, r};
    return Rings{2, 2, 2};
}

template <int FMT, int BT, bool PAIR = false>
struct Smem {
    // Dequantized weight stages in tensor memory (written with tcgen05.st, read by the MMA as its
    // A operand) where the two accumulator buffers leave room for them: single CTAs with BT <= 128.
    // This keeps the 16 KB per k-block of dequantized weights off the shared-memory pipe twice
    // (the dequantizers' stores and the MMA's reads). A TMEM_A stage holds KPS = 4 k-blocks (one
    // raw super-block, decoded by one dequantizer group; the groups alternate stages) and one
    // barrier pair serves the activations and the weights of the stage, so the MMA issuer and the
    // dequantizers wait once per four k-blocks (an mbarrier wait costs about as much issue time as
    // four M=128, N=32 MMAs).
    //
    // CTA pairs with 256-row activation tiles use tensor-memory stages too (the M = 256 MMA reads
    // each CTA's 128 weight rows from that CTA's tensor memory): one 256-column accumulator per
    // CTA (NACC = 1) leaves room for two stages. A pair then decodes every weight tile once per
    // 256 activation rows and each SM's MMA (128 x 256 x 64 per k-block) outlasts its decoding.
    static constexpr bool TMEM_A = FMT != FMT_F16 && (PAIR ? BT == 256 : BT <= 128);
    static constexpr int KPS = TMEM_A ? 4 : 1;  // k-blocks per stage: one raw super-block
    static constexpr int B_ATOM = (PAIR ? BT / 2 : BT) * 128;  // one k-block of activations (a pair CTA: half the rows)
    static constexpr int B_STAGE = KPS * B_ATOM;
    static constexpr int raw_bytes = RawTile<FMT>::bytes;
    // accumulator buffers (the epilogue of one tile overlaps the MMAs of the next when there are 2)
    // (one accumulator when two would leave fewer than JK_MIN_TMEM_STAGES weight stages)
    static constexpr int NACC = TMEM_A && 2 * BT + JK_MIN_TMEM_STAGES * 32 * KPS > 512 ? 1 : 2;
    static constexpr uint32_t TMEM_A0 = NACC * BT;  // first tensor-memory column of the A stages
    static constexpr Rings rings = TMEM_A ? pick_rings_tmem(B_STAGE, raw_bytes, (512 - NACC * BT) / (32 * KPS))
                                          : pick_rings(B_STAGE, raw_bytes);
    static constexpr int SX = rings.sx, SA = rings.sa, R = rings.r;
    // Groups of 4 dequantizer warps. A TMEM_A group waits on a stage's empty barrier by phase
    // parity, which is only sound if no group can reach a stage while the stage S places earlier
    // is still unconsumed: group g fills stage st after its own stage st - G, whose stage was
    // freed by the MMAs of stage st - G - S, so G <= S keeps every waiter within one phase.
    static constexpr int DQ_GROUPS = TMEM_A ? (SA < 3 ? SA : 3) : 2;
    static constexpr int THREADS = TMEM_A ? 32 * (8 + 4 * DQ_GROUPS) : 512;
    static_assert(!TMEM_A || (DQ_GROUPS >= 2 && DQ_GROUPS <= SA), "dequantizer groups vs stages");
    static_assert(FMT != FMT_F16 || SX == SA, "FP16 weights share the activation ring");
    static constexpr uint32_t TMEM_COLS = TMEM_A ? 512 : NACC * BT;
    static_assert(!TMEM_A || (SX == SA && TMEM_A0 + 32 * KPS * SA <= TMEM_COLS), "tensor memory budget");
    static constexpr int off_b = 0;
    static constexpr int off_a = off_b + SX * B_STAGE;
    static constexpr int off_raw = off_a + (TMEM_A ? 0 : SA * A_STAGE_BYTES);
    static constexpr int off_bar = off_raw + R * raw_bytes;
    // Stream-K fix-up: an owner's final segment is the CTA's last, so by then the operand and raw
    // stages [0, off_bar) are idle. They hold a ring of FIX_NB chunks for the contributor partials
    // (bulk-copied, FIX_CH activation rows x BW f32 each, contiguous in the workspace), then two
    // output staging buffers of the same size from which the epilogue threads write whole output
    // rows with 16-byte stores.
    static constexpr int FIX_CH = BT < 32 ? BT : 32;
    static constexpr int FIX_CHUNK = FIX_CH * BW * 4;
    static constexpr int FIX_NB = off_bar / FIX_CHUNK - 2 < 16 ? off_bar / FIX_CHUNK - 2 : 16;
    static constexpr int off_fix_out = FIX_NB * FIX_CHUNK;
    static_assert(FIX_NB >= 1, "fix-up ring");
    // full_b/empty_b x SX | full_a/empty_a x SA | raw_full/empty x R | acc_full/empty x 2 | fix-up ring
    static constexpr int n_bar = 2 * SX + 2 * SA + 2 * R + 4 + FIX_NB;
    static constexpr int bar_full_b = 0, bar_empty_b = SX, bar_full_a = 2 * SX, bar_empty_a = 2 * SX + SA,
                         bar_raw_full = 2 * SX + 2 * SA, bar_raw_empty = bar_raw_full + R,
                         bar_acc_full = bar_raw_empty + R, bar_acc_empty = bar_acc_full + 2, bar_fix = bar_acc_empty + 2;
    static constexpr int off_tmem = off_bar + 8 * n_bar;
    static constexpr int total = off_tmem + 16 + 1024;  // + base alignment slack
    static_assert(total <= SMEM_LIMIT, "shared memory budget");
};

// ------------------------------------------------------------------------------------------------
// Work schedule shared by every warp role (each role walks the same segments in the same order).
// ------------------------------------------------------------------------------------------------
struct Sched {
    int64_t tiles;     // weight tiles * activation tiles
    int tiles_m;       // activation-row tiles (grouped: jobs, an upper bound)
    int kbt;           // k-blocks per tile
    int G;             // CTAs
    int sk;            // 1 = stream-K, 0 = whole tiles
    // Expert-grouped products (whole tiles only): activation rows are expert-sorted; job j covers
    // sorted rows [jobs[2j+2], min(jobs[2j+2] + BT, offsets[e+1])) of expert e = jobs[2j+1]
    // (jobs[0] = job count, read on the device) and writes output rows sorted[s].
    const uint32_t* jobs;     // null: dense product
    const uint32_t* offsets;
    const uint32_t* sorted;
    int64_t n_exp;            // weight rows (output columns) per expert
    int job_rows;             // rows per job (<= BT)
    int64_t njobs;            // grouped: the job count jobs[0], read once per thread in the kernel
};

// Where a tile sits: its first weight row in the matrix, the first output column, its
// activation rows [m0, mend) and (grouped) whether its job exists.
struct TileAt {
    int64_t wrow0, col0, m0, mend;
    bool live;
};
template <int TW, int BT>
__device__ __forceinline__ TileAt tile_at(const Sched& s, int64_t tile, int rank, int64_t m) {
    TileAt t;
    const int64_t wt = tile / s.tiles_m, mt = tile % s.tiles_m;
    t.col0 = wt * TW + rank * 128;
    if (!s.jobs) {
        t.wrow0 = t.col0;
        t.m0 = mt * BT;
        t.mend = m;
        t.live = true;
    } else {
        t.live = mt < s.njobs;
        const int64_t e = t.live ? __ldg(s.jobs + 1 + 2 * mt) : 0;
        t.m0 = t.live ? __ldg(s.jobs + 2 + 2 * mt) : 0;
        const int64_t end = t.live ? __ldg(s.offsets + e + 1) : 0;
        t.mend = end < t.m0 + s.job_rows ? end : t.m0 + s.job_rows;
        t.wrow0 = e * s.n_exp + t.col0;
    }
    return t;
}

// Programmatic dependent launch (the launch sets cudaLaunchAttributeProgrammaticStreamSerialization):
// gdc_launch lets the next kernel on the stream start on SMs this grid frees; gdc_wait blocks until
// the previous kernel on the stream has completed and its memory is visible (a no-op without the
// attribute).
__device__ __forceinline__ void gdc_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void gdc_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

struct Seg {
    int64_t tile;
    int kb_lo, kb_hi;
};

struct SegState {
    int64_t next;      // SK: next iteration; DP: next tile
    int64_t end;       // SK: end iteration
};

__device__ __forceinline__ int64_t sk_start(const Sched& s, int c) {
    return (int64_t)c * (s.tiles * s.kbt) / s.G;
}

__device__ __forceinline__ void seg_init(const Sched& s, int c, SegState& st) {
    if (s.sk) {
        st.next = sk_start(s, c);
        st.end = sk_start(s, c + 1);
    } else {
        st.next = c;
        st.end = s.tiles;
    }
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}


// ---- CTA pairs (tcgen05 cta_group::2): the two CTAs of a cluster share one 256-row MMA ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// the shared::cluster address of `addr` (a shared::cta address of this CTA's layout) in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(dst_smem), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A (128 rows from each CTA's smem) x B^T (N/2 rows from each CTA's smem)
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p; }"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// the same with A read from tensor memory: each CTA's tensor memory holds its 128 rows of A at the
// same address (two 16-bit values per 32-bit column in k order)
__device__ __forceinline__ void mma_f16_ta_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p; }"
        :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// arrive on the mbarrier at offset `bar` in both CTAs of the pair once the issued MMAs complete
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 :: "r"(bar), "h"((unsigned short)3) : "memory");
}
// this CTA's half of a pair operand tile; the transaction bytes count on the leader CTA's barrier
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m, int32_t c0, int32_t c1,
                                                 uint32_t leader_bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(dst), "l"(m), "r"(c0), "r"(c1), "r"(leader_bar) : "memory");
}

__device__ __forceinline__ bool seg_next(const Sched& s, SegState& st, Seg& g) {
    if (st.next >= st.end) return false;
    if (s.sk) {
        g.tile = st.next / s.kbt;
        g.kb_lo = (int)(st.next % s.kbt);
        const int64_t left = st.end - st.next;
        g.kb_hi = left < (int64_t)(s.kbt - g.kb_lo) ? g.kb_lo + (int)left : s.kbt;
        st.next += g.kb_hi - g.kb_lo;
    } else {
        if (s.jobs) {  // grouped: every role skips the tiles of jobs past the device-side count
            while (st.next < st.end && st.next % s.tiles_m >= s.njobs) st.next += s.G;
            if (st.next >= st.end) return false;
        }
        g.tile = st.next;
        g.kb_lo = 0;
        g.kb_hi = s.kbt;
        st.next += s.G;
    }
    return true;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void epi_bar() {  // the 4 epilogue warps only
    asm volatile("bar.sync 1, %0;" :: "n"(EPI_THREADS) : "memory");
}

// 16 columns of 32-bit accumulators: thread i of the warp gets lane (taddr.lane + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

// Per-thread dequantizer of one weight row's super-blocks (256 k-elements = 4 k-blocks). A k-block
// is written in two halves (PART 0/1), rounded to bf16/f16, into the row's 128-byte swizzled line
// of the operand tile. Everything a super-block needs beyond the raw TMA stage (block
// scales kept in global memory) is loaded one super-block ahead (prefetch) so no global load sits
// on the critical path; Q4_K's header is decoded once per super-block into 8 (d*sc, dmin*m) pairs.
//   Q4_K part p: qs bytes 32j + 16p .. +16 -> low-nibble chunks 2p, 2p+1 and high-nibble chunks
//                2p+4, 2p+5 of k-block j (sub-blocks 2j and 2j+1)
//   others part p: chunks 4p .. 4p+3 of k-block j
// Destinations of a dequantized weight row's k-block (8 chunks of 8 16-bit values, k order):
// SmemRow writes the row of a 128-byte swizzled shared-memory A stage; RegRow keeps the 32 words in
// registers for one tcgen05.st into a tensor-memory A stage.
struct SmemRow {
    uint8_t* arow;
    int sw;
    __device__ __forceinline__ void put(int c, uint4 v) { *reinterpret_cast<uint4*>(arow + 16 * (c ^ sw)) = v; }
};
struct RegRow {
    uint32_t w[32];
    __device__ __forceinline__ void put(int c, uint4 v) {
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
    }
};
template <bool BF16, class O>
__device__ __forceinline__ void put8(O& o, int c, const float (&v)[8]) {
    uint4 pk;
    pk.x = pack2<BF16>(v[0], v[1]);
    pk.y = pack2<BF16>(v[2], v[3]);
    pk.z = pack2<BF16>(v[4], v[5]);
    pk.w = pack2<BF16>(v[6], v[7]);
    o.put(c, pk);
}

// 8 exact values (d*sc)*q - dmin*m (as fma, see jk_decode.cuh) of the 4 nibble-bytes of w0, w1
__device__ __forceinline__ void q4k_vals(uint32_t w0, uint32_t w1, float dd, float mm, float (&v)[8]) {
    const uint32_t ws[2] = {w0, w1};
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int i = 0; i < 4; i += 2) {
            const float2 q = sub2(make_float2(magic_byte(ws[t], i), magic_byte(ws[t], i + 1)), make_float2(MAGIC, MAGIC));
            const float2 r = fma2(make_float2(dd, dd), q, make_float2(-mm, -mm));
            v[4 * t + i] = r.x;
            v[4 * t + i + 1] = r.y;
        }
}

template <int FMT, bool BF16>
struct SbDequant;

// Packed 16-bit arithmetic for the operand tiles: x2 = two bf16 (BF16) or two f16 values.
template <bool BF16>
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t r;
    if constexpr (BF16) asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    else asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
template <bool BF16>
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    if constexpr (BF16) asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    else asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
// Exponent byte of the 16-bit magic M (bf16 0x4300 = 128, f16 0x6400 = 1024): a byte b < 128
// placed in the low byte gives the value M + b exactly. (Only the bf16 form is used for Q4_K.)
template <bool BF16>
constexpr uint32_t H2_MAGIC_HI = BF16 ? 0x43434343u : 0x64646464u;
template <bool BF16>
constexpr uint32_t H2_MAGIC = BF16 ? 0x43004300u : 0x64006400u;

// Q4_K: 8 weights (the nibble bytes of w0, w1 -- each byte one 4-bit quant) as bf16/f16, packed in
// k order. q is recovered exactly ((M + q) - M), then w = q * dd - mm in one rounding, with dd =
// d*sc and mm = dmin*m rounded to the operand type: the error is within two roundings of the
// 16-bit result (the per-element product tolerance covers it; jk_qmatrix_dequantize stays exact).
template <bool BF16>
__device__ __forceinline__ uint4 q4k_pack8(uint32_t w0, uint32_t w1, uint32_t dd2, uint32_t nmm2) {
    constexpr uint32_t HI = H2_MAGIC_HI<BF16>, M = H2_MAGIC<BF16>;
    uint4 r;
    r.x = h2_fma<BF16>(h2_sub<BF16>(__byte_perm(w0, HI, 0x4140), M), dd2, nmm2);
    r.y = h2_fma<BF16>(h2_sub<BF16>(__byte_perm(w0, HI, 0x4342), M), dd2, nmm2);
    r.z = h2_fma<BF16>(h2_sub<BF16>(__byte_perm(w1, HI, 0x4140), M), dd2, nmm2);
    r.w = h2_fma<BF16>(h2_sub<BF16>(__byte_perm(w1, HI, 0x4342), M), dd2, nmm2);
    return r;
}

// bf16 operands: packed 16-bit decode (q4k_pack8). FP16 operands keep the exact f32 decode
// rounded once: f16's range could overflow d*sc on its own where the f32 product does not.
template <bool BF16>
struct SbDequant<FMT_Q4K, BF16> {
    uint32_t dd2[8], nmm2[8];  // bf16: (d*sc, d*sc) and (-dmin*m, -dmin*m) pairs per sub-block
    float dd[8], mm[8];        // f16: exact f32 scale and min
    __device__ __forceinline__ void prefetch(const WView&, int64_t, int) {}
    __device__ __forceinline__ void begin(const uint8_t* raw_row, const WView&, int64_t, bool, int) {
        const uint4 hdr = *reinterpret_cast<const uint4*>(raw_row);
        const float d = half_bits_to_float(hdr.x & 0xFFFFu);
        const float dmin = half_bits_to_float(hdr.x >> 16);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t sc, mn;
            q4k_scale_min(hdr.y, hdr.z, hdr.w, j, sc, mn);  // j is a compile-time constant here
            const float a = __fmul_rn(d, (float)sc), b = __fmul_rn(dmin, (float)mn);
            if constexpr (BF16) {
                dd2[j] = pack2<true>(a, a);
                nmm2[j] = pack2<true>(-b, -b);
            } else {
                dd[j] = a;
                mm[j] = b;
            }
        }
    }
    template <int J, int PART, class O>
    __device__ __forceinline__ void kblock(const uint8_t* raw_row, int, int, O& o) {
        const uint4 q = *reinterpret_cast<const uint4*>(raw_row + 16 + 32 * J + 16 * PART);
        if constexpr (BF16) {
            const uint32_t dlo = dd2[2 * J], mlo = nmm2[2 * J], dhi = dd2[2 * J + 1], mhi = nmm2[2 * J + 1];
            o.put(2 * PART, q4k_pack8<true>(q.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, dlo, mlo));
            o.put(2 * PART + 1, q4k_pack8<true>(q.z & 0x0F0F0F0Fu, q.w & 0x0F0F0F0Fu, dlo, mlo));
            o.put(2 * PART + 4, q4k_pack8<true>((q.x >> 4) & 0x0F0F0F0Fu, (q.y >> 4) & 0x0F0F0F0Fu, dhi, mhi));
            o.put(2 * PART + 5, q4k_pack8<true>((q.z >> 4) & 0x0F0F0F0Fu, (q.w >> 4) & 0x0F0F0F0Fu, dhi, mhi));
        } else {
            float v[8];
            q4k_vals(q.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, dd[2 * J], mm[2 * J], v);
            put8<false>(o, 2 * PART, v);
            q4k_vals(q.z & 0x0F0F0F0Fu, q.w & 0x0F0F0F0Fu, dd[2 * J], mm[2 * J], v);
            put8<false>(o, 2 * PART + 1, v);
            q4k_vals((q.x >> 4) & 0x0F0F0F0Fu, (q.y >> 4) & 0x0F0F0F0Fu, dd[2 * J + 1], mm[2 * J + 1], v);
            put8<false>(o, 2 * PART + 4, v);
            q4k_vals((q.z >> 4) & 0x0F0F0F0Fu, (q.w >> 4) & 0x0F0F0F0Fu, dd[2 * J + 1], mm[2 * J + 1], v);
            put8<false>(o, 2 * PART + 5, v);
        }
    }
};

template <bool BF16>
struct SbDequant<FMT_Q6K, BF16> {
    uint32_t d_next = 0;
    float d = 0.f;
    __device__ __forceinline__ void prefetch(const WView& w, int64_t rr, int sb) {
        d_next = __ldg(w.d + rr * (w.k / 256) + sb);
    }
    __device__ __forceinline__ void begin(const uint8_t*, const WView&, int64_t, bool row_ok, int) {
        d = row_ok ? half_bits_to_float(d_next) : 0.f;
    }
    template <int J, int PART, class O>
    __device__ __forceinline__ void kblock(const uint8_t* body, int, int, O& o) {
        Q6KBlock bq;
        bq.load(body, d, J);
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            bq.chunk(4 * PART + i, v);
            put8<BF16>(o, 4 * PART + i, v);
        }
    }
};

template <bool BF16>
struct SbDequant<FMT_Q8_0, BF16> {
    uint4 d_next = make_uint4(0, 0, 0, 0);  // f16 scales of the super-block's 8 blocks
    uint4 dcur = make_uint4(0, 0, 0, 0);
    __device__ __forceinline__ void prefetch(const WView& w, int64_t rr, int sb) {
        const uint16_t* p = w.d + rr * (w.k / 32) + 8 * sb;
        if ((w.k & 255) == 0) {
            d_next = __ldg(reinterpret_cast<const uint4*>(p));
        } else {  // row not 16-byte aligned or partial super-block: load the valid pairs
            uint32_t t[4] = {0u, 0u, 0u, 0u};
            const int64_t nb = w.k / 32 - 8 * (int64_t)sb;
            for (int i = 0; i < 4; ++i)
                if (2 * i < nb) t[i] = __ldg(reinterpret_cast<const uint32_t*>(p) + i);
            d_next = make_uint4(t[0], t[1], t[2], t[3]);
        }
    }
    __device__ __forceinline__ void begin(const uint8_t*, const WView&, int64_t, bool row_ok, int) {
        dcur = row_ok ? d_next : make_uint4(0, 0, 0, 0);
    }
    template <int J, int PART, class O>
    __device__ __forceinline__ void kblock(const uint8_t* raw_row_half0, int row, int, O& o) {
        // k-block J: 128-byte swizzled half J/2 of the stage (the caller points raw_row_half0 at
        // half 0's row; half 1 starts BW * 128 bytes later), logical chunks 4 (J%2) ..
        const uint32_t dw = (J >> 1) == 0 ? ((J & 1) ? dcur.y : dcur.x) : ((J & 1) ? dcur.w : dcur.z);
        Q80Block bq;
        bq.load_sw(raw_row_half0 + (J >> 1) * (BW * 128), 4 * (J & 1), row, half_bits_to_float(dw & 0xFFFFu),
                   half_bits_to_float(dw >> 16));
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            bq.chunk(4 * PART + i, v);
            put8<BF16>(o, 4 * PART + i, v);
        }
    }
};

template <bool BF16>
struct SbDequant<FMT_Q5_0, BF16> {
    uint4 d_next = make_uint4(0, 0, 0, 0), h_next0 = make_uint4(0, 0, 0, 0), h_next1 = make_uint4(0, 0, 0, 0);
    uint4 dcur = make_uint4(0, 0, 0, 0), h0 = make_uint4(0, 0, 0, 0), h1 = make_uint4(0, 0, 0, 0);
    __device__ __forceinline__ void prefetch(const WView& w, int64_t rr, int sb) {
        const int64_t nb = w.k / 32 - 8 * (int64_t)sb;
        const uint16_t* pd = w.d + rr * (w.k / 32) + 8 * sb;
        const uint32_t* ph = w.h + rr * (w.k / 32) + 8 * sb;
        uint32_t t[4] = {0u, 0u, 0u, 0u}, a[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
        for (int i = 0; i < 4; ++i)
            if (2 * i < nb) t[i] = __ldg(reinterpret_cast<const uint32_t*>(pd) + i);
        for (int i = 0; i < 8; ++i)
            if (i < nb) a[i] = __ldg(ph + i);
        d_next = make_uint4(t[0], t[1], t[2], t[3]);
        h_next0 = make_uint4(a[0], a[1], a[2], a[3]);
        h_next1 = make_uint4(a[4], a[5], a[6], a[7]);
    }
    __device__ __forceinline__ void begin(const uint8_t*, const WView&, int64_t, bool row_ok, int) {
        dcur = row_ok ? d_next : make_uint4(0, 0, 0, 0);
        h0 = h_next0;
        h1 = h_next1;
    }
    template <int J, int PART, class O>
    __device__ __forceinline__ void kblock(const uint8_t* rowp, int, int sw, O& o) {
        // 128-byte swizzled row of the super-block; k-block J = logical chunks 2J, 2J+1
        const uint32_t dw = (J >> 1) == 0 ? ((J & 1) ? dcur.y : dcur.x) : ((J & 1) ? dcur.w : dcur.z);
        const uint32_t ha = J == 0 ? h0.x : J == 1 ? h0.z : J == 2 ? h1.x : h1.z;
        const uint32_t hb = J == 0 ? h0.y : J == 1 ? h0.w : J == 2 ? h1.y : h1.w;
        Q50Block bq;
        bq.load_words(*reinterpret_cast<const uint4*>(rowp + 16 * ((2 * J) ^ sw)),
                      *reinterpret_cast<const uint4*>(rowp + 16 * ((2 * J + 1) ^ sw)), ha, hb,
                      half_bits_to_float(dw & 0xFFFFu), half_bits_to_float(dw >> 16));
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            bq.chunk(4 * PART + i, v);
            put8<BF16>(o, 4 * PART + i, v);
        }
    }
};

// Dequantizer role: DQ_WARPS warps in two groups of 4 (one thread per weight row of the tile). The
// groups take alternating k-blocks of the CTA's k-block sequence, so two weight tiles are decoded
// at once; a thread decodes its row's whole k-block (64 weights). Both groups read every raw
// super-block stage and each warp releases it once.
template <int FMT, bool BF16, int BT, bool PAIR>
__device__ __forceinline__ void dequant_role(const Sched& sched, SegState& ss, uint8_t* smem, int row_in_tile, int grp,
                                             int rank, const WView& w, uint32_t* err, bool& ok, uint32_t bar0, int lane) {
    using L = Smem<FMT, BT, PAIR>;
    constexpr int TW = PAIR ? 2 * BW : BW;  // weight rows per tile
    constexpr int SA = L::SA, R = L::R;
    auto full_a = [&](int s) { return bar0 + 8u * (L::bar_full_a + s); };
    auto empty_a = [&](int s) { return bar0 + 8u * (L::bar_empty_a + s); };
    auto raw_full = [&](int r) { return bar0 + 8u * (L::bar_raw_full + r); };
    auto raw_empty = [&](int r) { return bar0 + 8u * (L::bar_raw_empty + r); };
    const int sw = row_in_tile & 7;
    SbDequant<FMT, BF16> dq;
    int it = 0, raw_n = 0;
    Seg sg;
    while (ok && seg_next(sched, ss, sg)) {
        const int64_t row = tile_at<TW, BT>(sched, sg.tile, rank, 0).wrow0 + row_in_tile;
        const bool row_ok = row < w.rows;
        const int64_t rr = row_ok ? row : 0;
        const int sb_lo = sg.kb_lo >> 2, sb_hi = (sg.kb_hi - 1) >> 2;
        dq.prefetch(w, rr, sb_lo);
        for (int sb = sb_lo; sb <= sb_hi && ok; ++sb) {
            const int r = raw_n++;
            const int slot = r % R;
            ok = __all_sync(0xFFFFFFFFu, mbar_wait(raw_full(slot), (r / R) & 1, err));
            if (!ok) break;
            const uint8_t* raw = smem + L::off_raw + slot * L::raw_bytes;
            const uint8_t* raw_row = raw + row_in_tile * (FMT == FMT_Q4K ? 144 : FMT == FMT_Q6K ? 208 : 128);
            dq.begin(raw_row, w, rr, row_ok, sb);
            if (sb < sb_hi) dq.prefetch(w, rr, sb + 1);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kb = 4 * sb + j;
                if (kb < sg.kb_lo || kb >= sg.kb_hi) continue;
                const int my = (it & 1) == grp;
                const int s = it % SA;
                ++it;
                if (!my) continue;
                const int it0 = it - 1;
                if (it0 >= SA) ok = __all_sync(0xFFFFFFFFu, mbar_wait(empty_a(s), ((it0 / SA) - 1) & 1, err));
                if (!ok) break;
                JK_TRACE_POINT(6, it0);
                {
                    SmemRow o{smem + L::off_a + s * A_STAGE_BYTES + row_in_tile * 128, sw};
                    switch (j) {
                    case 0: dq.template kblock<0, 0>(raw_row, row_in_tile, sw, o); dq.template kblock<0, 1>(raw_row, row_in_tile, sw, o); break;
                    case 1: dq.template kblock<1, 0>(raw_row, row_in_tile, sw, o); dq.template kblock<1, 1>(raw_row, row_in_tile, sw, o); break;
                    case 2: dq.template kblock<2, 0>(raw_row, row_in_tile, sw, o); dq.template kblock<2, 1>(raw_row, row_in_tile, sw, o); break;
                    default: dq.template kblock<3, 0>(raw_row, row_in_tile, sw, o); dq.template kblock<3, 1>(raw_row, row_in_tile, sw, o); break;
                    }
                    fence_proxy_async_smem();
                }
                __syncwarp();
                JK_TRACE_POINT(9, it0);
                if (lane == 0) {
                    if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(full_a(s), 0));  // the leader issues the MMA
                    else mbar_arrive(full_a(s));
                }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(raw_empty(slot));
        }
    }
}

// Dequantizer role with tensor-memory A stages (Smem::TMEM_A). A stage is one raw super-block
// (KPS = 4 k-blocks, the stage and raw-ring counters advance together) and the G groups take
// turns: group g decodes the whole stage st with st % G == g (one super-block header decode, one
// raw wait and one empty wait per 4 k-blocks per group) into TMEM lanes of its rows, one
// tcgen05.st of 32 columns per k-block, then arrives once on the stage's full barrier.
template <int FMT, bool BF16, int BT, bool PAIR>
__device__ __forceinline__ void dequant_role_tmem(const Sched& sched, SegState& ss, uint8_t* smem, int row_in_tile,
                                                  int grp, int rank, const WView& w, uint32_t* err, bool& ok,
                                                  uint32_t bar0, int lane, uint32_t tmem) {
    using L = Smem<FMT, BT, PAIR>;
    constexpr int TW = PAIR ? 2 * BW : BW;  // weight rows per tile
    constexpr int S = L::SX, R = L::R, KPS = L::KPS;
    static_assert(KPS == 4, "a stage is one raw super-block");
    constexpr int G = L::DQ_GROUPS;
    auto full = [&](int st) { return bar0 + 8u * (L::bar_full_b + st); };
    auto empty = [&](int st) { return bar0 + 8u * (L::bar_empty_b + st); };
    auto raw_full = [&](int r) { return bar0 + 8u * (L::bar_raw_full + r); };
    auto raw_empty = [&](int r) { return bar0 + 8u * (L::bar_raw_empty + r); };
    const int sw = row_in_tile & 7;
    const uint32_t tlanes = tmem + ((uint32_t)(row_in_tile & ~31) << 16) + L::TMEM_A0;
    SbDequant<FMT, BF16> dq;
    int st = 0;  // stage = raw super-block counter
    Seg sg;
    // Expert-grouped products look the next segment's weight row up (its expert, from the
    // device-side job table) one segment ahead, so the table load of a tile switch overlaps this
    // segment's decode instead of delaying the next tile's first stage. Dense products compute it.
    bool have = seg_next(sched, ss, sg);
    int64_t wrow0 = have && sched.jobs ? tile_at<TW, BT>(sched, sg.tile, rank, 0).wrow0 : 0;
    while (ok && have) {
        Seg sg_n = sg;
        bool have_n = false;
        int64_t wrow0_n = 0;
        if (sched.jobs) {
            have_n = seg_next(sched, ss, sg_n);
            if (have_n) wrow0_n = tile_at<TW, BT>(sched, sg_n.tile, rank, 0).wrow0;
        } else {
            wrow0 = tile_at<TW, BT>(sched, sg.tile, rank, 0).wrow0;
        }
        const int64_t row = wrow0 + row_in_tile;
        const bool row_ok = row < w.rows;
        const int64_t rr = row_ok ? row : 0;
        const int sb_lo = sg.kb_lo >> 2, sb_hi = (sg.kb_hi - 1) >> 2;
        const int first_own = sb_lo + (grp - st % G + G) % G;
        if (first_own <= sb_hi) dq.prefetch(w, rr, first_own);
        for (int sb = sb_lo; sb <= sb_hi && ok; ++sb, ++st) {
            if (st % G != grp) continue;
            const int s = st % S, slot = st % R;
            ok = __all_sync(0xFFFFFFFFu, mbar_wait(raw_full(slot), (st / R) & 1, err));
            if (!ok) break;
            JK_TRACE_POINT(10, st);
            const uint8_t* raw_row = smem + L::off_raw + slot * L::raw_bytes +
                                     row_in_tile * (FMT == FMT_Q4K ? 144 : FMT == FMT_Q6K ? 208 : 128);
            dq.begin(raw_row, w, rr, row_ok, sb);
            if (sb + G <= sb_hi) dq.prefetch(w, rr, sb + G);
            JK_TRACE_POINT(11, st);
            if (st >= S) ok = __all_sync(0xFFFFFFFFu, mbar_wait(empty(s), ((st / S) - 1) & 1, err));
            if (!ok) break;
            JK_TRACE_POINT(6, st);
            tc_fence_after();  // the MMAs that read the stage before have completed
            const int kb_lo = 4 * sb > sg.kb_lo ? 4 * sb : sg.kb_lo;
            const int kb_hi = 4 * sb + 4 < sg.kb_hi ? 4 * sb + 4 : sg.kb_hi;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kb = 4 * sb + j;
                if (kb < kb_lo || kb >= kb_hi) continue;
                RegRow o;
                switch (j) {
                case 0: dq.template kblock<0, 0>(raw_row, row_in_tile, sw, o); dq.template kblock<0, 1>(raw_row, row_in_tile, sw, o); break;
                case 1: dq.template kblock<1, 0>(raw_row, row_in_tile, sw, o); dq.template kblock<1, 1>(raw_row, row_in_tile, sw, o); break;
                case 2: dq.template kblock<2, 0>(raw_row, row_in_tile, sw, o); dq.template kblock<2, 1>(raw_row, row_in_tile, sw, o); break;
                default: dq.template kblock<3, 0>(raw_row, row_in_tile, sw, o); dq.template kblock<3, 1>(raw_row, row_in_tile, sw, o); break;
                }
                tmem_st32(tlanes + (uint32_t)(32 * (KPS * s + j)), o.w);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            JK_TRACE_POINT(9, st);
            if (lane == 0) {
                if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(full(s), 0));  // the leader issues the MMA
                else mbar_arrive(full(s));
                mbar_arrive(raw_empty(slot));
            }
        }
        if (sched.jobs) {
            sg = sg_n;
            wrow0 = wrow0_n;
            have = have_n;
        } else {
            have = seg_next(sched, ss, sg);
        }
    }
}

// PAIR: launched as clusters of 2 CTAs sharing each 256-weight-row tile (tcgen05 cta_group::2).
// Each CTA dequantizes its own 128 weight rows and loads half of the activation rows; the leader
// (cluster rank 0) issues M=256 MMAs that read both CTAs' shared memory and write each CTA's
// 128-row accumulator; completions are committed to both CTAs. Halving the activation bytes each
// SM loads per k-block is the point: at BT=256 those tiles, not the MMAs, bound the main loop.
// MODE: 0 dense product, whole tiles; 1 dense product, stream-K; 2 expert-grouped product, whole
// tiles. Each schedule is its own instantiation, compiled without the other schedules' code paths
// (the whole-tile kernel without them measured 1.7-3 us faster per product at m = 256).
template <int FMT, bool BF16, int BT, bool PAIR, int MODE>
__global__ void __launch_bounds__(Smem<FMT, BT, PAIR>::THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, WView w,
               float* __restrict__ out, int64_t m, int64_t ldo, Sched sched_in, float* __restrict__ ws_part,
               uint32_t* __restrict__ ws_flag, uint32_t* err) {
    // the schedule's mode as compile-time constants: the other modes' branches fold away
    Sched sched = sched_in;
    if constexpr (MODE != 2) sched.jobs = nullptr;
    sched.sk = MODE == 1 ? 1 : 0;
    constexpr bool SK = MODE == 1;
    using L = Smem<FMT, BT, PAIR>;
    constexpr int SX = L::SX, SA = L::SA;
    constexpr bool QUANT = FMT != FMT_F16;
    static_assert(!PAIR || QUANT, "pairs are for quantized weights");
    constexpr int TW = PAIR ? 2 * BW : BW;  // weight rows per tile
    constexpr uint32_t TMEM_COLS = L::TMEM_COLS;
    constexpr uint32_t IDESC = idesc_f16(BF16, TW, BT);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::off_bar;
    auto full_b = [&](int s) { return bar0 + 8u * (L::bar_full_b + s); };
    auto empty_b = [&](int s) { return bar0 + 8u * (L::bar_empty_b + s); };
    auto full_a = [&](int s) { return bar0 + 8u * (L::bar_full_a + s); };
    auto empty_a = [&](int s) { return bar0 + 8u * (L::bar_empty_a + s); };
    constexpr int R = L::R;
    auto raw_full = [&](int r) { return bar0 + 8u * (L::bar_raw_full + r); };
    auto raw_empty = [&](int r) { return bar0 + 8u * (L::bar_raw_empty + r); };
    auto acc_full = [&](int b) { return bar0 + 8u * (L::bar_acc_full + b); };
    auto acc_empty = [&](int b) { return bar0 + 8u * (L::bar_acc_empty + b); };
    auto fix_full = [&](int i) { return bar0 + 8u * (L::bar_fix + i); };
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::off_tmem);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int cta = blockIdx.x;                          // partial-tile slot and flag of this CTA
    const int rank = PAIR ? (int)cluster_ctarank() : 0;  // 128-row half of the pair's weight rows
    const int unit = PAIR ? cta >> 1 : cta;              // schedule unit (CTA or pair)
    auto cid = [&](int u) { return PAIR ? 2 * u + rank : u; };  // CTA of unit u holding our half

    if (threadIdx.x == 0) {
        for (int s = 0; s < SX; ++s) {
            // TMEM_A: the stage's producer arrival (with its bytes) and the warps of the
            // dequantizer group that decodes the stage (in both CTAs of a pair, on the leader's barrier)
            mbar_init(full_b(s), L::TMEM_A ? 1 + 4 * (PAIR ? 2 : 1) : 1);
            mbar_init(empty_b(s), 1);
        }
        for (int s = 0; s < SA; ++s) {
            // one group of dequantizer warps per k-block (in both CTAs of a pair)
            mbar_init(full_a(s), (PAIR ? 2 : 1) * DQ_WARPS / 2);
            mbar_init(empty_a(s), 1);
        }
        for (int r = 0; r < R; ++r) {
            mbar_init(raw_full(r), 1);
            // every dequantizer warp reads each raw super-block, except with TMEM_A stages, where
            // one group decodes it
            mbar_init(raw_empty(r), L::TMEM_A ? 4 : DQ_WARPS);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full(b), 1);
            mbar_init(acc_empty(b), (PAIR ? 2 : 1) * EPI_WARPS);
        }
        for (int i = 0; i < L::FIX_NB; ++i) mbar_init(fix_full(i), 1);
        mbar_fence_init();
    }
    if (warp == MMA_WARP) {
        if constexpr (PAIR) {
            tmem_alloc_pair(smem_u32(tmem_holder), TMEM_COLS);  // both CTAs of the pair, same holder offset
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before any remote arrive or copy
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    JK_TRACE_POINT(14, 0);
    // The next product may start on the SMs this grid frees and fill its pipeline (raw weights,
    // dequantized stages) while this grid's last tiles finish. Everything that reads what the
    // previous kernel on the stream wrote -- the activations (the producer), the grouped job table
    // (every role), the stream-K flags and partials (epilogues, after their MMAs and so after the
    // producer) -- waits for it first; weights are read-only for the whole product.
    gdc_launch();
    if (sched.jobs) {
        gdc_wait();
        // the job count cannot change during the product: one load here instead of one per
        // segment in every role (a dependent load at each tile switch)
        sched.njobs = (int64_t)__ldg(sched.jobs);
    }

    bool ok = true;
    SegState ss;
    seg_init(sched, unit, ss);
    Seg sg;

    // The producer, raw-producer and MMA roles run their loops with the whole warp converged (waits
    // on every lane, warp-uniform addresses and descriptors); one lane issues the TMA copies, the
    // MMAs and the commits.
    const bool leader = lane == 0;
    if (warp == PRODUCER_WARP) {
        // --------------------- activation (and FP16 weight) producer ---------------------
        gdc_wait();  // the activations may come from the previous kernel
        if (leader) {
            tma_prefetch(&tm_x);
            tma_prefetch(&tm_w);
        }
        int it = 0;
        if constexpr (L::TMEM_A) {
            constexpr int KPS = L::KPS;
            while (ok && seg_next(sched, ss, sg)) {
                const int32_t m0 =
                    (int32_t)(tile_at<TW, BT>(sched, sg.tile, rank, m).m0 + (PAIR ? rank * (BT / 2) : 0));
                for (int p = sg.kb_lo / KPS; p <= (sg.kb_hi - 1) / KPS && ok; ++p) {
                    const int s = it % SX;
                    if (it >= SX) ok = __all_sync(0xFFFFFFFFu, mbar_wait(empty_b(s), ((it / SX) - 1) & 1, err));
                    if (!ok) break;
                    JK_TRACE_POINT(1, it);
                    const int lo = p * KPS > sg.kb_lo ? p * KPS : sg.kb_lo;
                    const int hi = p * KPS + KPS < sg.kb_hi ? p * KPS + KPS : sg.kb_hi;
                    if (elect_one()) {
                        if constexpr (PAIR) {
                            // both CTAs' halves count on the leader's barrier; only the leader expects them
                            if (rank == 0) mbar_expect_tx(full_b(s), (uint32_t)(2 * (hi - lo) * L::B_ATOM));
                            const uint32_t lbar = mapa_shared(full_b(s), 0);
                            for (int kb = lo; kb < hi; ++kb)
                                tma_load_2d_pair(sbase + L::off_b + s * L::B_STAGE + (kb % KPS) * L::B_ATOM, &tm_x,
                                                 kb * KB, m0, lbar);
                        } else {
                            mbar_expect_tx(full_b(s), (uint32_t)((hi - lo) * L::B_ATOM));
                            for (int kb = lo; kb < hi; ++kb)
                                tma_load_2d(sbase + L::off_b + s * L::B_STAGE + (kb % KPS) * L::B_ATOM, &tm_x, kb * KB,
                                            m0, full_b(s));
                        }
                    }
                    __syncwarp();
                    ++it;
                }
            }
        } else
        while (ok && seg_next(sched, ss, sg)) {
            const TileAt ta = tile_at<TW, BT>(sched, sg.tile, rank, m);
            const int32_t n0 = (int32_t)ta.wrow0;
            const int32_t m0 = (int32_t)(ta.m0 + (PAIR ? rank * (BT / 2) : 0));
            for (int kb = sg.kb_lo; kb < sg.kb_hi && ok; ++kb) {
                const int s = it % SX;
                if (it >= SX) ok = __all_sync(0xFFFFFFFFu, mbar_wait(empty_b(s), ((it / SX) - 1) & 1, err));
                if (!ok) break;
                JK_TRACE_POINT(1, it);
                if constexpr (PAIR) {
                    // both halves count on the leader's full barrier; only the leader expects them
                    if (elect_one()) {
                        if (rank == 0) mbar_expect_tx(full_b(s), 2 * L::B_STAGE);
                        tma_load_2d_pair(sbase + L::off_b + s * L::B_STAGE, &tm_x, kb * KB, m0,
                                         mapa_shared(full_b(s), 0));
                    }
                } else if (elect_one()) {
                    if constexpr (FMT == FMT_F16) {
                        mbar_expect_tx(full_b(s), L::B_STAGE + A_STAGE_BYTES);
                        tma_load_2d(sbase + L::off_a + s * A_STAGE_BYTES, &tm_w, kb * KB, n0, full_b(s));
                    } else {
                        mbar_expect_tx(full_b(s), L::B_STAGE);
                    }
                    tma_load_2d(sbase + L::off_b + s * L::B_STAGE, &tm_x, kb * KB, m0, full_b(s));
                }
                __syncwarp();
                ++it;
            }
        }
        // drain: every copy this warp issued lands before the CTA may exit (a pair peer's copies
        // complete on the leader's barrier; the final cluster barrier covers them)
        if (!ok && (!PAIR || rank == 0))
            for (int i = it - SX < 0 ? 0 : it - SX; i < it; ++i) mbar_wait(full_b(i % SX), (i / SX) & 1, err);
    } else if (warp == RAW_WARP<L::TMEM_A>) {
        // --------------------- raw weight producer: runs up to R super-blocks ahead ---------------------
        if constexpr (QUANT) {
            int raw_n = 0;
            while (ok && seg_next(sched, ss, sg)) {
                const int32_t n0 = (int32_t)tile_at<TW, BT>(sched, sg.tile, rank, m).wrow0;
                for (int kb = sg.kb_lo; kb < sg.kb_hi && ok; ++kb) {
                    if (kb != sg.kb_lo && (kb & 3) != 0) continue;
                    const int r = raw_n;
                    const int slot = r % R;
                    if (r >= R) ok = __all_sync(0xFFFFFFFFu, mbar_wait(raw_empty(slot), ((r / R) - 1) & 1, err));
                    if (!ok) break;
                    ++raw_n;
                    JK_TRACE_POINT(2, r);
                    const int sb = kb >> 2;
                    const uint32_t dst = sbase + L::off_raw + slot * L::raw_bytes;
                    if (elect_one()) {
                        mbar_expect_tx(raw_full(slot), L::raw_bytes);
                        if constexpr (FMT == FMT_Q4K) {
                            tma_load_2d(dst, &tm_w, sb * 36, n0, raw_full(slot));
                        } else if constexpr (FMT == FMT_Q6K) {
                            tma_load_2d(dst, &tm_w, sb * 52, n0, raw_full(slot));
                        } else if constexpr (FMT == FMT_Q8_0) {
                            tma_load_2d(dst, &tm_w, sb * 256, n0, raw_full(slot));
                            tma_load_2d(dst + BW * 128, &tm_w, sb * 256 + 128, n0, raw_full(slot));
                        } else {
                            tma_load_2d(dst, &tm_w, sb * 128, n0, raw_full(slot));
                        }
                    }
                    __syncwarp();
                }
            }
            if (!ok)
                for (int r = raw_n - R < 0 ? 0 : raw_n - R; r < raw_n; ++r) mbar_wait(raw_full(r % R), (r / R) & 1, err);
        }
    } else if (warp == MMA_WARP && (!PAIR || rank == 0)) {
        // ------------------------------ MMA issuer (a pair's leader only) ------------------------------
        int it = 0, seg_i = 0;
        bool issued = false;
        auto commit = [&](uint32_t bar) {  // arrives once the MMAs issued so far complete
            if constexpr (PAIR) mma_commit_pair(bar);
            else mma_commit(bar);
        };
        constexpr int NACC = L::NACC;
        while (ok && seg_next(sched, ss, sg)) {
            const int b = seg_i % NACC;
            if (seg_i >= NACC) ok = __all_sync(0xFFFFFFFFu, mbar_wait(acc_empty(b), ((seg_i / NACC) - 1) & 1, err));
            if (!ok) break;
            tc_fence_after();
            const uint32_t acc = tmem + (uint32_t)(b * BT);
            if constexpr (L::TMEM_A) {
                // one wait and one commit per stage of KPS k-blocks; A from tensor memory (8 columns
                // = 16 values per lane per K=16 step), B from the stage's activation atoms
                constexpr int KPS = L::KPS;
                for (int p = sg.kb_lo / KPS; p <= (sg.kb_hi - 1) / KPS; ++p) {
                    const int s = it % SX;
                    JK_TRACE_POINT(2, it);
                    // (a pair's stage is complete when the other CTA's dequantizers have arrived too)
                    ok = __all_sync(0xFFFFFFFFu, PAIR ? mbar_wait_cluster(full_b(s), (uint32_t)((it / SX) & 1), err)
                                                      : mbar_wait(full_b(s), (uint32_t)((it / SX) & 1), err));
                    if (!ok) break;
                    JK_TRACE_POINT(4, it);
                    tc_fence_after();
                    // Operands are computed by the whole (converged) warp and one elected lane issues:
                    // warp-uniform descriptors let the MMAs go out back to back (from a lane-0 branch
                    // each MMA costs about twice its tensor-pipe time at N = 32).
                    const uint32_t at = tmem + L::TMEM_A0 + (uint32_t)(32 * KPS * s);
                    const uint64_t bd = sw128_kmajor_desc(sbase + L::off_b + s * L::B_STAGE);
                    if (elect_one()) {
#pragma unroll
                        for (int j = 0; j < KPS; ++j) {
                            const int kb = p * KPS + j;
                            if (kb < sg.kb_lo || kb >= sg.kb_hi) continue;
#pragma unroll
                            for (int k = 0; k < KB / 16; ++k) {
                                const uint32_t a_k = at + (uint32_t)(32 * j + 8 * k);
                                const uint64_t b_k = bd + (uint64_t)(j * (L::B_ATOM >> 4) + 2 * k);
                                const uint32_t accum = (kb > sg.kb_lo || k > 0) ? 1u : 0u;
                                if constexpr (PAIR) mma_f16_ta_pair(acc, a_k, b_k, IDESC, accum);
                                else mma_f16_ta(acc, a_k, b_k, IDESC, accum);
                            }
                        }
                        JK_TRACE_POINT(0, it);
                        commit(empty_b(s));
                    }
                    __syncwarp();
                    issued = true;
                    ++it;
                }
            } else
            // k-blocks go to the tensor pipe MMA_BATCH at a time: the waits, commits and loop
            // overhead of a batch are paid once while the previous batch's MMAs execute
            for (int kb = sg.kb_lo; kb < sg.kb_hi;) {
                const int nb = kb + MMA_BATCH <= sg.kb_hi ? MMA_BATCH : sg.kb_hi - kb;
                JK_TRACE_POINT(2, it);
                bool got = true;
#pragma unroll
                for (int q = 0; q < MMA_BATCH; ++q) {
                    if (q < nb && got) got = mbar_wait(full_b((it + q) % SX), (uint32_t)(((it + q) / SX) & 1), err);
                    if (q < nb && got && QUANT) got = mbar_wait(full_a((it + q) % SA), (uint32_t)(((it + q) / SA) & 1), err);
                }
                ok = __all_sync(0xFFFFFFFFu, got);
                if (!ok) break;
                JK_TRACE_POINT(4, it);
                tc_fence_after();
                uint64_t bdq[MMA_BATCH], adq[MMA_BATCH];
#pragma unroll
                for (int q = 0; q < MMA_BATCH; ++q) {
                    bdq[q] = sw128_kmajor_desc(sbase + L::off_b + ((it + q) % SX) * L::B_STAGE);
                    adq[q] = sw128_kmajor_desc(sbase + L::off_a + ((it + q) % SA) * A_STAGE_BYTES);
                }
                if (elect_one()) {
#pragma unroll
                    for (int q = 0; q < MMA_BATCH; ++q) {
                        if (q >= nb) break;
                        const uint64_t bd = bdq[q], ad = adq[q];
#pragma unroll
                        for (int k = 0; k < KB / 16; ++k) {  // +32 bytes per K=16 step inside the swizzle atom
                            const uint32_t accum = (kb + q > sg.kb_lo || k > 0) ? 1u : 0u;
                            if constexpr (PAIR)
                                mma_f16_pair(acc, ad + 2u * k, bd + 2u * k, IDESC, accum);
                            else
                                mma_f16(acc, ad + 2u * k, bd + 2u * k, IDESC, accum);
                        }
                    }
                    JK_TRACE_POINT(0, it);
#pragma unroll
                    for (int q = 0; q < MMA_BATCH; ++q) {
                        if (q >= nb) break;
                        commit(empty_b((it + q) % SX));
                        if constexpr (QUANT) commit(empty_a((it + q) % SA));
                    }
                    JK_TRACE_POINT(1, it);
                }
                __syncwarp();
                issued = true;
                kb += nb;
                it += nb;
            }
            if (!ok) break;
            if (elect_one()) commit(acc_full(b));  // arrives when this segment's MMAs are complete
            __syncwarp();
            JK_TRACE_POINT(12, seg_i);
            ++seg_i;
        }
        if (!ok && issued) {
            // Error path: drain the MMAs issued so far before TMEM is released. The commit arrives on
            // acc_full(b) of the unfinished segment; wait for it.
            const int b = seg_i % NACC;
            if (leader) commit(acc_full(b));
            __syncwarp();
            mbar_wait(acc_full(b), (seg_i / NACC) & 1, err);
        }
    } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + EPI_WARPS) {
        // ------------------------------ epilogue ------------------------------
        const int quarter = warp & 3;                 // TMEM lanes this warp may read
        const int row_in_tile = 32 * quarter + lane;  // weight row within the tile
        const bool issuer = threadIdx.x == 32 * EPI_WARP0;
        // output rows are 16-byte aligned: the staged epilogue writes them with 16-byte stores
        const bool vec_out = ((reinterpret_cast<uintptr_t>(out) | (uintptr_t)(ldo * 4)) & 15) == 0;
        __shared__ int fix_bad;
        int seg_i = 0;
        int fix_q = 0;  // fix-up chunks consumed so far (ring parity)
        while (ok && seg_next(sched, ss, sg)) {
            const int b = seg_i % L::NACC;
            ok = __all_sync(0xFFFFFFFFu, mbar_wait_sleepy(acc_full(b), (seg_i / L::NACC) & 1, err));
            tc_fence_after();
            if (!ok) break;
            JK_TRACE_POINT(7, seg_i);
            const TileAt ta = tile_at<TW, BT>(sched, sg.tile, rank, m);
            const int64_t n0 = ta.col0;  // output column of TMEM lane 0 (dense: also its weight row)
            const int64_t m0 = ta.m0;
            const int64_t wrow = n0 + row_in_tile;
            const bool contributor = SK && sg.kb_lo > 0;
            const bool owner = SK && sg.kb_lo == 0 && sg.kb_hi < sched.kbt;
            // contributors of an owned tile: the following units whose ranges start inside it (a
            // pair CTA combines with the same-rank CTA of each contributing pair)
            int u_last = unit;
            if (owner) {
                const int64_t tile_end = (sg.tile + 1) * sched.kbt;
                while (u_last + 1 < sched.G && sk_start(sched, u_last + 1) < tile_end) ++u_last;
                __shared__ int flags_ok;
                if (threadIdx.x == 32 * EPI_WARP0) {
                    bool good = true;
                    for (int u = unit + 1; u <= u_last && good; ++u) {
                        const int c = cid(u);
                        const uint64_t t0 = globaltimer();
                        while (ld_acquire(ws_flag + c) == 0u) {
                            if (globaltimer() - t0 > WAIT_LIMIT_NS) {
                                atomicOr(err, ERR_WAIT_TIMEOUT);
                                good = false;
                                break;
                            }
                        }
                    }
                    flags_ok = good ? 1 : 0;
                }
                epi_bar();
                ok = flags_ok != 0;
                JK_TRACE_POINT(10, seg_i);
            }
            if (ok) {
                const uint32_t tbase = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(b * BT);
                // CH columns per round: all TMEM loads of the round are issued before one wait, and an
                // owner loads all contributor partials of the round before adding them.
                constexpr int CH = L::FIX_CH;
                // Owner of the CTA's last segment: the contributor partials arrive in shared memory by
                // bulk copies (round-major, contributor-minor chunks through a FIX_NB ring) instead of
                // per-thread loads, so a whole ring of them is in flight at once.
                const int nc = u_last - unit;
                const bool bulk_fix = owner && nc > 0 && ss.next >= ss.end;
                // The CTA's last tile: the pipeline's shared memory is idle, so the output rows are
                // staged there and written whole, 16 bytes per thread and store (per-element column
                // stores of a 128 x 128 f32 tile took ~6 us on the exposed tail of a product; bulk
                // row copies from shared memory ~3 us, and they held the CTA until they had read
                // it; thread stores let the CTA leave as soon as they are issued, 0.3-1.3 us less
                // per product).
                const bool staged = !contributor && vec_out && !sched.jobs && ss.next >= ss.end;
                const int nchunks = bulk_fix ? (BT / CH) * nc : 0;
                auto issue_chunk = [&](int q) {
                    const int r = q / nc, ci = q - r * nc;
                    const int g = fix_q + q, buf = g % L::FIX_NB;
                    const float* src = ws_part + (int64_t)cid(unit + 1 + ci) * BT * BW + (int64_t)(r * CH) * BW;
                    mbar_expect_tx(fix_full(buf), (uint32_t)L::FIX_CHUNK);
                    bulk_g2s(sbase + (uint32_t)(buf * L::FIX_CHUNK), src, (uint32_t)L::FIX_CHUNK, fix_full(buf));
                };
                int issued_q = 0;
                bool dead = false;
                if (bulk_fix) {
                    if (issuer) {
                        fix_bad = 0;
                        fence_proxy_async_smem();
                        for (; issued_q < nchunks && issued_q < L::FIX_NB; ++issued_q) issue_chunk(issued_q);
                    }
                }
#pragma unroll 1
                for (int c0 = 0; c0 < BT; c0 += CH) {
                    uint32_t v[CH];
#pragma unroll
                    for (int q = 0; q < CH / 16; ++q) {
                        uint32_t (&vq)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[16 * q]);
                        tmem_ld16(tbase + (uint32_t)(c0 + 16 * q), vq);
                    }
                    tmem_ld_wait();
                    JK_TRACE_POINT(5, c0 / CH);
                    if (contributor) {
                        float* slot = ws_part + (int64_t)cta * BT * BW + (int64_t)c0 * BW + row_in_tile;
#pragma unroll
                        for (int j = 0; j < CH; ++j) slot[j * BW] = __uint_as_float(v[j]);
                    } else {
                        float acc[CH];
#pragma unroll
                        for (int j = 0; j < CH; ++j) acc[j] = __uint_as_float(v[j]);
                        if (bulk_fix) {
                            for (int ci = 0; ci < nc; ++ci) {
                                const int q = (c0 / CH) * nc + ci;
                                const int g = fix_q + q, buf = g % L::FIX_NB;
                                if (!dead) dead = !mbar_wait(fix_full(buf), (uint32_t)((g / L::FIX_NB) & 1), err);
                                if (!dead) {
                                    const float* sp = reinterpret_cast<const float*>(smem + buf * L::FIX_CHUNK) + row_in_tile;
#pragma unroll
                                    for (int j = 0; j < CH; ++j) acc[j] += sp[j * BW];
                                }
                                epi_bar();  // every reader is done with this buffer
                                if (issuer && !dead && issued_q < nchunks) {
                                    fence_proxy_async_smem();
                                    issue_chunk(issued_q++);
                                }
                            }
                        } else {
                            for (int u = unit + 1; u <= u_last; ++u) {
                                const float* slot = ws_part + (int64_t)cid(u) * BT * BW + (int64_t)c0 * BW + row_in_tile;
                                float p[CH];
#pragma unroll
                                for (int j = 0; j < CH; ++j) p[j] = __ldcg(slot + j * BW);
#pragma unroll
                                for (int j = 0; j < CH; ++j) acc[j] += p[j];
                            }
                        }
                        JK_TRACE_POINT(13, c0 / CH);
                        if (staged) {
                            // stage the round as [row of out][BW]; the two staging buffers alternate
                            // between rounds
                            float* tp = reinterpret_cast<float*>(smem + L::off_fix_out + ((c0 / CH) & 1) * L::FIX_CHUNK);
                            // the threads read the buffer back themselves (synchronously) and post
                            // 16-byte global stores: nothing outlives the CTA's shared memory, so
                            // the CTA leaves once its stores are issued
#pragma unroll
                            for (int j = 0; j < CH; ++j) tp[j * BW + row_in_tile] = acc[j];
                            epi_bar();
                            const int64_t cols = w.rows - n0 < BW ? w.rows - n0 : BW;
                            const int64_t mleft = m - (m0 + c0);
                            const int nrows = mleft < CH ? (int)mleft : CH;
                            for (int idx = row_in_tile; idx < nrows * (BW / 4); idx += EPI_THREADS) {
                                const int j = idx / (BW / 4), c = idx % (BW / 4);
                                if (4 * c < cols)
                                    *reinterpret_cast<float4*>(out + (m0 + c0 + j) * ldo + n0 + 4 * c) =
                                        *reinterpret_cast<const float4*>(tp + j * BW + 4 * c);
                            }
                        } else if (!sched.jobs) {
                            if (wrow < w.rows) {
                                float* o = out + (m0 + c0) * ldo + wrow;
                                const int64_t mleft = m - (m0 + c0);
#pragma unroll
                                for (int j = 0; j < CH; ++j)
                                    if (j < mleft) o[j * ldo] = acc[j];
                            }
                        } else if (wrow < sched.n_exp) {
                            // grouped: sorted row s goes to output row sorted[s] (its assignment)
                            const int64_t mleft = ta.mend - (m0 + c0);
                            const uint32_t* srow = sched.sorted + m0 + c0;
#pragma unroll
                            for (int j = 0; j < CH; ++j)
                                if (j < mleft) out[(int64_t)__ldg(srow + j) * ldo + wrow] = acc[j];
                        }
                    }
                }
                if (bulk_fix) {
                    if (dead) atomicOr(&fix_bad, 1);
                    epi_bar();
                    if (fix_bad) {
                        ok = false;
                        // a chunk never arrived: give the copies still in flight a bounded wait
                        if (issuer)
                            for (int q = 0; q < issued_q; ++q) {
                                const int g = fix_q + q;
                                (void)mbar_wait(fix_full(g % L::FIX_NB), (uint32_t)((g / L::FIX_NB) & 1), err);
                            }
                    }
                    fix_q += nchunks;
                }
                JK_TRACE_POINT(11, seg_i);
                if (contributor) {
                    // every partial store of the tile precedes the barrier; the flag writer's
                    // gpu-scope release store then publishes them all (cumulativity through
                    // bar.sync; a full fence before it measured 0.4 us slower per product)
                    epi_bar();
                    if (issuer) st_release(ws_flag + cta, 1u);
                } else if (owner) {
                    epi_bar();  // all partial reads done: clear the flags for the next launch
                    if (threadIdx.x == 32 * EPI_WARP0)
                        for (int u = unit + 1; u <= u_last; ++u) ws_flag[cid(u)] = 0u;
                }
            }
            tc_fence_before();
            __syncwarp();
            JK_TRACE_POINT(8, seg_i);
            if (lane == 0) {  // the MMA issuer (a pair's leader) may overwrite this accumulator
                if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(acc_empty(b), 0));
                else mbar_arrive(acc_empty(b));
            }
            ++seg_i;
        }
    } else if (dq_slot<L::TMEM_A>(warp) >= 0) {
        // ------------------------------ dequantizers ------------------------------
        if constexpr (QUANT) {
            const int t = 32 * dq_slot<L::TMEM_A>(warp) + lane;  // 0..255
            const int row_in_tile = t & (BW - 1);
            if constexpr (L::TMEM_A)
                dequant_role_tmem<FMT, BF16, BT, PAIR>(sched, ss, smem, row_in_tile, t / BW, rank, w, err, ok, bar0, lane,
                                                       tmem);
            else
                dequant_role<FMT, BF16, BT, PAIR>(sched, ss, smem, row_in_tile, t / BW, rank, w, err, ok, bar0, lane);
        }
    }

    tc_fence_before();
    __syncthreads();
    // a pair CTA may still receive the peer's arrives and have its shared memory read by the
    // leader's MMAs until both are here
    if constexpr (PAIR) cluster_sync();
    JK_TRACE_POINT(15, 0);
    if (warp == MMA_WARP) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem, TMEM_COLS);
        else tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Shared-memory opt-in and CTAs per SM, once per (kernel instantiation, device): `cache` must be
// a static of the instantiation's own launcher (all instantiations share one function type).
template <class K>
int prepare_kernel(K kern, int smem, int threads, int device, int (&cache)[64]) {
    if (device < 0 || device >= 64) return -1;
    if (cache[device] == 0) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -1;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
            return -1;
        cache[device] = per_sm;
    }
    return cache[device];
}


template <int FMT, bool BF16, int BT, bool PAIR, int MODE>
jk_status launch_tc_k(const LaunchArgs& a) {
    using L = Smem<FMT, BT, PAIR>;
    auto kern = gemm_tc_kernel<FMT, BF16, BT, PAIR, MODE>;
    constexpr int TW = PAIR ? 2 * BW : BW;
    int dev = 0;
    cudaGetDevice(&dev);
    static int per_sm_cache[64] = {};
    const int per_sm = prepare_kernel(kern, L::total, L::THREADS, dev, per_sm_cache);
    if (per_sm < 0) return cuda_fail(cudaGetLastError(), "gemm kernel attributes");
    const WView& w = a.wq->view;
    Sched s{};
    if (a.jobs) {
        s.tiles_m = (int)a.max_jobs;
        s.tiles = ((a.n_exp + TW - 1) / TW) * s.tiles_m;
        s.jobs = a.jobs;
        s.offsets = a.offsets;
        s.sorted = a.sorted;
        s.n_exp = a.n_exp;
        s.job_rows = a.job_rows;
    } else {
        s.tiles_m = (int)((a.m + BT - 1) / BT);
        s.tiles = ((w.rows + TW - 1) / TW) * s.tiles_m;
    }
    s.kbt = (int)(w.k / KB);
    s.sk = a.stream_k ? 1 : 0;
    const int64_t work = s.sk ? s.tiles * s.kbt : s.tiles;
    if constexpr (PAIR) {
        cudaLaunchConfig_t cfg = {};
        cfg.blockDim = dim3(L::THREADS);
        cfg.dynamicSmemBytes = L::total;
        cfg.stream = a.stream;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        // pairs that can be resident at once (a GPC with an odd SM count leaves one SM unpaired)
        static int pairs_cache[64] = {};
        if (dev < 0 || dev >= 64) return fail(JK_ERR_INVALID, "device index out of range");
        if (!pairs_cache[dev]) {
            cfg.gridDim = dim3(2 * ((unsigned)sm_count(dev) / 2));
            int clusters = 0;
            cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
            if (e != cudaSuccess) return cuda_fail(e, "gemm pair occupancy");
            if (clusters < 1) return fail(JK_ERR_UNSUPPORTED, "gemm: no CTA pair fits on this device");
            pairs_cache[dev] = clusters;
        }
        int64_t g = pairs_cache[dev];
        const int64_t budget = sm_budget(dev) / 2;
        if (g > budget) g = budget;
        if (a.grid_cap > 0 && 2 * g > a.grid_cap) g = a.grid_cap / 2;
        if (g > work) g = work;
        if (g < 1) g = 1;
        s.G = (int)g;
        cfg.gridDim = dim3(2 * (unsigned)s.G);
        // programmatic dependent launch, as for single CTAs: the next product's pairs start on the
        // SMs this grid frees and fill their weight stages while its last tiles finish
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 2;
        cudaError_t e = cudaLaunchKernelEx(&cfg, kern, *a.tm_x, a.wq->tm_w, w, a.out, a.m, a.ldo, s, a.ws_part,
                                           a.ws_flag, device_error_word(a.wq->device));
        if (e != cudaSuccess) return cuda_fail(e, "gemm pair launch");
        return cuda_fail(cudaGetLastError(), "gemm pair launch");
    } else {
        int64_t g = (int64_t)sm_budget(dev) * per_sm;
        if (a.grid_cap > 0 && g > a.grid_cap) g = a.grid_cap;
        if (g > work) g = work;
        s.G = (int)g;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)s.G);
        cfg.blockDim = dim3(L::THREADS);
        cfg.dynamicSmemBytes = L::total;
        cfg.stream = a.stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, kern, *a.tm_x, a.wq->tm_w, w, a.out, a.m, a.ldo, s, a.ws_part,
                                           a.ws_flag, device_error_word(a.wq->device));
        if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
        return cuda_fail(cudaGetLastError(), "gemm launch");
    }
}

template <int FMT, bool BF16, int BT, bool PAIR>
jk_status launch_tc(const LaunchArgs& a) {
    if (a.jobs) return launch_tc_k<FMT, BF16, BT, PAIR, 2>(a);
    return a.stream_k ? launch_tc_k<FMT, BF16, BT, PAIR, 1>(a) : launch_tc_k<FMT, BF16, BT, PAIR, 0>(a);
}

template <int FMT, bool BF16>
jk_status launch_tc_bt(const LaunchArgs& a, int bt) {
    if constexpr (FMT != FMT_F16) {
        if (a.pair) {
            if (bt == 128) return launch_tc<FMT, BF16, 128, true>(a);
            if (bt == 256) return launch_tc<FMT, BF16, 256, true>(a);
        }
    }
    switch (bt) {
    case 32: return launch_tc<FMT, BF16, 32, false>(a);
    case 64: return launch_tc<FMT, BF16, 64, false>(a);
    case 96: return launch_tc<FMT, BF16, 96, false>(a);
    case 128: return launch_tc<FMT, BF16, 128, false>(a);
    default: return launch_tc<FMT, BF16, 256, false>(a);
    }
}

}  // namespace tc
}  // namespace jk
