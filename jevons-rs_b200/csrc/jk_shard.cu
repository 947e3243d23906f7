// jk_shard.cu -- the column-sharded product with its f32 output all-gathered over NVLink
// (jk_sharded_matmul_allgather), and the inter-process buffer plumbing it runs on (jk_ipc_*).
//
// The reference runs on one GPU; its large-N projections (the vocabulary head, the FFN up
// projection) split by output column because a super-block never spans weight rows. Here rank r
// of `world` holds weight rows [r n_r, (r+1) n_r) and every rank ends with the whole output in a
// rank-major buffer [world][m][n_r] (rank p's columns are rows [p m, (p+1) m) of it).
//
// B200 design: the exchange uses the copy engines, not SMs. The persistent tensor-core product
// holds every SM, so a collective kernel (NCCL's all-gather) can only run between products; copy
// engines push each finished row chunk of this rank's shard straight into every peer's buffer
// (cudaMemcpyAsync to peer memory mapped with CUDA IPC, NSUB copy streams per peer) while the next
// chunk's product runs. The copy streams carry copies only: a kernel there would wait for an SM
// the persistent products hold. A wait (jk_allgather_wait, or a call with wait != 0) then
// increments this rank's counter word in every peer (flags[rank] += 1, a system-scope release
// reduction by a one-thread kernel ordered after all copies issued to that peer since the last
// wait) and polls its own flags: each rank's own slot flags[rank] counts the waits it has done,
// and the wait kernel (one warp) waits with system-scope acquires until every peer's counter
// reaches flags[rank] + 1, then advances flags[rank]. The counters live on the device, so a CUDA
// graph that replays a captured step stays in step with the peers (no host-side epoch is baked
// into the graph). Every wait is bounded (2 s):
// on expiry the kernel records ERR_WAIT_TIMEOUT in the device error word and returns, so a rank
// that never arrives surfaces as an error instead of a hung GPU.
#include "jk_internal.h"

#include <cstdio>
#include <cstring>
#include <mutex>

namespace jk {
namespace {

constexpr int MAX_WORLD = 8;
constexpr int MAX_CHUNKS = 16;
// Copy streams per peer: one copy engine moves a few-MB peer copy at a fraction of the link rate,
// so each chunk's copy to a peer is split in NSUB row ranges on NSUB streams (engines).
constexpr int NSUB = 4;
constexpr uint64_t FLAG_WAIT_NS = 2000000000ull;  // 2 s

// peer_flags[rank] += 1 in a peer's flag array, after this stream's copies to that peer
__global__ void signal_peer_kernel(uint32_t* word) {
    if (threadIdx.x == 0) {
        __threadfence_system();
        asm volatile("red.release.sys.global.add.u32 [%0], 1;" :: "l"(word) : "memory");
    }
}

// Waits until flags[p] >= flags[rank] + 1 for every peer p (each peer's counter of signals), then
// advances flags[rank], this rank's count of waits. One warp, lane p polls peer p.
__global__ void wait_peers_kernel(uint32_t* flags, int world, int rank, uint32_t* err) {
    const int p = threadIdx.x;
    const uint32_t target = flags[rank] + 1;  // only this rank writes its own slot
    bool ok = true;
    if (p < world && p != rank) {
        const uint64_t t0 = globaltimer();
        for (uint32_t i = 0;; ++i) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + p) : "memory");
            if ((int32_t)(v - target) >= 0) break;
            if ((i & 255u) == 255u && globaltimer() - t0 > FLAG_WAIT_NS) {
                ok = false;
                break;
            }
            __nanosleep(128);
        }
    }
    if (!ok) atomicOr(err, ERR_WAIT_TIMEOUT);
    __syncwarp();
    if (p == 0) flags[rank] = target;
}

// Copy streams (NSUB per peer) and events, created once per device.
// Copy of this rank's rows [r0, r1) of its shard into every peer's gathered buffer by the SMs
// (16-byte loads and peer stores over NVLink): grid.y = peer index (this rank skipped).
struct PeerRows {
    float4* d[MAX_WORLD];
};
__global__ void __launch_bounds__(256) push_rows_kernel(const float4* __restrict__ src, PeerRows dst, int rank,
                                                        size_t n4) {
    const int p = (int)blockIdx.y < rank ? (int)blockIdx.y : (int)blockIdx.y + 1;
    float4* __restrict__ d = dst.d[p];
    for (size_t i = (size_t)blockIdx.x * 256 + threadIdx.x; i < n4; i += (size_t)gridDim.x * 256) d[i] = src[i];
}

struct ShardState {
    bool ready = false;
    cudaStream_t cs[MAX_WORLD][NSUB] = {};
    cudaEvent_t sub[MAX_WORLD][NSUB] = {};
    cudaEvent_t chunk[MAX_CHUNKS] = {};
    cudaEvent_t done[MAX_WORLD] = {};
    cudaEvent_t pushed = {};
};

jk_status shard_state(int device, ShardState** out) {
    static std::mutex mu;
    static ShardState st[64];
    if (device < 0 || device >= 64) return fail(JK_ERR_INVALID, "device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    ShardState& s = st[device];
    if (!s.ready) {
        if (cudaEventCreateWithFlags(&s.pushed, cudaEventDisableTiming) != cudaSuccess)
            return cuda_fail(cudaGetLastError(), "sharded product: event set-up");
        for (int p = 0; p < MAX_WORLD; ++p) {
            cudaError_t e = cudaEventCreateWithFlags(&s.done[p], cudaEventDisableTiming);
            for (int q = 0; q < NSUB && e == cudaSuccess; ++q) {
                e = cudaStreamCreateWithFlags(&s.cs[p][q], cudaStreamNonBlocking);
                if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.sub[p][q], cudaEventDisableTiming);
            }
            if (e != cudaSuccess) return cuda_fail(e, "sharded product: copy stream set-up");
        }
        for (int i = 0; i < MAX_CHUNKS; ++i) {
            cudaError_t e = cudaEventCreateWithFlags(&s.chunk[i], cudaEventDisableTiming);
            if (e != cudaSuccess) return cuda_fail(e, "sharded product: event set-up");
        }
        s.ready = true;
    }
    *out = &s;
    return JK_OK;
}

size_t dtype_bytes(int dt) { return dt == JK_DTYPE_F32 ? 4 : 2; }

}  // namespace
}  // namespace jk

using jk::fail;

extern "C" jk_status jk_ipc_alloc(int device, size_t bytes, void** dev_ptr, uint8_t handle[64]) {
    if (!dev_ptr || !handle || bytes == 0) return fail(JK_ERR_INVALID, "ipc alloc: null pointer or zero size");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
    jk::DeviceGuard g(device);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return jk::cuda_fail(e, "ipc alloc");
    }
    memcpy(handle, &h, 64);
    *dev_ptr = p;
    return JK_OK;
}

extern "C" jk_status jk_ipc_free(int device, void* dev_ptr) {
    if (!dev_ptr) return JK_OK;
    jk::DeviceGuard g(device);
    return jk::cuda_fail(cudaFree(dev_ptr), "ipc free");
}

extern "C" jk_status jk_ipc_open(int device, const uint8_t handle[64], void** dev_ptr) {
    if (!handle || !dev_ptr) return fail(JK_ERR_INVALID, "ipc open: null pointer");
    jk::DeviceGuard g(device);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, 64);
    return jk::cuda_fail(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "ipc open");
}

extern "C" jk_status jk_ipc_close(int device, void* dev_ptr) {
    if (!dev_ptr) return JK_OK;
    jk::DeviceGuard g(device);
    return jk::cuda_fail(cudaIpcCloseMemHandle(dev_ptr), "ipc close");
}

extern "C" jk_status jk_allgather_wait(int device, uint32_t* const* flags_peers, int world, int rank, void* stream) {
    if (world < 1 || world > jk::MAX_WORLD || rank < 0 || rank >= world)
        return fail(JK_ERR_INVALID, "allgather wait: rank / world out of range (world <= 8)");
    if (world == 1) return JK_OK;
    if (!flags_peers) return fail(JK_ERR_INVALID, "allgather wait: null flag table");
    for (int p = 0; p < world; ++p)
        if (!flags_peers[p]) return fail(JK_ERR_INVALID, "allgather wait: null flags");
    jk::DeviceGuard g(device);
    jk::ShardState* ss = nullptr;
    jk_status st = jk::shard_state(device, &ss);
    if (st != JK_OK) return st;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    for (int p = 0; p < world; ++p) {
        if (p == rank) continue;
        // peer p's first copy stream joins the others; after every copy issued to p since the last
        // wait: flags_peers[p][rank] += 1; then `stream` joins that stream
        cudaError_t e = cudaSuccess;
        for (int q = 1; q < jk::NSUB && e == cudaSuccess; ++q) {
            e = cudaEventRecord(ss->sub[p][q], ss->cs[p][q]);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(ss->cs[p][0], ss->sub[p][q], 0);
        }
        if (e == cudaSuccess) {
            jk::signal_peer_kernel<<<1, 32, 0, ss->cs[p][0]>>>(flags_peers[p] + rank);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaEventRecord(ss->done[p], ss->cs[p][0]);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, ss->done[p], 0);
        if (e != cudaSuccess) return jk::cuda_fail(e, "allgather wait: signal peers");
    }
    jk::wait_peers_kernel<<<1, 32, 0, cs>>>(flags_peers[rank], world, rank, jk::device_error_word(device));
    return jk::cuda_fail(cudaGetLastError(), "allgather wait launch");
}

extern "C" jk_status jk_sharded_matmul_allgather(const jk_qmatrix* w_shard, const void* x, int x_dtype, size_t x_len,
                                                 size_t m, int rank, int world, float* const* out_peers,
                                                 uint32_t* const* flags_peers, int chunks, int wait,
                                                 jk_split_scratch* scratch, void* stream) {
    if (!w_shard) return fail(JK_ERR_INVALID, "null matrix");
    if (world < 1 || world > jk::MAX_WORLD || rank < 0 || rank >= world)
        return fail(JK_ERR_INVALID, "sharded product: rank / world out of range (world <= 8)");
    if (chunks < 1 || chunks > jk::MAX_CHUNKS) return fail(JK_ERR_INVALID, "sharded product: chunks must be 1..16");
    if (!out_peers || !flags_peers) return fail(JK_ERR_INVALID, "sharded product: null peer tables");
    for (int p = 0; p < world; ++p)
        if (!out_peers[p] || !flags_peers[p]) return fail(JK_ERR_INVALID, "sharded product: null peer buffer");
    if (x_dtype != JK_DTYPE_F32 && x_dtype != JK_DTYPE_F16 && x_dtype != JK_DTYPE_BF16)
        return fail(JK_ERR_INVALID, "unknown activation dtype");
    if (m > (size_t)INT32_MAX) return fail(JK_ERR_INVALID, "m too large");
    const size_t n_r = w_shard->n, k = w_shard->k;
    if (x_len < m * k) return fail(JK_ERR_INVALID, "sharded product: activation buffer too small");
    if (m == 0) return JK_OK;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    jk::DeviceGuard dg(w_shard->device);
    jk::ShardState* ss = nullptr;
    jk_status st = jk::shard_state(w_shard->device, &ss);
    if (st != JK_OK) return st;
    // row chunks: multiples of 32 rows (the smallest row tile), as even as possible
    const size_t unit = 32, units = (m + unit - 1) / unit;
    const int nchunk = (int)(units < (size_t)chunks ? units : (size_t)chunks);
    const size_t esz = jk::dtype_bytes(x_dtype);
    float* mine = out_peers[rank] + (size_t)rank * m * n_r;
    // With 4 or more chunks the last quarter of them is pushed by the SMs once the products are
    // done: the copy engines are still busy with the earlier chunks then, and the SMs are idle.
    const int n_sm = world > 1 && nchunk >= 4 ? nchunk / 4 : 0;
    size_t r_sm = m;  // first row pushed by the SMs
    for (int i = 0; i < nchunk; ++i) {
        const size_t r0 = (size_t)i * units / nchunk * unit, r1e = (size_t)(i + 1) * units / nchunk * unit;
        const size_t r1 = r1e < m ? r1e : m;
        if (r1 <= r0) continue;
        const size_t rows = r1 - r0;
        st = jk_matmul(w_shard, static_cast<const char*>(x) + r0 * k * esz, x_dtype, rows * k, rows, mine + r0 * n_r,
                       rows * n_r, scratch, stream);
        if (st != JK_OK) return st;
        if (world == 1) continue;
        if (i >= nchunk - n_sm) {
            if (r0 < r_sm) r_sm = r0;
            continue;
        }
        cudaError_t e = cudaEventRecord(ss->chunk[i], cs);
        for (int p = 0; p < world && e == cudaSuccess; ++p) {
            if (p == rank) continue;
            for (int q = 0; q < jk::NSUB && e == cudaSuccess; ++q) {
                const size_t q0 = r0 + rows * q / jk::NSUB, q1 = r0 + rows * (q + 1) / jk::NSUB;
                if (q1 <= q0) continue;
                e = cudaStreamWaitEvent(ss->cs[p][q], ss->chunk[i], 0);
                if (e == cudaSuccess)
                    e = cudaMemcpyAsync(out_peers[p] + (size_t)rank * m * n_r + q0 * n_r, mine + q0 * n_r,
                                        (q1 - q0) * n_r * 4, cudaMemcpyDeviceToDevice, ss->cs[p][q]);
            }
        }
        if (e != cudaSuccess) return jk::cuda_fail(e, "sharded product: chunk copies");
    }
    if (world == 1) return JK_OK;
    if (r_sm < m) {
        jk::PeerRows pr{};
        for (int p = 0; p < world; ++p)
            pr.d[p] = reinterpret_cast<float4*>(out_peers[p] + (size_t)rank * m * n_r + r_sm * n_r);
        const size_t n4 = (m - r_sm) * n_r / 4;
        const unsigned gx = (unsigned)jk::sm_count(w_shard->device) * 2;
        jk::push_rows_kernel<<<dim3(gx, (unsigned)(world - 1)), 256, 0, cs>>>(
            reinterpret_cast<const float4*>(mine + r_sm * n_r), pr, rank, n4);
        cudaError_t e = cudaGetLastError();
        // the peers' signals (jk_allgather_wait, on the first copy stream of each peer) follow
        // these stores
        if (e == cudaSuccess) e = cudaEventRecord(ss->pushed, cs);
        for (int p = 0; p < world && e == cudaSuccess; ++p)
            if (p != rank) e = cudaStreamWaitEvent(ss->cs[p][0], ss->pushed, 0);
        if (e != cudaSuccess) return jk::cuda_fail(e, "sharded product: SM copies");
    }
    if (wait) return jk_allgather_wait(w_shard->device, flags_peers, world, rank, stream);
    return JK_OK;
}
