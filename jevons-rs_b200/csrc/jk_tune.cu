// jk_tune.cu -- measured launch plans for the dense and expert-grouped products (host code only).
//
// The reference's Tuner (crates/jevons-gemma4-diffusion/src/gpu/tune.rs) times the candidate
// plans of every weight shape the model uses on the device at start-up, keyed by a row-count
// bucket, keeps the heuristic plan unless a candidate is clearly faster, and stores the table in a
// text file keyed by a device profile. This is that tuner for the B200 kernels:
//
//   bucket            tune.rs:74-76      plans measured at m = bucket serve (bucket/2, bucket]
//   candidates        tune.rs:499-531    this library's tiles: bm 32..256, bn 128/256, splits 1..8
//   pick (5% margin)  tune.rs:548-562
//   time              tune.rs:564-589    here: CUDA events on the caller's stream, best of 3
//                                        batches of >= 2 ms, after one untimed run
//   Tuner::dense      tune.rs:162-175    lookup, falling back to Plan::heuristic
//   tune_dense        tune.rs:231-269
//   Tuner::grouped    tune.rs:177-192    default GroupPlan {bm 32, bn 128}
//   tune_grouped      tune.rs:271-346    tiles bm 32..256 x bn 128/256 over the caller's routes
//   load / save       tune.rs:358-446    same line formats ("dense ...", "grouped ...")
//
// Tuning never changes a result a caller relies on being exact: row-invariant requests only
// consider plans without split-K (whole tiles), whose per-row accumulation order does not depend
// on the tile shape.
#include "jk_internal.h"

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <map>
#include <mutex>
#include <sstream>
#include <tuple>
#include <vector>

namespace {

constexpr int TUNE_VERSION = 1;
constexpr double MARGIN = 0.05;

// (fmt, n, k, bucket, row_invariant)
using DenseKey = std::tuple<int, size_t, size_t, size_t, int>;
// (fmt, n, k, experts, bucket)
using GroupKey = std::tuple<int, size_t, size_t, size_t, size_t>;

size_t bucket_of(size_t m) {
    size_t b = 1;
    while (b < m) b <<= 1;
    return b < 4 ? 4 : b;
}

bool same_plan(const jk_plan& a, const jk_plan& b) { return a.bm == b.bm && a.bn == b.bn && a.splits == b.splits; }

// Index of the plan to keep: the fastest, unless the baseline is within MARGIN of it.
long pick_index(const double* times, const jk_plan* plans, size_t count, const jk_plan& baseline) {
    if (count == 0) return -1;
    size_t best = 0;
    for (size_t i = 1; i < count; ++i)
        if (times[i] < times[best]) best = i;
    for (size_t i = 0; i < count; ++i)
        if (same_plan(plans[i], baseline) && times[best] > times[i] * (1.0 - MARGIN)) return (long)i;
    return (long)best;
}

}  // namespace

struct jk_tuner {
    int device;
    std::string path;  // empty: memory only
    std::string profile;
    std::map<DenseKey, jk_plan> dense;
    std::map<GroupKey, jk_plan> grouped;  // splits always 1
    std::mutex mu;
};

namespace {

std::string profile_key(int device) {
    cudaDeviceProp p{};
    if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return std::string();
    char buf[400];
    snprintf(buf, sizeof buf, "v%d abi=%d device=%d name=%s sms=%d cc=%d.%d smem=%zu l2=%d", TUNE_VERSION,
             jk_abi_version(), device, p.name, p.multiProcessorCount, p.major, p.minor, p.sharedMemPerBlockOptin,
             p.l2CacheSize);
    for (char* c = buf; *c; ++c)
        if (*c == '\n') *c = ' ';
    return buf;
}

void load_table(jk_tuner* t) {
    std::ifstream f(t->path);
    if (!f) return;
    std::string line;
    if (!std::getline(f, line) || line != t->profile) return;
    while (std::getline(f, line)) {
        std::istringstream in(line);
        std::string kind;
        long long v[8];
        if (!(in >> kind) || (kind != "dense" && kind != "grouped")) continue;
        const int fields = kind == "dense" ? 8 : 7;
        bool ok = true;
        for (int j = 0; j < fields; ++j) ok = ok && (in >> v[j]);
        std::string extra;
        if (!ok || (in >> extra) || v[0] < 0 || v[1] <= 0 || v[2] <= 0 || v[3] <= 0 || v[4] < 0) continue;
        if (kind == "dense")
            t->dense[DenseKey{(int)v[0], (size_t)v[1], (size_t)v[2], (size_t)v[3], v[4] != 0}] =
                jk_plan{(int32_t)v[5], (int32_t)v[6], (int32_t)v[7]};
        else
            t->grouped[GroupKey{(int)v[0], (size_t)v[1], (size_t)v[2], (size_t)v[3], (size_t)v[4]}] =
                jk_plan{(int32_t)v[5], (int32_t)v[6], 1};
    }
}

// Candidate plans for an m-row product (tune.rs:499-531, with this library's tiles).
std::vector<jk_plan> candidates(const jk_qmatrix* w, size_t m, bool row_invariant) {
    std::vector<jk_plan> out;
    if (!row_invariant && m <= JK_GEMV_ROWS) out.push_back({0, 128, 1});
    const size_t steps = w->k / 64;
    for (int bm : {32, 64, 96, 128, 256}) {
        if (bm > 32 && (size_t)bm / 2 >= m) continue;  // taller than the rows only wastes work
        for (int bn : {128, 256}) {
            for (int splits : {1, 2, 4, 8}) {
                if (row_invariant && splits > 1) continue;
                if (splits > 1 && steps / (size_t)splits < 4) continue;
                const jk_plan p{bm, bn, splits};
                if (jk_plan_valid_for(&p, w, m)) out.push_back(p);
            }
        }
    }
    return out;
}

}  // namespace

using jk::DeviceGuard;
using jk::fail;

extern "C" size_t jk_tune_bucket(size_t m) { return bucket_of(m); }

extern "C" jk_status jk_tune_pick(const double* times, const jk_plan* plans, size_t count, jk_plan baseline,
                                  jk_plan* out) {
    if (!out || (count && (!times || !plans))) return fail(JK_ERR_INVALID, "tune_pick: null pointer");
    const long i = pick_index(times, plans, count, baseline);
    if (i < 0) return fail(JK_ERR_INVALID, "tune_pick: no candidates");
    *out = plans[i];
    return JK_OK;
}

extern "C" jk_status jk_tuner_create(int device, const char* path, int load, jk_tuner** out) {
    if (!out) return fail(JK_ERR_INVALID, "null pointer");
    *out = nullptr;
    std::string key = profile_key(device);
    if (key.empty()) return fail(JK_ERR_CUDA, "tuner: cannot read the device properties");
    jk_tuner* t = new jk_tuner();
    t->device = device;
    t->path = path ? path : "";
    t->profile = key;
    if (load && !t->path.empty()) load_table(t);
    *out = t;
    return JK_OK;
}

extern "C" void jk_tuner_destroy(jk_tuner* t) { delete t; }

extern "C" size_t jk_tuner_size(const jk_tuner* t) {
    if (!t) return 0;
    std::lock_guard<std::mutex> lock(const_cast<jk_tuner*>(t)->mu);
    return t->dense.size() + t->grouped.size();
}

extern "C" jk_status jk_tuner_plan(const jk_tuner* t, const jk_qmatrix* w, size_t m, int row_invariant,
                                   jk_plan* out) {
    if (!t || !w || !out) return fail(JK_ERR_INVALID, "null pointer");
    const DenseKey key{w->type, w->n, w->k, bucket_of(m), row_invariant != 0};
    {
        std::lock_guard<std::mutex> lock(const_cast<jk_tuner*>(t)->mu);
        auto it = t->dense.find(key);
        if (it != t->dense.end() && jk_plan_valid_for(&it->second, w, m) &&
            (!row_invariant || (it->second.bm > 0 && it->second.splits == 1))) {
            *out = it->second;
            return JK_OK;
        }
    }
    return jk_plan_heuristic(w, m, row_invariant, 0, out);
}

extern "C" jk_status jk_tuner_tune(jk_tuner* t, const jk_qmatrix* const* ws, size_t count, size_t m,
                                   int row_invariant, const void* x, int x_dtype, size_t x_len, float* out,
                                   size_t out_len, jk_split_scratch* scratch, void* stream, jk_plan* chosen) {
    if (!t || !ws || count == 0 || !ws[0]) return fail(JK_ERR_INVALID, "tuner: no matrices");
    const jk_qmatrix* w = ws[0];
    for (size_t i = 1; i < count; ++i)
        if (!ws[i] || ws[i]->type != w->type || ws[i]->n != w->n || ws[i]->k != w->k || ws[i]->device != w->device)
            return fail(JK_ERR_INVALID, "tuner: matrices of one call must share type, shape and device");
    if (w->device != t->device) return fail(JK_ERR_INVALID, "tuner: matrix on another device");
    if (m == 0) return fail(JK_ERR_INVALID, "tuner: m must be positive");
    const size_t b = bucket_of(m);
    if (x_len < b * w->k || out_len < b * w->n)
        return fail(JK_ERR_INVALID, "tuner: x and out must hold bucket(m) rows");
    DeviceGuard g(t->device);
    auto s = static_cast<cudaStream_t>(stream);
    jk_plan baseline;
    if (jk_status st = jk_plan_heuristic(w, b, row_invariant, 0, &baseline)) return st;
    std::vector<jk_plan> cands = candidates(w, b, row_invariant != 0);
    bool has_base = false;
    for (const jk_plan& p : cands) has_base = has_base || same_plan(p, baseline);
    if (!has_base && jk_plan_valid_for(&baseline, w, b)) cands.push_back(baseline);

    cudaEvent_t e0, e1;
    if (cudaEventCreate(&e0) != cudaSuccess) return jk::cuda_fail(cudaGetLastError(), "tuner event");
    if (cudaEventCreate(&e1) != cudaSuccess) {
        cudaEventDestroy(e0);
        return jk::cuda_fail(cudaGetLastError(), "tuner event");
    }
    std::vector<double> times;
    jk_status st = JK_OK;
    auto run = [&](const jk_plan& p) -> jk_status {
        for (size_t i = 0; i < count; ++i)
            if (jk_status r = jk_matmul_plan(ws[i], x, x_dtype, x_len, b, out, out_len, scratch, p, stream)) return r;
        return JK_OK;
    };
    auto batch = [&](const jk_plan& p, int reps, double* ms) -> jk_status {
        cudaEventRecord(e0, s);
        for (int r = 0; r < reps; ++r)
            if (jk_status q = run(p)) return q;
        cudaEventRecord(e1, s);
        cudaError_t ce = cudaEventSynchronize(e1);
        if (ce != cudaSuccess) return jk::cuda_fail(ce, "tuner timing");
        float f = 0.f;
        cudaEventElapsedTime(&f, e0, e1);
        *ms = (double)f / reps;
        return JK_OK;
    };
    for (const jk_plan& p : cands) {
        double once = 0.0, best = 1e30;
        if ((st = run(p)) || (st = batch(p, 1, &once))) break;  // untimed first run, then one probe
        int reps = once > 0.0 ? (int)(2.0 / once) + 1 : 32;
        reps = reps < 1 ? 1 : reps > 32 ? 32 : reps;
        for (int i = 0; i < 3 && !st; ++i) {
            double ms = 0.0;
            st = batch(p, reps, &ms);
            if (ms < best) best = ms;
        }
        if (st) break;
        times.push_back(best);
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (st) return st;
    const long i = pick_index(times.data(), cands.data(), cands.size(), baseline);
    if (i < 0) return fail(JK_ERR_UNSUPPORTED, "tuner: no valid plan for this shape");
    {
        std::lock_guard<std::mutex> lock(t->mu);
        t->dense[DenseKey{w->type, w->n, w->k, b, row_invariant != 0}] = cands[i];
    }
    if (chosen) *chosen = cands[i];
    return JK_OK;
}

extern "C" jk_status jk_tuner_save(const jk_tuner* t) {
    if (!t) return fail(JK_ERR_INVALID, "null pointer");
    if (t->path.empty()) return JK_OK;
    std::ostringstream o;
    o << t->profile << '\n';
    {
        std::lock_guard<std::mutex> lock(const_cast<jk_tuner*>(t)->mu);
        for (const auto& [k, p] : t->dense)
            o << "dense " << std::get<0>(k) << ' ' << std::get<1>(k) << ' ' << std::get<2>(k) << ' ' << std::get<3>(k)
              << ' ' << std::get<4>(k) << ' ' << p.bm << ' ' << p.bn << ' ' << p.splits << '\n';
        for (const auto& [k, p] : t->grouped)
            o << "grouped " << std::get<0>(k) << ' ' << std::get<1>(k) << ' ' << std::get<2>(k) << ' '
              << std::get<3>(k) << ' ' << std::get<4>(k) << ' ' << p.bm << ' ' << p.bn << '\n';
    }
    const std::string tmp = t->path + ".tmp";
    {
        std::ofstream f(tmp, std::ios::trunc);
        if (!(f << o.str())) return fail(JK_ERR_INVALID, "tuner: cannot write " + tmp);
    }
    if (std::rename(tmp.c_str(), t->path.c_str()) != 0) return fail(JK_ERR_INVALID, "tuner: cannot store " + t->path);
    return JK_OK;
}

// Tuner::grouped (tune.rs:177-192): the stored tile shape for w and bucket(rows) when n is a
// multiple of its bn, else the reference's default GroupPlan { bm: 32, bn: 128 }.
extern "C" jk_status jk_tuner_group_plan(const jk_tuner* t, const jk_qmatrix* w, size_t rows, jk_plan* out) {
    if (!t || !w || !out) return fail(JK_ERR_INVALID, "null pointer");
    const GroupKey key{w->type, w->n, w->k, w->experts, bucket_of(rows)};
    std::lock_guard<std::mutex> lock(const_cast<jk_tuner*>(t)->mu);
    auto it = t->grouped.find(key);
    *out = it != t->grouped.end() && it->second.bn > 0 && w->n % (size_t)it->second.bn == 0 ? it->second
                                                                                            : jk_plan{32, 128, 1};
    return JK_OK;
}

// Tuner::tune_grouped (tune.rs:271-346): for `m` tokens routed top_k ways by the first
// a = bucket(m) * top_k ids of `ids`, groups the routes for each candidate tile (bm 32..256,
// bn 128/256), then times the grouped product over all `count` expert matrices (rows of x: one
// per route, in_div 1) and stores the pick against the default {32, 128}.
extern "C" jk_status jk_tuner_tune_grouped(jk_tuner* t, const jk_qmatrix* const* ws, size_t count, size_t m,
                                           size_t top_k, const uint32_t* ids, size_t ids_len, const void* x,
                                           int x_dtype, size_t x_len, float* out, size_t out_len, uint32_t* sorted,
                                           uint32_t* offsets, uint32_t* jobs, size_t jobs_len,
                                           jk_split_scratch* scratch, void* stream, jk_plan* chosen) {
    if (!t || !ws || count == 0 || !ws[0]) return fail(JK_ERR_INVALID, "tuner: no matrices");
    const jk_qmatrix* w = ws[0];
    for (size_t i = 1; i < count; ++i)
        if (!ws[i] || ws[i]->type != w->type || ws[i]->n != w->n || ws[i]->k != w->k ||
            ws[i]->experts != w->experts || ws[i]->device != w->device)
            return fail(JK_ERR_INVALID, "tuner: matrices of one call must share type, shape and device");
    if (w->device != t->device) return fail(JK_ERR_INVALID, "tuner: matrix on another device");
    if (m == 0 || top_k == 0) return fail(JK_ERR_INVALID, "tuner: m and top_k must be positive");
    const size_t b = bucket_of(m), a = b * top_k;
    if (ids_len < a || x_len < a * w->k || out_len < a * w->n)
        return fail(JK_ERR_INVALID, "tuner: ids, x and out must hold bucket(m) * top_k routes");
    DeviceGuard g(t->device);
    auto s = static_cast<cudaStream_t>(stream);
    const jk_plan baseline{32, 128, 1};
    std::vector<jk_plan> cands;
    for (int bm : {32, 64, 128, 256})
        for (int bn : {128, 256}) {
            const jk_plan p{bm, bn, 1};
            if (w->n % (size_t)bn == 0 && jk_plan_valid_for(&p, w, a) &&
                1 + 2 * jk_group_max_jobs(a, w->experts, bm) <= jobs_len)
                cands.push_back(p);
        }
    cudaEvent_t e0, e1;
    if (cudaEventCreate(&e0) != cudaSuccess) return jk::cuda_fail(cudaGetLastError(), "tuner event");
    if (cudaEventCreate(&e1) != cudaSuccess) {
        cudaEventDestroy(e0);
        return jk::cuda_fail(cudaGetLastError(), "tuner event");
    }
    std::vector<double> times;
    std::vector<jk_plan> timed;
    jk_status st = JK_OK;
    for (const jk_plan& p : cands) {
        if ((st = jk_group_experts(t->device, ids, a, w->experts, p.bm, sorted, offsets, jobs, jobs_len, stream))) break;
        const jk_groups grp{sorted, offsets, jobs, jk_group_max_jobs(a, w->experts, p.bm), 1, a};
        auto run = [&]() -> jk_status {
            for (size_t i = 0; i < count; ++i)
                if (jk_status r = jk_matmul_grouped(ws[i], x, x_dtype, x_len, &grp, out, out_len, p.bm, p.bn, 1,
                                                    scratch, stream))
                    return r;
            return JK_OK;
        };
        auto batch = [&](int reps, double* ms) -> jk_status {
            cudaEventRecord(e0, s);
            for (int r = 0; r < reps; ++r)
                if (jk_status q = run()) return q;
            cudaEventRecord(e1, s);
            cudaError_t ce = cudaEventSynchronize(e1);
            if (ce != cudaSuccess) return jk::cuda_fail(ce, "tuner timing");
            float f = 0.f;
            cudaEventElapsedTime(&f, e0, e1);
            *ms = (double)f / reps;
            return JK_OK;
        };
        double once = 0.0, best = 1e30;
        if ((st = run()) || (st = batch(1, &once))) break;
        int reps = once > 0.0 ? (int)(2.0 / once) + 1 : 32;
        reps = reps < 1 ? 1 : reps > 32 ? 32 : reps;
        for (int i = 0; i < 3 && !st; ++i) {
            double ms = 0.0;
            st = batch(reps, &ms);
            if (ms < best) best = ms;
        }
        if (st) break;
        times.push_back(best);
        timed.push_back(p);
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (st) return st;
    const long i = pick_index(times.data(), timed.data(), timed.size(), baseline);
    if (i < 0) return fail(JK_ERR_UNSUPPORTED, "tuner: no valid grouped plan for this shape");
    {
        std::lock_guard<std::mutex> lock(t->mu);
        t->grouped[GroupKey{w->type, w->n, w->k, w->experts, b}] = timed[i];
    }
    if (chosen) *chosen = timed[i];
    return JK_OK;
}
