// jk_api.cu -- the C ABI of include/jk.h: argument validation with the reference's error
// messages, GGML -> B200 layout repacking and upload, launch plans, and dispatch to the kernels.
//
// Reference items mirrored here (paths within zojeda/jevons-rs):
//   TensorType::block            crates/jevons-formats/src/gguf.rs:134-145
//   quant::{q4k_scale_min, packed_words, pack}   crates/jevons-formats/src/quant.rs:14-23,128-193
//   QMatrix::{upload, from_packed, f16_view}     crates/jevons-kernels/src/gemm.rs:832-948
//   Plan::{heuristic, valid_for}                 gemm.rs:981-1038
//   matmul / matmul_plan / matvec / matmul_tiled gemm.rs:1067-1168
//   SplitScratch                                 gemm.rs:1040-1065
//   f16_linear / plan                            crates/jevons-burn/src/kernels.rs:16-31,47-114
#include "jk_internal.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_last_error;

// Per-device error word written by bounded waits that run out (see jk_common.cuh).
__device__ uint32_t g_jk_device_error;

constexpr int MAX_DEVICES = 64;

const char* type_name(int t) {
    switch (t) {
    case JK_TYPE_F32: return "F32";
    case JK_TYPE_F16: return "F16";
    case JK_TYPE_Q5_0: return "Q5_0";
    case JK_TYPE_Q8_0: return "Q8_0";
    case JK_TYPE_Q4_K: return "Q4K";
    case JK_TYPE_Q6_K: return "Q6K";
    default: return "Other";
    }
}

bool block_of(int t, uint64_t& elems, uint64_t& bytes) {
    switch (t) {
    case JK_TYPE_F32: elems = 1; bytes = 4; return true;
    case JK_TYPE_F16: elems = 1; bytes = 2; return true;
    case JK_TYPE_Q4_K: elems = 256; bytes = 144; return true;
    case JK_TYPE_Q5_0: elems = 32; bytes = 22; return true;
    case JK_TYPE_Q6_K: elems = 256; bytes = 210; return true;
    case JK_TYPE_Q8_0: elems = 32; bytes = 34; return true;
    default: elems = bytes = 0; return false;
    }
}

int fmt_of(int t) {
    switch (t) {
    case JK_TYPE_Q4_K: return jk::FMT_Q4K;
    case JK_TYPE_Q6_K: return jk::FMT_Q6K;
    case JK_TYPE_Q5_0: return jk::FMT_Q5_0;
    case JK_TYPE_Q8_0: return jk::FMT_Q8_0;
    case JK_TYPE_F16: return jk::FMT_F16;
    default: return -1;
    }
}

std::string shape_str(int type, size_t experts, size_t n, size_t k) {
    char buf[160];
    snprintf(buf, sizeof buf, "%s [%zux%zu, %zu]", type_name(type), experts, n, k);
    return buf;
}

uint16_t le16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
uint32_t le32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else {
            int e = -1;
            do { man <<= 1; ++e; } while (!(man & 0x400));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// IEEE binary32 -> binary16, round to nearest even (exact for values that came from f16, which is
// the case for QMatrix::from_packed's f32 scale region).
uint16_t float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520 -> inf
    if (absx < 0x38800000u) {                                        // subnormal or zero in f16
        if (absx < 0x33000000u) return (uint16_t)sign;               // < 2^-25 -> 0
        const uint32_t e = absx >> 23;
        const uint32_t man = (absx & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e;  // 14 - (e - 127) + 13 - 1 ... aligns to 2^-24 units
        uint32_t r = man >> (shift);
        const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((absx >> 13) - ((127 - 15) << 10));
    const uint32_t rem = absx & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
    return (uint16_t)(sign | r);
}

using jk::DeviceGuard;

// Runs f(begin, end) over [0, count) on up to 16 host threads (host-side repacking).
template <class F>
void parallel_for(size_t count, F f) {
    unsigned hw = std::thread::hardware_concurrency();
    size_t nt = std::min<size_t>(hw ? hw : 1, 16);
    if (count < (1u << 16) || nt <= 1) {
        f(size_t(0), count);
        return;
    }
    std::vector<std::thread> ts;
    const size_t chunk = (count + nt - 1) / nt;
    for (size_t i = 0; i < nt; ++i) {
        const size_t b = i * chunk, e = std::min(count, b + chunk);
        if (b >= e) break;
        ts.emplace_back([=] { f(b, e); });
    }
    for (auto& t : ts) t.join();
}

}  // namespace

namespace jk {

jk_status fail(jk_status st, const std::string& msg) {
    g_last_error = msg;
    return st;
}

jk_status cuda_fail(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return JK_OK;
    return fail(JK_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

uint32_t* device_error_word(int device) {
    static std::mutex mu;
    static uint32_t* words[MAX_DEVICES] = {};
    if (device < 0 || device >= MAX_DEVICES) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!words[device]) {
        DeviceGuard g(device);
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_jk_device_error) == cudaSuccess) words[device] = static_cast<uint32_t*>(p);
    }
    return words[device];
}

int sm_count(int device) {
    static std::mutex mu;
    static int counts[MAX_DEVICES] = {};
    if (device < 0 || device >= MAX_DEVICES) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (!counts[device]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
        counts[device] = v;
    }
    return counts[device];
}

static std::atomic<int> g_sm_cap[MAX_DEVICES];

int sm_budget(int device) {
    const int total = sm_count(device);
    if (device < 0 || device >= MAX_DEVICES) return total;
    const int cap = g_sm_cap[device].load(std::memory_order_relaxed);
    return cap > 0 && cap < total ? cap : total;
}

jk_status encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, uint64_t dim0, uint64_t dim1,
                         uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swizzle,
                         const void* base) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!encode) return fail(JK_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {dim0, dim1};
    const cuuint64_t strides[1] = {stride1_bytes};
    const cuuint32_t box[2] = {box0, box1};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[200];
        snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d) for dims %llu x %llu, box %u x %u", (int)r,
                 (unsigned long long)dim0, (unsigned long long)dim1, box0, box1);
        return fail(JK_ERR_CUDA, buf);
    }
    return JK_OK;
}

}  // namespace jk

using jk::fail;
using jk::cuda_fail;

// ================================================================================================
// errors / library
// ================================================================================================
extern "C" const char* jk_last_error(void) { return g_last_error.c_str(); }
extern "C" int jk_abi_version(void) { return JK_ABI_VERSION; }

extern "C" jk_status jk_set_max_ctas(int device, int max_sms) {
    if (device < 0 || device >= MAX_DEVICES) return fail(JK_ERR_INVALID, "device index out of range");
    if (max_sms < 0) return fail(JK_ERR_INVALID, "max_sms must be >= 0");
    jk::g_sm_cap[device].store(max_sms, std::memory_order_relaxed);
    return JK_OK;
}

extern "C" jk_status jk_get_max_ctas(int device, int* max_sms, int* sm_total) {
    if (device < 0 || device >= MAX_DEVICES) return fail(JK_ERR_INVALID, "device index out of range");
    if (max_sms) *max_sms = jk::g_sm_cap[device].load(std::memory_order_relaxed);
    if (sm_total) *sm_total = jk::sm_count(device);
    return JK_OK;
}

// ================================================================================================
// block formats (host)
// ================================================================================================
extern "C" jk_status jk_tensor_type_block(int type, uint64_t* elements, uint64_t* bytes) {
    if (!elements || !bytes) return fail(JK_ERR_INVALID, "null output pointer");
    if (!block_of(type, *elements, *bytes)) return fail(JK_ERR_UNSUPPORTED, "unsupported tensor type");
    return JK_OK;
}

extern "C" jk_status jk_q4k_scale_min(int j, const uint8_t scales[12], uint8_t* scale, uint8_t* min) {
    if (!scales || !scale || !min) return fail(JK_ERR_INVALID, "null pointer");
    if (j < 0 || j >= 8) return fail(JK_ERR_INVALID, "q4k_scale_min: j must be in 0..8");
    const uint8_t* q = scales;
    if (j < 4) {
        *scale = q[j] & 63;
        *min = q[j + 4] & 63;
    } else {
        *scale = (uint8_t)((q[j + 4] & 15) | ((q[j - 4] >> 6) << 4));
        *min = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
    return JK_OK;
}

static void packed_words_of(int type, size_t w[4]) {
    w[0] = w[1] = w[2] = w[3] = 0;
    switch (type) {
    case JK_TYPE_Q4_K: w[0] = 36; break;
    case JK_TYPE_Q6_K: w[0] = 32; w[1] = 16; w[2] = 4; w[3] = 1; break;
    case JK_TYPE_Q5_0: w[0] = 4; w[1] = 1; w[3] = 1; break;
    case JK_TYPE_Q8_0: w[0] = 8; w[3] = 1; break;
    default: break;
    }
}

extern "C" jk_status jk_packed_words(int type, size_t words[4]) {
    if (!words) return fail(JK_ERR_INVALID, "null pointer");
    packed_words_of(type, words);
    return JK_OK;
}

extern "C" jk_status jk_pack(int type, const void* ggml_bytes, size_t len, uint32_t* q, size_t q_words, uint32_t* h,
                             size_t h_words, uint32_t* s, size_t s_words, float* d, size_t d_words) {
    uint64_t be, bb;
    if (!block_of(type, be, bb)) return fail(JK_ERR_UNSUPPORTED, "unsupported tensor type");
    if (type != JK_TYPE_Q4_K && type != JK_TYPE_Q6_K && type != JK_TYPE_Q5_0 && type != JK_TYPE_Q8_0)
        return fail(JK_ERR_UNSUPPORTED, std::string(type_name(type)) + " has no GPU block layout");
    if (len % bb) return fail(JK_ERR_SHAPE, "tensor is not a whole number of blocks");
    if (len && !ggml_bytes) return fail(JK_ERR_INVALID, "null input");
    const size_t blocks = len / bb;
    size_t w[4];
    packed_words_of(type, w);
    if (q_words < blocks * w[0] || h_words < blocks * w[1] || s_words < blocks * w[2] || d_words < blocks * w[3])
        return fail(JK_ERR_INVALID, "pack: output regions too small");
    if ((blocks * w[0] != 0 && !q) || (blocks * w[1] != 0 && !h) || (blocks * w[2] != 0 && !s) ||
        (blocks * w[3] != 0 && !d))
        return fail(JK_ERR_INVALID, "pack: null output region");
    const uint8_t* raw = static_cast<const uint8_t*>(ggml_bytes);
    parallel_for(blocks, [&](size_t b0, size_t b1) {
        for (size_t i = b0; i < b1; ++i) {
            const uint8_t* b = raw + i * bb;
            switch (type) {
            case JK_TYPE_Q4_K:
                for (int t = 0; t < 36; ++t) q[i * 36 + t] = le32(b + 4 * t);
                break;
            case JK_TYPE_Q6_K:
                for (int t = 0; t < 32; ++t) q[i * 32 + t] = le32(b + 4 * t);
                for (int t = 0; t < 16; ++t) h[i * 16 + t] = le32(b + 128 + 4 * t);
                for (int t = 0; t < 4; ++t) s[i * 4 + t] = le32(b + 192 + 4 * t);
                d[i] = half_to_float(le16(b + 208));
                break;
            case JK_TYPE_Q5_0:
                d[i] = half_to_float(le16(b));
                h[i] = le32(b + 2);
                for (int t = 0; t < 4; ++t) q[i * 4 + t] = le32(b + 6 + 4 * t);
                break;
            case JK_TYPE_Q8_0:
                d[i] = half_to_float(le16(b));
                for (int t = 0; t < 8; ++t) q[i * 8 + t] = le32(b + 2 + 4 * t);
                break;
            }
        }
    });
    return JK_OK;
}

// Host dequantization of whole blocks, quant::dequantize (crates/jevons-formats/src/quant.rs:83-101)
// with the block decoders of quant.rs:25-80. Every product of a scale and a quant is exact in f32
// (d has 11 significant bits, the other factor at most 13), so the only rounding is Q4_K's final
// subtraction; the operations below keep the reference's order (the library is compiled with
// -ffp-contract=off, so the multiply and the subtraction stay two operations).
namespace {

void host_block_q4k(const uint8_t* b, float* out) {
    const float d = half_to_float(le16(b)), dmin = half_to_float(le16(b + 2));
    const uint8_t* sc = b + 4;
    const uint8_t* qs = b + 16;
    for (int pair = 0; pair < 4; ++pair) {
        float dd[2], mm[2];
        for (int h = 0; h < 2; ++h) {
            uint8_t s, m;
            jk_q4k_scale_min(2 * pair + h, sc, &s, &m);
            dd[h] = d * (float)s;
            mm[h] = dmin * (float)m;
        }
        for (int l = 0; l < 32; ++l) {
            const uint8_t q = qs[32 * pair + l];
            const float lo = dd[0] * (float)(q & 15), hi = dd[1] * (float)(q >> 4);
            out[64 * pair + l] = lo - mm[0];
            out[64 * pair + 32 + l] = hi - mm[1];
        }
    }
}

void host_block_q6k(const uint8_t* b, float* out) {
    const float d = half_to_float(le16(b + 208));
    for (int h = 0; h < 2; ++h) {
        const uint8_t* ql = b + 64 * h;
        const uint8_t* qh = b + 128 + 32 * h;
        const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192 + 8 * h);
        float* o = out + 128 * h;
        for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            const int q[4] = {((ql[l] & 15) | ((qh[l] & 3) << 4)) - 32, ((ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4)) - 32,
                              ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32,
                              ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32};
            for (int j = 0; j < 4; ++j) {
                const float ds = d * (float)sc[is + 2 * j];
                o[l + 32 * j] = ds * (float)q[j];
            }
        }
    }
}

void host_block_q5_0(const uint8_t* b, float* out) {
    const float d = half_to_float(le16(b));
    const uint32_t qh = le32(b + 2);
    const uint8_t* qs = b + 6;
    for (int j = 0; j < 16; ++j) {
        const uint32_t h0 = ((qh >> j) << 4) & 0x10u, h1 = (qh >> (j + 12)) & 0x10u;
        out[j] = d * (float)((int)((qs[j] & 15u) | h0) - 16);
        out[j + 16] = d * (float)((int)((qs[j] >> 4) | h1) - 16);
    }
}

void host_block_q8_0(const uint8_t* b, float* out) {
    const float d = half_to_float(le16(b));
    for (int j = 0; j < 32; ++j) out[j] = d * (float)(int8_t)b[2 + j];
}

}  // namespace

extern "C" jk_status jk_dequantize(int type, const void* bytes, size_t len, float* out, size_t out_len) {
    uint64_t be, bb;
    if (!block_of(type, be, bb)) return fail(JK_ERR_UNSUPPORTED, "unsupported tensor type");
    if (len % bb || out_len != len / bb * be) return fail(JK_ERR_SHAPE, "dequantization size mismatch");
    if (len && (!bytes || !out)) return fail(JK_ERR_INVALID, "null pointer");
    const uint8_t* raw = static_cast<const uint8_t*>(bytes);
    parallel_for(len / bb, [&](size_t b0, size_t b1) {
        for (size_t i = b0; i < b1; ++i) {
            const uint8_t* src = raw + i * bb;
            float* dst = out + i * be;
            switch (type) {
            case JK_TYPE_F32: memcpy(dst, src, 4); break;
            case JK_TYPE_F16: dst[0] = half_to_float(le16(src)); break;
            case JK_TYPE_Q4_K: host_block_q4k(src, dst); break;
            case JK_TYPE_Q6_K: host_block_q6k(src, dst); break;
            case JK_TYPE_Q5_0: host_block_q5_0(src, dst); break;
            default: host_block_q8_0(src, dst); break;
            }
        }
    });
    return JK_OK;
}

// ================================================================================================
// device
// ================================================================================================
extern "C" jk_status jk_gpu_init(int device) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= count) {
        char buf[96];
        snprintf(buf, sizeof buf, "CUDA device %d: no such device (%d visible)", device, count);
        return fail(JK_ERR_INVALID, buf);
    }
    cudaDeviceProp p;
    e = cudaGetDeviceProperties(&p, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    if (p.major != 10) {
        char buf[400];  // the device name is up to 256 characters
        snprintf(buf, sizeof buf, "CUDA device %d (%s, sm_%d%d): the kernels are built for sm_100a (B200)", device,
                 p.name, p.major, p.minor);
        return fail(JK_ERR_UNSUPPORTED, buf);
    }
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    if (!jk::device_error_word(device)) return fail(JK_ERR_CUDA, "device error word unavailable");
    return JK_OK;
}

extern "C" jk_status jk_gpu_sync(void* stream) {
    return cuda_fail(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "device sync");
}

extern "C" jk_status jk_device_error(int device, uint32_t* code) {
    if (!code) return fail(JK_ERR_INVALID, "null pointer");
    DeviceGuard g(device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "device sync");
    uint32_t* word = jk::device_error_word(device);
    if (!word) return fail(JK_ERR_CUDA, "device error word unavailable");
    e = cudaMemcpy(code, word, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "read device error word");
    const uint32_t zero = 0;
    e = cudaMemcpy(word, &zero, 4, cudaMemcpyHostToDevice);
    return cuda_fail(e, "clear device error word");
}

// ================================================================================================
// quantized matrices
// ================================================================================================
namespace {

jk_status finish_matrix(jk_qmatrix* m) {
    m->view.rows = (int64_t)(m->experts * m->n);
    m->view.n = (int64_t)m->n;
    m->view.k = (int64_t)m->k;
    m->view.q_row_bytes = jk::q_row_bytes(m->view.fmt, (int64_t)m->k);
    jk_status st = jk::make_weight_tmap(m->view, &m->tm_w);
    m->has_tmap = st == JK_OK;
    return st;
}

struct HostLayout {
    std::vector<uint8_t> q;
    std::vector<uint16_t> d;
    std::vector<uint32_t> h;
};

jk_status upload_layout(int device, int type, size_t n, size_t k, size_t experts, HostLayout& hl, const void* q_src,
                        size_t q_bytes, jk_qmatrix** out) {
    DeviceGuard g(device);
    jk_status st = jk_gpu_init(device);
    if (st != JK_OK) return st;
    auto* m = new (std::nothrow) jk_qmatrix();
    if (!m) return fail(JK_ERR_INVALID, "out of host memory");
    m->type = type;
    m->device = device;
    m->n = n;
    m->k = k;
    m->experts = experts;
    m->view.fmt = fmt_of(type);
    const size_t d_bytes = hl.d.size() * 2, h_bytes = hl.h.size() * 4;
    // The small-row kernel copies the scale / high-bit words of a row segment rounded out to
    // 16-byte boundaries, so those arrays carry 64 bytes of slack past their end.
    cudaError_t e = cudaMalloc(&m->q_alloc, q_bytes ? q_bytes : 16);
    if (e == cudaSuccess && d_bytes) e = cudaMalloc(&m->d_alloc, d_bytes + 64);
    if (e == cudaSuccess && h_bytes) e = cudaMalloc(&m->h_alloc, h_bytes + 64);
    if (e == cudaSuccess) e = cudaMemcpy(m->q_alloc, q_src, q_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && d_bytes) e = cudaMemcpy(m->d_alloc, hl.d.data(), d_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && h_bytes) e = cudaMemcpy(m->h_alloc, hl.h.data(), h_bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        jk_qmatrix_destroy(m);
        return cuda_fail(e, "weight upload");
    }
    m->view.q = static_cast<const uint8_t*>(m->q_alloc);
    m->view.d = static_cast<const uint16_t*>(m->d_alloc);
    m->view.h = static_cast<const uint32_t*>(m->h_alloc);
    m->device_bytes = q_bytes + d_bytes + h_bytes;
    st = finish_matrix(m);
    if (st != JK_OK) {
        jk_qmatrix_destroy(m);
        return st;
    }
    *out = m;
    return JK_OK;
}

jk_status check_shape(int type, size_t n, size_t k, size_t experts, uint64_t blk) {
    if (n == 0 || k == 0 || experts == 0 || k % 64 || n % 64 || k % blk)
        return fail(JK_ERR_SHAPE, shape_str(type, experts, n, k) + " has an unsupported shape");
    return JK_OK;
}

}  // namespace

extern "C" jk_status jk_qmatrix_upload(int device, int type, size_t n, size_t k, size_t experts, const void* ggml_bytes,
                                       size_t len, jk_qmatrix** out) {
    if (!out) return fail(JK_ERR_INVALID, "null output pointer");
    *out = nullptr;
    uint64_t be, bb;
    if (!block_of(type, be, bb)) return fail(JK_ERR_UNSUPPORTED, "unsupported type");
    if (fmt_of(type) < 0 || type == JK_TYPE_F16)
        return fail(JK_ERR_UNSUPPORTED, std::string(type_name(type)) + " weights are not supported");
    // QMatrix::upload's byte-count check (gemm.rs:841-845) comes first, then from_packed's shape rules.
    if (k % be != 0 || len != experts * n * k / be * bb)
        return fail(JK_ERR_SHAPE, shape_str(type, experts, n, k) + " has the wrong byte count");
    jk_status st = check_shape(type, n, k, experts, be);
    if (st != JK_OK) return st;
    if (!ggml_bytes) return fail(JK_ERR_INVALID, "null weight bytes");
    const uint8_t* raw = static_cast<const uint8_t*>(ggml_bytes);
    const size_t blocks = len / bb;
    HostLayout hl;
    switch (type) {
    case JK_TYPE_Q4_K:
        return upload_layout(device, type, n, k, experts, hl, raw, len, out);
    case JK_TYPE_Q6_K:
        hl.q.resize(blocks * 208);
        hl.d.resize(blocks);
        parallel_for(blocks, [&](size_t b0, size_t b1) {
            for (size_t i = b0; i < b1; ++i) {
                memcpy(&hl.q[i * 208], raw + i * 210, 208);
                hl.d[i] = le16(raw + i * 210 + 208);
            }
        });
        break;
    case JK_TYPE_Q8_0:
        hl.q.resize(blocks * 32);
        hl.d.resize(blocks);
        parallel_for(blocks, [&](size_t b0, size_t b1) {
            for (size_t i = b0; i < b1; ++i) {
                hl.d[i] = le16(raw + i * 34);
                memcpy(&hl.q[i * 32], raw + i * 34 + 2, 32);
            }
        });
        break;
    case JK_TYPE_Q5_0:
        hl.q.resize(blocks * 16);
        hl.d.resize(blocks);
        hl.h.resize(blocks);
        parallel_for(blocks, [&](size_t b0, size_t b1) {
            for (size_t i = b0; i < b1; ++i) {
                hl.d[i] = le16(raw + i * 22);
                hl.h[i] = le32(raw + i * 22 + 2);
                memcpy(&hl.q[i * 16], raw + i * 22 + 6, 16);
            }
        });
        break;
    }
    return upload_layout(device, type, n, k, experts, hl, hl.q.data(), hl.q.size(), out);
}

extern "C" jk_status jk_qmatrix_from_packed(int device, int type, size_t n, size_t k, size_t experts, const uint32_t* q,
                                            size_t q_words, const uint32_t* h, size_t h_words, const uint32_t* s,
                                            size_t s_words, const float* d, size_t d_words, jk_qmatrix** out) {
    if (!out) return fail(JK_ERR_INVALID, "null output pointer");
    *out = nullptr;
    uint64_t be, bb;
    if (fmt_of(type) < 0 || type == JK_TYPE_F16 || !block_of(type, be, bb)) {
        return fail(JK_ERR_UNSUPPORTED, std::string(type_name(type)) + " weights are not supported");
    }
    size_t w[4];
    packed_words_of(type, w);
    const size_t blocks = experts * n * k / be;
    if (check_shape(type, n, k, experts, be) != JK_OK || q_words != blocks * w[0] || h_words != blocks * w[1] ||
        s_words != blocks * w[2] || d_words != blocks * w[3])
        return fail(JK_ERR_SHAPE, shape_str(type, experts, n, k) + " has an unsupported shape");
    if ((q_words && !q) || (h_words && !h) || (s_words && !s) || (d_words && !d))
        return fail(JK_ERR_INVALID, "null packed region");
    HostLayout hl;
    switch (type) {
    case JK_TYPE_Q4_K:
        return upload_layout(device, type, n, k, experts, hl, q, q_words * 4, out);
    case JK_TYPE_Q6_K:
        hl.q.resize(blocks * 208);
        hl.d.resize(blocks);
        parallel_for(blocks, [&](size_t b0, size_t b1) {
            for (size_t i = b0; i < b1; ++i) {
                memcpy(&hl.q[i * 208], q + i * 32, 128);
                memcpy(&hl.q[i * 208 + 128], h + i * 16, 64);
                memcpy(&hl.q[i * 208 + 192], s + i * 4, 16);
                hl.d[i] = float_to_half(d[i]);
            }
        });
        break;
    case JK_TYPE_Q8_0:
        hl.q.resize(blocks * 32);
        hl.d.resize(blocks);
        parallel_for(blocks, [&](size_t b0, size_t b1) {
            for (size_t i = b0; i < b1; ++i) {
                memcpy(&hl.q[i * 32], q + i * 8, 32);
                hl.d[i] = float_to_half(d[i]);
            }
        });
        break;
    case JK_TYPE_Q5_0:
        hl.q.resize(blocks * 16);
        hl.d.resize(blocks);
        hl.h.resize(blocks);
        parallel_for(blocks, [&](size_t b0, size_t b1) {
            for (size_t i = b0; i < b1; ++i) {
                memcpy(&hl.q[i * 16], q + i * 4, 16);
                hl.h[i] = h[i];
                hl.d[i] = float_to_half(d[i]);
            }
        });
        break;
    }
    return upload_layout(device, type, n, k, experts, hl, hl.q.data(), hl.q.size(), out);
}

extern "C" jk_status jk_qmatrix_f16_view(int device, size_t n, size_t k, const void* f16_weights_dev,
                                         jk_qmatrix** out) {
    if (!out) return fail(JK_ERR_INVALID, "null output pointer");
    *out = nullptr;
    if (k % 64 || n % 64 || n == 0 || k == 0) {
        char buf[96];
        snprintf(buf, sizeof buf, "F16 [%zu, %zu] has an unsupported shape", n, k);
        return fail(JK_ERR_SHAPE, buf);
    }
    if (!f16_weights_dev || (reinterpret_cast<uintptr_t>(f16_weights_dev) & 15))
        return fail(JK_ERR_INVALID, "F16 weights must be a 16-byte aligned device pointer");
    DeviceGuard g(device);
    jk_status st = jk_gpu_init(device);
    if (st != JK_OK) return st;
    auto* m = new (std::nothrow) jk_qmatrix();
    if (!m) return fail(JK_ERR_INVALID, "out of host memory");
    m->type = JK_TYPE_F16;
    m->device = device;
    m->n = n;
    m->k = k;
    m->experts = 1;
    m->view.fmt = jk::FMT_F16;
    m->view.q = static_cast<const uint8_t*>(f16_weights_dev);
    m->device_bytes = n * k * 2;
    st = finish_matrix(m);
    if (st != JK_OK) {
        delete m;
        return st;
    }
    *out = m;
    return JK_OK;
}

extern "C" void jk_qmatrix_destroy(jk_qmatrix* w) {
    if (!w) return;
    {
        DeviceGuard g(w->device);
        if (w->q_alloc) cudaFree(w->q_alloc);
        if (w->d_alloc) cudaFree(w->d_alloc);
        if (w->h_alloc) cudaFree(w->h_alloc);
    }
    delete w;
}

extern "C" jk_status jk_qmatrix_info(const jk_qmatrix* w, int* type, size_t* n, size_t* k, size_t* experts,
                                     size_t* device_bytes) {
    if (!w) return fail(JK_ERR_INVALID, "null matrix");
    if (type) *type = w->type;
    if (n) *n = w->n;
    if (k) *k = w->k;
    if (experts) *experts = w->experts;
    if (device_bytes) *device_bytes = w->device_bytes;
    return JK_OK;
}

extern "C" jk_status jk_qmatrix_dequantize(const jk_qmatrix* w, float* out_dev, size_t out_len, void* stream) {
    if (!w || !out_dev) return fail(JK_ERR_INVALID, "null pointer");
    if (out_len != w->experts * w->n * w->k) return fail(JK_ERR_INVALID, "dequantization size mismatch");
    DeviceGuard g(w->device);
    return jk::launch_dequant(w->view, out_dev, static_cast<cudaStream_t>(stream));
}

// ================================================================================================
// plans
// ================================================================================================
namespace {

constexpr int ROW_TILES[4] = {32, 64, 128, 256};

int row_tile_for(size_t m) {
    for (int t : ROW_TILES)
        if (m <= (size_t)t) return t;
    return 256;
}

bool plan_valid(const jk_plan& p, const jk_qmatrix* w, size_t m) {
    if (p.bm == 0) return m <= JK_GEMV_ROWS && p.splits == 1 && w->k / 32 <= 1u << 20;
    const bool bm_ok = p.bm == 32 || p.bm == 64 || p.bm == 96 || p.bm == 128 || p.bm == 256;
    // bn: weight rows per tile. 128 = one CTA per tile; 256 = a CTA pair (tcgen05 cta_group::2,
    // each CTA dequantizes 128 rows and loads half the activation rows) for block-quantized
    // weights at bm >= 128.
    const bool bn_ok = p.bn == 128 || (p.bn == 256 && w->type != JK_TYPE_F16 && p.bm >= 128);
    return bm_ok && bn_ok && p.splits >= 1 && p.splits <= 16 && w->k / 64 >= (size_t)p.splits;
}

jk_status check_launch(const jk_qmatrix* w, const void* x, int x_dtype, size_t x_len, size_t m, const float* out,
                       size_t out_len) {
    if (!w) return fail(JK_ERR_INVALID, "null matrix");
    if (x_dtype != JK_DTYPE_F32 && x_dtype != JK_DTYPE_F16 && x_dtype != JK_DTYPE_BF16)
        return fail(JK_ERR_INVALID, "unknown activation dtype");
    // m is bounded first so that m * k and m * n below cannot wrap around
    if (m > (size_t)INT32_MAX) return fail(JK_ERR_INVALID, "m too large");
    if (x_len < m * w->k || out_len < m * w->n) {
        char buf[200];
        snprintf(buf, sizeof buf, "%s: buffers too small for m=%zu (x %zu < %zu or out %zu < %zu)",
                 shape_str(w->type, w->experts, w->n, w->k).c_str(), m, x_len, m * w->k, out_len, m * w->n);
        return fail(JK_ERR_INVALID, buf);
    }
    if (m && (!x || !out)) return fail(JK_ERR_INVALID, "null activation or output pointer");
    return JK_OK;
}

// The dense products use expert 0's rows (gemm.rs:591 with expert = 0).
jk::WView dense_view(const jk_qmatrix* w) {
    jk::WView v = w->view;
    v.rows = (int64_t)w->n;
    return v;
}

}  // namespace

// Plan::heuristic (gemm.rs:989-1004), adapted to this kernel. Row-invariant plans: the smallest
// activation-row tile >= m, capped at 128 for block-quantized weights (there the dequantized weights
// live in tensor memory next to two accumulators, which measures faster than 256-row tiles with
// shared-memory weight stages). Otherwise, for block-quantized weights, a small cost model picks the
// row tile and the schedule: whole tiles of bm rows take ceil(tiles / SMs) waves of k-blocks at the
// main loop's measured cycles per k-block for that tile (32: 338, 64: 400, 96: 491, 128: 555), and
// stream-K (bm = min(row tile, 128), splits = 2) spreads the same k-blocks evenly over the SMs but
// pays a fixed ~20000 cycles (its fix-up and the pipeline fill it can no longer overlap with the
// previous product). On B200 this reproduces the measured best plan of every shape tried (Q4_K
// N=10240, K=2560 at m = 32..768: e.g. bm 64 at m=160-192, 96 at m=224-288 and 448, 128 at 320-384
// and 512-768; Q6_K N=2560, K=10240: stream-K; Q8_0 at m=750: 96 or 64). FP16 weights keep the
// rule of growing the row tile with m, with stream-K only when whole tiles leave most SMs idle.
extern "C" jk_status jk_plan_heuristic(const jk_qmatrix* w, size_t m, int row_invariant, int sms, jk_plan* out) {
    if (!w || !out) return fail(JK_ERR_INVALID, "null pointer");
    int bm = row_tile_for(m);
    if (w->type != JK_TYPE_F16 && bm > 128) bm = 128;
    const int bn = 128;
    if (row_invariant) {
        *out = {bm, bn, 1};
        return JK_OK;
    }
    if (m <= 2) {
        *out = {0, bn, 1};
        return JK_OK;
    }
    const size_t target = sms > 0 ? (size_t)sms : (size_t)jk::sm_count(w->device);
    const size_t wt = (w->n + 127) / 128;
    const size_t kbt = w->k / 64;
    if (w->type != JK_TYPE_F16) {
        static const int TILE[4] = {32, 64, 96, 128};
        static const double CYC[4] = {338.0, 400.0, 491.0, 555.0};
        int best = 3;
        double best_cost = 0.0;
        for (int t = 3; t >= 0; --t) {  // ties go to the larger tile
            const size_t tiles = wt * ((m + TILE[t] - 1) / TILE[t]);
            const double cost = (double)((tiles + target - 1) / target) * (double)kbt * CYC[t];
            if (t == 3 || cost < best_cost) {
                best = t;
                best_cost = cost;
            }
        }
        if (kbt >= 8) {
            const int tsk = bm == 32 ? 0 : bm == 64 ? 1 : bm == 96 ? 2 : 3;
            const size_t tiles = wt * ((m + bm - 1) / bm);
            const double sk_cost = (double)tiles * (double)kbt / (double)target * CYC[tsk] + 20000.0;
            if (sk_cost < best_cost) {
                *out = {bm, bn, 2};
                return JK_OK;
            }
        }
        *out = {TILE[best], bn, 1};
        return JK_OK;
    }
    const size_t tiles = wt * ((m + bm - 1) / bm);
    const bool enough_tiles = tiles * 2 >= target;
    *out = {bm, bn, enough_tiles || kbt < 8 ? 1 : 2};
    return JK_OK;
}

extern "C" int jk_plan_valid_for(const jk_plan* plan, const jk_qmatrix* w, size_t m) {
    if (!plan || !w) return 0;
    return plan_valid(*plan, w, m) ? 1 : 0;
}

// ================================================================================================
// split-K scratch
// ================================================================================================
extern "C" jk_status jk_split_scratch_create(int device, jk_split_scratch** out) {
    if (!out) return fail(JK_ERR_INVALID, "null output pointer");
    auto* s = new (std::nothrow) jk_split_scratch();
    if (!s) return fail(JK_ERR_INVALID, "out of host memory");
    s->device = device;
    *out = s;
    return JK_OK;
}

extern "C" void jk_split_scratch_destroy(jk_split_scratch* s) {
    if (!s) return;
    if (s->buf) {
        DeviceGuard g(s->device);
        cudaFree(s->buf);
    }
    delete s;
}

// Grows the scratch to `bytes` (cudaMalloc, synchronising the device) and zeroes it, so the
// stream-K flag words at its start begin at zero.
jk_status jk::scratch_reserve(jk_split_scratch* s, size_t bytes, void** out) {
    if (s->bytes < bytes) {
        DeviceGuard g(s->device);
        if (s->buf) {
            cudaError_t e = cudaDeviceSynchronize();
            if (e != cudaSuccess) return cuda_fail(e, "scratch growth sync");
            cudaFree(s->buf);
            s->buf = nullptr;
            s->bytes = 0;
        }
        cudaError_t e = cudaMalloc(&s->buf, bytes);
        if (e != cudaSuccess) return cuda_fail(e, "split-K scratch allocation");
        e = cudaMemset(s->buf, 0, bytes);
        if (e != cudaSuccess) return cuda_fail(e, "split-K scratch clear");
        s->bytes = bytes;
    }
    *out = s->buf;
    return JK_OK;
}

// ================================================================================================
// products
// ================================================================================================
extern "C" jk_status jk_matvec(const jk_qmatrix* w, const void* x, int x_dtype, size_t x_len, size_t m, float* out,
                               size_t out_len, void* stream) {
    jk_status st = check_launch(w, x, x_dtype, x_len, m, out, out_len);
    if (st != JK_OK) return st;
    if (m > JK_GEMV_ROWS) {
        char buf[96];
        snprintf(buf, sizeof buf, "matvec takes at most %d rows (got %zu)", JK_GEMV_ROWS, m);
        return fail(JK_ERR_INVALID, buf);
    }
    if (m == 0) return JK_OK;
    DeviceGuard g(w->device);
    return jk::launch_gemv(dense_view(w), x, x_dtype, m, out, static_cast<cudaStream_t>(stream));
}

extern "C" jk_status jk_matmul_plan(const jk_qmatrix* w, const void* x, int x_dtype, size_t x_len, size_t m,
                                    float* out, size_t out_len, jk_split_scratch* scratch, jk_plan plan,
                                    void* stream) {
    jk_status st = check_launch(w, x, x_dtype, x_len, m, out, out_len);
    if (st != JK_OK) return st;
    if (!plan_valid(plan, w, m)) {
        char buf[160];
        snprintf(buf, sizeof buf, "plan {bm %d, bn %d, splits %d} is not valid for %s at m=%zu", plan.bm, plan.bn,
                 plan.splits, shape_str(w->type, w->experts, w->n, w->k).c_str(), m);
        return fail(JK_ERR_INVALID, buf);
    }
    if (m == 0) return JK_OK;
    if (plan.bm == 0) return jk_matvec(w, x, x_dtype, x_len, m, out, out_len, stream);
    if (m > (size_t)INT32_MAX) return fail(JK_ERR_INVALID, "m too large");
    DeviceGuard g(w->device);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    // Operand type of the tensor-core kernel: FP16 weights need f16 activations; quantized weights
    // take bf16 or f16 activations as given, f32 activations are rounded to bf16 first.
    const bool f16_weights = w->type == JK_TYPE_F16;
    const bool want_bf16 = f16_weights ? false : x_dtype != JK_DTYPE_F16;
    const bool convert = f16_weights ? x_dtype != JK_DTYPE_F16 : x_dtype == JK_DTYPE_F32;
    // Scratch layout: [stream-K workspace (flags first) | bf16 copy of f32 activations].
    const bool stream_k = plan.splits > 1;
    const size_t ws_bytes = stream_k ? jk::stream_k_workspace_bytes(w->device, plan.bm) : 0;
    const size_t conv_bytes = convert ? (m * w->k * 2 + 255) / 256 * 256 : 0;
    void* sbuf = nullptr;
    if (ws_bytes + conv_bytes) {
        if (!scratch) return fail(JK_ERR_INVALID, "this plan needs a split-K scratch (splits > 1 or f32 activations)");
        if (scratch->device != w->device) return fail(JK_ERR_INVALID, "scratch belongs to another device");
        st = jk::scratch_reserve(scratch, ws_bytes + conv_bytes, &sbuf);
        if (st != JK_OK) return st;
    }
    const void* xk = x;
    if (convert) {
        if (f16_weights) return fail(JK_ERR_UNSUPPORTED, "FP16 weights need FP16 activations");
        void* xc = static_cast<char*>(sbuf) + ws_bytes;
        st = jk::launch_convert_to_bf16(x, x_dtype, m * w->k, xc, cs);
        if (st != JK_OK) return st;
        xk = xc;
    }
    if ((reinterpret_cast<uintptr_t>(xk) & 15) != 0) return fail(JK_ERR_INVALID, "activations must be 16-byte aligned");
    jk_qmatrix dense = *w;
    dense.view = dense_view(w);
    return jk::launch_gemm(&dense, xk, want_bf16, m, out, plan.bm, plan.bn == 256, stream_k, sbuf, ws_bytes, cs);
}

// ================================================================================================
// expert-grouped products
// ================================================================================================
extern "C" size_t jk_group_max_jobs(size_t assignments, size_t experts, int bm) {
    if (bm < 1) return 0;
    return (assignments + (size_t)bm - 1) / (size_t)bm + (experts < assignments ? experts : assignments);
}

extern "C" jk_status jk_group_experts(int device, const uint32_t* ids, size_t assignments, size_t experts, int bm,
                                      uint32_t* sorted, uint32_t* offsets, uint32_t* jobs, size_t jobs_len,
                                      void* stream) {
    if (experts == 0 || experts > jk::GROUP_MAX_EXPERTS)
        return fail(JK_ERR_UNSUPPORTED, "grouping takes 1..1024 experts");
    if (bm < 1) return fail(JK_ERR_INVALID, "grouping row tile must be positive");
    if (assignments > (size_t)INT32_MAX) return fail(JK_ERR_INVALID, "too many assignments");
    if (!offsets || !jobs || (assignments && (!ids || !sorted))) return fail(JK_ERR_INVALID, "null grouping buffer");
    const size_t need = jk_group_max_jobs(assignments, experts, bm);
    if (jobs_len < 1 + 2 * need) {
        char buf[160];
        snprintf(buf, sizeof buf, "jobs buffer holds %zu words; %zu routes over %zu experts at bm=%d need %zu", jobs_len,
                 assignments, experts, bm, 1 + 2 * need);
        return fail(JK_ERR_INVALID, buf);
    }
    DeviceGuard g(device);
    return jk::launch_group_experts(ids, assignments, experts, bm, (jobs_len - 1) / 2 < (size_t)UINT32_MAX
                                        ? (jobs_len - 1) / 2 : (size_t)UINT32_MAX,
                                    sorted, offsets, jobs, jk::device_error_word(device),
                                    static_cast<cudaStream_t>(stream));
}

namespace {

// Shared checks of the grouped products; sets *x_rows to the activation rows x holds.
jk_status check_grouped(const jk_qmatrix* w, const void* x, int x_dtype, size_t x_len, const jk_groups* g,
                        const float* out, size_t out_len, size_t* x_rows) {
    if (!w || !g) return fail(JK_ERR_INVALID, "null matrix or groups");
    if (x_dtype != JK_DTYPE_F32 && x_dtype != JK_DTYPE_F16 && x_dtype != JK_DTYPE_BF16)
        return fail(JK_ERR_INVALID, "unknown activation dtype");
    if (g->in_div < 1) return fail(JK_ERR_INVALID, "groups: in_div must be >= 1");
    const size_t need_x = (g->rows + g->in_div - 1) / g->in_div;
    if (out_len < g->rows * w->n || x_len < need_x * w->k) {
        char buf[220];
        snprintf(buf, sizeof buf, "%s: buffers too small for %zu grouped rows (x %zu < %zu or out %zu < %zu)",
                 shape_str(w->type, w->experts, w->n, w->k).c_str(), g->rows, x_len, need_x * w->k, out_len,
                 g->rows * w->n);
        return fail(JK_ERR_INVALID, buf);
    }
    if (g->rows && (!x || !out || !g->sorted || !g->offsets || !g->jobs))
        return fail(JK_ERR_INVALID, "null activation, output or grouping pointer");
    if (g->rows > (size_t)INT32_MAX || g->max_jobs > (size_t)INT32_MAX) return fail(JK_ERR_INVALID, "groups too large");
    *x_rows = x_len / w->k;
    return JK_OK;
}

}  // namespace

extern "C" jk_status jk_matmul_grouped(const jk_qmatrix* w, const void* x, int x_dtype, size_t x_len,
                                       const jk_groups* g, float* out, size_t out_len, int bm, int bn, int splits,
                                       jk_split_scratch* scratch, void* stream) {
    size_t x_rows = 0;
    jk_status st = check_grouped(w, x, x_dtype, x_len, g, out, out_len, &x_rows);
    if (st != JK_OK) return st;
    const jk_plan plan{bm, bn, splits};
    if (bm == 0 || !plan_valid(plan, w, 1)) {
        char buf[160];
        snprintf(buf, sizeof buf, "grouped plan {bm %d, bn %d, splits %d} is not valid for %s", bm, bn, splits,
                 shape_str(w->type, w->experts, w->n, w->k).c_str());
        return fail(JK_ERR_INVALID, buf);
    }
    if (g->rows == 0 || g->max_jobs == 0) return JK_OK;
    const bool f16_weights = w->type == JK_TYPE_F16;
    if (f16_weights && x_dtype != JK_DTYPE_F16) return fail(JK_ERR_UNSUPPORTED, "FP16 weights need FP16 activations");
    if (!scratch) return fail(JK_ERR_INVALID, "grouped products need a scratch for the sorted activation rows");
    if (scratch->device != w->device) return fail(JK_ERR_INVALID, "scratch belongs to another device");
    DeviceGuard dg(w->device);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    // operand type: f16 activations stay f16, bf16 and f32 go to bf16 (as in jk_matmul_plan)
    const bool want_bf16 = x_dtype != JK_DTYPE_F16;
    // the sorted rows go after the stream-K flag words, which other products on this scratch
    // expect to find zero
    const size_t flags = jk::stream_k_flag_bytes(w->device);
    void* sbuf = nullptr;
    st = jk::scratch_reserve(scratch, flags + (g->rows * w->k * 2 + 255) / 256 * 256, &sbuf);
    if (st != JK_OK) return st;
    void* xs = static_cast<char*>(sbuf) + flags;
    st = jk::launch_gather_rows(x, x_dtype, x_rows, w->k, g->sorted, g->rows, g->in_div, xs, want_bf16, cs);
    if (st != JK_OK) return st;
    return jk::launch_gemm_grouped(w, xs, want_bf16, g->rows, g->sorted, g->offsets, g->jobs, g->max_jobs, bm, out,
                                   bm, bn == 256, cs);
}

extern "C" jk_status jk_matvec_grouped(const jk_qmatrix* w, const void* x, int x_dtype, size_t x_len,
                                       const jk_groups* g, float* out, size_t out_len, int mr, void* stream) {
    size_t x_rows = 0;
    jk_status st = check_grouped(w, x, x_dtype, x_len, g, out, out_len, &x_rows);
    if (st != JK_OK) return st;
    if (mr < 1 || mr > JK_GEMV_ROWS) {
        char buf[96];
        snprintf(buf, sizeof buf, "matvec_grouped takes job tiles of 1..%d rows (got %d)", JK_GEMV_ROWS, mr);
        return fail(JK_ERR_INVALID, buf);
    }
    if (g->rows == 0 || g->max_jobs == 0) return JK_OK;
    DeviceGuard dg(w->device);
    return jk::launch_gemv_grouped(w->view, x, x_dtype, x_rows, g->sorted, g->offsets, g->jobs, g->max_jobs,
                                   g->in_div, mr, g->rows, out, static_cast<cudaStream_t>(stream));
}

extern "C" jk_status jk_matmul(const jk_qmatrix* w, const void* x, int x_dtype, size_t x_len, size_t m, float* out,
                               size_t out_len, jk_split_scratch* scratch, void* stream) {
    jk_plan p;
    jk_status st = jk_plan_heuristic(w, m, 0, 0, &p);
    if (st != JK_OK) return st;
    if (p.splits > 1 && !scratch) p.splits = 1;  // no scratch given: keep the product in place
    return jk_matmul_plan(w, x, x_dtype, x_len, m, out, out_len, scratch, p, stream);
}

extern "C" jk_status jk_matmul_tiled(const jk_qmatrix* w, const void* x, int x_dtype, size_t x_len, size_t m,
                                     float* out, size_t out_len, int bm, int bn, void* stream) {
    jk_plan p{bm, bn, 1};
    return jk_matmul_plan(w, x, x_dtype, x_len, m, out, out_len, nullptr, p, stream);
}

extern "C" jk_status jk_f16_linear(const void* x_f16, size_t m, size_t k, const void* w_f16, size_t n, float* out,
                                   void* stream) {
    if (k % 64 || n % 64) {
        char buf[96];
        snprintf(buf, sizeof buf, "F16 [%zu, %zu] has an unsupported shape", n, k);
        return fail(JK_ERR_SHAPE, buf);
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    jk_qmatrix* w = nullptr;
    jk_status st = jk_qmatrix_f16_view(dev, n, k, w_f16, &w);
    if (st != JK_OK) return st;
    // Fixed row-invariant plan (kernels.rs:16-31): the activation-row tile grows with m, never split-K.
    jk_plan p{row_tile_for(m), 128, 1};
    st = jk_matmul_plan(w, x_f16, JK_DTYPE_F16, m * k, m, out, m * n, nullptr, p, stream);
    jk_qmatrix_destroy(w);
    return st;
}
