// C ABI of the packed-affine matrix path: the reference's dispatch-layer
// rules restated for a CUDA device (rucin93/qwen-mlx-runner v0.7.3,
// src/gpu.rs), then the B200 launchers.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/qmr.h"
#include "qmr_internal.h"

namespace qmr {

namespace {

thread_local std::string t_last_error;

struct Modes {
    bool reference = false;
    int gemv = QMR_GEMV_ALIGNED;
    bool meta_bf16 = false;
    int block = QMR_BLOCK_LEGACY;
    bool batched_delta = true;
    bool parallel_norm = false;
    bool parallel_attention = false;
    int stream_path = kPathMma;  // streaming kernel of the fast path
    bool initialised = false;
};

std::mutex g_modes_mu;
Modes g_modes;

Modes modes() {
    std::lock_guard<std::mutex> lock(g_modes_mu);
    return g_modes;
}

// ---- overflow-checked arithmetic (usize in the reference) -----------------
bool mul_ok(uint64_t a, uint64_t b, uint64_t *out) { return !__builtin_mul_overflow(a, b, out); }
bool add_ok(uint64_t a, uint64_t b, uint64_t *out) { return !__builtin_add_overflow(a, b, out); }

const char *gemv_name(int g) {
    return g == QMR_GEMV_PACKED4 ? "packed4" : (g == QMR_GEMV_STREAM ? "stream" : "aligned");
}
const char *block_name(int m) {
    return m == QMR_BLOCK_SHARED ? "shared" : (m == QMR_BLOCK_MLP_R2 ? "mlp-r2" : "legacy");
}

bool ends_with(const std::string &s, const char *suffix) {
    const size_t n = strlen(suffix);
    return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}
bool starts_with(const std::string &s, const char *prefix) { return s.rfind(prefix, 0) == 0; }

}  // namespace

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

// supported_bf16_quantization (src/gpu/metadata.rs:16-18).
static bool supported_bf16_quantization(uint32_t bits, uint64_t group) {
    return (bits == 4 || bits == 8) && (group == 32 || group == 64 || group == 128);
}

// dispatch_layout (src/gpu.rs:1041-1294).  Fills sizes and the expected
// logical thread count; returns QMR_OK or a QMR_E* code with a message.
static int dispatch_layout(const std::string &name, const uint32_t *p, size_t np,
                           std::vector<uint64_t> &sizes, uint64_t &threads) {
    size_t count;
    if (name == "matvec_f16" || name == "embed_f16" || name == "rms_norm" || name == "conv_silu" ||
        name == "split_q_gate" || name == "softmax")
        count = 2;
    else if (name == "matvec_affine" || name == "embed_affine" || name == "matvec_affine_bf16" ||
             name == "embed_affine_bf16" || name == "delta_step" || name == "attn_scores" ||
             name == "attn_values")
        count = 4;
    else if (name == "delta_norm" || name == "gated_rms" || name == "head_rms" || name == "kv_append" ||
             name == "matmul_f16")
        count = 3;
    else if (name == "rope" || name == "matmul_affine" || name == "matmul_affine_bf16" ||
             name == "delta_step_block")
        count = 5;
    else if (name == "add" || name == "swiglu" || name == "copy_f32")
        count = 1;
    else
        return fail(QMR_EUNSUPPORTED, "Unknown GPU kernel %s", name.c_str());
    if (np != count) return fail(QMR_EINVAL, "%s: expected %zu parameters", name.c_str(), count);

    auto n = [&](size_t i) -> uint64_t { return p[i]; };
    bool ok = true;
    int code = QMR_OK;
    auto product = [&](std::initializer_list<uint64_t> v) -> uint64_t {
        uint64_t acc = 1;
        for (uint64_t x : v) {
            if (!mul_ok(acc, x, &acc)) {
                if (ok) code = fail(QMR_ERANGE, "GPU shape overflow");
                ok = false;
                return 0;
            }
        }
        if (acc > 0xffffffffull) {
            if (ok) code = fail(QMR_ERANGE, "GPU element index overflow");
            ok = false;
            return 0;
        }
        return acc;
    };
    auto f = [&](uint64_t elements) -> uint64_t {
        uint64_t out;
        if (!mul_ok(elements, 4, &out)) {
            if (ok) code = fail(QMR_ERANGE, "GPU byte size overflow");
            ok = false;
            return 0;
        }
        return out;
    };
    auto positive = [&](std::initializer_list<size_t> idx) -> bool {
        for (size_t i : idx)
            if (p[i] == 0) {
                code = fail(QMR_EINVAL, "%s: dimensions must be nonzero", name.c_str());
                return false;
            }
        return true;
    };
    auto eps = [&](size_t i) -> bool {
        float v;
        memcpy(&v, &p[i], 4);
        if (!(std::isfinite(v) && v > 0.f)) {
            code = fail(QMR_EINVAL, "%s: epsilon must be finite and positive", name.c_str());
            return false;
        }
        return true;
    };
#define QMR_CHECK(cond)                        \
    do {                                       \
        if (!(cond)) return code;              \
        if (!ok) return code;                  \
    } while (0)
#define QMR_ENSURE(cond, c, ...)                      \
    do {                                              \
        if (!(cond)) return fail((c), __VA_ARGS__);   \
    } while (0)

    sizes.clear();
    if (name == "matvec_f16" || name == "embed_f16" || name == "matvec_affine" || name == "embed_affine" ||
        name == "matvec_affine_bf16" || name == "embed_affine_bf16") {
        QMR_CHECK(positive({1}));
        const bool embedding = starts_with(name, "embed");
        uint64_t rows;
        if (embedding) {
            QMR_ENSURE(add_ok(n(0), 1, &rows), QMR_ERANGE, "Embedding row overflow");
        } else {
            QMR_CHECK(positive({0}));
            rows = n(0);
        }
        const uint64_t total = product({rows, n(1)});
        QMR_CHECK(true);
        const uint64_t output = embedding ? n(1) : n(0);
        const bool bf16 = ends_with(name, "_bf16");
        if (ends_with(name, "affine") || bf16) {
            QMR_ENSURE((p[2] == 4 || p[2] == 8) && p[3] > 0, QMR_EINVAL, "Only affine 4/8-bit quantization supported");
            QMR_ENSURE(n(1) % (32 / n(2)) == 0 && n(1) % n(3) == 0, QMR_EINVAL, "Invalid packed matrix alignment");
            QMR_ENSURE(!bf16 || supported_bf16_quantization(p[2], n(3)), QMR_EINVAL,
                       "BF16 metadata supports only affine Q4/Q8 groups 32, 64 or 128");
            uint64_t meta;
            QMR_ENSURE(mul_ok(total / n(3), bf16 ? 2 : 4, &meta), QMR_ERANGE, "Affine metadata byte size overflow");
            uint64_t packed;
            QMR_ENSURE(mul_ok(total, n(2), &packed), QMR_ERANGE, "Packed byte size overflow");
            sizes = {packed / 8, meta, meta};
        } else {
            uint64_t dense;
            QMR_ENSURE(mul_ok(total, 2, &dense), QMR_ERANGE, "Dense byte size overflow");
            sizes = {dense};
        }
        if (!embedding) sizes.push_back(f(n(1)));
        sizes.push_back(f(output));
        threads = embedding ? output : product({output, 32});
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "matmul_affine" || name == "matmul_affine_bf16" || name == "matmul_f16") {
        QMR_CHECK(positive({0, 1}));
        const bool affine = name != "matmul_f16";
        const uint64_t batch = n(affine ? 4 : 2);
        QMR_ENSURE(batch >= 1 && batch <= 4, QMR_EINVAL, "Matrix blocks support one through four RHS");
        const uint64_t total = product({n(0), n(1)});
        QMR_CHECK(true);
        if (affine) {
            QMR_ENSURE(supported_bf16_quantization(p[2], n(3)), QMR_EINVAL,
                       "Matrix blocks support affine Q4/Q8 groups 32, 64 or 128");
            QMR_ENSURE(n(1) % (32 / n(2)) == 0 && n(1) % n(3) == 0, QMR_EINVAL, "Invalid packed matrix alignment");
            uint64_t meta;
            QMR_ENSURE(mul_ok(total / n(3), ends_with(name, "_bf16") ? 2 : 4, &meta), QMR_ERANGE,
                       "Affine block metadata byte size overflow");
            uint64_t packed;
            QMR_ENSURE(mul_ok(total, n(2), &packed), QMR_ERANGE, "Packed block byte size overflow");
            sizes = {packed / 8, meta, meta};
        } else {
            uint64_t dense;
            QMR_ENSURE(mul_ok(total, 2, &dense), QMR_ERANGE, "Dense block byte size overflow");
            sizes = {dense};
        }
        sizes.push_back(f(product({batch, n(1)})));
        sizes.push_back(f(product({batch, n(0)})));
        threads = product({n(0), 32});
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "copy_f32") {
        QMR_CHECK(positive({0}));
        sizes = {f(n(0)), f(n(0))};
        threads = n(0);
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "rms_norm") {
        QMR_CHECK(positive({0}));
        QMR_CHECK(eps(1));
        sizes = {f(n(0)), f(n(0)), f(n(0))};
        threads = 32;
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "add" || name == "swiglu") {
        QMR_CHECK(positive({0}));
        sizes = {f(n(0)), f(n(0)), f(n(0))};
        threads = n(0);
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "conv_silu") {
        QMR_CHECK(positive({0, 1}));
        sizes = {f(n(0)), f(product({n(0), n(1)})), f(product({n(0), n(1) - 1})), f(n(0))};
        threads = n(0);
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "delta_norm") {
        QMR_CHECK(positive({0, 1}));
        QMR_CHECK(eps(2));
        sizes = {f(product({2, n(0), n(1)}))};
        threads = product({n(0), 32});
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "delta_step" || name == "delta_step_block") {
        QMR_CHECK(positive({0, 1, 2, 3}));
        QMR_ENSURE(n(1) % n(0) == 0, QMR_EINVAL, "Value heads must be divisible by key heads");
        const uint64_t values = product({n(1), n(3)});
        const uint64_t keys2 = product({2, n(0), n(2)});
        QMR_CHECK(true);
        uint64_t qkv;
        QMR_ENSURE(add_ok(keys2, values, &qkv), QMR_ERANGE, "QKV shape overflow");
        QMR_ENSURE(qkv <= 0xffffffffull, QMR_ERANGE, "QKV index overflow");
        uint64_t batch = 1;
        if (name == "delta_step_block") {
            QMR_ENSURE(n(2) <= 128, QMR_EINVAL, "DeltaNet block key dimension must be <=128");
            QMR_ENSURE(n(4) >= 1 && n(4) <= 4, QMR_EINVAL, "DeltaNet block width must be 1..=4");
            batch = n(4);
        }
        sizes = {f(product({qkv, batch})), f(product({n(1), batch})), f(product({n(1), batch})), f(n(1)), f(n(1)),
                 f(product({values, n(2)})), f(product({values, batch}))};
        if (name == "delta_step_block") sizes.push_back(f(product({values, n(2), batch})));
        threads = product({values, 32});
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "gated_rms") {
        QMR_CHECK(positive({0, 1}));
        QMR_CHECK(eps(2));
        const uint64_t len = f(product({n(0), n(1)}));
        sizes = {len, len, f(n(1)), len};
        threads = product({n(0), 32});
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "head_rms") {
        QMR_CHECK(positive({0, 1}));
        QMR_CHECK(eps(2));
        sizes = {f(product({n(0), n(1)})), f(n(1))};
        threads = product({n(0), 32});
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "split_q_gate") {
        QMR_CHECK(positive({0, 1}));
        const uint64_t len = product({n(0), n(1)});
        sizes = {f(product({len, 2})), f(len), f(len)};
        threads = len;
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "rope") {
        QMR_CHECK(positive({0, 1, 2}));
        QMR_ENSURE(p[2] % 2 == 0 && p[2] <= p[1], QMR_EINVAL, "Invalid rotary dimension");
        float theta;
        memcpy(&theta, &p[4], 4);
        QMR_ENSURE(std::isfinite(theta) && theta > 0.f, QMR_EINVAL, "Invalid RoPE theta");
        sizes = {f(product({n(0), n(1)}))};
        threads = product({n(0), n(2) / 2});
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "kv_append") {
        QMR_CHECK(positive({0, 1}));
        const uint64_t len = product({n(0), n(1)});
        const uint64_t cap = product({n(2) + 1, len});
        sizes = {f(len), f(len), f(cap), f(cap)};
        threads = len;
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "attn_scores" || name == "attn_values") {
        QMR_CHECK(positive({0, 1, 2, 3}));
        QMR_ENSURE(n(0) % n(1) == 0, QMR_EINVAL, "Attention heads must be divisible by KV heads");
        const uint64_t q = f(product({n(0), n(2)}));
        const uint64_t kv = f(product({n(3), n(1), n(2)}));
        const uint64_t score = product({n(0), n(3)});
        if (name == "attn_scores") {
            sizes = {q, kv, f(score)};
            threads = product({score, 32});
        } else {
            sizes = {f(score), kv, q, q};
            threads = product({n(0), n(2)});
        }
        QMR_CHECK(true);
        return QMR_OK;
    }
    if (name == "softmax") {
        QMR_CHECK(positive({0, 1}));
        sizes = {f(product({n(0), n(1)}))};
        threads = product({n(0), 32});
        QMR_CHECK(true);
        return QMR_OK;
    }
#undef QMR_CHECK
#undef QMR_ENSURE
    return fail(QMR_EUNSUPPORTED, "Unknown GPU kernel %s", name.c_str());
}

// checked_buffer_range (src/gpu.rs:879-889).
static int checked_buffer_range(uint64_t offset, uint64_t minimum, uint64_t length) {
    if (offset % 4 != 0) return fail(QMR_EALIGN, "GPU buffer offsets must be 4-byte aligned");
    uint64_t end;
    if (!add_ok(offset, minimum, &end)) return fail(QMR_ERANGE, "GPU buffer view byte range overflow");
    if (end > length)
        return fail(QMR_ERANGE, "GPU buffer view ends at %llu bytes but buffer has %llu", (unsigned long long)end,
                    (unsigned long long)length);
    return QMR_OK;
}

// ranges_overlap (src/gpu.rs:891-894); views were overflow-checked first.
static bool ranges_overlap(uint64_t a, uint64_t a_len, uint64_t b, uint64_t b_len) {
    return a < b + b_len && b < a + a_len;
}

// specialized_matmul (src/gpu.rs:896-999).
static const char *specialized_matmul(const std::string &name, const uint32_t *p, bool aligned, int mode) {
    static const char *f16[] = {"matmul_f16_b1", "matmul_f16_b2", "matmul_f16_b3", "matmul_f16_b4"};
    if (name == "matmul_f16") return (p[2] >= 1 && p[2] <= 4) ? f16[p[2] - 1] : nullptr;
    const bool bf16 = ends_with(name, "_bf16");
    if (aligned && p[0] % 4 == 0 && p[1] % 512 == 0 && p[2] == 4 && p[3] == 64 &&
        (uint64_t)p[0] * p[1] <= 0x7fffffffull && (uint64_t)p[1] * p[4] <= 0x7fffffffull) {
        if (mode == QMR_BLOCK_MLP_R2 && name == "matmul_affine_bf16" && p[4] == 3 &&
            ((p[0] == 17408 && p[1] == 5120) || (p[0] == 5120 && p[1] == 17408)))
            return "matmul_q4_g64_b3_mlp_r2_aligned_bf16";
        if (mode == QMR_BLOCK_SHARED) {
            if (p[4] == 2) return bf16 ? "matmul_q4_g64_b2_shared_aligned_bf16" : "matmul_q4_g64_b2_shared_aligned";
            if (p[4] == 3) return bf16 ? "matmul_q4_g64_b3_shared_aligned_bf16" : "matmul_q4_g64_b3_shared_aligned";
        }
        static const char *al[] = {"matmul_q4_g64_b1_aligned", "matmul_q4_g64_b2_aligned",
                                   "matmul_q4_g64_b3_aligned", "matmul_q4_g64_b4_aligned"};
        static const char *al16[] = {"matmul_q4_g64_b1_aligned_bf16", "matmul_q4_g64_b2_aligned_bf16",
                                     "matmul_q4_g64_b3_aligned_bf16", "matmul_q4_g64_b4_aligned_bf16"};
        if (p[4] >= 1 && p[4] <= 4) return bf16 ? al16[p[4] - 1] : al[p[4] - 1];
        return nullptr;
    }
    if (!(p[2] == 4 || p[2] == 8) || !(p[3] == 32 || p[3] == 64 || p[3] == 128) || p[4] < 1 || p[4] > 4)
        return nullptr;
    // Names of the generic block table, e.g. matmul_q8_g64_b3_bf16.
    static thread_local char buf[64];
    snprintf(buf, sizeof buf, "matmul_q%u_g%u_b%u%s", p[2], p[3], p[4], bf16 ? "_bf16" : "");
    return buf;
}

// specialized_matvec / specialized_matvec_bf16 (src/gpu.rs:1003-1037).
static const char *specialized_matvec(const uint32_t *p, bool aligned, bool bf16) {
    aligned = aligned && p[0] % 4 == 0 && p[1] % 512 == 0 && (uint64_t)p[0] * p[1] <= 0x7fffffffull;
    const bool bits_ok = p[2] == 4 || p[2] == 8;
    const bool group_ok = p[3] == 32 || p[3] == 64 || p[3] == 128;
    if (!bits_ok || !group_ok) return nullptr;
    static thread_local char buf[64];
    if (bf16) {
        if (aligned && p[2] == 4 && p[3] == 64) return "matvec_q4_g64_aligned_bf16";
        snprintf(buf, sizeof buf, "matvec_q%u_g%u_bf16", p[2], p[3]);
        return buf;
    }
    if (aligned && p[2] == 4) {
        snprintf(buf, sizeof buf, "matvec_q4_g%u_aligned", p[3]);
        return buf;
    }
    snprintf(buf, sizeof buf, "matvec_q%u_g%u", p[2], p[3]);
    return buf;
}

static const char *stream_variant(uint32_t group) {
    switch (group) {
        case 32: return "matvec_q4_g32_stream";
        case 64: return "matvec_q4_g64_stream";
        case 128: return "matvec_q4_g128_stream";
        default: return nullptr;
    }
}

// BlockKernelMode::parse / parse_for_device (src/gpu.rs:49-78).
static int parse_block_mode(const char *device_name, const char *matmul, const char *delta, int *mode,
                            bool *batched) {
    const char *m = matmul ? matmul : (strcmp(device_name ? device_name : "", "Apple M5 Pro") == 0 ? "mlp-r2" : "legacy");
    const char *d = delta ? delta : "batched";
    if (strcmp(m, "legacy") == 0)
        *mode = QMR_BLOCK_LEGACY;
    else if (strcmp(m, "shared") == 0)
        *mode = QMR_BLOCK_SHARED;
    else if (strcmp(m, "mlp-r2") == 0)
        *mode = QMR_BLOCK_MLP_R2;
    else
        return fail(QMR_EINVAL, "QWEN_METAL_BLOCK_MATMUL must be legacy, shared or mlp-r2");
    if (strcmp(d, "sequential") != 0 && strcmp(d, "batched") != 0)
        return fail(QMR_EINVAL, "QWEN_METAL_BLOCK_DELTA must be sequential or batched");
    *batched = strcmp(d, "batched") == 0;
    return QMR_OK;
}

static int check_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return QMR_OK;
    return fail(QMR_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Launch one matrix product through the B200 kernels.
static int launch_matrix(const void *w, const void *s, const void *b, const float *x, float *y, uint32_t rows,
                         uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, bool bf16, bool reference,
                         bool r2, cudaStream_t stream) {
    if (!reference && fast_eligible(w, cols, bits, group)) {
        FastCall c = {};
        c.w = w;
        c.s = s;
        c.b = b;
        c.x = x;
        c.y = y;
        c.rows = rows;
        c.cols = cols;
        c.bits = bits;
        c.group = group;
        c.batch = batch;
        c.bf16 = bf16;
        c.r2 = r2;
        c.epilogue = 0;
        c.path = modes().stream_path;
        return run_fast(c, stream);
    }
    return run_generic(w, s, b, x, y, rows, cols, bits, group, batch, bf16, stream);
}

// The current modes as the decode engine needs them.
bool modes_meta_bf16() { return modes().meta_bf16; }
bool modes_gemv_aligned() { return modes().gemv == QMR_GEMV_ALIGNED && !modes().reference; }
int modes_stream_path() { return modes().stream_path; }

}  // namespace qmr

using namespace qmr;

extern "C" {

int qmr_abi_version(void) { return QMR_ABI_VERSION; }

const char *qmr_last_error(void) { return t_last_error.c_str(); }

int qmr_parse_block_mode(const char *device_name, const char *matmul, const char *delta, int *matmul_mode,
                         int *batched_delta) {
    int m = 0;
    bool b = true;
    const int rc = parse_block_mode(device_name, matmul, delta, &m, &b);
    if (rc != QMR_OK) return rc;
    if (matmul_mode) *matmul_mode = m;
    if (batched_delta) *batched_delta = b ? 1 : 0;
    return QMR_OK;
}

int qmr_init(int device, uint32_t flags) {
    auto env = [](const char *k) -> const char * { return getenv(k); };
    Modes m;
    const char *ref = env("QWEN_METAL_REFERENCE");
    m.reference = (flags & QMR_INIT_REFERENCE) != 0 || (ref != nullptr && strcmp(ref, "1") == 0);
    const char *gemv = env("QWEN_METAL_GEMV");
    if (gemv == nullptr) gemv = "aligned";
    if (strcmp(gemv, "packed4") == 0)
        m.gemv = QMR_GEMV_PACKED4;
    else if (strcmp(gemv, "aligned") == 0)
        m.gemv = QMR_GEMV_ALIGNED;
    else if (strcmp(gemv, "stream") == 0)
        m.gemv = QMR_GEMV_STREAM;
    else
        return fail(QMR_EINVAL, "QWEN_METAL_GEMV must be packed4, aligned or stream");
    const char *norm = env("QWEN_METAL_NORM");
    if (norm == nullptr) norm = "serial";
    if (strcmp(norm, "parallel") != 0 && strcmp(norm, "serial") != 0)
        return fail(QMR_EINVAL, "QWEN_METAL_NORM must be parallel or serial");
    m.parallel_norm = strcmp(norm, "parallel") == 0;
    const char *attn = env("QWEN_METAL_ATTN_VALUES");
    if (attn == nullptr) attn = "serial";
    if (strcmp(attn, "parallel") != 0 && strcmp(attn, "serial") != 0)
        return fail(QMR_EINVAL, "QWEN_METAL_ATTN_VALUES must be parallel or serial");
    m.parallel_attention = strcmp(attn, "parallel") == 0;
    const char *meta = env("QWEN_METAL_METADATA");
    if (meta == nullptr) meta = "f32";
    if (strcmp(meta, "f32") != 0 && strcmp(meta, "bf16") != 0)
        return fail(QMR_EINVAL, "QWEN_METAL_METADATA must be f32 or bf16");
    m.meta_bf16 = strcmp(meta, "bf16") == 0;
    int rc = check_cuda(cudaSetDevice(device), "cudaSetDevice");
    if (rc != QMR_OK) return rc;
    cudaDeviceProp prop;
    rc = check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (rc != QMR_OK) return rc;
    bool batched = true;
    rc = parse_block_mode(prop.name, env("QWEN_METAL_BLOCK_MATMUL"), env("QWEN_METAL_BLOCK_DELTA"), &m.block, &batched);
    if (rc != QMR_OK) return rc;
    m.batched_delta = batched;
    m.initialised = true;
    std::lock_guard<std::mutex> lock(g_modes_mu);
    m.stream_path = g_modes.stream_path;
    g_modes = m;
    return QMR_OK;
}

int qmr_set_modes(const char *gemv, const char *metadata, const char *block_matmul, const char *block_delta) {
    std::lock_guard<std::mutex> lock(g_modes_mu);
    Modes m = g_modes;
    if (gemv) {
        if (strcmp(gemv, "packed4") == 0)
            m.gemv = QMR_GEMV_PACKED4;
        else if (strcmp(gemv, "aligned") == 0)
            m.gemv = QMR_GEMV_ALIGNED;
        else if (strcmp(gemv, "stream") == 0)
            m.gemv = QMR_GEMV_STREAM;
        else
            return fail(QMR_EINVAL, "QWEN_METAL_GEMV must be packed4, aligned or stream");
    }
    if (metadata) {
        if (strcmp(metadata, "f32") != 0 && strcmp(metadata, "bf16") != 0)
            return fail(QMR_EINVAL, "QWEN_METAL_METADATA must be f32 or bf16");
        m.meta_bf16 = strcmp(metadata, "bf16") == 0;
    }
    if (block_matmul || block_delta) {
        int mode = m.block;
        bool batched = m.batched_delta;
        const int rc = parse_block_mode("", block_matmul ? block_matmul : block_name(m.block),
                                        block_delta ? block_delta : (m.batched_delta ? "batched" : "sequential"),
                                        &mode, &batched);
        if (rc != QMR_OK) return rc;
        m.block = mode;
        m.batched_delta = batched;
    }
    g_modes = m;
    return QMR_OK;
}

int qmr_get_modes(char *out, size_t out_len) {
    const Modes m = modes();
    const int n = snprintf(out, out_len, "gemv=%s,metadata=%s,block_matmul=%s,block_delta=%s,reference=%d",
                           m.reference ? "reference" : gemv_name(m.gemv), m.meta_bf16 ? "bf16" : "f32",
                           block_name(m.block), m.batched_delta ? "batched" : "sequential", m.reference ? 1 : 0);
    if (n < 0 || (size_t)n >= out_len) return fail(QMR_ERANGE, "mode string buffer too small");
    return QMR_OK;
}

int qmr_dispatch_layout(const char *name, const uint32_t *params, size_t nparams, uint64_t *sizes, size_t *count,
                        uint64_t *threads) {
    if (name == nullptr || (params == nullptr && nparams > 0)) return fail(QMR_EINVAL, "null argument");
    std::vector<uint64_t> s;
    uint64_t t = 0;
    const int rc = dispatch_layout(name, params, nparams, s, t);
    if (rc != QMR_OK) return rc;
    if (count) *count = s.size();
    if (sizes)
        for (size_t i = 0; i < s.size(); ++i) sizes[i] = s[i];
    if (threads) *threads = t;
    return QMR_OK;
}

int qmr_checked_buffer_range(uint64_t offset, uint64_t minimum, uint64_t length) {
    return checked_buffer_range(offset, minimum, length);
}

int qmr_select(const char *name, const uint32_t *params, size_t nparams, int aligned, int mode, char *out,
               size_t out_len) {
    if (name == nullptr || params == nullptr || out == nullptr) return fail(QMR_EINVAL, "null argument");
    const std::string n = name;
    const char *sel = nullptr;
    if (starts_with(n, "matmul_")) {
        if ((n == "matmul_f16" && nparams != 3) || (n != "matmul_f16" && nparams != 5))
            return fail(QMR_EINVAL, "%s: wrong parameter count", name);
        sel = specialized_matmul(n, params, aligned != 0, mode);
    } else if (n == "matvec_affine" || n == "matvec_affine_bf16") {
        if (nparams != 4) return fail(QMR_EINVAL, "%s: wrong parameter count", name);
        sel = specialized_matvec(params, aligned != 0, n == "matvec_affine_bf16");
    } else {
        return fail(QMR_EUNSUPPORTED, "no specialisation table for %s", name);
    }
    if (sel == nullptr) return fail(QMR_EUNSUPPORTED, "Unsupported specialization for %s", name);
    if (strlen(sel) + 1 > out_len) return fail(QMR_ERANGE, "name buffer too small");
    strcpy(out, sel);
    return QMR_OK;
}

int qmr_pack_bf16_exact(const float *values, uint64_t n, uint16_t *out) {
    for (uint64_t i = 0; i < n; ++i) {
        uint32_t u;
        memcpy(&u, &values[i], 4);
        if ((u & 0x7f800000u) == 0x7f800000u || (u & 0xffffu) != 0) return 0;
    }
    for (uint64_t i = 0; i < n; ++i) {
        uint32_t u;
        memcpy(&u, &values[i], 4);
        out[i] = (uint16_t)(u >> 16);
    }
    return 1;
}

int qmr_encode(const char *cname, const qmr_buffer *buffers, const uint64_t *offsets, size_t nbuffers,
               const uint32_t *params, size_t nparams, uint64_t threads, uint64_t group_size, void *stream_) {
    if (cname == nullptr || (buffers == nullptr && nbuffers > 0) || (params == nullptr && nparams > 0))
        return fail(QMR_EINVAL, "null argument");
    const Modes m = modes();
    if (!m.initialised) return fail(QMR_ENOTINIT, "qmr_init was not called");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const std::string name = cname;
    std::vector<uint64_t> sizes;
    uint64_t expected_threads = 0;
    int rc = dispatch_layout(name, params, nparams, sizes, expected_threads);
    if (rc != QMR_OK) return rc;
    if (m.reference && starts_with(name, "matmul_"))
        return fail(QMR_EUNSUPPORTED, "Block matrix dispatch is unavailable in reference mode");
    if (sizes.size() != nbuffers)
        return fail(QMR_EINVAL, "%s: expected %zu buffers, got %zu", cname, sizes.size(), nbuffers);
    auto off = [&](size_t i) -> uint64_t { return offsets ? offsets[i] : 0; };
    for (size_t i = 0; i < nbuffers; ++i) {
        rc = checked_buffer_range(off(i), sizes[i], buffers[i].length);
        if (rc != QMR_OK) return fail(rc, "%s: buffer %zu: %s", cname, i, qmr_last_error());
    }
    if (starts_with(name, "matmul_") || name == "copy_f32") {
        const size_t out = nbuffers - 1;
        for (size_t i = 0; i < out; ++i) {
            if (buffers[i].ptr == buffers[out].ptr) {
                const bool identical_copy = name == "copy_f32" && off(i) == off(out);
                if (!identical_copy && ranges_overlap(off(i), sizes[i], off(out), sizes[out]))
                    return fail(QMR_EOVERLAP, "%s: output overlaps input buffer %zu", cname, i);
            }
        }
    }
    if (name == "delta_step_block") {
        for (size_t out : {5, 6, 7})
            for (size_t i = 0; i < nbuffers; ++i)
                if (i != out && buffers[i].ptr == buffers[out].ptr &&
                    ranges_overlap(off(i), sizes[i], off(out), sizes[out]))
                    return fail(QMR_EOVERLAP, "%s: output %zu overlaps buffer %zu", cname, out, i);
    }
    if (m.reference && ends_with(name, "_bf16"))
        return fail(QMR_EUNSUPPORTED, "BF16 metadata dispatch is unavailable in reference mode");

    // Specialisation, as the reference names it (src/gpu.rs:693-746).
    const char *specialized = nullptr;
    bool r2 = false;
    if (starts_with(name, "matmul_")) {
        const bool aligned = m.gemv == QMR_GEMV_ALIGNED && off(0) % 8 == 0 &&
                             off(name == "matmul_f16" ? 1 : 3) % 16 == 0;
        specialized = specialized_matmul(name, params, aligned, m.block);
        if (specialized == nullptr) return fail(QMR_EUNSUPPORTED, "Unsupported matrix block specialization");
        r2 = strcmp(specialized, "matmul_q4_g64_b3_mlp_r2_aligned_bf16") == 0;
    } else if (name == "matvec_affine_bf16") {
        if (off(3) % 16 != 0) return fail(QMR_EALIGN, "BF16 matvec input requires a 16-byte aligned offset");
        specialized = specialized_matvec(params, m.gemv == QMR_GEMV_ALIGNED && off(0) % 8 == 0, true);
        if (specialized == nullptr) return fail(QMR_EUNSUPPORTED, "Unsupported BF16 affine quantization");
    } else if (!m.reference && name == "matvec_affine" && off(3) % 16 == 0) {
        const char *s = nullptr;
        if (m.gemv == QMR_GEMV_STREAM && off(0) % 8 == 0 && params[2] == 4 &&
            (uint64_t)params[0] * params[1] <= 0x7fffffffull)
            s = stream_variant(params[3]);
        specialized = s ? s : specialized_matvec(params, m.gemv == QMR_GEMV_ALIGNED && off(0) % 8 == 0, false);
    }
    if (threads != expected_threads)
        return fail(QMR_EINVAL, "%s: expected %llu threads, got %llu", cname, (unsigned long long)expected_threads,
                    (unsigned long long)threads);
    if (!(group_size >= 32 && group_size % 32 == 0 && group_size <= 1024))
        return fail(QMR_EINVAL, "%s: invalid threadgroup size %llu", cname, (unsigned long long)group_size);

    auto at = [&](size_t i) -> char * { return static_cast<char *>(buffers[i].ptr) + off(i); };
    if (name == "matvec_affine" || name == "matvec_affine_bf16" || name == "matmul_affine" ||
        name == "matmul_affine_bf16") {
        const bool bf16 = ends_with(name, "_bf16");
        const uint32_t batch = starts_with(name, "matmul_") ? params[4] : 1;
        // Reference mode and the unspecialised matvec run the per-element kernel.
        const bool reference_semantics = specialized == nullptr;
        return launch_matrix(at(0), at(1), at(2), reinterpret_cast<const float *>(at(3)),
                             reinterpret_cast<float *>(at(4)), params[0], params[1], params[2], params[3], batch,
                             bf16, reference_semantics, r2, stream);
    }
    if (name == "embed_affine" || name == "embed_affine_bf16")
        return run_embed(at(0), at(1), at(2), params[0], reinterpret_cast<float *>(at(3)), params[1], params[2],
                         params[3], ends_with(name, "_bf16"), stream);
    if (name == "copy_f32") {
        if (buffers[0].ptr == buffers[1].ptr && off(0) == off(1)) return QMR_OK;
        return run_copy_f32(reinterpret_cast<const float *>(at(0)), reinterpret_cast<float *>(at(1)), params[0],
                            stream);
    }
    return fail(QMR_EUNSUPPORTED, "%s: validated, but this build implements only the packed-affine matrix kernels",
                cname);
}

// ---- typed entry points ----------------------------------------------------

static int validate_typed(const char *name, const uint32_t *params, size_t np) {
    std::vector<uint64_t> sizes;
    uint64_t threads = 0;
    return dispatch_layout(name, params, np, sizes, threads);
}

int qmr_matvec_affine(const void *w, const void *scales, const void *biases, const float *x, float *y, uint32_t rows,
                      uint32_t cols, uint32_t bits, uint32_t group, int meta_bf16, void *stream) {
    const uint32_t p[4] = {rows, cols, bits, group};
    int rc = validate_typed(meta_bf16 ? "matvec_affine_bf16" : "matvec_affine", p, 4);
    if (rc != QMR_OK) return rc;
    const Modes m = modes();
    if (m.reference && meta_bf16) return fail(QMR_EUNSUPPORTED, "BF16 metadata dispatch is unavailable in reference mode");
    return launch_matrix(w, scales, biases, x, y, rows, cols, bits, group, 1, meta_bf16 != 0, m.reference, false,
                         static_cast<cudaStream_t>(stream));
}

int qmr_matmul_affine(const void *w, const void *scales, const void *biases, const float *x, float *y, uint32_t rows,
                      uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, int meta_bf16, void *stream) {
    const uint32_t p[5] = {rows, cols, bits, group, batch};
    int rc = validate_typed(meta_bf16 ? "matmul_affine_bf16" : "matmul_affine", p, 5);
    if (rc != QMR_OK) return rc;
    const Modes m = modes();
    if (m.reference) return fail(QMR_EUNSUPPORTED, "Block matrix dispatch is unavailable in reference mode");
    const char *sel = specialized_matmul(meta_bf16 ? "matmul_affine_bf16" : "matmul_affine", p,
                                         m.gemv == QMR_GEMV_ALIGNED, m.block);
    const bool r2 = sel != nullptr && strcmp(sel, "matmul_q4_g64_b3_mlp_r2_aligned_bf16") == 0;
    return launch_matrix(w, scales, biases, x, y, rows, cols, bits, group, batch, meta_bf16 != 0, false, r2,
                         static_cast<cudaStream_t>(stream));
}

int qmr_matmul_affine_static(const void *w, const void *scales, const void *biases, const float *x, float *y,
                             uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch,
                             int meta_bf16, void *stream) {
    const uint32_t p[5] = {rows, cols, bits, group, batch};
    int rc = validate_typed(meta_bf16 ? "matmul_affine_bf16" : "matmul_affine", p, 5);
    if (rc != QMR_OK) return rc;
    const Modes m = modes();
    if (m.reference) return fail(QMR_EUNSUPPORTED, "Block matrix dispatch is unavailable in reference mode");
    const char *sel = specialized_matmul(meta_bf16 ? "matmul_affine_bf16" : "matmul_affine", p,
                                         m.gemv == QMR_GEMV_ALIGNED, m.block);
    const bool r2 = sel != nullptr && strcmp(sel, "matmul_q4_g64_b3_mlp_r2_aligned_bf16") == 0;
    return matmul_static(w, scales, biases, x, y, rows, cols, bits, group, batch, meta_bf16 != 0, r2, m.stream_path,
                         static_cast<cudaStream_t>(stream));
}

int qmr_embed_affine(const void *w, const void *scales, const void *biases, uint32_t row, float *y, uint32_t cols,
                     uint32_t bits, uint32_t group, int meta_bf16, void *stream) {
    const uint32_t p[4] = {row, cols, bits, group};
    int rc = validate_typed(meta_bf16 ? "embed_affine_bf16" : "embed_affine", p, 4);
    if (rc != QMR_OK) return rc;
    return run_embed(w, scales, biases, row, y, cols, bits, group, meta_bf16 != 0, static_cast<cudaStream_t>(stream));
}

static int typed_fast_check(const void *w, uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch,
                            int meta_bf16, const char *what) {
    const uint32_t p[5] = {rows, cols, bits, group, batch};
    int rc = validate_typed(meta_bf16 ? "matmul_affine_bf16" : "matmul_affine", p, 5);
    if (rc != QMR_OK) return rc;
    if (!fast_eligible(w, cols, bits, group))
        return fail(QMR_EALIGN, "%s needs 16-byte aligned weights with 16-byte multiple rows", what);
    return QMR_OK;
}

int qmr_gateup_swiglu(const void *w_gate, const void *s_gate, const void *b_gate, const void *w_up, const void *s_up,
                      const void *b_up, const float *x, float *act, uint32_t rows, uint32_t cols, uint32_t bits,
                      uint32_t group, uint32_t batch, int meta_bf16, void *stream) {
    int rc = typed_fast_check(w_gate, rows, cols, bits, group, batch, meta_bf16, "qmr_gateup_swiglu");
    if (rc != QMR_OK) return rc;
    if (!fast_eligible(w_up, cols, bits, group))
        return fail(QMR_EALIGN, "qmr_gateup_swiglu needs 16-byte aligned up weights");
    FastCall c = {};
    c.w = w_gate;
    c.s = s_gate;
    c.b = b_gate;
    c.w2 = w_up;
    c.s2 = s_up;
    c.b2 = b_up;
    c.x = x;
    c.y = act;
    c.rows = rows;
    c.cols = cols;
    c.bits = bits;
    c.group = group;
    c.batch = batch;
    c.bf16 = meta_bf16 != 0;
    c.epilogue = 1;
    c.path = modes().stream_path;
    return run_fast(c, static_cast<cudaStream_t>(stream));
}

int qmr_head_argmax(const void *w, const void *scales, const void *biases, const float *x, float *logits,
                    int32_t *argmax, uint64_t *best_key, uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group,
                    uint32_t batch, int meta_bf16, uint32_t row_base, void *stream) {
    int rc = typed_fast_check(w, rows, cols, bits, group, batch, meta_bf16, "qmr_head_argmax");
    if (rc != QMR_OK) return rc;
    if ((uint64_t)row_base + rows > 0xffffffffull) return fail(QMR_ERANGE, "row_base + rows exceeds u32 token ids");
    FastCall c = {};
    c.w = w;
    c.s = scales;
    c.b = biases;
    c.x = x;
    c.y = logits;
    c.argmax = argmax;
    c.best_key = best_key;
    c.rows = rows;
    c.cols = cols;
    c.bits = bits;
    c.group = group;
    c.batch = batch;
    c.row_base = row_base;
    c.bf16 = meta_bf16 != 0;
    c.epilogue = 2;
    c.path = modes().stream_path;
    return run_fast(c, static_cast<cudaStream_t>(stream));
}

uint64_t qmr_prepared_bytes(uint32_t bits, uint32_t cols, uint32_t batch) {
    if ((bits != 4 && bits != 8) || batch < 1 || batch > 4 || cols == 0) return 0;
    return scratch_bytes((int)bits, cols, batch);
}

int qmr_prepare_activations(const float *x, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch,
                            void *prepared, uint64_t prepared_bytes, void *stream) {
    if (bits != 4 && bits != 8) return fail(QMR_EINVAL, "prepared activations support 4 or 8 bits");
    if (group != 32 && group != 64 && group != 128) return fail(QMR_EINVAL, "group must be 32, 64 or 128");
    if (cols % group != 0) return fail(QMR_EINVAL, "cols must be a multiple of the group");
    if (batch < 1 || batch > 4) return fail(QMR_EINVAL, "Matrix blocks support one through four RHS");
    if (cols == 0 || cols % (128 / bits) != 0)
        return fail(QMR_EINVAL, "cols must be a nonzero multiple of %u", 128 / bits);
    if (x == nullptr || prepared == nullptr) return fail(QMR_EINVAL, "null pointer");
    if (reinterpret_cast<uintptr_t>(prepared) % 256 != 0)
        return fail(QMR_EALIGN, "prepared activations must be 256-byte aligned");
    if (prepared_bytes < scratch_bytes((int)bits, cols, batch))
        return fail(QMR_ERANGE, "prepared buffer of %llu bytes is smaller than %llu", (unsigned long long)prepared_bytes,
                    (unsigned long long)scratch_bytes((int)bits, cols, batch));
    return run_prepare(x, cols, bits, group, batch, prepared, modes().stream_path, static_cast<cudaStream_t>(stream));
}

int qmr_matmul_prepared(const void *w, const void *scales, const void *biases, const void *prepared, float *y,
                        uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, int meta_bf16,
                        uint32_t flags, void *stream) {
    int rc = typed_fast_check(w, rows, cols, bits, group, batch, meta_bf16, "qmr_matmul_prepared");
    if (rc != QMR_OK) return rc;
    if (prepared == nullptr || reinterpret_cast<uintptr_t>(prepared) % 256 != 0)
        return fail(QMR_EALIGN, "prepared activations must be 256-byte aligned");
    const Modes m = modes();
    const uint32_t p[5] = {rows, cols, bits, group, batch};
    const char *sel = specialized_matmul(meta_bf16 ? "matmul_affine_bf16" : "matmul_affine", p,
                                         m.gemv == QMR_GEMV_ALIGNED, m.block);
    FastCall c = {};
    c.w = w;
    c.s = scales;
    c.b = biases;
    c.y = y;
    c.rows = rows;
    c.cols = cols;
    c.bits = bits;
    c.group = group;
    c.batch = batch;
    c.bf16 = meta_bf16 != 0;
    c.r2 = sel != nullptr && strcmp(sel, "matmul_q4_g64_b3_mlp_r2_aligned_bf16") == 0;
    c.epilogue = 0;
    c.path = m.stream_path;
    c.overlap = (flags & QMR_PREPARED_OVERLAP) != 0;
    return run_stream(c, const_cast<void *>(prepared), static_cast<cudaStream_t>(stream));
}

int qmr_copy_f32(const float *x, float *y, uint32_t n, void *stream) {
    if (n == 0) return fail(QMR_EINVAL, "copy_f32: dimensions must be nonzero");
    if (x == y) return QMR_OK;
    return run_copy_f32(x, y, n, static_cast<cudaStream_t>(stream));
}

int qmr_set_stream_path(const char *path) {
    if (path == nullptr) return fail(QMR_EINVAL, "null path");
    int p;
    if (strcmp(path, "mma") == 0)
        p = kPathMma;
    else if (strcmp(path, "tma") == 0)
        p = kPathTile;
    else if (strcmp(path, "registers") == 0)
        p = kPathRegisters;
    else
        return fail(QMR_EINVAL, "stream path must be mma, tma or registers");
    std::lock_guard<std::mutex> lock(g_modes_mu);
    g_modes.stream_path = p;
    return QMR_OK;
}

int qmr_device_error(int *code, int clear) {
    if (code == nullptr) return fail(QMR_EINVAL, "null code");
    return device_error(code, clear != 0);
}

int qmr_stream_sync(void *stream) {
    return check_cuda(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "stream synchronize");
}

// ---- sharded calls with the output exchange over peer memory -------------

int qmr_exchange_alloc(size_t bytes, void **dev_ptr) {
    if (dev_ptr == nullptr || bytes == 0) return fail(QMR_EINVAL, "qmr_exchange_alloc needs a size and an out pointer");
    *dev_ptr = nullptr;
    void *p = nullptr;
    int rc = check_cuda(cudaMalloc(&p, bytes), "exchange buffer allocation");
    if (rc != QMR_OK) return rc;
    rc = check_cuda(cudaMemset(p, 0, bytes), "exchange buffer clear");
    if (rc != QMR_OK) {
        cudaFree(p);
        return rc;
    }
    *dev_ptr = p;
    return QMR_OK;
}

int qmr_exchange_free(void *dev_ptr) { return check_cuda(cudaFree(dev_ptr), "exchange buffer free"); }

int qmr_ipc_handle(const void *dev_ptr, void *handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == QMR_IPC_HANDLE_BYTES, "IPC handle size");
    if (dev_ptr == nullptr || handle == nullptr) return fail(QMR_EINVAL, "qmr_ipc_handle: null pointer");
    cudaIpcMemHandle_t h;
    const int rc = check_cuda(cudaIpcGetMemHandle(&h, const_cast<void *>(dev_ptr)), "cudaIpcGetMemHandle");
    if (rc != QMR_OK) return rc;
    memcpy(handle, &h, sizeof(h));
    return QMR_OK;
}

int qmr_ipc_open(const void *handle, void **dev_ptr) {
    if (dev_ptr == nullptr || handle == nullptr) return fail(QMR_EINVAL, "qmr_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return check_cuda(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int qmr_ipc_close(void *dev_ptr) { return check_cuda(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle"); }

static int check_exchange(const QmrExchange *ex, bool head) {
    if (ex == nullptr) return fail(QMR_EINVAL, "null exchange");
    if (ex->world < 2 || ex->world > QMR_MAX_RANKS || ex->rank >= ex->world)
        return fail(QMR_EINVAL, "exchange needs 2..%d ranks and rank < world", QMR_MAX_RANKS);
    if (ex->epoch == nullptr) return fail(QMR_EINVAL, "exchange epoch word is null");
    for (uint32_t p = 0; p < ex->world; ++p) {
        if (ex->flags[p] == nullptr) return fail(QMR_EINVAL, "exchange flags of rank %u are null", p);
        if (head ? ex->keys[p] == nullptr : ex->out[p] == nullptr)
            return fail(QMR_EINVAL, "exchange %s of rank %u are null", head ? "keys" : "outputs", p);
    }
    return QMR_OK;
}

int qmr_matmul_affine_exchange(const void *w, const void *scales, const void *biases, const float *x, uint32_t rows,
                               uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, int meta_bf16,
                               const QmrExchange *ex, void *stream) {
    int rc = typed_fast_check(w, rows, cols, bits, group, batch, meta_bf16, "qmr_matmul_affine_exchange");
    if (rc == QMR_OK) rc = check_exchange(ex, false);
    if (rc != QMR_OK) return rc;
    if ((uint64_t)ex->row_base + rows > ex->total_rows) return fail(QMR_ERANGE, "shard rows exceed the full output");
    FastCall c = {};
    c.w = w;
    c.s = scales;
    c.b = biases;
    c.x = x;
    c.y = ex->out[ex->rank] + ex->row_base;
    c.ystride = ex->total_rows;
    c.rows = rows;
    c.cols = cols;
    c.bits = bits;
    c.group = group;
    c.batch = batch;
    c.bf16 = meta_bf16 != 0;
    c.epilogue = 0;
    c.path = kPathMma;
    c.ex = ex;
    return run_fast(c, static_cast<cudaStream_t>(stream));
}

int qmr_gateup_swiglu_exchange(const void *w_gate, const void *s_gate, const void *b_gate, const void *w_up,
                               const void *s_up, const void *b_up, const float *x, uint32_t rows, uint32_t cols,
                               uint32_t bits, uint32_t group, uint32_t batch, int meta_bf16, const QmrExchange *ex,
                               void *stream) {
    int rc = typed_fast_check(w_gate, rows, cols, bits, group, batch, meta_bf16, "qmr_gateup_swiglu_exchange");
    if (rc == QMR_OK && !fast_eligible(w_up, cols, bits, group))
        rc = fail(QMR_EALIGN, "qmr_gateup_swiglu_exchange needs 16-byte aligned up weights");
    if (rc == QMR_OK) rc = check_exchange(ex, false);
    if (rc != QMR_OK) return rc;
    if ((uint64_t)ex->row_base + rows > ex->total_rows) return fail(QMR_ERANGE, "shard rows exceed the full output");
    FastCall c = {};
    c.w = w_gate;
    c.s = s_gate;
    c.b = b_gate;
    c.w2 = w_up;
    c.s2 = s_up;
    c.b2 = b_up;
    c.x = x;
    c.y = ex->out[ex->rank] + ex->row_base;
    c.ystride = ex->total_rows;
    c.rows = rows;
    c.cols = cols;
    c.bits = bits;
    c.group = group;
    c.batch = batch;
    c.bf16 = meta_bf16 != 0;
    c.epilogue = 1;
    c.path = kPathMma;
    c.ex = ex;
    return run_fast(c, static_cast<cudaStream_t>(stream));
}

int qmr_head_argmax_exchange(const void *w, const void *scales, const void *biases, const float *x, float *logits,
                             uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch,
                             int meta_bf16, const QmrExchange *ex, void *stream) {
    int rc = typed_fast_check(w, rows, cols, bits, group, batch, meta_bf16, "qmr_head_argmax_exchange");
    if (rc == QMR_OK) rc = check_exchange(ex, true);
    if (rc != QMR_OK) return rc;
    if ((uint64_t)ex->row_base + rows > 0xffffffffull) return fail(QMR_ERANGE, "row_base + rows exceeds u32 token ids");
    FastCall c = {};
    c.w = w;
    c.s = scales;
    c.b = biases;
    c.x = x;
    c.y = logits;
    c.rows = rows;
    c.cols = cols;
    c.bits = bits;
    c.group = group;
    c.batch = batch;
    c.row_base = ex->row_base;
    c.bf16 = meta_bf16 != 0;
    c.epilogue = 2;
    c.path = kPathMma;
    c.ex = ex;
    return run_fast(c, static_cast<cudaStream_t>(stream));
}

int qmr_exchange_wait(const QmrExchange *ex, uint32_t batch, int32_t *argmax, uint64_t *best_key, void *stream) {
    const bool head = ex != nullptr && ex->keys[0] != nullptr;
    int rc = check_exchange(ex, head);
    if (rc != QMR_OK) return rc;
    if (batch < 1 || batch > 4) return fail(QMR_EINVAL, "Matrix blocks support one through four RHS");
    return launch_exchange_wait(*ex, batch, head ? argmax : nullptr, head ? best_key : nullptr,
                                static_cast<cudaStream_t>(stream));
}

}  // extern "C"
