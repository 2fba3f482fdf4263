// Launchers for the packed-affine kernels: kernel choice and launch shape for
// B200, the prepared-activation scratch, and programmatic dependent launch of
// the streaming kernel behind its prep pass.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>
#include <utility>

#include "matrix_kernels.cuh"
#include "qmr_internal.h"
#include "rowlane.cuh"

namespace qmr {

namespace {

struct Scratch {
    void *base = nullptr;
    size_t bytes = 0;
};

std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

constexpr int kConsumers = 8;  // consumer warps of the row-lane kernel
constexpr int kSmemBudget = 220 * 1024;
constexpr int kMinRowsPerSm = 96;  // below this, split K across CTAs

int log2i(uint32_t v) {
    int r = 0;
    while ((1u << r) < v) ++r;
    return r;
}

int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    return n;
}

void scratch_layout(void *base, int bits, uint32_t cols, uint32_t batch, ScratchView *v) {
    const size_t nchunks = (size_t)cols * bits / 128;
    char *p = static_cast<char *>(base);
    v->xp = reinterpret_cast<float *>(p);
    p += align_up((size_t)batch * cols * sizeof(float));
    v->xs = reinterpret_cast<float *>(p);
    p += align_up((size_t)batch * nchunks * sizeof(float));
    v->cf = reinterpret_cast<float *>(p);
    p += align_up(8 * sizeof(float));
    v->keys = reinterpret_cast<unsigned long long *>(p);
    v->done = reinterpret_cast<unsigned int *>(p + 4 * sizeof(unsigned long long));
    p += align_up(4 * sizeof(unsigned long long) + sizeof(unsigned int));
    v->counters = reinterpret_cast<unsigned int *>(p);
    p += align_up(kCounterCount * sizeof(unsigned int));
    v->partial = reinterpret_cast<float *>(p);
}

}  // namespace

size_t scratch_bytes(int bits, uint32_t cols, uint32_t batch) {
    const size_t nchunks = (size_t)cols * bits / 128;
    return align_up((size_t)batch * cols * sizeof(float)) + align_up((size_t)batch * nchunks * sizeof(float)) +
           align_up(8 * sizeof(float)) + align_up(4 * sizeof(unsigned long long) + sizeof(unsigned int)) +
           align_up(kCounterCount * sizeof(unsigned int)) + align_up(kPartialFloats * sizeof(float));
}

// Per (device, stream) scratch.  The first call on a stream reserves enough
// for cols <= 65536 at batch 4; larger shapes grow it after draining the
// stream, which is not allowed while the stream is being captured.
int acquire_scratch(cudaStream_t stream, size_t need, void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(QMR_ECUDA, "cudaGetDevice failed");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    Scratch &s = g_scratch[{dev, stream}];
    if (s.bytes >= need) {
        *out = s.base;
        return QMR_OK;
    }
    const size_t floor_bytes = scratch_bytes(4, 65536, 4);
    const size_t want = need > floor_bytes ? need : floor_bytes;
    if (s.base != nullptr) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(stream, &cs);
        if (cs != cudaStreamCaptureStatusNone)
            return fail(QMR_EUNSUPPORTED,
                        "activation scratch must grow, which cannot happen during stream capture; "
                        "make one call with the largest shape before capturing");
        if (cudaStreamSynchronize(stream) != cudaSuccess) return fail(QMR_ECUDA, "stream synchronize failed");
        cudaFree(s.base);
        s.base = nullptr;
        s.bytes = 0;
    }
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaMalloc of activation scratch failed: %s", cudaGetErrorString(e));
    e = cudaMemset(p, 0, want);  // counters start at zero
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaMemset of activation scratch failed: %s", cudaGetErrorString(e));
    s.base = p;
    s.bytes = want;
    *out = p;
    return QMR_OK;
}

bool fast_eligible(const void *w, uint32_t cols, uint32_t bits, uint32_t group) {
    if (bits != 4 && bits != 8) return false;
    if (group != 32 && group != 64 && group != 128) return false;
    if (cols % group != 0) return false;
    if (((uint64_t)cols * bits / 8) % 16 != 0) return false;
    if (reinterpret_cast<uintptr_t>(w) % 16 != 0) return false;
    return true;
}

namespace {

template <int BITS>
int launch_prep(const float *x, uint32_t cols, uint32_t batch, const ScratchView &sv, cudaStream_t stream) {
    const int nchunks = (int)((uint64_t)cols * BITS / 128);
    prep_kernel<BITS><<<batch, 512, 0, stream>>>(x, (int)cols, nchunks, sv);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "prep launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    return attr;
}

// ---- register-streaming fallback ------------------------------------------

template <int BITS, int B, int R, bool BF16, int EPI>
int launch_stream_t(const StreamArgs &a, bool overlap, cudaStream_t stream) {
    const int warps = (a.rows + R - 1) / R;
    const int blocks = (warps + 7) / 8;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = overlap ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, stream_kernel<BITS, B, R, BF16, EPI>, a);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "stream kernel launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

template <int BITS, bool BF16, int EPI>
int launch_stream_b(const StreamArgs &a, uint32_t batch, bool ov, cudaStream_t stream) {
    switch (batch) {
        case 1: return launch_stream_t<BITS, 1, 2, BF16, EPI>(a, ov, stream);
        case 2: return launch_stream_t<BITS, 2, 2, BF16, EPI>(a, ov, stream);
        case 3: return launch_stream_t<BITS, 3, 2, BF16, EPI>(a, ov, stream);
        default: return launch_stream_t<BITS, 4, 2, BF16, EPI>(a, ov, stream);
    }
}

template <int EPI>
int launch_stream(const StreamArgs &a, int bits, bool bf16, uint32_t batch, bool ov, cudaStream_t stream) {
    if (bits == 4)
        return bf16 ? launch_stream_b<4, true, EPI>(a, batch, ov, stream)
                    : launch_stream_b<4, false, EPI>(a, batch, ov, stream);
    return bf16 ? launch_stream_b<8, true, EPI>(a, batch, ov, stream) : launch_stream_b<8, false, EPI>(a, batch, ov, stream);
}

// ---- row-lane TMA kernel ----------------------------------------------------

template <int BITS, int B, int R, bool BF16, int EPI>
int launch_rowlane_t(RowlaneArgs a, bool overlap, cudaStream_t stream) {
    constexpr int NM = (EPI == 1) ? 2 : 1;
    constexpr int TR = 32 * R;
    constexpr int CE = Chunk<BITS>::elems;
    const RowlaneLayout L = rowlane_layout(NM, TR, a.slice_chunks, CE, B, a.group_shift, a.meta_bytes);
    const size_t red = (size_t)(kConsumers + 1) * NM * B * R * 32 * sizeof(float);
    int stages = (int)((kSmemBudget - red) / (L.stage_bytes + 2 * sizeof(uint64_t)));
    if (stages > 8) stages = 8;
    if (stages < 2) return fail(QMR_EUNSUPPORTED, "a %u-byte stage does not fit shared memory", L.stage_bytes);
    a.stages = stages;
    const size_t smem = (size_t)stages * L.stage_bytes + (size_t)stages * 2 * sizeof(uint64_t) + red;
    // Split-K bookkeeping: at most 4 tiles per row range use the counters.
    const int rows_per_range = (a.rows + a.ranges - 1) / a.ranges;
    if (a.ksplit > 1 && ((rows_per_range + TR - 1) / TR > 4 || a.ranges > 256))
        return fail(QMR_EUNSUPPORTED, "split-K launch shape exceeds the counter space");
    auto kern = rowlane_kernel<BITS, B, R, kConsumers, BF16, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.ranges * a.ksplit, 1, 1);
    cfg.blockDim = dim3(32 * (kConsumers + 1), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = overlap ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "row-lane kernel launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

template <int BITS, bool BF16, int EPI>
int launch_rowlane_b(const RowlaneArgs &a, uint32_t batch, int R, bool ov, cudaStream_t stream) {
    if constexpr (EPI != 1) {
        if (R == 4) {
            switch (batch) {
                case 1: return launch_rowlane_t<BITS, 1, 4, BF16, EPI>(a, ov, stream);
                case 2: return launch_rowlane_t<BITS, 2, 4, BF16, EPI>(a, ov, stream);
                case 3: return launch_rowlane_t<BITS, 3, 4, BF16, EPI>(a, ov, stream);
                default: return launch_rowlane_t<BITS, 4, 4, BF16, EPI>(a, ov, stream);
            }
        }
    }
    switch (batch) {
        case 1: return launch_rowlane_t<BITS, 1, 2, BF16, EPI>(a, ov, stream);
        case 2: return launch_rowlane_t<BITS, 2, 2, BF16, EPI>(a, ov, stream);
        case 3: return launch_rowlane_t<BITS, 3, 2, BF16, EPI>(a, ov, stream);
        default: return launch_rowlane_t<BITS, 4, 2, BF16, EPI>(a, ov, stream);
    }
}

template <int EPI>
int launch_rowlane(const RowlaneArgs &a, int bits, bool bf16, uint32_t batch, int R, bool ov, cudaStream_t stream) {
    if (bits == 4)
        return bf16 ? launch_rowlane_b<4, true, EPI>(a, batch, R, ov, stream)
                    : launch_rowlane_b<4, false, EPI>(a, batch, R, ov, stream);
    return bf16 ? launch_rowlane_b<8, true, EPI>(a, batch, R, ov, stream)
                : launch_rowlane_b<8, false, EPI>(a, batch, R, ov, stream);
}

bool rowlane_eligible(const FastCall &c, int slice_chunks) {
    const uint32_t gpc = c.group / (128 / c.bits);
    const uint64_t meta = c.bf16 ? 2 : 4;
    const uint64_t nchunks = (uint64_t)c.cols * c.bits / 128;
    if (nchunks % 4 != 0) return false;                  // chunk-sum slices of 16-byte multiples
    if ((nchunks / gpc) * meta % 16 != 0) return false;  // metadata row bytes
    if (((uint64_t)slice_chunks / gpc) * meta % 16 != 0) return false;
    auto al = [](const void *p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
    return al(c.w) && al(c.s) && al(c.b) && al(c.w2) && al(c.s2) && al(c.b2);
}

}  // namespace

int run_prepare(const float *x, uint32_t cols, uint32_t bits, uint32_t batch, void *base, cudaStream_t stream) {
    ScratchView sv;
    scratch_layout(base, (int)bits, cols, batch, &sv);
    return bits == 4 ? launch_prep<4>(x, cols, batch, sv, stream) : launch_prep<8>(x, cols, batch, sv, stream);
}

int run_stream(const FastCall &c, void *base, cudaStream_t stream) {
    ScratchView sv;
    scratch_layout(base, (int)c.bits, c.cols, c.batch, &sv);
    const int ce = 128 / (int)c.bits;
    const int gpc = (int)c.group / ce;
    const int meta = c.bf16 ? 2 : 4;
    const int nchunks = (int)((uint64_t)c.cols * c.bits / 128);
    int slice_chunks = 2 * kConsumers;
    if (gpc * 16 / meta > slice_chunks) slice_chunks = gpc * 16 / meta;
    if (!c.legacy_kernel && rowlane_eligible(c, slice_chunks)) {
        const int NM = c.epilogue == 1 ? 2 : 1;
        const int sms = sm_count();
        const int nslices = (nchunks + slice_chunks - 1) / slice_chunks;
        int ksplit = 1;
        if ((int)c.rows < kMinRowsPerSm * sms) {
            ksplit = (kMinRowsPerSm * sms + (int)c.rows - 1) / (int)c.rows;
            if (ksplit > 4) ksplit = 4;
            if (ksplit > nslices) ksplit = nslices;
            while (ksplit > 1 && (size_t)ksplit * NM * c.batch * c.rows > kPartialFloats) --ksplit;
        }
        int ranges = sms / ksplit;
        if (ranges > (int)c.rows) ranges = (int)c.rows;
        if (ranges < 1) ranges = 1;
        const int rows_per_range = ((int)c.rows + ranges - 1) / ranges;
        const int R = (c.r2 || c.epilogue == 1 || rows_per_range <= 64) ? 2 : 4;
        RowlaneArgs a = {};
        a.w = static_cast<const uint8_t *>(c.w);
        a.s = static_cast<const uint8_t *>(c.s);
        a.b = static_cast<const uint8_t *>(c.b);
        a.w2 = static_cast<const uint8_t *>(c.w2);
        a.s2 = static_cast<const uint8_t *>(c.s2);
        a.b2 = static_cast<const uint8_t *>(c.b2);
        a.xp = sv.xp;
        a.xs = sv.xs;
        a.cf = sv.cf;
        a.y = c.y;
        a.partial = sv.partial;
        a.range_counter = sv.counters;
        a.done_counter = sv.done;
        a.keys = sv.keys;
        a.argmax = c.argmax;
        a.best_key_out = reinterpret_cast<unsigned long long *>(c.best_key);
        a.rows = (int)c.rows;
        a.nchunks = nchunks;
        a.group_shift = log2i((uint32_t)gpc);
        a.meta_bytes = meta;
        a.ystride = (int)c.rows;
        a.row_base = (int)c.row_base;
        a.ranges = ranges;
        a.ksplit = ksplit;
        a.slice_chunks = slice_chunks;
        switch (c.epilogue) {
            case 0: return launch_rowlane<0>(a, (int)c.bits, c.bf16, c.batch, R, c.overlap, stream);
            case 1: return launch_rowlane<1>(a, (int)c.bits, c.bf16, c.batch, R, c.overlap, stream);
            default: return launch_rowlane<2>(a, (int)c.bits, c.bf16, c.batch, R, c.overlap, stream);
        }
    }
    StreamArgs a = {};
    a.w = static_cast<const uint4 *>(c.w);
    a.s = c.s;
    a.bias = c.b;
    a.w2 = static_cast<const uint4 *>(c.w2);
    a.s2 = c.s2;
    a.bias2 = c.b2;
    a.xp = sv.xp;
    a.xs = sv.xs;
    a.cf = sv.cf;
    a.y = c.y;
    a.keys = sv.keys;
    a.done = sv.done;
    a.argmax = c.argmax;
    a.best_key_out = reinterpret_cast<unsigned long long *>(c.best_key);
    a.rows = (int)c.rows;
    a.nchunks = nchunks;
    a.group_shift = log2i((uint32_t)gpc);
    a.ystride = (int)c.rows;
    a.row_base = (int)c.row_base;
    switch (c.epilogue) {
        case 0: return launch_stream<0>(a, (int)c.bits, c.bf16, c.batch, c.overlap, stream);
        case 1: return launch_stream<1>(a, (int)c.bits, c.bf16, c.batch, c.overlap, stream);
        default: return launch_stream<2>(a, (int)c.bits, c.bf16, c.batch, c.overlap, stream);
    }
}

int run_fast(const FastCall &c, cudaStream_t stream) {
    const size_t need = scratch_bytes((int)c.bits, c.cols, c.batch);
    void *base = c.scratch;
    if (base == nullptr) {
        const int rc = acquire_scratch(stream, need, &base);
        if (rc != QMR_OK) return rc;
    } else if (c.scratch_bytes < need) {
        return fail(QMR_ERANGE, "scratch of %zu bytes is smaller than the %zu required", c.scratch_bytes, need);
    }
    const int rc = run_prepare(c.x, c.cols, c.bits, c.batch, base, stream);
    if (rc != QMR_OK) return rc;
    FastCall behind_prep = c;
    behind_prep.overlap = true;  // the preceding kernel is our prep, which writes no weights
    return run_stream(behind_prep, base, stream);
}

int device_error(int *code, bool clear) {
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_qmr_device_error, sizeof v);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "reading the device error word: %s", cudaGetErrorString(e));
    if (clear && v != 0) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_qmr_device_error, &zero, sizeof zero);
        if (e != cudaSuccess) return fail(QMR_ECUDA, "clearing the device error word: %s", cudaGetErrorString(e));
    }
    *code = (int)v;
    return QMR_OK;
}

int run_generic(const void *w, const void *s, const void *b, const float *x, float *y, uint32_t rows, uint32_t cols,
                uint32_t bits, uint32_t group, uint32_t batch, bool bf16, cudaStream_t stream) {
    const uint64_t threads = (uint64_t)rows * 32;
    const uint64_t blocks = (threads + 255) / 256;
    if (blocks > 0x7fffffffull) return fail(QMR_EINVAL, "too many rows for one launch");
    if (bf16)
        generic_kernel<true><<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, x, y, rows,
                                                                   cols, bits, group, batch);
    else
        generic_kernel<false><<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, x, y, rows,
                                                                    cols, bits, group, batch);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "generic launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

int run_embed(const void *w, const void *s, const void *b, uint32_t row, float *y, uint32_t cols, uint32_t bits,
              uint32_t group, bool bf16, cudaStream_t stream) {
    const unsigned blocks = (cols + 255) / 256;
    if (bf16)
        embed_kernel<true><<<blocks, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, y, row, cols, bits, group);
    else
        embed_kernel<false><<<blocks, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, y, row, cols, bits,
                                                        group);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "embed launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

}  // namespace qmr
