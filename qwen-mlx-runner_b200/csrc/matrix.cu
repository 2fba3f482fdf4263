// Launchers for the packed-affine kernels: kernel choice for B200, the
// activation scratch, and programmatic dependent launch of the streaming
// kernel after its prep pass.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>
#include <utility>

#include "matrix_kernels.cuh"
#include "qmr_internal.h"
#include "tma_stream.cuh"

namespace qmr {


namespace {

struct Scratch {
    void *base = nullptr;
    size_t bytes = 0;
};

std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;

constexpr size_t kScratchAlign = 256;

size_t align_up(size_t v) { return (v + kScratchAlign - 1) / kScratchAlign * kScratchAlign; }

}  // namespace

size_t scratch_bytes(int bits, uint32_t cols, uint32_t batch) {
    const size_t elems = 128 / bits;
    const size_t nchunks = (size_t)cols * bits / 128;
    const size_t nblocks = (nchunks + 31) / 32;
    const size_t xp = batch * nblocks * 32 * elems * sizeof(float);
    const size_t xs = batch * nchunks * sizeof(float4);
    return align_up(xp) + align_up(xs) + align_up(4 * sizeof(unsigned long long) + sizeof(unsigned int));
}

void scratch_layout(void *base, int bits, uint32_t cols, uint32_t batch, ScratchView *v) {
    const size_t elems = 128 / bits;
    const size_t nchunks = (size_t)cols * bits / 128;
    const size_t nblocks = (nchunks + 31) / 32;
    const size_t xp = align_up(batch * nblocks * 32 * elems * sizeof(float));
    const size_t xs = align_up(batch * nchunks * sizeof(float4));
    char *p = static_cast<char *>(base);
    v->xp = reinterpret_cast<float4 *>(p);
    v->xs = reinterpret_cast<float4 *>(p + xp);
    v->keys = reinterpret_cast<unsigned long long *>(p + xp + xs);
    v->counter = reinterpret_cast<unsigned int *>(v->keys + 4);
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
    const size_t want = need > scratch_bytes(4, 65536, 4) ? need : scratch_bytes(4, 65536, 4);
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
    const cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaMalloc of activation scratch failed: %s", cudaGetErrorString(e));
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

int log2i(uint32_t v) {
    int r = 0;
    while ((1u << r) < v) ++r;
    return r;
}

template <int BITS>
int launch_prep(const float *x, uint32_t cols, uint32_t batch, const ScratchView &sv, bool argmax,
                cudaStream_t stream) {
    constexpr int elems = Chunk<BITS>::elems;
    const int nchunks = (int)((uint64_t)cols * BITS / 128);
    const int tasks = (int)batch * nchunks;
    const int warps = (tasks * elems + 31) / 32;
    int blocks = (warps + 7) / 8;
    if (blocks < 1) blocks = 1;
    if (blocks > 1184) blocks = 1184;
    prep_kernel<BITS><<<blocks, 256, 0, stream>>>(x, (int)cols, (int)batch, nchunks, sv.xp, sv.xs,
                                                  argmax ? sv.keys : nullptr, sv.counter);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "prep launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

template <int BITS, int B, int R, bool BF16, int EPI>
int launch_stream_t(const StreamArgs &a, cudaStream_t stream) {
    const int warps = (a.rows + R - 1) / R;
    const int blocks = (warps + 7) / 8;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, stream_kernel<BITS, B, R, BF16, EPI>, a);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "stream kernel launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

// Rows per warp for each (block width, epilogue); `r2` forces two rows per
// warp (the reference's selective R2 schedule).  Results do not depend on it.
template <int BITS, bool BF16, int EPI>
int launch_stream_b(const StreamArgs &a, uint32_t batch, bool r2, cudaStream_t stream) {
    if (r2) {
        switch (batch) {
            case 1: return launch_stream_t<BITS, 1, 2, BF16, EPI>(a, stream);
            case 2: return launch_stream_t<BITS, 2, 2, BF16, EPI>(a, stream);
            case 3: return launch_stream_t<BITS, 3, 2, BF16, EPI>(a, stream);
            default: return launch_stream_t<BITS, 4, 2, BF16, EPI>(a, stream);
        }
    }
    if constexpr (EPI == 1) {
        switch (batch) {
            case 1: return launch_stream_t<BITS, 1, 2, BF16, EPI>(a, stream);
            case 2: return launch_stream_t<BITS, 2, 2, BF16, EPI>(a, stream);
            case 3: return launch_stream_t<BITS, 3, 2, BF16, EPI>(a, stream);
            default: return launch_stream_t<BITS, 4, 2, BF16, EPI>(a, stream);
        }
    } else {
        switch (batch) {
            case 1: return launch_stream_t<BITS, 1, 4, BF16, EPI>(a, stream);
            case 2: return launch_stream_t<BITS, 2, 4, BF16, EPI>(a, stream);
            case 3: return launch_stream_t<BITS, 3, 4, BF16, EPI>(a, stream);
            default: return launch_stream_t<BITS, 4, 2, BF16, EPI>(a, stream);
        }
    }
}

template <int EPI>
int launch_stream(const StreamArgs &a, int bits, bool bf16, uint32_t batch, bool r2, cudaStream_t stream) {
    if (bits == 4) {
        return bf16 ? launch_stream_b<4, true, EPI>(a, batch, r2, stream)
                    : launch_stream_b<4, false, EPI>(a, batch, r2, stream);
    }
    return bf16 ? launch_stream_b<8, true, EPI>(a, batch, r2, stream)
                : launch_stream_b<8, false, EPI>(a, batch, r2, stream);
}

constexpr int kTmaConsumers = 8;
constexpr int kTmaSliceChunks = 64;
constexpr int kTmaSmemBudget = 200 * 1024;

int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    return n;
}

template <int BITS, int B, int R, bool BF16, int EPI>
int launch_tma_t(const TmaArgs &a0, cudaStream_t stream) {
    constexpr int NM = (EPI == 1) ? 2 : 1;
    constexpr int TR = kTmaConsumers * R;
    TmaArgs a = a0;
    a.slice_chunks = kTmaSliceChunks;
    const StageLayout L = stage_layout(NM, TR, a.slice_chunks, a.group_shift, a.meta_bytes);
    int stages = kTmaSmemBudget / (int)L.stage_bytes;
    if (stages > 8) stages = 8;
    if (stages < 2) return fail(QMR_EUNSUPPORTED, "stage of %u bytes does not fit shared memory", L.stage_bytes);
    a.stages = stages;
    const size_t smem = (size_t)stages * L.stage_bytes + (size_t)stages * 2 * sizeof(uint64_t);
    auto kern = tma_stream_kernel<BITS, B, R, kTmaConsumers, BF16, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    int grid = (a.rows + TR - 1) / TR;
    const int sms = sm_count();
    if (grid > sms) grid = sms;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(32 * (kTmaConsumers + 1), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "TMA stream kernel launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

template <int BITS, bool BF16, int EPI>
int launch_tma_b(const TmaArgs &a, uint32_t batch, bool r2, cudaStream_t stream) {
    if constexpr (EPI == 1) {
        switch (batch) {
            case 1: return launch_tma_t<BITS, 1, 2, BF16, EPI>(a, stream);
            case 2: return launch_tma_t<BITS, 2, 2, BF16, EPI>(a, stream);
            case 3: return launch_tma_t<BITS, 3, 2, BF16, EPI>(a, stream);
            default: return launch_tma_t<BITS, 4, 2, BF16, EPI>(a, stream);
        }
    } else {
        if (r2 && EPI == 0) {
            switch (batch) {
                case 1: return launch_tma_t<BITS, 1, 2, BF16, EPI>(a, stream);
                case 2: return launch_tma_t<BITS, 2, 2, BF16, EPI>(a, stream);
                case 3: return launch_tma_t<BITS, 3, 2, BF16, EPI>(a, stream);
                default: return launch_tma_t<BITS, 4, 2, BF16, EPI>(a, stream);
            }
        }
        switch (batch) {
            case 1: return launch_tma_t<BITS, 1, 4, BF16, EPI>(a, stream);
            case 2: return launch_tma_t<BITS, 2, 4, BF16, EPI>(a, stream);
            case 3: return launch_tma_t<BITS, 3, 4, BF16, EPI>(a, stream);
            default: return launch_tma_t<BITS, 4, 4, BF16, EPI>(a, stream);
        }
    }
}

template <int EPI>
int launch_tma(const TmaArgs &a, int bits, bool bf16, uint32_t batch, bool r2, cudaStream_t stream) {
    if (bits == 4)
        return bf16 ? launch_tma_b<4, true, EPI>(a, batch, r2, stream) : launch_tma_b<4, false, EPI>(a, batch, r2, stream);
    return bf16 ? launch_tma_b<8, true, EPI>(a, batch, r2, stream) : launch_tma_b<8, false, EPI>(a, batch, r2, stream);
}

}  // namespace

int run_prepare(const float *x, uint32_t cols, uint32_t bits, uint32_t batch, void *base, bool argmax,
                cudaStream_t stream) {
    ScratchView sv;
    scratch_layout(base, (int)bits, cols, batch, &sv);
    return bits == 4 ? launch_prep<4>(x, cols, batch, sv, argmax, stream)
                     : launch_prep<8>(x, cols, batch, sv, argmax, stream);
}

bool tma_eligible(const FastCall &c) {
    const uint32_t gpc = c.group / (128 / c.bits);
    const uint64_t meta = c.bf16 ? 2 : 4;
    const uint64_t nchunks = (uint64_t)c.cols * c.bits / 128;
    if ((nchunks / gpc) * meta % 16 != 0) return false;            // metadata row bytes
    if ((kTmaSliceChunks / gpc) * meta % 16 != 0) return false;    // metadata slice bytes
    auto al = [](const void *p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
    return al(c.w) && al(c.s) && al(c.b) && al(c.w2) && al(c.s2) && al(c.b2);
}

int run_stream(const FastCall &c, void *base, cudaStream_t stream) {
    ScratchView sv;
    scratch_layout(base, (int)c.bits, c.cols, c.batch, &sv);
    if (!c.legacy_kernel && tma_eligible(c)) {
        TmaArgs t = {};
        t.w = static_cast<const uint8_t *>(c.w);
        t.s = static_cast<const uint8_t *>(c.s);
        t.b = static_cast<const uint8_t *>(c.b);
        t.w2 = static_cast<const uint8_t *>(c.w2);
        t.s2 = static_cast<const uint8_t *>(c.s2);
        t.b2 = static_cast<const uint8_t *>(c.b2);
        t.xp = sv.xp;
        t.xs = sv.xs;
        t.y = c.y;
        t.keys = sv.keys;
        t.counter = sv.counter;
        t.argmax = c.argmax;
        t.best_key_out = reinterpret_cast<unsigned long long *>(c.best_key);
        t.rows = (int)c.rows;
        t.nchunks = (int)((uint64_t)c.cols * c.bits / 128);
        t.group_shift = log2i(c.group / (128 / c.bits));
        t.meta_bytes = c.bf16 ? 2 : 4;
        t.ystride = (int)c.rows;
        t.row_base = (int)c.row_base;
        switch (c.epilogue) {
            case 0: return launch_tma<0>(t, (int)c.bits, c.bf16, c.batch, c.r2, stream);
            case 1: return launch_tma<1>(t, (int)c.bits, c.bf16, c.batch, c.r2, stream);
            default: return launch_tma<2>(t, (int)c.bits, c.bf16, c.batch, c.r2, stream);
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
    a.y = c.y;
    a.keys = sv.keys;
    a.counter = sv.counter;
    a.argmax = c.argmax;
    a.best_key_out = reinterpret_cast<unsigned long long *>(c.best_key);
    a.rows = (int)c.rows;
    a.nchunks = (int)((uint64_t)c.cols * c.bits / 128);
    a.group_shift = log2i(c.group / (128 / c.bits));
    a.ystride = (int)c.rows;
    a.row_base = (int)c.row_base;
    switch (c.epilogue) {
        case 0: return launch_stream<0>(a, (int)c.bits, c.bf16, c.batch, c.r2, stream);
        case 1: return launch_stream<1>(a, (int)c.bits, c.bf16, c.batch, c.r2, stream);
        default: return launch_stream<2>(a, (int)c.bits, c.bf16, c.batch, c.r2, stream);
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
    const int rc = run_prepare(c.x, c.cols, c.bits, c.batch, base, c.epilogue == 2, stream);
    if (rc != QMR_OK) return rc;
    return run_stream(c, base, stream);
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

int run_generic(const void *w, const void *s, const void *b, const float *x, float *y, uint32_t rows,
                uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, bool bf16,
                cudaStream_t stream) {
    const uint64_t threads = (uint64_t)rows * 32;
    const uint64_t blocks = (threads + 255) / 256;
    if (blocks > 0x7fffffffull) return fail(QMR_EINVAL, "too many rows for one launch");
    if (bf16)
        generic_kernel<true><<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, x, y,
                                                                   rows, cols, bits, group, batch);
    else
        generic_kernel<false><<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, x, y,
                                                                    rows, cols, bits, group, batch);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "generic launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

int run_embed(const void *w, const void *s, const void *b, uint32_t row, float *y, uint32_t cols,
              uint32_t bits, uint32_t group, bool bf16, cudaStream_t stream) {
    const unsigned blocks = (cols + 255) / 256;
    if (bf16)
        embed_kernel<true><<<blocks, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, y, row, cols, bits,
                                                       group);
    else
        embed_kernel<false><<<blocks, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, y, row, cols, bits,
                                                        group);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "embed launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

}  // namespace qmr
