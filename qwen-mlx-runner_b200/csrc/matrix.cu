// Launchers for the packed-affine kernels: kernel choice and launch shape for
// B200, the prepared-activation scratch, and programmatic dependent launch of
// the streaming kernel behind its prep pass.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "matrix_kernels.cuh"
#include "qmr_internal.h"
#include "launch.h"

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



size_t prepared_floats(int bits, uint32_t cols, uint32_t batch) {
    const size_t nchunks = (size_t)cols * bits / 128;
    const size_t nblocks = (nchunks + kBlockChunks - 1) / kBlockChunks;
    const size_t bf = bits == 4 ? prepared_block_floats<4>() : prepared_block_floats<8>();
    return batch * nblocks * bf;
}

// Bytes of the MMA-path activations: 8 RHS-part columns of fp16 per input
// column, then the group sums (sized for the smallest group, 32).
size_t mma_prepared_bytes(uint32_t cols, uint32_t batch) {
    return align_up((size_t)cols * 8 * sizeof(__half)) + align_up((size_t)batch * (cols / 32) * sizeof(float));
}

// The activation region holds either path's layout.
size_t prepared_region(int bits, uint32_t cols, uint32_t batch) {
    const size_t a = align_up(prepared_floats(bits, cols, batch) * sizeof(float));
    const size_t b = mma_prepared_bytes(cols, batch);
    return a > b ? a : b;
}

void scratch_layout(void *base, int bits, uint32_t cols, uint32_t batch, ScratchView *v, MmaPrepView *mv = nullptr) {
    char *p = static_cast<char *>(base);
    v->xp = reinterpret_cast<float *>(p);
    if (mv != nullptr) {
        mv->xh = reinterpret_cast<__half *>(p);
        mv->xs = reinterpret_cast<float *>(p + align_up((size_t)cols * 8 * sizeof(__half)));
    }
    p += prepared_region(bits, cols, batch);
    v->cf = reinterpret_cast<float *>(p);
    if (mv != nullptr) mv->cf = v->cf;
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
    return prepared_region(bits, cols, batch) + align_up(8 * sizeof(float)) +
           align_up(4 * sizeof(unsigned long long) + sizeof(unsigned int)) +
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

cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    return attr;
}

int launch_mma_prep_bits(int bits, const float *x, uint32_t cols, uint32_t group, uint32_t batch,
                         const MmaPrepView &v, cudaStream_t stream) {
    return bits == 4 ? launch_mma_prep4(x, cols, group, batch, v, stream)
                     : launch_mma_prep8(x, cols, group, batch, v, stream);
}

int launch_mma_bits(int bits, const MmaArgs &a, bool bf16, uint32_t group, uint32_t batch, int epi, bool overlap,
                    cudaStream_t stream) {
    return bits == 4 ? launch_mma4(a, bf16, group, batch, epi, overlap, stream)
                     : launch_mma8(a, bf16, group, batch, epi, overlap, stream);
}

int run_prepare(const float *x, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, void *base, int path,
                cudaStream_t stream) {
    ScratchView sv;
    MmaPrepView mv;
    scratch_layout(base, (int)bits, cols, batch, &sv, &mv);
    if (path == kPathMma) {
        // The argmax keys and the CTA counter start each call at zero.
        const cudaError_t e = cudaMemsetAsync(sv.keys, 0, 4 * sizeof(unsigned long long) + sizeof(unsigned int), stream);
        if (e != cudaSuccess) return fail(QMR_ECUDA, "clearing argmax keys: %s", cudaGetErrorString(e));
        return launch_mma_prep_bits((int)bits, x, cols, group, batch, mv, stream);
    }
    return launch_prep_fp32(x, cols, bits, batch, sv, stream);
}

int run_stream(const FastCall &c, void *base, cudaStream_t stream) {
    ScratchView sv;
    MmaPrepView mv;
    scratch_layout(base, (int)c.bits, c.cols, c.batch, &sv, &mv);
    const int ce = 128 / (int)c.bits;
    const int gpc = (int)c.group / ce;
    const int meta = c.bf16 ? 2 : 4;
    const int nchunks = (int)((uint64_t)c.cols * c.bits / 128);
    if (c.path == kPathMma) {
        MmaArgs a = {};
        a.w = static_cast<const uint32_t *>(c.w);
        a.w2 = static_cast<const uint32_t *>(c.w2);
        a.s = c.s;
        a.b = c.b;
        a.s2 = c.s2;
        a.b2 = c.b2;
        a.xh = mv.xh;
        a.xs = mv.xs;
        a.cf = mv.cf;
        a.y = c.y;
        a.keys = sv.keys;
        a.done = sv.done;
        a.argmax = c.argmax;
        a.best_key_out = reinterpret_cast<unsigned long long *>(c.best_key);
        a.rows = (int)c.rows;
        a.cols = (int)c.cols;
        a.ystride = (int)c.rows;
        a.row_base = (int)c.row_base;
        const int units = ((int)c.rows + 15) / 16;
        const int sms = sm_count();
        a.ranges = units < sms ? units : sms;
        return launch_mma_bits((int)c.bits, a, c.bf16, c.group, c.batch, c.epilogue, c.overlap, stream);
    }
    if (c.path == kPathTile && tile_eligible(c)) return launch_tile_call(c, sv, stream);
    StreamArgs a = {};
    a.w = static_cast<const uint4 *>(c.w);
    a.s = c.s;
    a.bias = c.b;
    a.w2 = static_cast<const uint4 *>(c.w2);
    a.s2 = c.s2;
    a.bias2 = c.b2;
    a.xp = sv.xp;
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
    return launch_reg(a, (int)c.bits, c.bf16, c.batch, c.epilogue, c.overlap, stream);
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
    const int rc = run_prepare(c.x, c.cols, c.bits, c.group, c.batch, base, c.path, stream);
    if (rc != QMR_OK) return rc;
    FastCall behind_prep = c;
    behind_prep.overlap = true;  // the preceding kernel is our prep, which writes no weights
    return run_stream(behind_prep, base, stream);
}

}  // namespace qmr
