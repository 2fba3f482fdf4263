// The tensor-core streaming kernel and its activation prep, built once per
// bit width (QMR_MMA_BITS = 4 or 8) so the two halves compile in parallel.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>

#include "launch.h"

#ifndef QMR_MMA_BITS
#error "build with -DQMR_MMA_BITS=4 or -DQMR_MMA_BITS=8"
#endif

namespace qmr {

namespace {

constexpr int kBits = QMR_MMA_BITS;

template <int G>
int launch_prep_g(const float *x, uint32_t cols, uint32_t batch, int ngroups_pad, const MmaImageView &v,
                  cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((ngroups_pad + kPrepGroupsPerCta - 1) / kPrepGroupsPerCta), batch, 1);
    cfg.blockDim = dim3(4 * kPrepGroupsPerCta, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, mma_prep_kernel<kBits, G>, x, (int)cols, (int)batch, ngroups_pad, v);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "activation prep launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

// The shared-memory opt-in is a per-device function attribute: set it once per
// device for each instantiation.
template <typename Kern>
int opt_in_smem(Kern kern, std::atomic<uint64_t> &done) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(QMR_ECUDA, "cudaGetDevice failed");
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return QMR_OK;
    int max_optin = 0;
    cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, max_optin - (int)fa.sharedSizeBytes);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    done.fetch_or(bit, std::memory_order_acq_rel);
    return QMR_OK;
}

template <int G, int B, bool BF16, int EPI, int NW>
int launch_w(const MmaMaps &maps, const MmaArgs &a, const MmaPlan &p, bool overlap, cudaStream_t stream) {
    auto kern = mma_kernel<kBits, G, B, BF16, EPI, NW>;
    static std::atomic<uint64_t> opted{0};
    const int rc = opt_in_smem(kern, opted);
    if (rc != QMR_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)p.ctas, 1, 1);
    cfg.blockDim = dim3(32 * NW, 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (p.kc > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)p.kc;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    if (overlap) attr[na++] = pdl_attr();
    cfg.attrs = attr;
    cfg.numAttrs = na;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps, a);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "tensor-core kernel launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

template <int G, int B, bool BF16, int EPI>
int launch_t(const MmaMaps &m, const MmaArgs &a, const MmaPlan &p, bool overlap, cudaStream_t stream) {
    if (p.warps == kMmaWarps) return launch_w<G, B, BF16, EPI, kMmaWarps>(m, a, p, overlap, stream);
    // Two matrices per unit (gate/up), Q8 words and 128-column groups need
    // more registers than 12 warps leave; those never take the long plan.
    if constexpr (EPI != 1 && kBits == 4 && G <= 64)
        if (p.warps == kMmaWarpsLong) return launch_w<G, B, BF16, EPI, kMmaWarpsLong>(m, a, p, overlap, stream);
    return fail(QMR_EUNSUPPORTED, "no tensor-core kernel with %d warps", p.warps);
}

template <int G, bool BF16, int EPI>
int launch_b(const MmaMaps &m, const MmaArgs &a, const MmaPlan &p, uint32_t batch, bool ov, cudaStream_t stream) {
    switch (batch) {
        case 1: return launch_t<G, 1, BF16, EPI>(m, a, p, ov, stream);
        case 2: return launch_t<G, 2, BF16, EPI>(m, a, p, ov, stream);
        case 3: return launch_t<G, 3, BF16, EPI>(m, a, p, ov, stream);
        default: return launch_t<G, 4, BF16, EPI>(m, a, p, ov, stream);
    }
}

template <bool BF16, int EPI>
int launch_g(const MmaMaps &m, const MmaArgs &a, const MmaPlan &p, uint32_t group, uint32_t batch, bool ov,
             cudaStream_t stream) {
    switch (group) {
        case 32: return launch_b<32, BF16, EPI>(m, a, p, batch, ov, stream);
        case 64: return launch_b<64, BF16, EPI>(m, a, p, batch, ov, stream);
        default:
            // A Q8 window of 1024 columns needs 16 KiB slots, which the plan
            // never accepts; only Q4 instantiates group 128.
            if constexpr (kBits == 4) return launch_b<128, BF16, EPI>(m, a, p, batch, ov, stream);
            return fail(QMR_EUNSUPPORTED, "the tensor-core kernel does not take Q8 group 128");
    }
}

template <int EPI>
int launch_e(const MmaMaps &m, const MmaArgs &a, const MmaPlan &p, bool bf16, uint32_t group, uint32_t batch, bool ov,
             cudaStream_t stream) {
    return bf16 ? launch_g<true, EPI>(m, a, p, group, batch, ov, stream)
                : launch_g<false, EPI>(m, a, p, group, batch, ov, stream);
}

}  // namespace

#if QMR_MMA_BITS == 4
#define QMR_MMA_LAUNCH launch_mma4
#define QMR_MMA_PREP launch_mma_prep4
#else
#define QMR_MMA_LAUNCH launch_mma8
#define QMR_MMA_PREP launch_mma_prep8
#endif

int QMR_MMA_LAUNCH(const FastCall &c, const MmaPlan &p, const ScratchView &sv, const MmaImageView &v,
                   cudaStream_t stream) {
    const uint64_t row_words = (uint64_t)c.cols * kBits / 32;
    const uint64_t ngroups = c.cols / c.group;
    const uint32_t wg = (8 * c.group > 512 ? 8 * c.group : 512) / c.group;  // groups of one window
    const int msz = c.bf16 ? 2 : 4;
    MmaMaps maps;
    const int nm = c.epilogue == 1 ? 2 : 1;
    for (int q = 0; q < 2; ++q) {
        const bool second = q == 1 && nm == 2;
        const void *w = second ? c.w2 : c.w, *s = second ? c.s2 : c.s, *b = second ? c.b2 : c.b;
        int rc = tensor_map_2d(&maps.w[q], w, 4, row_words, c.rows, 32, kTileRows, true);
        if (rc == QMR_OK) rc = tensor_map_2d(&maps.s[q], s, msz, ngroups, c.rows, wg, kTileRows, false, c.meta_stride);
        if (rc == QMR_OK) rc = tensor_map_2d(&maps.b[q], b, msz, ngroups, c.rows, wg, kTileRows, false, c.meta_stride);
        if (rc != QMR_OK) return rc;
    }
    MmaArgs a = {};
    a.s = static_cast<const unsigned char *>(c.s);
    a.b = static_cast<const unsigned char *>(c.b);
    a.s2 = static_cast<const unsigned char *>(c.epilogue == 1 ? c.s2 : c.s);
    a.b2 = static_cast<const unsigned char *>(c.epilogue == 1 ? c.b2 : c.b);
    a.image = v.image;
    a.table = v.table;
    a.y = c.y;
    a.keys = sv.keys;
    a.done = sv.done;
    a.argmax = c.argmax;
    a.best_key_out = reinterpret_cast<unsigned long long *>(c.best_key);
    a.err = device_error_word();
    if (a.err == nullptr) return fail(QMR_ECUDA, "device error word is unavailable");
    a.rows = (int)c.rows;
    a.ngroups = (int)(c.cols / c.group);
    a.ngroups_pad = p.ngroups_pad;
    a.ystride = (int)(c.ystride != 0 ? c.ystride : c.rows);
    a.row_base = (int)c.row_base;
    if (c.ex != nullptr) {
        const QmrExchange &ex = *c.ex;
        a.xworld = (int)ex.world;
        a.xrank = (int)ex.rank;
        a.xepoch = ex.epoch;
        for (uint32_t p = 0; p < ex.world; ++p) {
            a.xflags[p] = ex.flags[p];
            a.xkeys[p] = reinterpret_cast<unsigned long long *>(ex.keys[p]);
            a.peer_y[p] = c.epilogue == 2 ? nullptr : ex.out[p] + ex.row_base;
        }
    }
    a.tiles = p.tiles;
    a.nwin = p.nwin;
    a.kc = p.kc;
    a.clusters = p.clusters;
    a.pieces = p.pieces;
    a.stages = p.stages;
    a.off_image = p.off_image;
    a.off_table = p.off_table;
    a.off_pieces = p.off_pieces;
    a.off_part = p.off_part;
    a.off_bars = p.off_bars;
    a.zero = 0u;
    a.row_scale = c.norm_w != nullptr ? v.row_scale : nullptr;
    a.resid = c.resid;
    a.x = c.x;
    a.norm_w = c.norm_w;
    a.eps = c.eps;
    a.build = c.build ? 1 : 0;
    a.red_slots = nullptr;
    a.red_flags = nullptr;
    a.red_epoch = nullptr;
    a.red_world = 0;
    a.x_out = nullptr;
    if (c.build && c.reduce != nullptr) {
        const QmrExchange &r = *c.reduce;
        a.red_slots = r.out[r.rank];
        a.red_flags = r.flags[r.rank];
        a.red_epoch = r.epoch;
        a.red_world = (int)r.world;
        a.x_out = c.x_out;
    }
    switch (c.epilogue) {
        case 0: return launch_e<0>(maps, a, p, c.bf16, c.group, c.batch, c.overlap, stream);
        case 1: return launch_e<1>(maps, a, p, c.bf16, c.group, c.batch, c.overlap, stream);
        default: return launch_e<2>(maps, a, p, c.bf16, c.group, c.batch, c.overlap, stream);
    }
}

#if QMR_MMA_BITS == 4
// Waits (one warp) until every rank has published this rank's current
// exchange epoch, then, for the head, merges the ranks' keys per RHS: the
// unsigned maximum is the highest logit under f32 total order with ties to
// the lowest index.  Bounded: after kWaitLimitNs it records kErrTimeoutPeer
// and returns.
__global__ void __launch_bounds__(32) exchange_wait_kernel(const unsigned int *flags, const unsigned int *epoch,
                                                           int world, const unsigned long long *keys, int batch,
                                                           int *argmax, unsigned long long *best_key,
                                                           unsigned int *err) {
    const int lane = threadIdx.x;
    const unsigned int e = *epoch;
    // After a wait has run out (a rank fell behind or stopped), later waits
    // return at once instead of each spending the full limit again.
    if (*(volatile unsigned int *)err != 0u) return;
    bool ok = true;
    if (lane < world) {
        const unsigned long long start = global_ns();
        for (;;) {
            unsigned int f;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(flags + lane) : "memory");
            if ((int)(f - e) >= 0) break;
            if (global_ns() - start > kWaitLimitNs) {
                ok = false;
                atomicCAS(err, 0u, kErrTimeoutPeer);
                break;
            }
            __nanosleep(200);
        }
    }
    if (!__all_sync(0xffffffffu, ok) || keys == nullptr || lane >= batch) return;
    // The lanes that acquired the flags are not the lanes that read the keys:
    // the keys are read with acquire semantics too, so each read is ordered
    // after the publishing rank's release of the flag this warp observed.
    __syncwarp();
    unsigned long long k = 0ull;
    for (int r = 0; r < world; ++r) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(keys + r * 4 + lane) : "memory");
        k = v > k ? v : k;
    }
    if (argmax) argmax[lane] = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
    if (best_key) best_key[lane] = k;
}

int launch_exchange_wait(const QmrExchange &ex, uint32_t batch, int32_t *argmax, uint64_t *best_key,
                         cudaStream_t stream) {
    unsigned int *err = device_error_word();
    if (err == nullptr) return fail(QMR_ECUDA, "device error word is unavailable");
    exchange_wait_kernel<<<1, 32, 0, stream>>>(ex.flags[ex.rank], ex.epoch, (int)ex.world,
                                               reinterpret_cast<const unsigned long long *>(ex.keys[ex.rank]),
                                               (int)batch, argmax, reinterpret_cast<unsigned long long *>(best_key),
                                               err);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "exchange wait launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

// How many clusters of kc CTAs can be resident at once.  Every plan holds
// more than half of an SM's shared memory (one CTA per SM), so the answer
// depends only on kc and on how the SMs group into GPCs: 148 SMs do not
// split into 37 co-resident clusters of 4.  Cached per (device, kc).
int mma_cluster_capacity(int kc) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || kc < 1 || kc > 8) return 0;
    static std::atomic<int> cache[64][9] = {};
    const int have = cache[dev][kc].load(std::memory_order_acquire);
    if (have != 0) return have;
    auto kern = mma_kernel<4, 64, 4, true, 0, kMmaWarps>;
    static std::atomic<uint64_t> opted{0};
    if (opt_in_smem(kern, opted) != QMR_OK) return 0;
    int max_optin = 0;
    cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return 0;
    const int sms = sm_count();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(sms / kc * kc), 1, 1);
    cfg.blockDim = dim3(32 * kMmaWarps, 1, 1);
    cfg.dynamicSmemBytes = (size_t)(max_optin - (int)fa.sharedSizeBytes);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)kc;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        return 0;
    }
    cache[dev][kc].store(n, std::memory_order_release);
    return n;
}
#endif

int QMR_MMA_PREP(const float *x, uint32_t cols, uint32_t group, uint32_t batch, int ngroups_pad,
                 const MmaImageView &v, cudaStream_t stream) {
    switch (group) {
        case 32: return launch_prep_g<32>(x, cols, batch, ngroups_pad, v, stream);
        case 64: return launch_prep_g<64>(x, cols, batch, ngroups_pad, v, stream);
        default: return launch_prep_g<128>(x, cols, batch, ngroups_pad, v, stream);
    }
}

}  // namespace qmr
