// The tensor-core streaming kernel and its activation prep, built once per
// bit width (QMR_MMA_BITS = 4 or 8) so the two halves compile in parallel.
#include <cuda_runtime.h>

#include "launch.h"

#ifndef QMR_MMA_BITS
#error "build with -DQMR_MMA_BITS=4 or -DQMR_MMA_BITS=8"
#endif

namespace qmr {

namespace {

template <int G>
int launch_mma_prep(const float *x, uint32_t cols, uint32_t batch, const MmaPrepView &v, cudaStream_t stream) {
    mma_prep_kernel<QMR_MMA_BITS, G><<<batch, 512, 0, stream>>>(x, (int)cols, (int)batch, v);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "prep launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

template <int G, int B, bool BF16, int EPI>
int launch_mma_t(const MmaArgs &a, bool overlap, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.ranges, 1, 1);
    cfg.blockDim = dim3(32 * kMmaWarps, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = overlap ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, mma_kernel<QMR_MMA_BITS, G, B, BF16, EPI>, a);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "mma kernel launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

template <int G, bool BF16, int EPI>
int launch_mma_b(const MmaArgs &a, uint32_t batch, bool ov, cudaStream_t stream) {
    switch (batch) {
        case 1: return launch_mma_t<G, 1, BF16, EPI>(a, ov, stream);
        case 2: return launch_mma_t<G, 2, BF16, EPI>(a, ov, stream);
        case 3: return launch_mma_t<G, 3, BF16, EPI>(a, ov, stream);
        default: return launch_mma_t<G, 4, BF16, EPI>(a, ov, stream);
    }
}

template <bool BF16, int EPI>
int launch_mma_g(const MmaArgs &a, uint32_t group, uint32_t batch, bool ov, cudaStream_t stream) {
    switch (group) {
        case 32: return launch_mma_b<32, BF16, EPI>(a, batch, ov, stream);
        case 64: return launch_mma_b<64, BF16, EPI>(a, batch, ov, stream);
        default: return launch_mma_b<128, BF16, EPI>(a, batch, ov, stream);
    }
}

template <int EPI>
int launch_mma_e(const MmaArgs &a, bool bf16, uint32_t group, uint32_t batch, bool ov, cudaStream_t stream) {
    return bf16 ? launch_mma_g<true, EPI>(a, group, batch, ov, stream) : launch_mma_g<false, EPI>(a, group, batch, ov, stream);
}

}  // namespace

#if QMR_MMA_BITS == 4
#define QMR_MMA_LAUNCH launch_mma4
#define QMR_MMA_PREP launch_mma_prep4
#else
#define QMR_MMA_LAUNCH launch_mma8
#define QMR_MMA_PREP launch_mma_prep8
#endif

int QMR_MMA_LAUNCH(const MmaArgs &a, bool bf16, uint32_t group, uint32_t batch, int epi, bool overlap,
                   cudaStream_t stream) {
    switch (epi) {
        case 0: return launch_mma_e<0>(a, bf16, group, batch, overlap, stream);
        case 1: return launch_mma_e<1>(a, bf16, group, batch, overlap, stream);
        default: return launch_mma_e<2>(a, bf16, group, batch, overlap, stream);
    }
}

int QMR_MMA_PREP(const float *x, uint32_t cols, uint32_t group, uint32_t batch, const MmaPrepView &v,
                 cudaStream_t stream) {
    switch (group) {
        case 32: return launch_mma_prep<32>(x, cols, batch, v, stream);
        case 64: return launch_mma_prep<64>(x, cols, batch, v, stream);
        default: return launch_mma_prep<128>(x, cols, batch, v, stream);
    }
}

}  // namespace qmr
