// FP32 kernels: activation prep, register-streaming block matmul, the
// generic per-element kernel and the embed kernel.
#include <cuda_runtime.h>

#include "launch.h"

namespace qmr {

namespace {

template <int BITS>
int launch_prep(const float *x, uint32_t cols, uint32_t batch, const ScratchView &sv, cudaStream_t stream) {
    const int nchunks = (int)((uint64_t)cols * BITS / 128);
    prep_kernel<BITS><<<batch, 512, 0, stream>>>(x, (int)cols, nchunks, sv);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "prep launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}


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

}  // namespace

int launch_prep_fp32(const float *x, uint32_t cols, uint32_t bits, uint32_t batch, const ScratchView &sv,
                     cudaStream_t stream) {
    return bits == 4 ? launch_prep<4>(x, cols, batch, sv, stream) : launch_prep<8>(x, cols, batch, sv, stream);
}

int launch_reg(const StreamArgs &a, int bits, bool bf16, uint32_t batch, int epi, bool overlap, cudaStream_t stream) {
    switch (epi) {
        case 0: return launch_stream<0>(a, bits, bf16, batch, overlap, stream);
        case 1: return launch_stream<1>(a, bits, bf16, batch, overlap, stream);
        default: return launch_stream<2>(a, bits, bf16, batch, overlap, stream);
    }
}

namespace {

// copy_f32 (kernels/matmul_block.metal:315-318): y[i] = x[i], 16-byte vectors
// when both ends are 16-byte aligned.  Launched behind the previous kernel
// (programmatic dependent launch): it lets the next kernel launch at once and
// waits for the previous one before reading x or writing y.  y may be pinned
// host memory (unified addressing): then this is the device-to-host copy,
// written straight over the host link.
__global__ void __launch_bounds__(256) copy_f32_kernel(const float *__restrict__ x, float *__restrict__ y, uint32_t n) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x, nt = (size_t)gridDim.x * blockDim.x;
    size_t done = 0;
    if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0) {
        const size_t n4 = n / 4;
        for (size_t i = tid; i < n4; i += nt)
            reinterpret_cast<float4 *>(y)[i] = __ldcg(reinterpret_cast<const float4 *>(x) + i);
        done = n4 * 4;
    }
    for (size_t i = done + tid; i < n; i += nt) y[i] = __ldcg(x + i);
}

}  // namespace

int run_copy_f32(const float *x, float *y, uint32_t n, cudaStream_t stream) {
    const uint64_t vec = ((uint64_t)n + 3) / 4;
    uint64_t blocks = (vec + 255) / 256;
    const uint64_t cap = 4ull * (uint64_t)sm_count();
    if (blocks > cap) blocks = cap;
    if (blocks == 0) blocks = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, copy_f32_kernel, x, y, n);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "copy_f32 launch failed: %s", cudaGetErrorString(e));
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
