// qmr_matmul_affine_static: qmr_matmul_affine without any device allocation.
//
// Who needs it: a caller that must not allocate device memory once it is
// running.  A serving engine that reserves its whole HBM budget (weights, KV
// cache, activations) at start-up treats any later cudaMalloc as an error,
// because it can fail under that budget and because it synchronises the
// device in the middle of a decode step.  A foreign-language binding may
// also have no way to own, size or free a scratch buffer for the library.
// qmr_matmul_affine grows a per-stream scratch buffer with cudaMalloc on
// first use (and on growth); this entry point instead uses one fixed,
// file-scope device array per device.
//
// Limits and rules:
//  * the array holds kStaticScratchBytes (3 MiB): enough for every shape with
//    cols <= 32768 at batch <= 4 (any bit width and group); larger shapes are
//    rejected with QMR_ERANGE before anything is launched;
//  * there is one array per device, shared by every stream and thread: calls
//    that overlap in time (two streams, or two host threads) race on it and
//    must be serialised by the caller;
//  * the first call on each device does the set-up (it looks the array's
//    address up with that device current, clears the array and waits for
//    the device to finish the clear), so it should come before any stream
//    capture;
//  * the address is looked up once per device and kept for the life of the
//    process: the entry point does not survive cudaDeviceReset (which
//    unloads the module that holds the array).
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "qmr_internal.h"

namespace qmr {

namespace {

constexpr size_t kStaticScratchBytes = 3u << 20;
constexpr uint32_t kStaticMaxCols = 32768;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
void *g_static_addr[64] = {};

// Address of this device's array, set up on first use: cudaGetSymbolAddress
// with the device current, then the whole array cleared (the argmax keys and
// the split-tile counters in it must start at zero) and the device
// synchronised, so the clear has finished before any stream -- a
// non-blocking one included -- runs a kernel on the array.
int static_scratch(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return fail(QMR_EUNSUPPORTED, "device %d is beyond the 64 the static scratch covers", dev);
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (g_static_addr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess)
            return fail(QMR_ECUDA, "cudaGetSymbolAddress of the static scratch: %s", cudaGetErrorString(e));
        if (reinterpret_cast<uintptr_t>(p) % 256 != 0)
            return fail(QMR_ECUDA, "static scratch is not 256-byte aligned");
        e = cudaMemset(p, 0, kStaticScratchBytes);
        if (e != cudaSuccess) return fail(QMR_ECUDA, "clearing the static scratch: %s", cudaGetErrorString(e));
        e = cudaDeviceSynchronize();
        if (e != cudaSuccess)
            return fail(QMR_ECUDA, "waiting for the static scratch clear: %s", cudaGetErrorString(e));
        g_static_addr[dev] = p;
    }
    *out = g_static_addr[dev];
    return QMR_OK;
}

}  // namespace

int matmul_static(const void *w, const void *s, const void *b, const float *x, float *y, uint32_t rows,
                  uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, bool bf16, bool r2, int path,
                  cudaStream_t stream) {
    if (!fast_eligible(w, cols, bits, group))
        return run_generic(w, s, b, x, y, rows, cols, bits, group, batch, bf16, stream);  // uses no scratch
    const size_t need = scratch_bytes((int)bits, cols, batch);
    if (cols > kStaticMaxCols || need > kStaticScratchBytes)
        return fail(QMR_ERANGE,
                    "qmr_matmul_affine_static: cols %u at batch %u needs %zu bytes of scratch; the fixed static "
                    "scratch holds %zu (cols up to %u at batch 4)",
                    cols, batch, need, kStaticScratchBytes, kStaticMaxCols);
    void *base = nullptr;
    const int rc = static_scratch(&base);
    if (rc != QMR_OK) return rc;
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
    c.path = path;
    c.scratch = base;
    c.scratch_bytes = kStaticScratchBytes;
    return run_fast(c, stream);
}

}  // namespace qmr
