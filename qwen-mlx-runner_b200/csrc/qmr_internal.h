// Internal interfaces shared by the C ABI (abi.cpp) and the launchers (matrix.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/qmr.h"

namespace qmr {

// Record a formatted message for qmr_last_error() and return `code`.
int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));

// One call of the streaming path (prep + streaming kernel).
struct FastCall {
    const void *w, *s, *b;     // matrix (gate for epilogue 1)
    const void *w2, *s2, *b2;  // up matrix for epilogue 1
    const float *x;
    float *y;                  // outputs (activations for epilogue 1, logits for 2)
    int32_t *argmax;           // epilogue 2
    uint64_t *best_key;        // epilogue 2
    uint32_t rows, cols, bits, group, batch, row_base;
    bool bf16;
    bool r2;                   // two rows per lane (the selective R2 schedule)
    int epilogue;              // 0 plain, 1 swiglu, 2 head argmax
    int path;                  // kPathMma, kPathTile or kPathRegisters
    bool overlap;              // programmatic dependent launch behind the previous kernel
    void *scratch;             // caller scratch or nullptr for the per-stream pool
    size_t scratch_bytes;
    uint32_t ystride;          // output row stride per RHS (0: rows)
    const QmrExchange *ex;     // output exchange over peer memory, or nullptr
    // Fused decode-step work (tensor-core path only): RMSNorm of x with
    // weight norm_w folded into the activation prep and the output factor,
    // and a residual added to every output (resid may equal y).
    const float *norm_w;
    float eps;
    const float *resid;
    // Metadata elements per row (0: cols / group).  A larger, 8-aligned
    // stride lets a column slice of a matrix keep 16-byte metadata rows;
    // tensor-core path only.
    uint32_t meta_stride;
    // An exchange of partial sums to all-reduce into x before it is used:
    // every rank's epoch is awaited, the slots [batch][world][cols] are
    // added to x in rank order and the reduced x is written to x_out (which
    // may be x itself only when the prep kernel runs); tensor-core path only.
    const QmrExchange *reduce;
    float *x_out;
    // The caller clears its scratch after any failed call, so calls with
    // the argmax or exchange epilogue may build their image in-kernel too.
    bool counted_build;
    // Set by run_fast: the streaming CTAs build the activation image in
    // their prologue from x (no prep kernel, no prepared image).
    bool build;
    // Optional: run_fast adds the number of kernels it launched.
    uint32_t *launch_count;
};
// The tensor-core path takes this call with the fused RMSNorm / residual
// epilogue (false: the caller must run them as separate kernels).
bool fused_supported(const FastCall &c);

// Streaming kernels of the fast path.
constexpr int kPathMma = 0;        // tensor-core weight streaming (default)
constexpr int kPathTile = 1;       // FP32 warp-specialised TMA pipeline
constexpr int kPathRegisters = 2;  // FP32 register streaming

// Fast (prep + streaming) path possible: Q4/Q8, group 32/64/128, 16-byte
// aligned weights with 16-byte multiple rows.
bool fast_eligible(const void *w, uint32_t cols, uint32_t bits, uint32_t group);
// Bytes of the prepared-activation buffer for (bits, cols, batch).
size_t scratch_bytes(int bits, uint32_t cols, uint32_t batch);
int acquire_scratch(cudaStream_t stream, size_t need, void **out);

int run_fast(const FastCall &c, cudaStream_t stream);
int run_prepare(const float *x, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, void *base, int path,
                cudaStream_t stream);
int run_stream(const FastCall &c, void *base, cudaStream_t stream);
int run_copy_f32(const float *x, float *y, uint32_t n, cudaStream_t stream);
int run_generic(const void *w, const void *s, const void *b, const float *x, float *y, uint32_t rows,
                uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, bool bf16, cudaStream_t stream);
int run_embed(const void *w, const void *s, const void *b, uint32_t row, float *y, uint32_t cols, uint32_t bits,
              uint32_t group, bool bf16, cudaStream_t stream);
int device_error(int *code, bool clear);
// The bounded wait for every rank's current exchange epoch (+ key merge).
int launch_exchange_wait(const QmrExchange &ex, uint32_t batch, int32_t *argmax, uint64_t *best_key,
                         cudaStream_t stream);
// Library modes (abi.cpp): QWEN_METAL_METADATA=bf16, QWEN_METAL_GEMV=aligned
// (and not reference mode), the selected streaming kernel.
bool modes_meta_bf16();
bool modes_gemv_aligned();
int modes_stream_path();
// qmr_matmul_affine on the fixed per-device static scratch (static_scratch.cu).
int matmul_static(const void *w, const void *s, const void *b, const float *x, float *y, uint32_t rows,
                  uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, bool bf16, bool r2, int path,
                  cudaStream_t stream);

}  // namespace qmr
