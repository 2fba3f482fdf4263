// Internal interfaces shared by the C ABI (abi.cpp) and the launchers.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/qmr.h"

namespace qmr {

// Record a formatted message for qmr_last_error() and return `code`.
int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));

struct ScratchView {
    float4 *xp;
    float4 *xs;
    unsigned long long *keys;
    unsigned int *counter;
};

// One call of the streaming path (prep + streaming kernel).
struct FastCall {
    const void *w, *s, *b;      // matrix (gate for epilogue 1)
    const void *w2, *s2, *b2;   // up matrix for epilogue 1
    const float *x;
    float *y;                   // outputs (activations for epilogue 1, logits for 2)
    int32_t *argmax;            // epilogue 2
    uint64_t *best_key;         // epilogue 2
    uint32_t rows, cols, bits, group, batch, row_base;
    bool bf16;
    bool r2;                    // two rows per warp (selective R2)
    int epilogue;               // 0 plain, 1 swiglu, 2 head argmax
    bool legacy_kernel;         // force the register-streaming kernel (tests and A/B runs)
    void *scratch;              // caller scratch or nullptr for the per-stream pool
    size_t scratch_bytes;
};

bool fast_eligible(const void *w, uint32_t cols, uint32_t bits, uint32_t group);
size_t scratch_bytes(int bits, uint32_t cols, uint32_t batch);
void scratch_layout(void *base, int bits, uint32_t cols, uint32_t batch, ScratchView *v);
int acquire_scratch(cudaStream_t stream, size_t need, void **out);

int run_fast(const FastCall &c, cudaStream_t stream);
int run_prepare(const float *x, uint32_t cols, uint32_t bits, uint32_t batch, void *base, bool argmax,
                cudaStream_t stream);
int run_stream(const FastCall &c, void *base, cudaStream_t stream);
int device_error(int *code, bool clear);
int run_generic(const void *w, const void *s, const void *b, const float *x, float *y, uint32_t rows,
                uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, bool bf16, cudaStream_t stream);
int run_embed(const void *w, const void *s, const void *b, uint32_t row, float *y, uint32_t cols, uint32_t bits,
              uint32_t group, bool bf16, cudaStream_t stream);

}  // namespace qmr
