// Internal interface of the decode-step kernels (decode.cu) used by the
// engine (engine.cpp).  Every activation, cache and recurrent state is FP32.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace qmr {

// Per-token control block in device memory.  Every kernel of a step reads
// the position from here, so one captured CUDA graph serves every token:
//   token of this step = prompt[pos] while pos < n_prompt, else `token`
//   (the previous step's greedy argmax, written by the head kernel).
// The step's last kernel appends the argmax to out[] and advances pos.
struct DecodeCtrl {
    uint32_t pos;
    int32_t token;     // argmax of the last step with a head
    uint32_t n_prompt;
    uint32_t n_out;    // tokens appended to out[]
    uint32_t pad[4];
};

struct DeltaArgs {
    const float *proj;   // [q: KH*K | k: KH*K | v: VH*V | z: VH*V | a: VH | b: VH]
    const float *conv_w; // [qkv channels][W]
    float *conv_state;   // [2 parities][qkv channels][W-1]
    float *state;        // [VH][V][K]
    const float *alog, *dt, *norm_w;
    float *out;          // [VH*V]
    const DecodeCtrl *ctrl;
    int KH, VH, K, V, W;
    float eps;
};

struct AttnArgs {
    const float *proj;   // [q|gate: NH*2*D | k: NKV*D | v: NKV*D]
    const float *qnorm, *knorm;
    float *kcache, *vcache;  // [context][NKV][D]
    float *part;             // [NKV][nchunks][G][D + 2]
    unsigned int *count;     // [NKV], zero between calls
    float *out;              // [NH*D]
    const DecodeCtrl *ctrl;
    int NH, NKV, D, RD, context, nchunks;
    float eps, theta;
};

constexpr int kAttnChunk = 64;  // positions per attention CTA

// Fill rows [row0, row0 + rows) of a Q4/g64 BF16-metadata matrix whose row
// stride is `cols` with the counter-based synthetic matrix (seed, mid).
int launch_synth_q4(uint32_t *w, uint16_t *s, uint16_t *b, uint64_t seed, uint32_t mid, uint32_t rows, uint32_t cols,
                    uint32_t row0, cudaStream_t stream);
int launch_fill_f32(float *p, uint64_t n, float v, cudaStream_t stream);
int launch_embed_token(const void *w, const void *s, const void *b, bool bf16, uint32_t cols, uint32_t bits,
                       uint32_t group, const DecodeCtrl *ctrl, const int32_t *prompt, float *x, cudaStream_t stream);
int launch_rms_norm(const float *x, const float *w, float *y, uint32_t n, float eps, cudaStream_t stream);
int launch_add(float *x, const float *r, uint32_t n, cudaStream_t stream);
int launch_delta_mixer(const DeltaArgs &a, cudaStream_t stream);
int launch_attention(const AttnArgs &a, cudaStream_t stream);
// record: append ctrl->token (the step's greedy argmax) to out[].
int launch_advance(DecodeCtrl *ctrl, int32_t *out, uint32_t out_cap, bool record, cudaStream_t stream);

}  // namespace qmr
