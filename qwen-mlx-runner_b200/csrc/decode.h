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

// One DeltaNet layer's mixer for nq consecutive tokens (1..4) at positions
// ctrl->pos .. ctrl->pos + nq - 1.  Single tokens (conv_snap == null) keep
// the convolution history double-buffered by position parity; a
// verification block (snapshots set) reads the live history and leaves
// every prefix's history in conv_snap and every prefix's recurrent state
// before token t in state_snap, for the rollback kernel to restore.
struct DeltaArgs {
    const float *proj;   // per token [q: KH*K | k: KH*K | v: VH*V | z: VH*V | a: VH | b: VH], stride proj_stride
    const float *conv_w; // [qkv channels][W]
    float *conv_state;   // [2 parities][qkv channels][W-1]
    float *state;        // [VH][V][K]
    const float *alog, *dt, *norm_w;
    float *out;          // [nq][VH*V]
    float *ybuf;         // [nq][VH*V] pre-norm outputs
    float *ssq;          // [VH][kDeltaSplit][4] sums of squares per part and token
    unsigned int *count; // [VH], zero between calls
    float *conv_snap;    // [nq + 1][qkv channels][W-1] or null
    float *state_snap;   // [nq][VH][V][K] or null
    const DecodeCtrl *ctrl;
    int KH, VH, K, V, W, nq, proj_stride;
    float eps;
};

// Decode attention for nq consecutive query tokens (1..4) at positions
// ctrl->pos + i, causal inside the block; their keys and values are appended
// to the caches.
struct AttnArgs {
    const float *proj;   // per token [q|gate: NH*2*D | k: NKV*D | v: NKV*D], stride proj_stride
    const float *qnorm, *knorm;
    float *kcache, *vcache;  // [context][NKV][D]
    float *part;             // [NKV][nchunks][nq][G][D + 2]
    unsigned int *count;     // [NKV], zero between calls
    float *out;              // [nq][NH*D]
    const DecodeCtrl *ctrl;
    int NH, NKV, D, RD, context, nchunks, nq, proj_stride;
    float eps, theta;
};

// The verification round's control words (device memory).
struct BlockCtrl {
    uint32_t pos_base;   // position of the block's first input
    uint32_t consumed;   // inputs kept after verification (1..nq)
    uint32_t accepted;   // drafts accepted
    uint32_t rounds;     // verification rounds run
    uint32_t drafts_accepted;  // over all rounds
    uint32_t pad[3];
};

constexpr int kAttnChunk = 64;  // positions per attention CTA
constexpr int kDeltaSplit = 4;  // CTAs per DeltaNet value head

// Fill rows [row0, row0 + rows) of a Q4/g64 BF16-metadata matrix whose row
// stride is `cols` with the counter-based synthetic matrix (seed, mid).
int launch_synth_q4(uint32_t *w, uint16_t *s, uint16_t *b, uint64_t seed, uint32_t mid, uint32_t rows, uint32_t cols,
                    uint32_t row0, cudaStream_t stream);
// Rows [r0, r0+nr) x columns [c0, c0+nc) of the synthetic matrix (seed,
// mid) of width full_cols into a destination with its own strides.
int launch_synth_region(uint32_t *w, uint16_t *s, uint16_t *b, uint64_t seed, uint32_t mid, uint32_t full_cols,
                        uint32_t r0, uint32_t nr, uint32_t c0, uint32_t nc, uint32_t dst_wstride, uint32_t dst_mstride,
                        uint32_t dst_row0, cudaStream_t stream);
// x[t][i] += the ranks' partial products in rank order (slots [t][world][H]).
int launch_partial_sum(float *x, const float *slots, int world, int H, int nq, cudaStream_t stream);
int launch_fill_f32(float *p, uint64_t n, float v, cudaStream_t stream);
int launch_embed_token(const void *w, const void *s, const void *b, bool bf16, uint32_t cols, uint32_t bits,
                       uint32_t group, const DecodeCtrl *ctrl, const int32_t *prompt, float *x, cudaStream_t stream);
// Embed a block.  prompt null (verification block): input 0 = ctrl->token
// (the anchor), input i >= 1 = drafts[ctrl->pos + i], and the block's base
// position goes to bctrl.  prompt set (prefill block): input i =
// prompt[ctrl->pos + i]; bctrl may be null.
int launch_embed_block(const void *w, const void *s, const void *b, bool bf16, uint32_t cols, uint32_t bits,
                       uint32_t group, const DecodeCtrl *ctrl, const int32_t *drafts, const int32_t *prompt,
                       BlockCtrl *bctrl, int nq, float *x, cudaStream_t stream);
// Greedy verification (src/speculative.rs:212-264 at temperature 0): accept
// drafts while each equals the argmax of the previous row, emit the accepted
// drafts and the next argmax, advance the position by the inputs consumed.
int launch_verify(DecodeCtrl *ctrl, BlockCtrl *bctrl, const int32_t *argmax, const int32_t *drafts, int nq,
                  int32_t *out, uint32_t out_cap, cudaStream_t stream);
// commit_block_prefix (src/engine/block.rs:335-390): restore every DeltaNet
// layer's state and convolution history to the consumed prefix.
// layer_ptrs: device array [nlayers][4] = {conv_state, state, conv_snap, state_snap}.
int launch_commit(const BlockCtrl *bctrl, float *const *layer_ptrs, int nlayers, int nq, size_t conv_elems,
                  size_t state_elems, cudaStream_t stream);
int launch_rms_norm(const float *x, const float *w, float *y, uint32_t n, float eps, cudaStream_t stream);
int launch_add(float *x, const float *r, uint32_t n, cudaStream_t stream);
int launch_delta_mixer(const DeltaArgs &a, cudaStream_t stream);
int launch_attention(const AttnArgs &a, cudaStream_t stream);
// record: append ctrl->token (the step's greedy argmax) to out[]; the
// position advances by `step` (a prefill block's width).
int launch_advance(DecodeCtrl *ctrl, int32_t *out, uint32_t out_cap, bool record, cudaStream_t stream, int step = 1);

}  // namespace qmr
