/*
 * qmr.h -- C ABI of the B200 (sm_100a) packed-affine matrix path.
 *
 * This library replaces the matrix half of the reference engine's GPU
 * dispatch layer (rucin93/qwen-mlx-runner v0.7.3, src/gpu.rs).  The reference
 * engine binds to it through `extern "C"` declarations of the entry points
 * below; each one names the reference interface it stands in for.
 *
 * Conventions shared by all entry points
 *   - Every pointer argument that names tensor data is a DEVICE pointer of
 *     the current CUDA device.  Streams are `cudaStream_t` passed as void*
 *     (NULL = the legacy default stream).  Calls are stream ordered and
 *     never synchronise the host.
 *   - Packed weights use the MLX affine layout the reference loads
 *     (src/weights.rs:292-351): u32 words, row-major, element c of a row at
 *     bits (c % (32/bits))*bits of word c/(32/bits), little-endian.  Scales
 *     and biases are one per (row, group): f32, or the high 16 bits of an
 *     f32 ("bf16 metadata", src/gpu/metadata.rs:6-14).
 *   - Block operands are token-major: X[b*cols + c], Y[b*rows + r]
 *     (kernels/matmul_block.metal:1-3).
 *   - Return value: QMR_OK (0) or a negative QMR_E* code.  All validation
 *     happens before any launch; on error nothing has been enqueued
 *     (src/gpu.rs:628-792).  qmr_last_error() gives the message of the last
 *     failure on the calling thread.
 */
#ifndef QMR_H
#define QMR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QMR_ABI_VERSION 1

enum {
    QMR_OK = 0,
    QMR_EINVAL = -1,       /* bad shape, parameter count, epsilon, batch ...   */
    QMR_ERANGE = -2,       /* buffer view beyond its allocation, size overflow */
    QMR_EALIGN = -3,       /* byte offset not 4-aligned (or 16 where required) */
    QMR_EOVERLAP = -4,     /* an output view overlaps an input view            */
    QMR_EUNSUPPORTED = -5, /* unknown kernel, no specialisation, mode forbids  */
    QMR_ECUDA = -6,        /* CUDA runtime error                               */
    QMR_ETIMEOUT = -7,     /* a bounded device-side wait ran out               */
    QMR_ENOTINIT = -8      /* qmr_init was not called on this device           */
};

/* Block-matmul schedules, src/gpu.rs:18-31 (BlockMatmulMode). */
enum { QMR_BLOCK_LEGACY = 0, QMR_BLOCK_SHARED = 1, QMR_BLOCK_MLP_R2 = 2 };

/* GEMV variants, src/gpu.rs:302-309 (QWEN_METAL_GEMV). */
enum { QMR_GEMV_PACKED4 = 0, QMR_GEMV_ALIGNED = 1, QMR_GEMV_STREAM = 2 };

/* qmr_init flags. */
#define QMR_INIT_FROM_ENV 0u  /* read QWEN_METAL_* like Gpu::new (gpu.rs:293-325) */
#define QMR_INIT_REFERENCE 1u /* force reference kernels, like new_with_reference(true) */

/* One device allocation as the dispatch ABI sees it: base pointer and byte
 * length.  Stands in for metal::Buffer; two views alias when their bases are
 * equal (gpu.rs:658-672 compares buffer identity). */
typedef struct qmr_buffer {
    void *ptr;
    uint64_t length;
} qmr_buffer;

/* ---- lifetime and modes ------------------------------------------------ */

/* Gpu::new / Gpu::new_with_reference (src/gpu.rs:293-437): bind `device`,
 * parse and validate QWEN_METAL_REFERENCE, QWEN_METAL_GEMV, QWEN_METAL_NORM,
 * QWEN_METAL_ATTN_VALUES, QWEN_METAL_METADATA, QWEN_METAL_BLOCK_MATMUL and
 * QWEN_METAL_BLOCK_DELTA with the reference's accepted values.  Safe to call
 * again; each call re-reads the environment. */
int qmr_init(int device, uint32_t flags);

/* Gpu::new_with_variant + set_block_kernel_mode (src/gpu.rs:305-309, 449-454):
 * override the modes.  Any argument may be NULL to keep the current value.
 * Values are the reference's strings ("aligned", "legacy", "mlp-r2", ...). */
int qmr_set_modes(const char *gemv, const char *metadata, const char *block_matmul,
                  const char *block_delta);

/* Current modes as "gemv=..,metadata=..,block_matmul=..,block_delta=..,reference=0|1"
 * (src/gpu.rs:439-470 kernel_mode/metadata_mode/block_kernel_mode). */
int qmr_get_modes(char *out, size_t out_len);

/* Message of the last failed call on this thread ("" if none). */
const char *qmr_last_error(void);

/* Library ABI version (QMR_ABI_VERSION). */
int qmr_abi_version(void);

/* ---- pure host logic (no GPU needed) ----------------------------------- */

/* BlockKernelMode::parse_for_device (src/gpu.rs:49-61): NULL matmul/delta
 * mean "unset"; the device default is mlp-r2 only for "Apple M5 Pro". */
int qmr_parse_block_mode(const char *device_name, const char *matmul, const char *delta,
                         int *matmul_mode, int *batched_delta);

/* dispatch_layout (src/gpu.rs:1041-1294): validates `params` for kernel
 * `name`, writes the minimum byte size of each buffer into sizes[0..*count)
 * and the logical thread count the reference expects.  sizes must hold 8. */
int qmr_dispatch_layout(const char *name, const uint32_t *params, size_t nparams,
                        uint64_t *sizes, size_t *count, uint64_t *threads);

/* checked_buffer_range (src/gpu.rs:879-889). */
int qmr_checked_buffer_range(uint64_t offset, uint64_t minimum, uint64_t length);

/* specialized_matmul / specialized_matvec / specialized_matvec_bf16
 * (src/gpu.rs:896-1037): the reference's specialised kernel name for
 * (name, params, aligned, mode), written into out.  QMR_EUNSUPPORTED when the
 * reference has none.  name is "matmul_affine[_bf16]", "matvec_affine" or
 * "matvec_affine_bf16"; mode is a QMR_BLOCK_* value. */
int qmr_select(const char *name, const uint32_t *params, size_t nparams, int aligned,
               int mode, char *out, size_t out_len);

/* pack_bf16_exact (src/gpu/metadata.rs:6-14): 1 and out filled when every
 * value is finite with zero low 16 bits, else 0. */
int qmr_pack_bf16_exact(const float *values, uint64_t n, uint16_t *out);

/* ---- the dispatch ABI -------------------------------------------------- */

/* DispatchEncoder::encode / encode_offsets (src/gpu.rs:120-174, 628-848):
 * validate and enqueue the named kernel.  offsets may be NULL (all zero).
 * Supported names: matvec_affine, matvec_affine_bf16, matmul_affine,
 * matmul_affine_bf16, embed_affine, embed_affine_bf16, copy_f32.  Other names
 * known to the reference validate and return QMR_EUNSUPPORTED. */
int qmr_encode(const char *name, const qmr_buffer *buffers, const uint64_t *offsets,
               size_t nbuffers, const uint32_t *params, size_t nparams, uint64_t threads,
               uint64_t group_size, void *stream);

/* ---- typed entry points (device pointers, no buffer lengths) ----------- */

/* Matrix::matvec (src/engine.rs:137-164): y[r] = sum_c (q*s+b)*x[c].
 * meta_bf16: 0 = f32 scales/biases, 1 = bf16 (high-half) scales/biases. */
int qmr_matvec_affine(const void *w, const void *scales, const void *biases, const float *x,
                      float *y, uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group,
                      int meta_bf16, void *stream);

/* Matrix::matmul_block (src/engine/block.rs:191-229): Y[b*rows+r] for
 * b < batch (1..4), every packed word read once for all batch rows. */
int qmr_matmul_affine(const void *w, const void *scales, const void *biases, const float *x,
                      float *y, uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group,
                      uint32_t batch, int meta_bf16, void *stream);

/* Matrix::embed (src/engine.rs:166-188), kernels embed_affine[_bf16]:
 * y[c] = float(q)*s + b for one row, bit-exact with the reference. */
int qmr_embed_affine(const void *w, const void *scales, const void *biases, uint32_t row,
                     float *y, uint32_t cols, uint32_t bits, uint32_t group, int meta_bf16,
                     void *stream);

/* qmr_matmul_affine that allocates no device memory (no reference
 * counterpart: the reference's Metal encoder never allocates per call).
 * For callers that must not allocate once running, e.g. an engine that
 * reserves its HBM budget at start-up (cudaMalloc would also synchronise the
 * device mid-step) or a binding that cannot own a scratch buffer.  Uses one
 * fixed 3 MiB device array per device: cols up to 32768 at batch <= 4,
 * larger shapes fail with QMR_ERANGE before any launch.  The array is shared
 * by all streams and threads, so calls that overlap in time race and must be
 * serialised by the caller.  The first call on each device does the set-up
 * (symbol lookup with the device current, clearing the array, then
 * cudaDeviceSynchronize so the clear is finished before any stream uses it)
 * and should come before any stream capture.  The array's address is kept
 * for the life of the process: do not use this entry point after
 * cudaDeviceReset. */
int qmr_matmul_affine_static(const void *w, const void *scales, const void *biases, const float *x,
                             float *y, uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group,
                             uint32_t batch, int meta_bf16, void *stream);

/* The gate/up projections plus swiglu of one MLP (src/engine.rs:755-763,
 * kernels/qwen.metal:91-94) in one pass: act[b*rows+r] =
 * silu(gate_b[r]) * up_b[r].  Both matrices share shape and format; x is
 * read once for both. */
int qmr_gateup_swiglu(const void *w_gate, const void *s_gate, const void *b_gate,
                      const void *w_up, const void *s_up, const void *b_up, const float *x,
                      float *act, uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group,
                      uint32_t batch, int meta_bf16, void *stream);

/* The head projection (src/engine.rs:777-780) plus greedy argmax
 * (src/chat.rs:383-390) in one pass: logits[b*rows+r] as qmr_matmul_affine,
 * and argmax[b] = index of the maximum logit of batch row b under f32 total
 * order, ties to the lowest index.  row_base is added to every reported index
 * (a vocabulary shard's first row).  best_key (optional, may be NULL)
 * receives the packed (total-order key << 32 | ~index) per batch row, the
 * value a cross-shard argmax reduces with a plain max. */
int qmr_head_argmax(const void *w, const void *scales, const void *biases, const float *x,
                    float *logits, int32_t *argmax, uint64_t *best_key, uint32_t rows,
                    uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch,
                    int meta_bf16, uint32_t row_base, void *stream);

/* ---- prepared activations (caller-owned workspace) ---------------------
 * The streaming kernels read activations in a pre-scaled, lane-interleaved
 * form.  The entry points above prepare it in a per-stream library
 * workspace.  Callers that apply several matrices to the same activations
 * (q/k/v, gate/up, DeltaNet in-projections), or that own their memory, can
 * prepare once into their own buffer and stream any number of matrices of
 * the same bits and cols from it.  These have no single reference
 * counterpart; they split Matrix::matvec / matmul_block
 * (src/engine.rs:137-164, src/engine/block.rs:191-229) into its two passes. */

/* Bytes of a prepared-activation buffer for (bits, cols, batch). */
uint64_t qmr_prepared_bytes(uint32_t bits, uint32_t cols, uint32_t batch);

/* Prepare x [batch, cols] (token-major f32) into `prepared` for matrices of
 * this bits and group (32/64/128); cols a multiple of the group and of
 * 128/bits.  `prepared` must be 256-byte aligned and hold
 * qmr_prepared_bytes(bits, cols, batch).  The layout depends on the stream
 * path (qmr_set_stream_path), which must not change before the matching
 * qmr_matmul_prepared calls. */
int qmr_prepare_activations(const float *x, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch,
                            void *prepared, uint64_t prepared_bytes, void *stream);

/* qmr_matmul_prepared flag: the kernel may start while the previous kernel
 * on the stream is still running and read the weights and metadata early
 * (programmatic dependent launch).  Set it only when the previous kernel
 * does not write this matrix; activations, outputs and the prepared buffer
 * are always read or written after the previous kernel completed. */
#define QMR_PREPARED_OVERLAP 1u

/* qmr_matmul_affine from prepared activations (same bits, cols, batch).
 * Weights must be 16-byte aligned with 16-byte multiple rows and group
 * 32/64/128; the result equals qmr_matmul_affine bit for bit.  Calls that
 * share one prepared buffer must not overlap on the GPU (it also holds the
 * split-K partial sums). */
int qmr_matmul_prepared(const void *w, const void *scales, const void *biases, const void *prepared, float *y,
                        uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch,
                        int meta_bf16, uint32_t flags, void *stream);

/* copy_f32 (kernels/matmul_block.metal:315-318): y[i] = x[i], i < n, as a
 * kernel chained behind the previous one on the stream (programmatic
 * dependent launch).  x and y may also be pinned host memory: copying a
 * result into pinned host memory this way is a device-to-host transfer
 * without a copy-engine round trip. */
int qmr_copy_f32(const float *x, float *y, uint32_t n, void *stream);

/* Select the streaming kernel of the fast path: "mma" (default; tensor-core
 * weight streaming, f16 subnormal weights x split-f16 activations, f32
 * accumulation), "tma" (FP32 warp-specialised TMA pipeline; needs 16-byte
 * aligned metadata with 16-byte multiple rows, else falls back to
 * "registers") or "registers" (FP32 register streaming).  All meet the same
 * oracle bound; each gives the same bits for a B-wide block and B GEMVs.
 * The switch exists for A/B measurement, in the spirit of QWEN_METAL_GEMV's
 * same-binary A/B variants (src/gpu.rs:302-309). */
int qmr_set_stream_path(const char *path);

/* Read (and optionally clear) the device error word that a kernel sets when
 * one of its bounded waits runs out (0 = none; 1/2/3 = full-stage,
 * empty-stage, drain timeout).  Synchronising; call between steps.  Stands in
 * for the command-status check of Gpu::finish (src/gpu.rs:861-865). */
int qmr_device_error(int *code, int clear);

/* Block until all work this library enqueued on `stream` finished, and
 * report a device error as QMR_ECUDA (Gpu::finish, src/gpu.rs:849-876). */
int qmr_stream_sync(void *stream);

/* ---- sharded calls with the output exchange over peer memory -------------
 * No single reference counterpart: the reference runs on one GPU.  These
 * carry the row-sharded MLP (gate/up and down split by output rows,
 * src/engine.rs:755-763 on n GPUs) and the vocabulary-sharded head
 * (src/engine.rs:777-780 + src/chat.rs:383-390) of the multi-GPU plan: one
 * process per GPU, each rank computing a contiguous block of output rows.
 * The streaming kernel itself stores every finished output row into every
 * rank's full output buffer (peer stores over NVLink through CUDA IPC
 * mappings; no multicast), and its last CTA publishes an epoch to every
 * rank's flag array.  qmr_exchange_wait, enqueued before the consumer,
 * waits (bounded, 2 s; QMR device error 4 on timeout) until every rank has
 * published the same epoch.  The head exchanges only its per-RHS argmax keys
 * and qmr_exchange_wait merges them (highest logit under f32 total order,
 * ties to the lowest vocabulary index), the single-GPU rule.
 *
 * Buffers come from qmr_exchange_alloc (zeroed device memory whose base is
 * an IPC allocation); every rank shares qmr_ipc_handle of each and maps the
 * peers' with qmr_ipc_open.  Exchanges on one QmrExchange must be issued by
 * every rank in the same order; a rank may reuse an output buffer only after
 * its own qmr_exchange_wait of the exchange after next (double-buffer the
 * outputs to overlap steps). */
#define QMR_MAX_RANKS 8
#define QMR_IPC_HANDLE_BYTES 64

typedef struct QmrExchange {
    uint32_t world;                      /* ranks, 2..QMR_MAX_RANKS */
    uint32_t rank;                       /* this rank */
    uint32_t total_rows;                 /* rows of the full output (the row stride per RHS) */
    uint32_t row_base;                   /* first output row of this rank's shard */
    float *out[QMR_MAX_RANKS];           /* every rank's full output [batch][total_rows]; NULL for the head */
    uint32_t *flags[QMR_MAX_RANKS];      /* every rank's flag array [world] (epoch per source rank) */
    uint64_t *keys[QMR_MAX_RANKS];       /* head: every rank's key array [world][4]; else NULL */
    uint32_t *epoch;                     /* this rank's exchange counter (zeroed device word) */
} QmrExchange;

int qmr_exchange_alloc(size_t bytes, void **dev_ptr);
int qmr_exchange_free(void *dev_ptr);
int qmr_ipc_handle(const void *dev_ptr, void *handle /* QMR_IPC_HANDLE_BYTES */);
int qmr_ipc_open(const void *handle, void **dev_ptr);
int qmr_ipc_close(void *dev_ptr);

/* qmr_matmul_affine / qmr_gateup_swiglu on this rank's rows (the matrices
 * are the shards: `rows` rows starting at ex->row_base of the full output),
 * writing the full outputs of all ranks.  Tensor-core path only
 * (QMR_EUNSUPPORTED for shapes it does not take). */
int qmr_matmul_affine_exchange(const void *w, const void *scales, const void *biases, const float *x,
                               uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch,
                               int meta_bf16, const QmrExchange *ex, void *stream);
int qmr_gateup_swiglu_exchange(const void *w_gate, const void *s_gate, const void *b_gate,
                               const void *w_up, const void *s_up, const void *b_up, const float *x,
                               uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch,
                               int meta_bf16, const QmrExchange *ex, void *stream);
/* The vocabulary shard's logits stay local (logits [batch][rows]); the
 * shard's best key per RHS goes to every rank. */
int qmr_head_argmax_exchange(const void *w, const void *scales, const void *biases, const float *x,
                             float *logits, uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group,
                             uint32_t batch, int meta_bf16, const QmrExchange *ex, void *stream);
/* Wait for every rank's current exchange; for the head also write the
 * merged argmax (token ids, may be NULL) and keys (may be NULL) per RHS. */
int qmr_exchange_wait(const QmrExchange *ex, uint32_t batch, int32_t *argmax, uint64_t *best_key, void *stream);

/* ---- checkpoints and the decode engine ---------------------------------
 * The per-token graph of the hybrid Qwen3.5 model (src/engine.rs:607-797):
 * DeltaNet and gated-attention layers in the config's 3:1 pattern, SwiGLU
 * MLPs, final norm and vocabulary head with greedy argmax.  All matrices run
 * through this library's packed-affine kernels; the other decode-step work
 * runs in this library's own kernels (one fused mixer launch per DeltaNet or
 * attention layer; RMSNorm folded into the next matrix's activation prep and
 * residual adds into the output epilogue where the tensor-core kernel takes
 * the matrix).  Activations, recurrent state and the KV cache are FP32.
 * Position and token live in device memory, so one captured CUDA graph per
 * step kind is replayed for every token.
 *
 * A QmrModel is bound to the CUDA device that is current when it is created;
 * its calls must come from one thread at a time (like the reference's
 * single-threaded Gpu). */
#define QMR_MAX_LAYERS 256

/* ModelConfig (src/config.rs:4-25) as the engine uses it. */
typedef struct QmrModelConfig {
    uint32_t hidden_size, intermediate_size, num_layers, num_heads, num_kv_heads, head_dim, vocab_size;
    uint32_t linear_key_heads, linear_value_heads, linear_key_dim, linear_value_dim, conv_width;
    uint32_t rotary_dim;                    /* head_dim * partial_rotary_factor */
    float rms_eps, rope_theta;
    uint8_t is_attention[QMR_MAX_LAYERS];   /* 1: full attention, 0: DeltaNet */
} QmrModelConfig;

typedef struct QmrCheckpoint QmrCheckpoint;
typedef struct QmrModel QmrModel;

/* Checkpoint::open (src/weights.rs:53-289): config.json plus one
 * .safetensors file or model.safetensors.index.json with its shards;
 * validates the config (src/config.rs:29-235), the safetensors headers and
 * the MLX affine quantisation metadata. */
int qmr_checkpoint_open(const char *dir, QmrCheckpoint **out);
void qmr_checkpoint_close(QmrCheckpoint *cp);
int qmr_checkpoint_config(const QmrCheckpoint *cp, QmrModelConfig *cfg, uint32_t *max_position, int *tied);
/* Checkpoint::matrix (src/weights.rs:292-351): shape and format of a packed
 * matrix; when w/s/b are non-NULL also its data: rows*cols*bits/32 u32 words
 * and rows*cols/group f32 scales and biases (F16/BF16/F32 widened). */
int qmr_checkpoint_matrix(const QmrCheckpoint *cp, const char *name, uint32_t *rows, uint32_t *cols, uint32_t *bits,
                          uint32_t *group, uint32_t *w, float *s, float *b);
/* Checkpoint::vector (src/weights.rs:353-368): n elements; data into out when
 * it is non-NULL and cap >= n. */
int qmr_checkpoint_vector(const QmrCheckpoint *cp, const char *name, float *out, uint64_t cap, uint64_t *n);

/* Engine::load (src/engine.rs:276-446): a checkpoint into device memory for
 * `context` positions (1..max_position_embeddings).  Metadata is compacted
 * to BF16 when QWEN_METAL_METADATA=bf16 and every value is BF16-exact
 * (src/gpu.rs:479-490, metadata.rs:6-14), as the reference does. */
int qmr_model_load(const char *dir, uint32_t context, QmrModel **out);
/* Engine::synthetic_qwen27b (src/engine/synthetic.rs:92-281) with distinct
 * seeded Q4/g64 BF16-metadata weights per layer and matrix (the counter
 * generator of the test oracle) and the reference's synthetic constants for
 * norms (1), conv (0.1), A_log and dt_bias (0). */
int qmr_model_synthetic(const QmrModelConfig *cfg, uint64_t seed, uint32_t context, QmrModel **out);
void qmr_model_free(QmrModel *m);
int qmr_model_config(const QmrModel *m, QmrModelConfig *cfg, uint32_t *context);
/* Engine::reset (src/engine.rs:561-584): clear recurrent state, position 0. */
int qmr_model_reset(QmrModel *m);
int qmr_model_position(const QmrModel *m, uint32_t *pos);
/* Engine::forward (src/engine.rs:586-605): one token at the current
 * position.  logits (host, vocab floats) and next (the greedy argmax,
 * src/chat.rs:383-390) may be NULL.  Fails before any launch for a token
 * outside the vocabulary or a full context. */
int qmr_model_forward(QmrModel *m, uint32_t token, float *logits, int32_t *next);
/* Prefill n prompt tokens then greedy-decode: out receives max_new tokens,
 * the first from the prompt's last logits (the reference's prefill + sample +
 * step loop, src/engine.rs:846-935, at temperature 0 and without EOS).  The
 * steps run as graph replays with no host round trip in between; the
 * prompt's positions before its last token run in blocks of 3 through the
 * batched path of verify_block (one weight stream per block, results equal
 * to single steps bit for bit); prefill_ms / decode_ms (may be NULL) are
 * device times. */
int qmr_model_generate(QmrModel *m, const uint32_t *prompt, uint32_t n_prompt, uint32_t max_new, uint32_t *out,
                       double *prefill_ms, double *decode_ms);
/* Engine::verify_block (src/engine/block.rs:296-333): evaluate inputs
 * tokens[0..n) (n = 1..4; the anchor and its drafts) at positions pos ..
 * pos+n-1 as one batch-n pass over every layer, matrices streamed once for
 * all inputs, DeltaNet state and convolution history saved before every
 * input.  logits (host, n*vocab, may be NULL) and argmax (host, n, may be
 * NULL) receive every row.  The state is tentative until
 * qmr_model_commit_block; no other step may run in between. */
int qmr_model_verify_block(QmrModel *m, const uint32_t *tokens, uint32_t n, float *logits, int32_t *argmax);
/* Engine::commit_block_prefix (src/engine/block.rs:335-390): keep the first
 * `consumed` inputs of the pending block; DeltaNet state and convolution
 * history are restored on the GPU, attention entries past the new position
 * are masked by it. */
int qmr_model_commit_block(QmrModel *m, uint32_t consumed);
/* Prefill, then greedy MTP-style decoding in verification rounds of `block`
 * inputs (2..4): each round evaluates [last token, drafts for the next
 * block-1 positions] with the drafts read from `drafts` (the draft token for
 * each absolute position; this library has no drafter), accepts drafts while
 * each equals the argmax of the row before it (src/speculative.rs:212-264 at
 * temperature 0), emits the accepted drafts plus the next argmax and rolls
 * the state back to the consumed prefix -- all on the device, one graph
 * replay per round.  out receives max_new tokens, the same tokens as
 * qmr_model_generate whatever the drafts; rounds and accepted (may be NULL)
 * count verification rounds and accepted drafts. */
int qmr_model_mtp_generate(QmrModel *m, const uint32_t *prompt, uint32_t n_prompt, uint32_t block, uint32_t max_new,
                           const uint32_t *drafts, uint32_t n_drafts, uint32_t *out, uint32_t *rounds,
                           uint32_t *accepted, double *prefill_ms, double *decode_ms);
/* Engine::mlp_r2_eligible_matrices (src/engine.rs:454-468). */
int qmr_model_mlp_r2_eligible(const QmrModel *m, uint32_t *count);
/* Gpu::metadata_stats (src/gpu.rs:473-478): matrices loaded with compacted
 * BF16 metadata and the bytes that saved. */
int qmr_model_metadata_stats(const QmrModel *m, uint64_t *matrices, uint64_t *saved_bytes);
/* Kernels the library launches per decode step with and without the head
 * (the captured graphs' node counts). */
int qmr_model_step_launches(const QmrModel *m, uint32_t *with_head, uint32_t *without_head);

/* ---- tensor-parallel decode over several GPUs --------------------------
 * No single reference counterpart (the reference decodes on one GPU): the
 * synthetic model of qmr_model_synthetic split over `world` processes, one
 * per GPU.  Rank r holds 1/world of the DeltaNet key and value heads, the
 * attention query heads (KV heads split too, or each replicated on the
 * world / num_kv_heads ranks that use it), the MLP rows and the vocabulary
 * rows; the residual stream is replicated.  out_proj, o_proj and down_proj
 * are split by input columns and their partial sums all-reduced over NVLink
 * by the streaming kernel's own output exchange (peer stores into every
 * rank's slot buffer, epoch release, bounded wait, a rank-ordered sum), so
 * every rank holds the same residual bits and emits the same tokens.  The
 * head's shard argmax keys are merged with the single-GPU rule.
 *
 * Set-up, every rank in lock step: qmr_model_synthetic_sharded (this
 * rank's weights and its exchange memory), qmr_model_exchange_handle
 * (QMR_IPC_HANDLE_BYTES to share with the other ranks), then
 * qmr_model_exchange_open with all ranks' handles in rank order (maps the
 * peers' memory and captures the step graphs; its warm-up steps exchange
 * with the peers).  After that every rank makes the same qmr_model_* calls
 * with the same arguments; logits are this rank's vocabulary rows
 * (qmr_model_shard).  A rank that falls more than 2 s behind makes the
 * others' waits run out (QMR_ETIMEOUT).  world = 1 is qmr_model_synthetic. */
int qmr_model_synthetic_sharded(const QmrModelConfig *cfg, uint64_t seed, uint32_t context, uint32_t world,
                                uint32_t rank, QmrModel **out);
int qmr_model_exchange_handle(const QmrModel *m, void *handle /* QMR_IPC_HANDLE_BYTES */);
int qmr_model_exchange_open(QmrModel *m, const void *handles /* world * QMR_IPC_HANDLE_BYTES */);
int qmr_model_shard(const QmrModel *m, uint32_t *world, uint32_t *rank, uint32_t *vocab_base, uint32_t *vocab_rows);

#ifdef __cplusplus
}
#endif

#endif /* QMR_H */
