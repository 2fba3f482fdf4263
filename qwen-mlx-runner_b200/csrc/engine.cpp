// The decode engine: the hybrid Qwen3.5 per-token graph on one B200.
//
// Restates the reference's Engine (rucin93/qwen-mlx-runner v0.7.3,
// src/engine.rs): the layer graph of forward_inner (:607-797), load (:276-
// 446), reset (:561-584), the synthetic 27B-shaped model
// (src/engine/synthetic.rs:92-281) and mlp_r2_eligible_matrices
// (:454-468).  The step is laid out for the GPU rather than after the
// reference's dispatch list:
//  * a DeltaNet layer's in-projections (qkv, z, a, b) are one concatenated
//    matrix, an attention layer's (q|gate, k, v) likewise, so each layer
//    streams its input-side weights in one call;
//  * the input RMSNorm of every matrix call on a hidden vector rides in that
//    call's activation prep and output factor, and the residual adds in the
//    out/o/down epilogues, whenever the tensor-core kernel takes the matrix
//    (otherwise separate rms_norm / add kernels run, as in the reference);
//  * the DeltaNet and attention mixers are one launch each (decode.cu);
//  * position and token are read on the device, so each kind of step (with
//    and without the vocabulary head) is captured once as a CUDA graph and
//    replayed for every token; prefill and greedy decode run as a sequence of
//    replays with no host round trip.
//
// Tensor-parallel decode over `world` GPUs (one process per GPU, the
// synthetic model): rank r holds 1/world of the DeltaNet key and value
// heads, of the attention query heads (KV heads split too, or replicated
// when there are fewer KV heads than ranks), of the MLP rows and of the
// vocabulary.  The residual stream x is replicated.  The in-projections and
// gate/up are split by output rows, so they read the full x and write local
// activations; out_proj, o_proj and down_proj are split along their input
// columns, so each rank's product is a partial sum of the full hidden
// vector.  Those partial sums are all-reduced by the streaming kernel's own
// exchange epilogue (every rank's partial row goes into slot `rank` of every
// rank's slot buffer over NVLink peer stores, then an epoch release), a
// bounded wait for every rank's epoch, and one kernel that adds the slots in
// rank order into x, so every rank keeps bit-identical x.  The head's shard
// argmax keys are exchanged the same way and merged by the wait kernel.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "checkpoint.h"
#include "decode.h"
#include "qmr_internal.h"

namespace qmr {

// Matrix slots of a layer and of the model; the synthetic generator's matrix
// id is slot-derived: layer * 16 + slot + 1, embedding 0x100000, head
// 0x100001 (the test oracle uses the same ids).
enum Slot { S_QKV, S_Z, S_A, S_B, S_OUT, S_Q, S_K, S_V, S_O, S_GATE, S_UP, S_DOWN };
constexpr uint32_t kMidEmbed = 0x100000u, kMidHead = 0x100001u;
inline uint32_t synth_mid(uint32_t layer, int slot) { return layer * 16u + (uint32_t)slot + 1u; }

struct DevMat {
    void *w = nullptr, *s = nullptr, *b = nullptr;
    uint32_t rows = 0, cols = 0, bits = 4, group = 64;
    uint32_t mstride = 0;  // metadata elements per row (0: cols / group); column slices pad it to 8
    bool bf16 = true;
};

constexpr int kMaxBlock = 4;  // inputs of one verification block (src/engine/block.rs:12)

struct LayerState {
    bool attn = false;
    float *conv_snap = nullptr, *state_snap = nullptr;  // verification-block prefixes
    DevMat in, out, gate, up, down;
    float *in_norm = nullptr, *post_norm = nullptr;
    float *conv_w = nullptr, *alog = nullptr, *dt = nullptr, *dnorm = nullptr;
    float *qnorm = nullptr, *knorm = nullptr;
    float *conv_state = nullptr, *state = nullptr;
    float *kcache = nullptr, *vcache = nullptr;
};

}  // namespace qmr

using namespace qmr;

struct QmrModel {
    int device = 0;
    QmrModelConfig cfg{};  // the model's configuration
    // This rank's shapes: cfg with the head counts, the MLP width and the
    // vocabulary divided among the ranks (cfg itself when world == 1).
    QmrModelConfig lc{};
    uint32_t world = 1, rank = 0;
    uint32_t kv0 = 0;     // first global KV head of this rank
    uint32_t vbase = 0;   // first vocabulary row of this rank
    // Exchange memory (world > 1): one IPC-shareable allocation holding two
    // slot buffers [kMaxBlock][world][hidden] f32, the flag arrays of the
    // partial-sum and head exchanges, the head key array [world][4] and the
    // two epoch words; the peers' copies are mapped in `peers`.
    uint8_t *xbuf = nullptr;
    size_t xslot = 0;     // bytes of one slot buffer (256-aligned)
    void *peers[QMR_MAX_RANKS] = {};
    QmrExchange xch[2] = {}, hxch = {};
    bool opened = true;   // sharded models are usable after qmr_model_exchange_open
    int xpar = 0;         // slot buffer of the next partial-sum exchange while recording
    // While recording: the partial-sum exchange whose all-reduce into x is
    // still to come (folded into the prep of the next matrix that reads x).
    const QmrExchange *pending_reduce = nullptr;
    uint32_t context = 0;
    std::vector<LayerState> layers;
    DevMat embed, head;
    float *final_norm = nullptr;
    float *x = nullptr, *proj = nullptr, *mixed = nullptr, *act = nullptr, *logits = nullptr;
    // The residual stream's second buffer: an all-reduce folded into a
    // streaming kernel's image build writes the reduced x to the other
    // buffer (its CTAs still read the old one).  xc: the buffer holding x at
    // the current point of a recording (the embedding writes x).
    float *x2 = nullptr, *xc = nullptr;
    float *normed = nullptr, *tmp = nullptr;
    float *attn_part = nullptr;
    unsigned int *attn_count = nullptr;
    float *delta_y = nullptr, *delta_ssq = nullptr;
    unsigned int *delta_count = nullptr;
    // Verification blocks (allocated on first use): snapshots per DeltaNet
    // layer, the round's control words, the per-row argmax, the draft table
    // (draft token for each position), device pointer table of the layers.
    bool block_ready = false;
    BlockCtrl *bctrl = nullptr;
    int32_t *block_argmax = nullptr;
    int32_t *drafts = nullptr;
    float **layer_ptrs = nullptr;
    int ndelta = 0;
    cudaGraph_t bgraph[2][kMaxBlock + 1] = {};
    cudaGraphExec_t bexec[2][kMaxBlock + 1] = {};  // [0] evaluate only, [1] round (evaluate, verify, commit)
    bool pending = false;  // an evaluated block awaits commit_block_prefix
    uint32_t pending_width = 0;
    int attn_chunks = 0;
    void *scratch = nullptr;
    size_t scratch_size = 0;
    DecodeCtrl *ctrl = nullptr;
    int32_t *prompt = nullptr, *out = nullptr;
    uint32_t out_cap = 0;
    int32_t *host_stage = nullptr;  // pinned: [0] token, [1] n_prompt
    cudaStream_t stream = nullptr;
    // [0] one token without the head, [1] one token with the head, [2] a
    // prefill block of kPrefillBlock prompt tokens without the head.
    cudaGraph_t graph[3] = {nullptr, nullptr, nullptr};
    cudaGraphExec_t exec[3] = {nullptr, nullptr, nullptr};
    uint32_t launches[3] = {0, 0, 0};
    uint32_t pos = 0;
    std::vector<void *> allocs;
    uint64_t compacted = 0, saved_bytes = 0;
    size_t qkv_channels = 0;

    ~QmrModel() {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        if (stream != nullptr) cudaStreamSynchronize(stream);
        for (int i = 0; i < 3; ++i) {
            if (exec[i] != nullptr) cudaGraphExecDestroy(exec[i]);
            if (graph[i] != nullptr) cudaGraphDestroy(graph[i]);
        }
        for (int i = 0; i < 2; ++i) {
            for (int b = 0; b <= kMaxBlock; ++b) {
                if (bexec[i][b] != nullptr) cudaGraphExecDestroy(bexec[i][b]);
                if (bgraph[i][b] != nullptr) cudaGraphDestroy(bgraph[i][b]);
            }
        }
        for (uint32_t r = 0; r < QMR_MAX_RANKS; ++r)
            if (peers[r] != nullptr) qmr_ipc_close(peers[r]);
        if (xbuf != nullptr) qmr_exchange_free(xbuf);
        for (void *p : allocs) cudaFree(p);
        if (host_stage != nullptr) cudaFreeHost(host_stage);
        if (stream != nullptr) cudaStreamDestroy(stream);
        cudaSetDevice(prev);
    }
};

namespace qmr {
namespace {

int cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) return fail(QMR_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    return QMR_OK;
}

template <typename T>
int dev_alloc(QmrModel *m, T **p, size_t count) {
    void *v = nullptr;
    const size_t bytes = count * sizeof(T) > 0 ? count * sizeof(T) : 16;
    int rc = cuda_check(cudaMalloc(&v, bytes), "cudaMalloc of model memory");
    if (rc != QMR_OK) return rc;
    m->allocs.push_back(v);
    rc = cuda_check(cudaMemsetAsync(v, 0, bytes, m->stream), "clearing model memory");
    *p = static_cast<T *>(v);
    return rc;
}

int upload(QmrModel *m, void *dst, const void *src, size_t bytes) {
    return cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, m->stream), "uploading model data");
}

int dev_vector(QmrModel *m, float **p, const std::vector<float> &v) {
    int rc = dev_alloc(m, p, v.size());
    if (rc == QMR_OK) rc = upload(m, *p, v.data(), v.size() * sizeof(float));
    if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "uploading model data");
    return rc;
}

int dev_const(QmrModel *m, float **p, size_t n, float value) {
    int rc = dev_alloc(m, p, n);
    if (rc == QMR_OK) rc = launch_fill_f32(*p, n, value, m->stream);
    return rc;
}

int alloc_matrix(QmrModel *m, DevMat *d, uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group, bool bf16,
                 uint32_t mstride = 0) {
    d->rows = rows;
    d->cols = cols;
    d->bits = bits;
    d->group = group;
    d->bf16 = bf16;
    d->mstride = mstride;
    const size_t wbytes = (size_t)rows * cols * bits / 8;
    const size_t groups = (size_t)rows * (mstride != 0 ? mstride : cols / group);
    uint8_t *w = nullptr, *s = nullptr, *b = nullptr;
    int rc = dev_alloc(m, &w, wbytes);
    if (rc == QMR_OK) rc = dev_alloc(m, &s, groups * (bf16 ? 2 : 4));
    if (rc == QMR_OK) rc = dev_alloc(m, &b, groups * (bf16 ? 2 : 4));
    d->w = w;
    d->s = s;
    d->b = b;
    return rc;
}

// Activations, recurrent state, KV cache and control memory for this
// rank's shapes.
int alloc_buffers(QmrModel *m, uint32_t context) {
    const QmrModelConfig &c = m->lc;
    const size_t H = c.hidden_size, F = c.intermediate_size;
    int rc = QMR_OK;
    const size_t KD = (size_t)c.linear_key_heads * c.linear_key_dim, VD = (size_t)c.linear_value_heads * c.linear_value_dim;
    const size_t QD = (size_t)c.num_heads * c.head_dim, KVD = (size_t)c.num_kv_heads * c.head_dim;
    m->qkv_channels = 2 * KD + VD;
    const size_t delta_in = 2 * KD + 2 * VD + 2 * c.linear_value_heads, attn_in = 2 * QD + 2 * KVD;
    size_t widest = H;
    for (size_t v : {F, VD, QD}) widest = v > widest ? v : widest;
    const size_t proj = delta_in > attn_in ? delta_in : attn_in;
    // Activations for up to kMaxBlock tokens (token-major).
    const size_t T = kMaxBlock;
    rc = dev_alloc(m, &m->x, T * H);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->x2, T * H);
    m->xc = m->x;
    if (rc == QMR_OK) rc = dev_alloc(m, &m->normed, T * widest);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->tmp, T * H);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->proj, T * proj);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->mixed, T * (VD > QD ? VD : QD));
    if (rc == QMR_OK) rc = dev_alloc(m, &m->act, T * F);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->logits, T * c.vocab_size);
    m->attn_chunks = (int)((context + kAttnChunk - 1) / kAttnChunk);
    const size_t G = c.num_heads / c.num_kv_heads;
    if (rc == QMR_OK)
        rc = dev_alloc(m, &m->attn_part, (size_t)c.num_kv_heads * m->attn_chunks * T * G * (c.head_dim + 2));
    if (rc == QMR_OK) rc = dev_alloc(m, &m->attn_count, c.num_kv_heads);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->delta_y, T * VD);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->delta_ssq, (size_t)c.linear_value_heads * kDeltaSplit * 4);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->delta_count, c.linear_value_heads);
    m->scratch_size = scratch_bytes(8, (uint32_t)widest, 4);
    uint8_t *scr = nullptr;
    if (rc == QMR_OK) rc = dev_alloc(m, &scr, m->scratch_size);
    m->scratch = scr;
    if (rc == QMR_OK) rc = dev_alloc(m, &m->ctrl, 1);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->bctrl, 1);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->block_argmax, T);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->drafts, (size_t)context + T);
    if (rc == QMR_OK) rc = dev_alloc(m, &m->prompt, context);
    m->out_cap = context;
    if (rc == QMR_OK) rc = dev_alloc(m, &m->out, context);
    if (rc == QMR_OK) rc = cuda_check(cudaMallocHost(&m->host_stage, 64), "pinned staging");
    if (rc != QMR_OK) return rc;
    m->layers.resize(c.num_layers);
    for (uint32_t l = 0; l < c.num_layers; ++l) {
        LayerState &L = m->layers[l];
        L.attn = c.is_attention[l] != 0;
        if (L.attn) {
            rc = dev_alloc(m, &L.kcache, (size_t)context * KVD);
            if (rc == QMR_OK) rc = dev_alloc(m, &L.vcache, (size_t)context * KVD);
        } else {
            rc = dev_alloc(m, &L.conv_state, 2 * m->qkv_channels * (c.conv_width - 1));
            if (rc == QMR_OK) rc = dev_alloc(m, &L.state, VD * c.linear_key_dim);
        }
        if (rc != QMR_OK) return rc;
    }
    return QMR_OK;
}

// This rank's shapes for a split over `world` ranks (see the file comment).
int shard_config(QmrModel *m, const QmrModelConfig &c, uint32_t world, uint32_t rank) {
    m->world = world;
    m->rank = rank;
    m->lc = c;
    m->kv0 = 0;
    m->vbase = 0;
    if (world == 1) return QMR_OK;
    if (world > QMR_MAX_RANKS || rank >= world) return fail(QMR_EINVAL, "world must be 1..%d and rank < world", QMR_MAX_RANKS);
    const uint32_t VD = c.linear_value_heads * c.linear_value_dim, QD = c.num_heads * c.head_dim;
    if (c.linear_key_heads % world || c.linear_value_heads % world || c.num_heads % world)
        return fail(QMR_EUNSUPPORTED, "DeltaNet key/value heads and attention heads must divide among %u ranks", world);
    if (c.num_kv_heads % world != 0 && world % c.num_kv_heads != 0)
        return fail(QMR_EUNSUPPORTED, "KV heads must divide among the ranks or the ranks among the KV heads");
    if (c.intermediate_size % (world * 64) || VD % (world * 64) || QD % (world * 64))
        return fail(QMR_EUNSUPPORTED, "MLP, DeltaNet value and attention widths must split into 64-column groups");
    if (c.vocab_size % (world * 16)) return fail(QMR_EUNSUPPORTED, "the vocabulary must split into 16-row tiles");
    QmrModelConfig &l = m->lc;
    l.linear_key_heads = c.linear_key_heads / world;
    l.linear_value_heads = c.linear_value_heads / world;
    l.num_heads = c.num_heads / world;
    if (c.num_kv_heads % world == 0) {
        l.num_kv_heads = c.num_kv_heads / world;
        m->kv0 = rank * l.num_kv_heads;
    } else {
        // Fewer KV heads than ranks: each KV head is replicated on the
        // world / num_kv_heads ranks whose query heads use it.
        l.num_kv_heads = 1;
        m->kv0 = rank / (world / c.num_kv_heads);
    }
    l.intermediate_size = c.intermediate_size / world;
    l.vocab_size = c.vocab_size / world;
    m->vbase = rank * l.vocab_size;
    return QMR_OK;
}

// Model-wide validation and the activations, state and control memory
// (sized for this rank's shapes, m->lc).
int create_common(QmrModel *m, const QmrModelConfig &gc, uint32_t context, uint32_t world = 1, uint32_t rank = 0) {
    const QmrModelConfig &c = gc;
    if (c.num_layers == 0 || c.num_layers > QMR_MAX_LAYERS) return fail(QMR_EINVAL, "layer count out of range");
    if (c.hidden_size == 0 || c.intermediate_size == 0 || c.vocab_size == 0 || c.num_heads == 0 ||
        c.num_kv_heads == 0 || c.head_dim == 0 || c.linear_key_heads == 0 || c.linear_value_heads == 0 ||
        c.linear_key_dim == 0 || c.linear_value_dim == 0 || c.conv_width == 0)
        return fail(QMR_EINVAL, "model dimensions must be positive");
    if (c.num_heads % c.num_kv_heads != 0 || c.num_heads / c.num_kv_heads > 8)
        return fail(QMR_EUNSUPPORTED, "attention needs at most 8 query heads per KV head");
    if (c.head_dim > 256 || c.rotary_dim == 0 || c.rotary_dim % 2 != 0 || c.rotary_dim > c.head_dim)
        return fail(QMR_EUNSUPPORTED, "head_dim must be <= 256 with an even rotary dimension that fits it");
    if (c.linear_key_dim > 128 || c.linear_value_heads % c.linear_key_heads != 0)
        return fail(QMR_EUNSUPPORTED, "DeltaNet needs key dim <= 128 and value heads a multiple of key heads");
    if (!(c.rms_eps > 0 && std::isfinite(c.rms_eps)) || !(c.rope_theta > 0 && std::isfinite(c.rope_theta)))
        return fail(QMR_EINVAL, "invalid RMS epsilon or RoPE theta");
    if (context == 0) return fail(QMR_EINVAL, "context must be positive");
    // Metal-era 32-bit index limits kept as the reference checks them (engine.rs:286-304).
    if ((uint64_t)c.num_heads * context * 32 > 0xffffffffull || (uint64_t)context * c.num_kv_heads * c.head_dim > 0xffffffffull)
        return fail(QMR_ERANGE, "context exceeds 32-bit indexing");
    m->cfg = gc;
    m->context = context;
    int rc = shard_config(m, gc, world, rank);
    if (rc != QMR_OK) return rc;
    rc = cuda_check(cudaGetDevice(&m->device), "cudaGetDevice");
    if (rc == QMR_OK) rc = cuda_check(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "stream");
    if (rc != QMR_OK) return rc;
    return alloc_buffers(m, context);
}
// Rows of the concatenated in-projection: DeltaNet [qkv; z; a; b], attention [q|gate; k; v].
uint32_t in_rows(const QmrModelConfig &c, bool attn) {
    if (attn) return 2 * c.num_heads * c.head_dim + 2 * c.num_kv_heads * c.head_dim;
    return 2 * c.linear_key_heads * c.linear_key_dim + 2 * c.linear_value_heads * c.linear_value_dim +
           2 * c.linear_value_heads;
}

// ---- one step --------------------------------------------------------------

struct StepCounter {
    uint32_t n = 0;
};

// y = W x for the engine, with the optional fused input RMSNorm (norm_w) and
// residual (resid == y), gate/up SwiGLU (epi 1, up = second matrix) or head
// argmax (epi 2, into argmax).
int flush_reduce(QmrModel *m, StepCounter *cnt, int nq);

float *other_x(QmrModel *m) { return m->xc == m->x ? m->x2 : m->x; }

int mat_call(QmrModel *m, const DevMat &W, const float *x, float *y, const float *norm_w, const float *resid, int epi,
             const DevMat *up, int32_t *argmax, StepCounter *cnt, int nq = 1) {
    FastCall c = {};
    c.w = W.w;
    c.s = W.s;
    c.b = W.b;
    if (epi == 1) {
        c.w2 = up->w;
        c.s2 = up->s;
        c.b2 = up->b;
    }
    c.x = x;
    c.y = y;
    c.argmax = argmax;
    c.rows = W.rows;
    c.cols = W.cols;
    c.bits = W.bits;
    c.group = W.group;
    c.batch = (uint32_t)nq;
    c.bf16 = W.bf16;
    c.epilogue = epi;
    c.counted_build = true;  // clear_state clears the scratch after any failed call
    c.path = modes_stream_path();
    c.scratch = m->scratch;
    c.scratch_bytes = m->scratch_size;
    c.eps = m->cfg.rms_eps;
    c.meta_stride = W.mstride;
    const bool reduce = m->pending_reduce != nullptr && x == m->xc;
    if (norm_w != nullptr || resid != nullptr || reduce) {
        FastCall f = c;
        f.norm_w = norm_w;
        f.resid = resid;
        f.reduce = reduce ? m->pending_reduce : nullptr;
        f.x_out = reduce ? other_x(m) : nullptr;
        if (fused_supported(f)) {
            f.launch_count = &cnt->n;
            const int rc = run_fast(f, m->stream);
            if (reduce) {
                m->pending_reduce = nullptr;
                m->xc = f.x_out;
            }
            return rc;
        }
    }
    int rc = reduce ? flush_reduce(m, cnt, nq) : QMR_OK;
    if (rc != QMR_OK) return rc;
    if (norm_w != nullptr) {
        for (int t = 0; t < nq && rc == QMR_OK; ++t) {
            rc = launch_rms_norm(x + (size_t)t * W.cols, norm_w, m->normed + (size_t)t * W.cols, W.cols,
                                 m->cfg.rms_eps, m->stream);
            ++cnt->n;
        }
        if (rc != QMR_OK) return rc;
        c.x = m->normed;
    }
    if (resid != nullptr) c.y = m->tmp;
    if (fast_eligible(W.w, W.cols, W.bits, W.group)) {
        c.launch_count = &cnt->n;
        rc = run_fast(c, m->stream);
    } else if (epi == 0) {
        rc = run_generic(W.w, W.s, W.b, c.x, c.y, W.rows, W.cols, W.bits, W.group, (uint32_t)nq, W.bf16, m->stream);
        cnt->n += 1;
    } else {
        rc = fail(QMR_EUNSUPPORTED, "fused gate/up and head need a packed shape the streaming kernels take");
    }
    if (rc != QMR_OK) return rc;
    if (resid != nullptr) {
        rc = launch_add(y, m->tmp, W.rows * (uint32_t)nq, m->stream);
        ++cnt->n;
    }
    return rc;
}

// The pending all-reduce as its own launches: the bounded wait for every
// rank's epoch, then the rank-ordered sum of the slots into x.
int flush_reduce(QmrModel *m, StepCounter *cnt, int nq) {
    const QmrExchange *ex = m->pending_reduce;
    if (ex == nullptr) return QMR_OK;
    m->pending_reduce = nullptr;
    int rc = launch_exchange_wait(*ex, (uint32_t)nq, nullptr, nullptr, m->stream);
    ++cnt->n;
    if (rc == QMR_OK) rc = launch_partial_sum(m->xc, ex->out[ex->rank], (int)m->world, (int)m->lc.hidden_size, nq, m->stream);
    ++cnt->n;
    return rc;
}

// x += W in for the matrices that feed the residual stream (out_proj,
// o_proj, down_proj).  One GPU: the residual epilogue.  Split over ranks:
// W is this rank's column slice, its partial product goes through the
// exchange into slot `rank` of every rank's slot buffer; the all-reduce
// into x (bounded wait for every rank's epoch, rank-ordered sum of the
// slots) is folded into the prep of the next matrix that reads x, or runs
// as its own launches at the end of the step.  Every exchange is thus
// waited for before the next one is issued, and the two slot buffers
// alternate, so a rank one exchange ahead never overwrites slots that a
// peer has not summed yet.
int mat_reduce(QmrModel *m, const DevMat &W, const float *in, StepCounter *cnt, int nq) {
    if (m->world == 1) return mat_call(m, W, in, m->xc, nullptr, m->xc, 0, nullptr, nullptr, cnt, nq);
    int rc = flush_reduce(m, cnt, nq);  // none pending in the step's order (in -> out, gate/up -> down)
    if (rc != QMR_OK) return rc;
    const QmrExchange &ex = m->xch[m->xpar];
    m->xpar ^= 1;
    FastCall c = {};
    c.w = W.w;
    c.s = W.s;
    c.b = W.b;
    c.x = in;
    c.y = ex.out[ex.rank] + ex.row_base;
    c.ystride = ex.total_rows;
    c.rows = W.rows;
    c.cols = W.cols;
    c.bits = W.bits;
    c.group = W.group;
    c.batch = (uint32_t)nq;
    c.bf16 = W.bf16;
    c.path = kPathMma;
    c.scratch = m->scratch;
    c.scratch_bytes = m->scratch_size;
    c.meta_stride = W.mstride;
    c.ex = &ex;
    c.counted_build = true;
    c.launch_count = &cnt->n;
    rc = run_fast(c, m->stream);
    m->pending_reduce = &ex;
    return rc;
}

// Final norm + head + greedy argmax into `argmax` (nq entries).  Split over
// ranks: each rank's vocabulary rows, its logits stay local, and the wait
// kernel merges the ranks' best keys (highest logit, ties to the lowest
// vocabulary index).
int head_call(QmrModel *m, int32_t *argmax, StepCounter *cnt, int nq) {
    if (m->world == 1)
        return mat_call(m, m->head, m->xc, m->logits, m->final_norm, nullptr, 2, nullptr, argmax, cnt, nq);
    const DevMat &W = m->head;
    FastCall c = {};
    c.w = W.w;
    c.s = W.s;
    c.b = W.b;
    c.x = m->xc;
    c.y = m->logits;
    c.rows = W.rows;
    c.cols = W.cols;
    c.bits = W.bits;
    c.group = W.group;
    c.batch = (uint32_t)nq;
    c.row_base = m->vbase;
    c.bf16 = W.bf16;
    c.epilogue = 2;
    c.path = kPathMma;
    c.scratch = m->scratch;
    c.scratch_bytes = m->scratch_size;
    c.norm_w = m->final_norm;
    c.eps = m->cfg.rms_eps;
    c.ex = &m->hxch;
    c.reduce = m->pending_reduce;
    c.x_out = c.reduce != nullptr ? other_x(m) : nullptr;
    c.counted_build = true;
    c.launch_count = &cnt->n;
    int rc = run_fast(c, m->stream);
    if (c.reduce != nullptr) m->xc = c.x_out;
    m->pending_reduce = nullptr;
    if (rc == QMR_OK) rc = launch_exchange_wait(m->hxch, (uint32_t)nq, argmax, nullptr, m->stream);
    ++cnt->n;
    return rc;
}

// Kinds of recorded step: one token without / with the head, a
// verification block evaluated, or a full verification round (evaluate,
// greedy verify, roll back to the consumed prefix).
// a prefill block (kPrefillBlock prompt tokens evaluated together, no head).
enum StepKind { kStepPlain, kStepHead, kStepBlockEval, kStepBlockRound, kStepPrefill };

// Prompt tokens per prefill block.  The matrices stream once for the block
// and a B-wide call equals B single calls bit for bit, so a block equals as
// many single steps; an odd width keeps the DeltaNet conv history's
// ping-pong buffer (chosen by position parity) where the next step reads it.
constexpr int kPrefillBlock = 3;

int record_step(QmrModel *m, StepKind kind, int nq, StepCounter *cnt) {
    const QmrModelConfig &c = m->lc;
    const bool block = kind == kStepBlockEval || kind == kStepBlockRound;
    const bool pre = kind == kStepPrefill;
    m->xc = m->x;  // the embedding writes x
    int rc;
    if (block || pre)
        rc = launch_embed_block(m->embed.w, m->embed.s, m->embed.b, m->embed.bf16, m->embed.cols, m->embed.bits,
                                m->embed.group, m->ctrl, m->drafts, pre ? m->prompt : nullptr,
                                pre ? nullptr : m->bctrl, nq, m->x, m->stream);
    else
        rc = launch_embed_token(m->embed.w, m->embed.s, m->embed.b, m->embed.bf16, m->embed.cols, m->embed.bits,
                                m->embed.group, m->ctrl, m->prompt, m->x, m->stream);
    ++cnt->n;
    for (uint32_t l = 0; l < c.num_layers && rc == QMR_OK; ++l) {
        LayerState &L = m->layers[l];
        // The in-projection writes [nq][in rows]; the mixers read it with that stride.
        rc = mat_call(m, L.in, m->xc, m->proj, L.in_norm, nullptr, 0, nullptr, nullptr, cnt, nq);
        if (rc != QMR_OK) break;
        if (L.attn) {
            AttnArgs a = {};
            a.proj = m->proj;
            a.qnorm = L.qnorm;
            a.knorm = L.knorm;
            a.kcache = L.kcache;
            a.vcache = L.vcache;
            a.part = m->attn_part;
            a.count = m->attn_count;
            a.out = m->mixed;
            a.ctrl = m->ctrl;
            a.NH = (int)c.num_heads;
            a.NKV = (int)c.num_kv_heads;
            a.D = (int)c.head_dim;
            a.RD = (int)c.rotary_dim;
            a.context = (int)m->context;
            a.nchunks = m->attn_chunks;
            a.nq = nq;
            a.proj_stride = (int)L.in.rows;
            a.eps = c.rms_eps;
            a.theta = c.rope_theta;
            rc = launch_attention(a, m->stream);
        } else {
            DeltaArgs a = {};
            a.proj = m->proj;
            a.conv_w = L.conv_w;
            a.conv_state = L.conv_state;
            a.state = L.state;
            a.alog = L.alog;
            a.dt = L.dt;
            a.norm_w = L.dnorm;
            a.out = m->mixed;
            a.ybuf = m->delta_y;
            a.ssq = m->delta_ssq;
            a.count = m->delta_count;
            a.conv_snap = block ? L.conv_snap : nullptr;
            a.state_snap = block ? L.state_snap : nullptr;
            a.ctrl = m->ctrl;
            a.KH = (int)c.linear_key_heads;
            a.VH = (int)c.linear_value_heads;
            a.K = (int)c.linear_key_dim;
            a.V = (int)c.linear_value_dim;
            a.W = (int)c.conv_width;
            a.nq = nq;
            a.proj_stride = (int)L.in.rows;
            a.eps = c.rms_eps;
            rc = launch_delta_mixer(a, m->stream);
        }
        ++cnt->n;
        if (rc == QMR_OK) rc = mat_reduce(m, L.out, m->mixed, cnt, nq);
        if (rc == QMR_OK) rc = mat_call(m, L.gate, m->xc, m->act, L.post_norm, nullptr, 1, &L.up, nullptr, cnt, nq);
        if (rc == QMR_OK) rc = mat_reduce(m, L.down, m->act, cnt, nq);
    }
    if (rc == QMR_OK && kind != kStepPlain && !pre)
        rc = head_call(m, block ? m->block_argmax : &m->ctrl->token, cnt, nq);
    if (rc == QMR_OK) rc = flush_reduce(m, cnt, nq);  // a step without the head: the last down's all-reduce
    m->pending_reduce = nullptr;
    if (rc == QMR_OK && !block) {
        rc = launch_advance(m->ctrl, m->out, m->out_cap, kind == kStepHead, m->stream, pre ? nq : 1);
        ++cnt->n;
    }
    if (rc == QMR_OK && kind == kStepBlockRound) {
        rc = launch_verify(m->ctrl, m->bctrl, m->block_argmax, m->drafts, nq, m->out, m->out_cap, m->stream);
        ++cnt->n;
        if (rc == QMR_OK && m->ndelta > 0) {
            const size_t VD = (size_t)c.linear_value_heads * c.linear_value_dim;
            rc = launch_commit(m->bctrl, m->layer_ptrs, m->ndelta, nq, m->qkv_channels * (c.conv_width - 1),
                               VD * c.linear_key_dim, m->stream);
            ++cnt->n;
        }
    }
    return rc;
}

int clear_state(QmrModel *m) {
    const QmrModelConfig &c = m->lc;
    const size_t VD = (size_t)c.linear_value_heads * c.linear_value_dim;
    int rc = QMR_OK;
    for (LayerState &L : m->layers) {
        if (L.attn) continue;
        if (rc == QMR_OK)
            rc = cuda_check(cudaMemsetAsync(L.conv_state, 0, 2 * m->qkv_channels * (c.conv_width - 1) * sizeof(float),
                                            m->stream), "reset");
        if (rc == QMR_OK) rc = cuda_check(cudaMemsetAsync(L.state, 0, VD * c.linear_key_dim * sizeof(float), m->stream), "reset");
    }
    if (rc == QMR_OK) rc = cuda_check(cudaMemsetAsync(m->ctrl, 0, sizeof(DecodeCtrl), m->stream), "reset");
    // The streaming kernels' CTA counters and argmax keys (the engine's
    // calls build their images in-kernel, without the prep that clears them).
    if (rc == QMR_OK) rc = cuda_check(cudaMemsetAsync(m->scratch, 0, m->scratch_size, m->stream), "reset");
    if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "reset");
    m->pos = 0;
    m->pending = false;
    return rc;
}

// One eager step of each kind (per-device kernel attributes and occupancy
// queries happen outside capture), then the three graphs, then a clean state.
int build_graphs(QmrModel *m) {
    int rc = QMR_OK;
    const StepKind kinds[3] = {kStepPlain, kStepHead, kStepPrefill};
    const int widths[3] = {1, 1, kPrefillBlock};
    // A context shorter than a prefill block has no prefill graph (its
    // prompts prefill token by token).
    const int nkinds = m->context >= (uint32_t)kPrefillBlock ? 3 : 2;
    for (int head = 0; head < nkinds && rc == QMR_OK; ++head) {
        // Each warm-up step starts at position 0, inside any context.
        StepCounter cnt;
        rc = clear_state(m);
        if (rc == QMR_OK) rc = record_step(m, kinds[head], widths[head], &cnt);
        if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "warm-up step");
    }
    for (int head = 0; head < nkinds && rc == QMR_OK; ++head) {
        StepCounter cnt;
        rc = cuda_check(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
        if (rc != QMR_OK) break;
        const int rs = record_step(m, kinds[head], widths[head], &cnt);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(m->stream, &g);
        if (rs != QMR_OK) {
            if (g != nullptr) cudaGraphDestroy(g);
            return rs;
        }
        rc = cuda_check(e, "end capture");
        if (rc != QMR_OK) break;
        m->graph[head] = g;
        rc = cuda_check(cudaGraphInstantiate(&m->exec[head], g, 0), "graph instantiate");
        m->launches[head] = cnt.n;
    }
    if (rc == QMR_OK) rc = clear_state(m);
    return rc;
}

// Verification-block resources (BlockState::new, src/engine/block.rs:45-135):
// prefix snapshots per DeltaNet layer, the device table of layer pointers,
// then the evaluate and round graphs of width nq.  The per-width kernels are
// first run eagerly on the matrices alone (they touch activations and
// scratch, never model state), so the capture sees no first-use set-up.
int ensure_block(QmrModel *m, int nq) {
    const QmrModelConfig &c = m->lc;
    int rc = QMR_OK;
    if (!m->block_ready) {
        const size_t conv = m->qkv_channels * (c.conv_width - 1);
        const size_t st = (size_t)c.linear_value_heads * c.linear_value_dim * c.linear_key_dim;
        std::vector<float *> ptrs;
        for (LayerState &L : m->layers) {
            if (L.attn) continue;
            rc = dev_alloc(m, &L.conv_snap, (size_t)(kMaxBlock + 1) * conv);
            if (rc == QMR_OK) rc = dev_alloc(m, &L.state_snap, (size_t)kMaxBlock * st);
            if (rc != QMR_OK) return rc;
            ptrs.insert(ptrs.end(), {L.conv_state, L.state, L.conv_snap, L.state_snap});
        }
        m->ndelta = (int)(ptrs.size() / 4);
        rc = dev_alloc(m, &m->layer_ptrs, ptrs.size() > 0 ? ptrs.size() : 1);
        if (rc == QMR_OK && !ptrs.empty()) rc = upload(m, m->layer_ptrs, ptrs.data(), ptrs.size() * sizeof(float *));
        if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "block set-up");
        if (rc != QMR_OK) return rc;
        m->block_ready = true;
    }
    if (m->bexec[1][nq] != nullptr) return QMR_OK;
    StepCounter warm;
    m->xc = m->x;
    bool seen[2] = {false, false};
    for (LayerState &L : m->layers) {
        if (seen[L.attn]) continue;
        seen[L.attn] = true;
        rc = mat_call(m, L.in, m->xc, m->proj, L.in_norm, nullptr, 0, nullptr, nullptr, &warm, nq);
        if (rc == QMR_OK) rc = mat_reduce(m, L.out, m->mixed, &warm, nq);
        if (rc == QMR_OK) rc = mat_call(m, L.gate, m->xc, m->act, L.post_norm, nullptr, 1, &L.up, nullptr, &warm, nq);
        if (rc == QMR_OK) rc = mat_reduce(m, L.down, m->act, &warm, nq);
        if (rc != QMR_OK) return rc;
    }
    rc = head_call(m, m->block_argmax, &warm, nq);
    if (rc == QMR_OK) rc = flush_reduce(m, &warm, nq);
    if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "block warm-up");
    for (int kind = 0; kind < 2 && rc == QMR_OK; ++kind) {
        StepCounter cnt;
        rc = cuda_check(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
        if (rc != QMR_OK) break;
        const int rs = record_step(m, kind == 0 ? kStepBlockEval : kStepBlockRound, nq, &cnt);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(m->stream, &g);
        if (rs != QMR_OK) {
            if (g != nullptr) cudaGraphDestroy(g);
            return rs;
        }
        rc = cuda_check(e, "end capture");
        if (rc != QMR_OK) break;
        m->bgraph[kind][nq] = g;
        rc = cuda_check(cudaGraphInstantiate(&m->bexec[kind][nq], g, 0), "graph instantiate");
    }
    return rc;
}

int check_device_error() {
    int code = 0;
    const int rc = device_error(&code, false);
    if (rc != QMR_OK) return rc;
    if (code != 0) return fail(QMR_ETIMEOUT, "a bounded device wait ran out (code %d)", code);
    return QMR_OK;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// ---- building from a checkpoint -----------------------------------------------

// Upload one or more checkpoint matrices as one concatenated device matrix
// (rows stacked).  Metadata is stored as BF16 when the library's metadata
// mode is bf16 and every part is BF16-exact (compact_metadata,
// src/gpu.rs:479-490), else as f32.
int load_matrix(QmrModel *m, const Checkpoint &cp, const std::vector<std::string> &names, DevMat *d) {
    std::vector<HostMatrix> parts(names.size());
    uint32_t rows = 0;
    for (size_t i = 0; i < names.size(); ++i) {
        const int rc = cp.matrix(names[i], &parts[i]);
        if (rc != QMR_OK) return rc;
        if (i > 0 && (parts[i].cols != parts[0].cols || parts[i].bits != parts[0].bits ||
                      parts[i].group != parts[0].group))
            return fail(QMR_EINVAL, "%s: parts of one projection differ in width or quantisation", names[i].c_str());
        rows += parts[i].rows;
    }
    const HostMatrix &p0 = parts[0];
    const bool supported = (p0.bits == 4 || p0.bits == 8) && (p0.group == 32 || p0.group == 64 || p0.group == 128);
    std::vector<std::vector<uint16_t>> cs(parts.size()), cb(parts.size());
    bool bf16 = modes_meta_bf16() && supported;
    for (size_t i = 0; i < parts.size() && bf16; ++i) {
        cs[i].resize(parts[i].scales.size());
        cb[i].resize(parts[i].biases.size());
        bf16 = qmr_pack_bf16_exact(parts[i].scales.data(), parts[i].scales.size(), cs[i].data()) == 1 &&
               qmr_pack_bf16_exact(parts[i].biases.data(), parts[i].biases.size(), cb[i].data()) == 1;
    }
    int rc = alloc_matrix(m, d, rows, p0.cols, p0.bits, p0.group, bf16);
    size_t woff = 0, moff = 0;
    for (size_t i = 0; i < parts.size() && rc == QMR_OK; ++i) {
        const HostMatrix &p = parts[i];
        rc = upload(m, static_cast<uint8_t *>(d->w) + woff, p.words.data(), p.words.size() * 4);
        const size_t esz = bf16 ? 2 : 4;
        const void *sp = bf16 ? (const void *)cs[i].data() : (const void *)p.scales.data();
        const void *bp = bf16 ? (const void *)cb[i].data() : (const void *)p.biases.data();
        if (rc == QMR_OK) rc = upload(m, static_cast<uint8_t *>(d->s) + moff, sp, p.scales.size() * esz);
        if (rc == QMR_OK) rc = upload(m, static_cast<uint8_t *>(d->b) + moff, bp, p.biases.size() * esz);
        if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "uploading a matrix");
        woff += p.words.size() * 4;
        moff += p.scales.size() * esz;
        if (bf16) {
            m->compacted += 1;
            m->saved_bytes += (p.scales.size() + p.biases.size()) * 2;
        }
    }
    return rc;
}

int load_vector(QmrModel *m, const Checkpoint &cp, const std::string &name, size_t n, float **out) {
    std::vector<float> v;
    int rc = cp.vector(name, &v);
    if (rc != QMR_OK) return rc;
    if (v.size() != n) return fail(QMR_EINVAL, "%s: expected %zu elements, got %zu", name.c_str(), n, v.size());
    return dev_vector(m, out, v);
}

int load_model(QmrModel *m, const std::string &dir, uint32_t context) {
    std::unique_ptr<Checkpoint> cp;
    int rc = Checkpoint::open(dir, &cp);
    if (rc != QMR_OK) return rc;
    const QmrModelConfig &c = cp->config();
    if (context == 0 || context > cp->max_position())
        return fail(QMR_EINVAL, "context must be in 1..=%u", cp->max_position());
    rc = create_common(m, c, context);
    if (rc != QMR_OK) return rc;
    const size_t H = c.hidden_size;
    rc = load_matrix(m, *cp, {"model.embed_tokens"}, &m->embed);
    if (rc == QMR_OK && (m->embed.rows != c.vocab_size || m->embed.cols != H))
        rc = fail(QMR_EINVAL, "model.embed_tokens: expected [%u,%zu]", c.vocab_size, H);
    for (uint32_t l = 0; l < c.num_layers && rc == QMR_OK; ++l) {
        LayerState &L = m->layers[l];
        const std::string p = "model.layers." + std::to_string(l);
        rc = load_vector(m, *cp, p + ".input_layernorm", H, &L.in_norm);
        if (rc == QMR_OK) rc = load_vector(m, *cp, p + ".post_attention_layernorm", H, &L.post_norm);
        if (rc == QMR_OK && L.attn) {
            const std::string a = p + ".self_attn.";
            rc = load_matrix(m, *cp, {a + "q_proj", a + "k_proj", a + "v_proj"}, &L.in);
            if (rc == QMR_OK) rc = load_matrix(m, *cp, {a + "o_proj"}, &L.out);
            if (rc == QMR_OK) rc = load_vector(m, *cp, a + "q_norm", c.head_dim, &L.qnorm);
            if (rc == QMR_OK) rc = load_vector(m, *cp, a + "k_norm", c.head_dim, &L.knorm);
        } else if (rc == QMR_OK) {
            const std::string a = p + ".linear_attn.";
            rc = load_matrix(m, *cp, {a + "in_proj_qkv", a + "in_proj_z", a + "in_proj_a", a + "in_proj_b"}, &L.in);
            if (rc == QMR_OK) rc = load_matrix(m, *cp, {a + "out_proj"}, &L.out);
            std::vector<float> conv;
            if (rc == QMR_OK) rc = cp->conv(a + "conv1d", (uint32_t)m->qkv_channels, c.conv_width, &conv);
            if (rc == QMR_OK) rc = dev_vector(m, &L.conv_w, conv);
            if (rc == QMR_OK) rc = load_vector(m, *cp, a + "A_log", c.linear_value_heads, &L.alog);
            if (rc == QMR_OK) rc = load_vector(m, *cp, a + "dt_bias", c.linear_value_heads, &L.dt);
            if (rc == QMR_OK) rc = load_vector(m, *cp, a + "norm", c.linear_value_dim, &L.dnorm);
        }
        if (rc == QMR_OK) rc = load_matrix(m, *cp, {p + ".mlp.gate_proj"}, &L.gate);
        if (rc == QMR_OK) rc = load_matrix(m, *cp, {p + ".mlp.up_proj"}, &L.up);
        if (rc == QMR_OK) rc = load_matrix(m, *cp, {p + ".mlp.down_proj"}, &L.down);
        if (rc == QMR_OK && (L.in.rows != in_rows(c, L.attn) || L.in.cols != H || L.out.rows != H ||
                             L.gate.rows != c.intermediate_size || L.gate.cols != H || L.up.rows != c.intermediate_size ||
                             L.down.rows != H || L.down.cols != c.intermediate_size ||
                             L.gate.bf16 != L.up.bf16 || L.gate.bits != L.up.bits || L.gate.group != L.up.group))
            rc = fail(QMR_EINVAL, "layer %u: matrix shapes do not match the config", l);
    }
    if (rc == QMR_OK) rc = load_vector(m, *cp, "model.norm", H, &m->final_norm);
    // A tied head is the embedding matrix itself (engine.rs:426-431).
    if (rc == QMR_OK) {
        if (cp->tied())
            m->head = m->embed;
        else
            rc = load_matrix(m, *cp, {"lm_head"}, &m->head);
    }
    if (rc == QMR_OK && (m->head.rows != c.vocab_size || m->head.cols != H))
        rc = fail(QMR_EINVAL, "lm_head: expected [%u,%zu]", c.vocab_size, H);
    return rc;
}

// ---- the synthetic model --------------------------------------------------------

// Rows [r0, r0 + nr) of synthetic matrix `mid` (full width `cols`), the
// parts stacked in order into one device matrix.
struct RowPart {
    uint32_t mid, r0, nr;
};

int synth_rows(QmrModel *m, DevMat *d, uint64_t seed, const std::vector<RowPart> &parts, uint32_t cols) {
    uint32_t rows = 0;
    for (const RowPart &p : parts) rows += p.nr;
    int rc = alloc_matrix(m, d, rows, cols, 4, 64, true);
    uint32_t dst = 0;
    for (const RowPart &p : parts) {
        if (rc != QMR_OK) break;
        rc = launch_synth_region(static_cast<uint32_t *>(d->w), static_cast<uint16_t *>(d->s),
                                 static_cast<uint16_t *>(d->b), seed, p.mid, cols, p.r0, p.nr, 0, cols, cols / 8,
                                 cols / 64, dst, m->stream);
        dst += p.nr;
    }
    return rc;
}

// Columns [c0, c0 + nc) of synthetic matrix `mid` (rows x full_cols): the
// input-side slice of a column-split matrix.  Its metadata rows are padded
// to a multiple of 8 groups (16-byte rows for the kernel's tensor maps).
int synth_cols(QmrModel *m, DevMat *d, uint64_t seed, uint32_t mid, uint32_t rows, uint32_t full_cols, uint32_t c0,
               uint32_t nc) {
    const uint32_t ng = nc / 64, mstride = (ng + 7) / 8 * 8;
    int rc = alloc_matrix(m, d, rows, nc, 4, 64, true, mstride == ng ? 0 : mstride);
    if (rc == QMR_OK)
        rc = launch_synth_region(static_cast<uint32_t *>(d->w), static_cast<uint16_t *>(d->s),
                                 static_cast<uint16_t *>(d->b), seed, mid, full_cols, 0, rows, c0, nc, nc / 8, mstride,
                                 0, m->stream);
    return rc;
}

// The synthetic model, or rank `rank`'s shard of it (the file comment gives
// the split); the matrices are regions of the same seeded matrices either way.
int synth_model(QmrModel *m, const QmrModelConfig &c, uint64_t seed, uint32_t context, uint32_t world = 1,
                uint32_t rank = 0) {
    if (c.hidden_size % 64 || c.intermediate_size % 64 || (c.linear_value_heads * c.linear_value_dim) % 64 ||
        (c.num_heads * c.head_dim) % 64)
        return fail(QMR_EINVAL, "synthetic Q4/g64 matrices need widths divisible by 64");
    int rc = create_common(m, c, context, world, rank);
    if (rc != QMR_OK) return rc;
    const QmrModelConfig &l = m->lc;
    const uint32_t H = c.hidden_size, F = c.intermediate_size, Fl = l.intermediate_size;
    const uint32_t KD = c.linear_key_heads * c.linear_key_dim, VD = c.linear_value_heads * c.linear_value_dim;
    const uint32_t KDl = l.linear_key_heads * l.linear_key_dim, VDl = l.linear_value_heads * l.linear_value_dim;
    const uint32_t QD = c.num_heads * c.head_dim, QDl = l.num_heads * l.head_dim;
    const uint32_t KVD = c.num_kv_heads * c.head_dim, KVDl = l.num_kv_heads * l.head_dim;
    const uint32_t VHl = l.linear_value_heads, r = rank, kvr0 = m->kv0 * c.head_dim;
    (void)KVD;
    rc = synth_rows(m, &m->embed, seed, {{kMidEmbed, 0, c.vocab_size}}, H);
    if (rc == QMR_OK) rc = synth_rows(m, &m->head, seed, {{kMidHead, m->vbase, l.vocab_size}}, H);
    if (rc == QMR_OK) rc = dev_const(m, &m->final_norm, H, 1.0f);
    for (uint32_t li = 0; li < c.num_layers && rc == QMR_OK; ++li) {
        LayerState &L = m->layers[li];
        rc = dev_const(m, &L.in_norm, H, 1.0f);
        if (rc == QMR_OK) rc = dev_const(m, &L.post_norm, H, 1.0f);
        if (rc == QMR_OK && L.attn) {
            // q|gate rows of this rank's query heads ([head][2][D]), k and v rows of its KV heads.
            rc = synth_rows(m, &L.in, seed,
                            {{synth_mid(li, S_Q), r * 2 * QDl, 2 * QDl}, {synth_mid(li, S_K), kvr0, KVDl},
                             {synth_mid(li, S_V), kvr0, KVDl}}, H);
            if (rc == QMR_OK) rc = synth_cols(m, &L.out, seed, synth_mid(li, S_O), H, QD, r * QDl, QDl);
            if (rc == QMR_OK) rc = dev_const(m, &L.qnorm, c.head_dim, 1.0f);
            if (rc == QMR_OK) rc = dev_const(m, &L.knorm, c.head_dim, 1.0f);
        } else if (rc == QMR_OK) {
            // q, k, v channels of this rank's key / value heads, then z, a, b of its value heads.
            rc = synth_rows(m, &L.in, seed,
                            {{synth_mid(li, S_QKV), r * KDl, KDl}, {synth_mid(li, S_QKV), KD + r * KDl, KDl},
                             {synth_mid(li, S_QKV), 2 * KD + r * VDl, VDl}, {synth_mid(li, S_Z), r * VDl, VDl},
                             {synth_mid(li, S_A), r * VHl, VHl}, {synth_mid(li, S_B), r * VHl, VHl}},
                            H);
            if (rc == QMR_OK) rc = synth_cols(m, &L.out, seed, synth_mid(li, S_OUT), H, VD, r * VDl, VDl);
            if (rc == QMR_OK) rc = dev_const(m, &L.conv_w, m->qkv_channels * c.conv_width, 0.1f);
            if (rc == QMR_OK) rc = dev_const(m, &L.alog, VHl, 0.0f);
            if (rc == QMR_OK) rc = dev_const(m, &L.dt, VHl, 0.0f);
            if (rc == QMR_OK) rc = dev_const(m, &L.dnorm, c.linear_value_dim, 1.0f);
        }
        if (rc == QMR_OK) rc = synth_rows(m, &L.gate, seed, {{synth_mid(li, S_GATE), r * Fl, Fl}}, H);
        if (rc == QMR_OK) rc = synth_rows(m, &L.up, seed, {{synth_mid(li, S_UP), r * Fl, Fl}}, H);
        if (rc == QMR_OK) rc = synth_cols(m, &L.down, seed, synth_mid(li, S_DOWN), H, F, r * Fl, Fl);
    }
    if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "generating the synthetic model");
    return rc;
}

// Exchange memory of a sharded model: its own allocation (IPC-shareable).
constexpr size_t kFlagsOff = 0, kHFlagsOff = 256, kKeysOff = 512, kEpochOff = 768, kHEpochOff = 772, kCtlBytes = 1024;

int alloc_exchange(QmrModel *m) {
    m->xslot = ((size_t)kMaxBlock * m->world * m->lc.hidden_size * 4 + 255) / 256 * 256;
    void *p = nullptr;
    const int rc = qmr_exchange_alloc(2 * m->xslot + kCtlBytes, &p);
    m->xbuf = static_cast<uint8_t *>(p);
    return rc;
}

// Fill the two partial-sum exchanges and the head exchange from every
// rank's exchange memory (this rank's own and the mapped peers').
void wire_exchanges(QmrModel *m, uint8_t *const *base) {
    const uint32_t H = m->lc.hidden_size;
    for (int par = 0; par < 2; ++par) {
        QmrExchange &x = m->xch[par];
        x = QmrExchange{};
        x.world = m->world;
        x.rank = m->rank;
        x.total_rows = m->world * H;
        x.row_base = m->rank * H;
        for (uint32_t p = 0; p < m->world; ++p) {
            x.out[p] = reinterpret_cast<float *>(base[p] + par * m->xslot);
            x.flags[p] = reinterpret_cast<uint32_t *>(base[p] + 2 * m->xslot + kFlagsOff);
        }
        x.epoch = reinterpret_cast<uint32_t *>(m->xbuf + 2 * m->xslot + kEpochOff);
    }
    QmrExchange &h = m->hxch;
    h = QmrExchange{};
    h.world = m->world;
    h.rank = m->rank;
    h.total_rows = m->cfg.vocab_size;
    h.row_base = m->vbase;
    for (uint32_t p = 0; p < m->world; ++p) {
        h.flags[p] = reinterpret_cast<uint32_t *>(base[p] + 2 * m->xslot + kHFlagsOff);
        h.keys[p] = reinterpret_cast<uint64_t *>(base[p] + 2 * m->xslot + kKeysOff);
    }
    h.epoch = reinterpret_cast<uint32_t *>(m->xbuf + 2 * m->xslot + kHEpochOff);
}

int finish_create(QmrModel *m, QmrModel **out) {
    int rc = build_graphs(m);
    if (rc == QMR_OK) rc = check_device_error();
    if (rc != QMR_OK) {
        delete m;
        return rc;
    }
    *out = m;
    return QMR_OK;
}

int replay(QmrModel *m, int kind, uint32_t times) {
    for (uint32_t i = 0; i < times; ++i) {
        const int rc = cuda_check(cudaGraphLaunch(m->exec[kind], m->stream), "graph launch");
        if (rc != QMR_OK) return rc;
    }
    return QMR_OK;
}

// Prompt positions without the head: prefill blocks, then single steps for
// the remainder.
int prefill(QmrModel *m, uint32_t n) {
    const uint32_t nb = m->exec[2] != nullptr ? n / (uint32_t)kPrefillBlock : 0u;
    int rc = replay(m, 2, nb);
    if (rc == QMR_OK) rc = replay(m, 0, n - nb * (uint32_t)kPrefillBlock);
    return rc;
}

}  // namespace
}  // namespace qmr

extern "C" {

int qmr_checkpoint_open(const char *dir, QmrCheckpoint **out) {
    if (dir == nullptr || out == nullptr) return fail(QMR_EINVAL, "null argument");
    std::unique_ptr<Checkpoint> cp;
    const int rc = Checkpoint::open(dir, &cp);
    if (rc != QMR_OK) return rc;
    *out = reinterpret_cast<QmrCheckpoint *>(cp.release());
    return QMR_OK;
}

void qmr_checkpoint_close(QmrCheckpoint *cp) { delete reinterpret_cast<Checkpoint *>(cp); }

int qmr_checkpoint_config(const QmrCheckpoint *cp, QmrModelConfig *cfg, uint32_t *max_position, int *tied) {
    if (cp == nullptr) return fail(QMR_EINVAL, "null checkpoint");
    const Checkpoint *c = reinterpret_cast<const Checkpoint *>(cp);
    if (cfg) *cfg = c->config();
    if (max_position) *max_position = c->max_position();
    if (tied) *tied = c->tied() ? 1 : 0;
    return QMR_OK;
}

int qmr_checkpoint_matrix(const QmrCheckpoint *cp, const char *name, uint32_t *rows, uint32_t *cols, uint32_t *bits,
                          uint32_t *group, uint32_t *w, float *s, float *b) {
    if (cp == nullptr || name == nullptr) return fail(QMR_EINVAL, "null argument");
    HostMatrix m;
    const int rc = reinterpret_cast<const Checkpoint *>(cp)->matrix(name, &m);
    if (rc != QMR_OK) return rc;
    if (rows) *rows = m.rows;
    if (cols) *cols = m.cols;
    if (bits) *bits = m.bits;
    if (group) *group = m.group;
    if (w) memcpy(w, m.words.data(), m.words.size() * 4);
    if (s) memcpy(s, m.scales.data(), m.scales.size() * 4);
    if (b) memcpy(b, m.biases.data(), m.biases.size() * 4);
    return QMR_OK;
}

int qmr_checkpoint_vector(const QmrCheckpoint *cp, const char *name, float *out, uint64_t cap, uint64_t *n) {
    if (cp == nullptr || name == nullptr) return fail(QMR_EINVAL, "null argument");
    std::vector<float> v;
    const int rc = reinterpret_cast<const Checkpoint *>(cp)->vector(name, &v);
    if (rc != QMR_OK) return rc;
    if (n) *n = v.size();
    if (out != nullptr) {
        if (cap < v.size()) return fail(QMR_ERANGE, "vector of %zu elements does not fit %llu", v.size(), (unsigned long long)cap);
        memcpy(out, v.data(), v.size() * 4);
    }
    return QMR_OK;
}

int qmr_model_load(const char *dir, uint32_t context, QmrModel **out) {
    if (dir == nullptr || out == nullptr) return fail(QMR_EINVAL, "null argument");
    QmrModel *m = new QmrModel();
    const int rc = load_model(m, dir, context);
    if (rc != QMR_OK) {
        delete m;
        return rc;
    }
    return finish_create(m, out);
}

int qmr_model_synthetic(const QmrModelConfig *cfg, uint64_t seed, uint32_t context, QmrModel **out) {
    if (cfg == nullptr || out == nullptr) return fail(QMR_EINVAL, "null argument");
    QmrModel *m = new QmrModel();
    const int rc = synth_model(m, *cfg, seed, context);
    if (rc != QMR_OK) {
        delete m;
        return rc;
    }
    return finish_create(m, out);
}

int qmr_model_synthetic_sharded(const QmrModelConfig *cfg, uint64_t seed, uint32_t context, uint32_t world,
                                uint32_t rank, QmrModel **out) {
    if (cfg == nullptr || out == nullptr) return fail(QMR_EINVAL, "null argument");
    if (world == 0 || world > QMR_MAX_RANKS || rank >= world)
        return fail(QMR_EINVAL, "world must be 1..%d and rank < world", QMR_MAX_RANKS);
    if (world == 1) return qmr_model_synthetic(cfg, seed, context, out);
    QmrModel *m = new QmrModel();
    int rc = synth_model(m, *cfg, seed, context, world, rank);
    if (rc == QMR_OK) rc = alloc_exchange(m);
    if (rc != QMR_OK) {
        delete m;
        return rc;
    }
    m->opened = false;
    *out = m;
    return QMR_OK;
}

int qmr_model_exchange_handle(const QmrModel *m, void *handle) {
    if (m == nullptr || handle == nullptr) return fail(QMR_EINVAL, "null argument");
    if (m->world < 2 || m->xbuf == nullptr) return fail(QMR_EINVAL, "the model is not sharded");
    DeviceGuard g(m->device);
    return qmr_ipc_handle(m->xbuf, handle);
}

int qmr_model_exchange_open(QmrModel *m, const void *handles) {
    if (m == nullptr || handles == nullptr) return fail(QMR_EINVAL, "null argument");
    if (m->world < 2 || m->xbuf == nullptr) return fail(QMR_EINVAL, "the model is not sharded");
    if (m->opened) return fail(QMR_EINVAL, "the exchange is already open");
    DeviceGuard g(m->device);
    uint8_t *base[QMR_MAX_RANKS] = {};
    const uint8_t *h = static_cast<const uint8_t *>(handles);
    int rc = QMR_OK;
    for (uint32_t r = 0; r < m->world && rc == QMR_OK; ++r) {
        if (r == m->rank) {
            base[r] = m->xbuf;
            continue;
        }
        void *p = nullptr;
        rc = qmr_ipc_open(h + (size_t)r * QMR_IPC_HANDLE_BYTES, &p);
        m->peers[r] = p;
        base[r] = static_cast<uint8_t *>(p);
    }
    if (rc != QMR_OK) return rc;
    wire_exchanges(m, base);
    m->opened = true;
    // The warm-up steps exchange with the peers: every rank opens together.
    rc = build_graphs(m);
    if (rc == QMR_OK) rc = check_device_error();
    if (rc != QMR_OK) m->opened = false;
    return rc;
}

int qmr_model_shard(const QmrModel *m, uint32_t *world, uint32_t *rank, uint32_t *vocab_base, uint32_t *vocab_rows) {
    if (m == nullptr) return fail(QMR_EINVAL, "null model");
    if (world) *world = m->world;
    if (rank) *rank = m->rank;
    if (vocab_base) *vocab_base = m->vbase;
    if (vocab_rows) *vocab_rows = m->lc.vocab_size;
    return QMR_OK;
}

void qmr_model_free(QmrModel *m) { delete m; }

int qmr_model_config(const QmrModel *m, QmrModelConfig *cfg, uint32_t *context) {
    if (m == nullptr) return fail(QMR_EINVAL, "null model");
    if (cfg) *cfg = m->cfg;
    if (context) *context = m->context;
    return QMR_OK;
}

int qmr_model_reset(QmrModel *m) {
    if (m == nullptr) return fail(QMR_EINVAL, "null model");
    if (!m->opened) return fail(QMR_EINVAL, "open the sharded model's exchange first");
    DeviceGuard g(m->device);
    return clear_state(m);
}

int qmr_model_position(const QmrModel *m, uint32_t *pos) {
    if (m == nullptr || pos == nullptr) return fail(QMR_EINVAL, "null argument");
    *pos = m->pos;
    return QMR_OK;
}

int qmr_model_forward(QmrModel *m, uint32_t token, float *logits, int32_t *next) {
    if (m == nullptr) return fail(QMR_EINVAL, "null model");
    if (!m->opened) return fail(QMR_EINVAL, "open the sharded model's exchange first");
    if (m->pending) return fail(QMR_EINVAL, "commit or reset the pending verification block before a normal forward");
    if (token >= m->cfg.vocab_size) return fail(QMR_EINVAL, "token %u outside vocabulary", token);
    if (m->pos >= m->context) return fail(QMR_ERANGE, "context capacity %u exhausted", m->context);
    DeviceGuard g(m->device);
    m->host_stage[0] = (int32_t)token;
    m->host_stage[1] = 0;  // n_prompt: the token comes from ctrl->token
    int rc = cuda_check(cudaMemcpyAsync(&m->ctrl->token, m->host_stage, 8, cudaMemcpyHostToDevice, m->stream),
                        "writing the step token");
    if (rc == QMR_OK) rc = replay(m, 1, 1);
    if (rc == QMR_OK && logits != nullptr)
        rc = cuda_check(cudaMemcpyAsync(logits, m->logits, (size_t)m->lc.vocab_size * 4, cudaMemcpyDeviceToHost,
                                        m->stream), "reading logits");
    if (rc == QMR_OK)
        rc = cuda_check(cudaMemcpyAsync(m->host_stage + 2, &m->ctrl->token, 4, cudaMemcpyDeviceToHost, m->stream),
                        "reading the argmax");
    if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "forward");
    if (rc == QMR_OK) rc = check_device_error();
    if (rc != QMR_OK) {
        // A failed step may have updated recurrent state; never reuse it (engine.rs:591-595).
        clear_state(m);
        return rc;
    }
    if (next) *next = m->host_stage[2];
    m->pos += 1;
    return QMR_OK;
}

int qmr_model_generate(QmrModel *m, const uint32_t *prompt, uint32_t n_prompt, uint32_t max_new, uint32_t *out,
                       double *prefill_ms, double *decode_ms) {
    if (m == nullptr || prompt == nullptr || out == nullptr) return fail(QMR_EINVAL, "null argument");
    if (n_prompt == 0 || max_new == 0) return fail(QMR_EINVAL, "empty prompt or max_new = 0");
    if (!m->opened) return fail(QMR_EINVAL, "open the sharded model's exchange first");
    if (m->pending) return fail(QMR_EINVAL, "commit or reset the pending verification block first");
    for (uint32_t i = 0; i < n_prompt; ++i)
        if (prompt[i] >= m->cfg.vocab_size) return fail(QMR_EINVAL, "prompt token %u outside vocabulary", prompt[i]);
    if ((uint64_t)m->pos + n_prompt + max_new - 1 > m->context)
        return fail(QMR_ERANGE, "prompt (%u tokens) plus max_new (%u) exceeds context %u", n_prompt, max_new, m->context);
    DeviceGuard g(m->device);
    std::vector<int32_t> p(prompt, prompt + n_prompt);
    int rc = cuda_check(cudaMemcpyAsync(m->prompt + m->pos, p.data(), (size_t)n_prompt * 4, cudaMemcpyHostToDevice,
                                        m->stream), "uploading the prompt");
    const uint32_t hdr[2] = {m->pos + n_prompt, 0u};  // n_prompt (absolute), n_out
    if (rc == QMR_OK)
        rc = cuda_check(cudaMemcpyAsync(&m->ctrl->n_prompt, hdr, 8, cudaMemcpyHostToDevice, m->stream), "control block");
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    for (int i = 0; i < 3 && rc == QMR_OK; ++i) rc = cuda_check(cudaEventCreate(&ev[i]), "event");
    if (rc == QMR_OK) rc = cuda_check(cudaEventRecord(ev[0], m->stream), "event");
    if (rc == QMR_OK) rc = prefill(m, n_prompt - 1);
    if (rc == QMR_OK) rc = replay(m, 1, 1);
    if (rc == QMR_OK) rc = cuda_check(cudaEventRecord(ev[1], m->stream), "event");
    if (rc == QMR_OK) rc = replay(m, 1, max_new - 1);
    if (rc == QMR_OK) rc = cuda_check(cudaEventRecord(ev[2], m->stream), "event");
    std::vector<int32_t> toks(max_new);
    if (rc == QMR_OK)
        rc = cuda_check(cudaMemcpyAsync(toks.data(), m->out, (size_t)max_new * 4, cudaMemcpyDeviceToHost, m->stream),
                        "reading tokens");
    if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "generate");
    if (rc == QMR_OK) rc = check_device_error();
    float t01 = 0, t12 = 0;
    if (rc == QMR_OK) rc = cuda_check(cudaEventElapsedTime(&t01, ev[0], ev[1]), "event time");
    if (rc == QMR_OK) rc = cuda_check(cudaEventElapsedTime(&t12, ev[1], ev[2]), "event time");
    for (auto e : ev)
        if (e != nullptr) cudaEventDestroy(e);
    if (rc != QMR_OK) {
        clear_state(m);
        return rc;
    }
    for (uint32_t i = 0; i < max_new; ++i) out[i] = (uint32_t)toks[i];
    if (prefill_ms) *prefill_ms = t01;
    if (decode_ms) *decode_ms = t12;
    m->pos += n_prompt + max_new - 1;
    return QMR_OK;
}

int qmr_model_verify_block(QmrModel *m, const uint32_t *tokens, uint32_t n, float *logits, int32_t *argmax) {
    if (m == nullptr || tokens == nullptr) return fail(QMR_EINVAL, "null argument");
    if (!m->opened) return fail(QMR_EINVAL, "open the sharded model's exchange first");
    if (m->pending) return fail(QMR_EINVAL, "commit or reset the pending verification block before another block");
    if (n < 1 || n > (uint32_t)kMaxBlock) return fail(QMR_EINVAL, "verification block width must be 1..=4");
    for (uint32_t i = 0; i < n; ++i)
        if (tokens[i] >= m->cfg.vocab_size) return fail(QMR_EINVAL, "verification block contains a token outside vocabulary");
    if ((uint64_t)m->pos + n > m->context)
        return fail(QMR_ERANGE, "verification block exceeds context capacity %u", m->context);
    DeviceGuard g(m->device);
    int rc = ensure_block(m, (int)n);
    // Input 0 is the anchor (ctrl->token); inputs 1.. come from the draft table.
    std::vector<int32_t> t(tokens, tokens + n);
    m->host_stage[0] = t[0];
    m->host_stage[1] = 0;
    if (rc == QMR_OK)
        rc = cuda_check(cudaMemcpyAsync(&m->ctrl->token, m->host_stage, 8, cudaMemcpyHostToDevice, m->stream),
                        "block anchor");
    if (rc == QMR_OK && n > 1)
        rc = cuda_check(cudaMemcpyAsync(m->drafts + m->pos + 1, t.data() + 1, (size_t)(n - 1) * 4,
                                        cudaMemcpyHostToDevice, m->stream), "block inputs");
    if (rc == QMR_OK) rc = cuda_check(cudaGraphLaunch(m->bexec[0][n], m->stream), "graph launch");
    if (rc == QMR_OK && logits != nullptr)
        rc = cuda_check(cudaMemcpyAsync(logits, m->logits, (size_t)n * m->lc.vocab_size * 4, cudaMemcpyDeviceToHost,
                                        m->stream), "reading logits");
    if (rc == QMR_OK && argmax != nullptr)
        rc = cuda_check(cudaMemcpyAsync(argmax, m->block_argmax, (size_t)n * 4, cudaMemcpyDeviceToHost, m->stream),
                        "reading argmax");
    if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "verify block");
    if (rc == QMR_OK) rc = check_device_error();
    if (rc != QMR_OK) {
        clear_state(m);
        return rc;
    }
    m->pending = true;
    m->pending_width = n;
    m->pos += n;
    return QMR_OK;
}

int qmr_model_commit_block(QmrModel *m, uint32_t consumed) {
    if (m == nullptr) return fail(QMR_EINVAL, "null model");
    if (!m->opened) return fail(QMR_EINVAL, "open the sharded model's exchange first");
    if (!m->pending) return fail(QMR_EINVAL, "there is no pending verification block");
    if (consumed > m->pending_width) return fail(QMR_EINVAL, "accepted prefix exceeds pending block length");
    DeviceGuard g(m->device);
    const uint32_t base = m->pos - m->pending_width;
    const QmrModelConfig &c = m->lc;
    m->host_stage[0] = (int32_t)consumed;
    m->host_stage[4] = (int32_t)(base + consumed);
    int rc = cuda_check(cudaMemcpyAsync(&m->bctrl->consumed, m->host_stage, 4, cudaMemcpyHostToDevice, m->stream),
                        "commit");
    if (rc == QMR_OK)
        rc = cuda_check(cudaMemcpyAsync(&m->ctrl->pos, m->host_stage + 4, 4, cudaMemcpyHostToDevice, m->stream), "commit");
    if (rc == QMR_OK)
        rc = launch_commit(m->bctrl, m->layer_ptrs, m->ndelta, (int)m->pending_width, m->qkv_channels * (c.conv_width - 1),
                           (size_t)c.linear_value_heads * c.linear_value_dim * c.linear_key_dim, m->stream);
    if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "commit");
    if (rc != QMR_OK) {
        clear_state(m);
        return rc;
    }
    m->pending = false;
    m->pos = base + consumed;
    return QMR_OK;
}

int qmr_model_mtp_generate(QmrModel *m, const uint32_t *prompt, uint32_t n_prompt, uint32_t block, uint32_t max_new,
                           const uint32_t *drafts, uint32_t n_drafts, uint32_t *out, uint32_t *rounds,
                           uint32_t *accepted, double *prefill_ms, double *decode_ms) {
    if (m == nullptr || prompt == nullptr || out == nullptr || drafts == nullptr) return fail(QMR_EINVAL, "null argument");
    if (!m->opened) return fail(QMR_EINVAL, "open the sharded model's exchange first");
    if (block < 2 || block > (uint32_t)kMaxBlock) return fail(QMR_EINVAL, "MTP block width must be 2..=4");
    if (n_prompt == 0 || max_new == 0) return fail(QMR_EINVAL, "empty prompt or max_new = 0");
    if (m->pending) return fail(QMR_EINVAL, "commit or reset the pending verification block first");
    for (uint32_t i = 0; i < n_prompt; ++i)
        if (prompt[i] >= m->cfg.vocab_size) return fail(QMR_EINVAL, "prompt token %u outside vocabulary", prompt[i]);
    for (uint32_t i = 0; i < n_drafts; ++i)
        if (drafts[i] >= m->cfg.vocab_size) return fail(QMR_EINVAL, "draft token %u outside vocabulary", drafts[i]);
    if ((uint64_t)m->pos + n_prompt + max_new - 1 + block > m->context)
        return fail(QMR_ERANGE, "prompt (%u) plus max_new (%u) plus a block (%u) exceeds context %u", n_prompt, max_new,
                    block, m->context);
    DeviceGuard g(m->device);
    int rc = ensure_block(m, (int)block);
    const uint32_t base = m->pos;
    std::vector<int32_t> p(prompt, prompt + n_prompt);
    if (rc == QMR_OK)
        rc = cuda_check(cudaMemcpyAsync(m->prompt + base, p.data(), (size_t)n_prompt * 4, cudaMemcpyHostToDevice,
                                        m->stream), "uploading the prompt");
    const uint32_t hdr[2] = {base + n_prompt, 0u};
    if (rc == QMR_OK)
        rc = cuda_check(cudaMemcpyAsync(&m->ctrl->n_prompt, hdr, 8, cudaMemcpyHostToDevice, m->stream), "control block");
    std::vector<int32_t> table(m->context + kMaxBlock, 0);
    for (uint32_t i = 0; i < n_drafts && i < m->context; ++i) table[i] = (int32_t)drafts[i];
    if (rc == QMR_OK)
        rc = cuda_check(cudaMemcpyAsync(m->drafts, table.data(), table.size() * 4, cudaMemcpyHostToDevice, m->stream),
                        "uploading the draft table");
    if (rc == QMR_OK) rc = cuda_check(cudaMemsetAsync(m->bctrl, 0, sizeof(BlockCtrl), m->stream), "block control");
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    for (int i = 0; i < 3 && rc == QMR_OK; ++i) rc = cuda_check(cudaEventCreate(&ev[i]), "event");
    if (rc == QMR_OK) rc = cuda_check(cudaEventRecord(ev[0], m->stream), "event");
    if (rc == QMR_OK) rc = prefill(m, n_prompt - 1);
    if (rc == QMR_OK) rc = replay(m, 1, 1);  // the prompt's last token emits the first output
    if (rc == QMR_OK) rc = cuda_check(cudaEventRecord(ev[1], m->stream), "event");
    // Rounds of verification, replayed in batches; every round emits 1..block
    // tokens, so a batch sized for full acceptance never overshoots by more
    // than one round.
    uint32_t n_out = 1, pos = base + n_prompt;
    while (rc == QMR_OK && n_out < max_new && (uint64_t)pos + block <= m->context) {
        uint32_t k = (max_new - n_out + block - 1) / block;
        const uint32_t room = (m->context - pos) / block;
        if (k > room) k = room;
        if (k == 0) break;
        for (uint32_t i = 0; i < k && rc == QMR_OK; ++i)
            rc = cuda_check(cudaGraphLaunch(m->bexec[1][block], m->stream), "graph launch");
        if (rc == QMR_OK)
            rc = cuda_check(cudaMemcpyAsync(m->host_stage, m->ctrl, 16, cudaMemcpyDeviceToHost, m->stream), "control");
        if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "verification rounds");
        pos = (uint32_t)m->host_stage[0];
        n_out = (uint32_t)m->host_stage[3];
    }
    if (rc == QMR_OK) rc = cuda_check(cudaEventRecord(ev[2], m->stream), "event");
    std::vector<int32_t> toks(n_out);
    BlockCtrl bc{};
    if (rc == QMR_OK)
        rc = cuda_check(cudaMemcpyAsync(toks.data(), m->out, (size_t)n_out * 4, cudaMemcpyDeviceToHost, m->stream),
                        "reading tokens");
    if (rc == QMR_OK) rc = cuda_check(cudaMemcpyAsync(&bc, m->bctrl, sizeof bc, cudaMemcpyDeviceToHost, m->stream), "stats");
    if (rc == QMR_OK) rc = cuda_check(cudaStreamSynchronize(m->stream), "mtp generate");
    if (rc == QMR_OK) rc = check_device_error();
    float t01 = 0, t12 = 0;
    if (rc == QMR_OK) rc = cuda_check(cudaEventElapsedTime(&t01, ev[0], ev[1]), "event time");
    if (rc == QMR_OK) rc = cuda_check(cudaEventElapsedTime(&t12, ev[1], ev[2]), "event time");
    for (auto e : ev)
        if (e != nullptr) cudaEventDestroy(e);
    if (rc != QMR_OK) {
        clear_state(m);
        return rc;
    }
    if (n_out < max_new) return fail(QMR_ERANGE, "context filled after %u of %u tokens", n_out, max_new);
    for (uint32_t i = 0; i < max_new; ++i) out[i] = (uint32_t)toks[i];
    if (rounds) *rounds = bc.rounds;
    if (accepted) *accepted = bc.drafts_accepted;
    if (prefill_ms) *prefill_ms = t01;
    if (decode_ms) *decode_ms = t12;
    m->pos = pos;
    return QMR_OK;
}

int qmr_model_mlp_r2_eligible(const QmrModel *m, uint32_t *count) {
    if (m == nullptr || count == nullptr) return fail(QMR_EINVAL, "null argument");
    uint32_t n = 0;
    if (modes_gemv_aligned())
        for (const LayerState &L : m->layers)
            for (const DevMat *d : {&L.gate, &L.up, &L.down})
                if (d->bf16 && d->bits == 4 && d->group == 64 &&
                    ((d->rows == 17408 && d->cols == 5120) || (d->rows == 5120 && d->cols == 17408)))
                    ++n;
    *count = n;
    return QMR_OK;
}

int qmr_model_metadata_stats(const QmrModel *m, uint64_t *matrices, uint64_t *saved_bytes) {
    if (m == nullptr) return fail(QMR_EINVAL, "null model");
    if (matrices) *matrices = m->compacted;
    if (saved_bytes) *saved_bytes = m->saved_bytes;
    return QMR_OK;
}

int qmr_model_step_launches(const QmrModel *m, uint32_t *with_head, uint32_t *without_head) {
    if (m == nullptr) return fail(QMR_EINVAL, "null model");
    if (with_head) *with_head = m->launches[1];
    if (without_head) *without_head = m->launches[0];
    return QMR_OK;
}

}  // extern "C"
