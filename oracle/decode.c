/*
 * FP64 oracle of one decode step of the hybrid Qwen3.5 graph.  TEST
 * INFRASTRUCTURE ONLY: tests, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg call it as the checker; the product (libqmr) never links it.
 *
 * It restates, in double precision throughout, the reference's per-token
 * graph (rucin93/qwen-mlx-runner v0.7.3, src/engine.rs:607-797) with the
 * element semantics of its kernels (kernels/qwen.metal:78-258) and of its
 * independent scalar oracle (scripts/make_fixture.py:77-151, `forward`):
 *   x = embed(token)                                      affine_bf16.metal:439-451
 *   per layer: n = rms(x) * w_in                          qwen.metal:78-86
 *     DeltaNet (qwen.metal:95-183, make_fixture.py:88-112):
 *       qkv, z, a, b = W n; conv_silu over the last `width` inputs per
 *       channel (oldest first); q /= sqrt(|q|^2+eps)*sqrt(K), k /= sqrt(|k|^2+eps);
 *       decay = exp(-exp(A_log) * softplus(a + dt)), beta = sigmoid(b);
 *       per value row: S = S*decay; delta = beta*(v - S.k); S += k*delta;
 *       y = S.q; y = rms(y)*w_norm * silu(z); out = W_out y
 *     attention (qwen.metal:184-258, make_fixture.py:113-131):
 *       q|gate per head, k, v = W n; head rms on q and k; partial
 *       rotate-half RoPE on the first rotary_dim dims (frequency exponent
 *       2i/rotary_dim); append k, v; softmax(q.k/sqrt(D)) over positions
 *       0..pos of the head's KV group; out = (p.v) * sigmoid(gate); W_o out
 *     x += out; n = rms(x) * w_post; x += W_down(silu(W_gate n) * (W_up n))
 *   logits = W_head (rms(x) * w_final)
 * Recurrent state, convolution history and the KV cache are FP64 here.
 *
 * Matrices are packed affine (Q4/Q8, f32 or BF16 metadata) as in the matrix
 * oracle, or synthetic: words and metadata generated on the fly by the
 * counter-based generator below, which the device generator reproduces bit
 * for bit.  Matrix-vector products use four interleaved FP64 partial sums per
 * row (the order differs from a left-to-right sum by about 1e-16 relative).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- counter-based synthetic generator (shared with the device) --------- */

static inline uint64_t sg_mix(uint64_t z) {
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ull;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBull;
    z ^= z >> 31;
    return z;
}

static inline uint64_t sg_key(uint64_t seed, uint64_t mid, uint64_t tag) {
    return sg_mix(seed ^ (mid * 0x9E3779B97F4A7C15ull) ^ (tag * 0xD1B54A32D192ED03ull));
}

static inline uint16_t sg_bf16_rne(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

static inline float sg_bf16_f32(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Word pair j (words 2j and 2j+1 of the flat [rows][cols*4/32] array). */
uint64_t or_synth_pair(uint64_t seed, uint32_t mid, uint64_t j) {
    return sg_mix(sg_key(seed, mid, 1) + (j + 1) * 0x9E3779B97F4A7C15ull);
}

/* Scale and bias (BF16 bits) of flat group g: scale uniform in [0.002, 0.02]
 * rounded to BF16; bias = BF16(-8*scale + 1e-3 * n), n an Irwin-Hall sum of
 * four 16-bit uniforms scaled to unit variance (a normal approximation that
 * is plain arithmetic, so it is reproducible on the device). */
void or_synth_meta(uint64_t seed, uint32_t mid, uint64_t g, uint16_t *scale, uint16_t *bias) {
    const uint64_t h = sg_mix(sg_key(seed, mid, 2) + (g + 1) * 0x9E3779B97F4A7C15ull);
    const double u = (double)(h >> 11) * (1.0 / 9007199254740992.0);
    const float s32 = (float)(0.002 + 0.018 * u);
    const uint16_t sb = sg_bf16_rne(s32);
    const uint64_t h2 = sg_mix(h ^ sg_key(seed, mid, 3));
    double n = 0.0;
    for (int k = 0; k < 4; ++k) n = n + ((double)((h2 >> (16 * k)) & 0xffffu) + 0.5) * (1.0 / 65536.0);
    n = (n - 2.0) * 1.7320508075688772;
    const float b32 = (float)(-8.0 * (double)sg_bf16_f32(sb) + 1e-3 * n);
    *scale = sb;
    *bias = sg_bf16_rne(b32);
}

/* Materialise a synthetic Q4/g64 matrix (for small shapes and for tests of
 * the generator itself). */
void or_synth_matrix(uint64_t seed, uint32_t mid, uint32_t rows, uint32_t cols, uint32_t *w, uint16_t *s,
                     uint16_t *b) {
    const uint64_t words = (uint64_t)rows * cols / 8;
    for (uint64_t j = 0; j < words / 2; ++j) {
        const uint64_t h = or_synth_pair(seed, mid, j);
        w[2 * j] = (uint32_t)h;
        w[2 * j + 1] = (uint32_t)(h >> 32);
    }
    const uint64_t groups = (uint64_t)rows * cols / 64;
    for (uint64_t g = 0; g < groups; ++g) or_synth_meta(seed, mid, g, &s[g], &b[g]);
}

/* ---- model ---------------------------------------------------------------- */

typedef struct {
    const uint32_t *w;
    const void *s, *b;
    int bf16;
    uint32_t rows, cols, bits, group;
    int synth;
    uint64_t seed;
    uint32_t mid;
} or_mat;

enum { M_QKV, M_Z, M_A, M_B, M_OUT, M_Q, M_K, M_V, M_O, M_GATE, M_UP, M_DOWN, M_COUNT };
enum { V_IN, V_POST, V_CONV, V_ALOG, V_DT, V_DNORM, V_QNORM, V_KNORM, V_COUNT };

typedef struct {
    /* config: hidden, inter, layers, heads, kv_heads, head_dim, vocab,
     * lin key heads, lin value heads, key dim, value dim, conv width, rotary dim */
    uint32_t H, F, L, NH, NKV, D, VOCAB, KH, VH, K, V, W, RD;
    double eps, theta;
    uint32_t context;
    uint8_t *is_attn;
    or_mat *mats;     /* [L][M_COUNT] */
    or_mat embed, head;
    const float **vecs; /* [L][V_COUNT] */
    const float *final_norm;
    /* state */
    double *conv;     /* per delta layer [qkv][W-1] */
    double *dstate;   /* per delta layer [VH][V][K] */
    double *kc, *vc;  /* per attention layer [context][NKV][D] */
    uint32_t pos;
} or_model;

or_model *or_model_new(const uint32_t *cfg, const double *fcfg, const uint8_t *is_attn, uint32_t context) {
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->H = cfg[0];
    m->F = cfg[1];
    m->L = cfg[2];
    m->NH = cfg[3];
    m->NKV = cfg[4];
    m->D = cfg[5];
    m->VOCAB = cfg[6];
    m->KH = cfg[7];
    m->VH = cfg[8];
    m->K = cfg[9];
    m->V = cfg[10];
    m->W = cfg[11];
    m->RD = cfg[12];
    m->eps = fcfg[0];
    m->theta = fcfg[1];
    m->context = context;
    m->is_attn = (uint8_t *)malloc(m->L);
    memcpy(m->is_attn, is_attn, m->L);
    m->mats = (or_mat *)calloc((size_t)m->L * M_COUNT, sizeof(or_mat));
    m->vecs = (const float **)calloc((size_t)m->L * V_COUNT, sizeof(float *));
    const size_t qkv = 2 * (size_t)m->KH * m->K + (size_t)m->VH * m->V;
    size_t ndelta = 0, nattn = 0;
    for (uint32_t l = 0; l < m->L; ++l) {
        if (m->is_attn[l])
            ++nattn;
        else
            ++ndelta;
    }
    m->conv = (double *)calloc(ndelta * qkv * (m->W - 1) + 1, sizeof(double));
    m->dstate = (double *)calloc(ndelta * (size_t)m->VH * m->V * m->K + 1, sizeof(double));
    m->kc = (double *)calloc(nattn * (size_t)context * m->NKV * m->D + 1, sizeof(double));
    m->vc = (double *)calloc(nattn * (size_t)context * m->NKV * m->D + 1, sizeof(double));
    return m;
}

void or_model_free(or_model *m) {
    if (!m) return;
    free(m->is_attn);
    free(m->mats);
    free(m->vecs);
    free(m->conv);
    free(m->dstate);
    free(m->kc);
    free(m->vc);
    free(m);
}

static or_mat *slot(or_model *m, int layer, int which) {
    if (layer < 0) return which == 0 ? &m->embed : &m->head;
    return &m->mats[(size_t)layer * M_COUNT + which];
}

void or_model_set_matrix(or_model *m, int layer, int which, const uint32_t *w, const void *s, const void *b,
                         int bf16, uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group) {
    or_mat *t = slot(m, layer, which);
    memset(t, 0, sizeof(*t));
    t->w = w;
    t->s = s;
    t->b = b;
    t->bf16 = bf16;
    t->rows = rows;
    t->cols = cols;
    t->bits = bits;
    t->group = group;
}

void or_model_set_synth(or_model *m, int layer, int which, uint64_t seed, uint32_t mid, uint32_t rows,
                        uint32_t cols) {
    or_mat *t = slot(m, layer, which);
    memset(t, 0, sizeof(*t));
    t->synth = 1;
    t->seed = seed;
    t->mid = mid;
    t->rows = rows;
    t->cols = cols;
    t->bits = 4;
    t->group = 64;
    t->bf16 = 1;
}

void or_model_set_vector(or_model *m, int layer, int which, const float *v) {
    if (layer < 0)
        m->final_norm = v;
    else
        m->vecs[(size_t)layer * V_COUNT + which] = v;
}

void or_model_reset(or_model *m) {
    const size_t qkv = 2 * (size_t)m->KH * m->K + (size_t)m->VH * m->V;
    size_t ndelta = 0, nattn = 0;
    for (uint32_t l = 0; l < m->L; ++l) {
        if (m->is_attn[l])
            ++nattn;
        else
            ++ndelta;
    }
    memset(m->conv, 0, (ndelta * qkv * (m->W - 1) + 1) * sizeof(double));
    memset(m->dstate, 0, (ndelta * (size_t)m->VH * m->V * m->K + 1) * sizeof(double));
    memset(m->kc, 0, (nattn * (size_t)m->context * m->NKV * m->D + 1) * sizeof(double));
    memset(m->vc, 0, (nattn * (size_t)m->context * m->NKV * m->D + 1) * sizeof(double));
    m->pos = 0;
}

uint32_t or_model_position(const or_model *m) { return m->pos; }

static inline double meta_at(const void *p, int bf16, size_t gi) {
    if (bf16) return (double)sg_bf16_f32(((const uint16_t *)p)[gi]);
    return (double)((const float *)p)[gi];
}

/* Dequantised row r of a matrix into out[cols] (FP64 q*s+b). */
static void row_values(const or_mat *t, uint32_t r, double *out) {
    const uint32_t cols = t->cols;
    if (t->synth) {
        const uint32_t wpr = cols / 8;
        const uint64_t base = (uint64_t)r * wpr / 2;
        for (uint32_t p = 0; p < wpr / 2; ++p) {
            const uint64_t h = or_synth_pair(t->seed, t->mid, base + p);
            for (int k = 0; k < 16; ++k) out[16 * p + k] = (double)((h >> (4 * k)) & 15u);
        }
        for (uint32_t g = 0; g < cols / 64; ++g) {
            uint16_t sb, bb;
            or_synth_meta(t->seed, t->mid, (uint64_t)r * (cols / 64) + g, &sb, &bb);
            const double s = (double)sg_bf16_f32(sb), b = (double)sg_bf16_f32(bb);
            for (uint32_t c = 64 * g; c < 64 * g + 64; ++c) out[c] = out[c] * s + b;
        }
        return;
    }
    const uint32_t pack = 32 / t->bits, mask = (1u << t->bits) - 1u;
    const uint32_t *wr = t->w + (size_t)r * (cols / pack);
    const uint32_t ng = cols / t->group;
    for (uint32_t c = 0; c < cols; ++c) {
        const double q = (double)((wr[c / pack] >> ((c % pack) * t->bits)) & mask);
        const size_t gi = (size_t)r * ng + c / t->group;
        out[c] = q * meta_at(t->s, t->bf16, gi) + meta_at(t->b, t->bf16, gi);
    }
}

/* y[r] = sum_c W[r,c] x[c] for rows [0, rows). */
static void matvec(const or_mat *t, const double *x, double *y) {
    const uint32_t cols = t->cols;
#pragma omp parallel
    {
        double *row = (double *)malloc((size_t)cols * sizeof(double));
#pragma omp for schedule(dynamic, 16)
        for (long long r = 0; r < (long long)t->rows; ++r) {
            row_values(t, (uint32_t)r, row);
            double a0 = 0, a1 = 0, a2 = 0, a3 = 0;
            uint32_t c = 0;
            for (; c + 4 <= cols; c += 4) {
                a0 += row[c] * x[c];
                a1 += row[c + 1] * x[c + 1];
                a2 += row[c + 2] * x[c + 2];
                a3 += row[c + 3] * x[c + 3];
            }
            for (; c < cols; ++c) a0 += row[c] * x[c];
            y[r] = (a0 + a1) + (a2 + a3);
        }
        free(row);
    }
}

static void rms_apply(const double *x, const float *w, uint32_t n, double eps, double *y) {
    double ss = 0;
    for (uint32_t i = 0; i < n; ++i) ss += x[i] * x[i];
    const double inv = 1.0 / sqrt(ss / n + eps);
    for (uint32_t i = 0; i < n; ++i) y[i] = x[i] * inv * (double)w[i];
}

static inline double sigmoid64(double v) { return 1.0 / (1.0 + exp(-v)); }
static inline double silu64d(double v) { return v * sigmoid64(v); }
static inline double softplus64(double v) { return v > 0 ? v + log1p(exp(-v)) : log1p(exp(v)); }

/* One token at the current position; logits (optional, vocab doubles) of
 * the next token.  Returns 0, or -1 for a token outside the vocabulary or a
 * full context (nothing is changed then). */
int or_model_forward(or_model *m, uint32_t token, double *logits) {
    if (token >= m->VOCAB || m->pos >= m->context) return -1;
    const uint32_t H = m->H, F = m->F, K = m->K, V = m->V, KH = m->KH, VH = m->VH, D = m->D, NH = m->NH,
                   NKV = m->NKV, W = m->W;
    const size_t qkvn = 2 * (size_t)KH * K + (size_t)VH * V;
    double *x = (double *)malloc(H * sizeof(double));
    double *n = (double *)malloc(H * sizeof(double));
    double *out = (double *)malloc(H * sizeof(double));
    size_t big = qkvn;
    if ((size_t)F > big) big = F;
    if ((size_t)2 * NH * D > big) big = (size_t)2 * NH * D;
    if ((size_t)VH * V > big) big = (size_t)VH * V;
    double *p1 = (double *)malloc(big * sizeof(double));
    double *p2 = (double *)malloc(big * sizeof(double));
    double *p3 = (double *)malloc(big * sizeof(double));
    double *p4 = (double *)malloc(big * sizeof(double));
    double *scores = (double *)malloc(((size_t)m->pos + 1) * sizeof(double));
    row_values(&m->embed, token, x);
    size_t di = 0, ai = 0;
    for (uint32_t l = 0; l < m->L; ++l) {
        const or_mat *mt = &m->mats[(size_t)l * M_COUNT];
        const float **vc = &m->vecs[(size_t)l * V_COUNT];
        rms_apply(x, vc[V_IN], H, m->eps, n);
        if (!m->is_attn[l]) {
            double *qkv = p1, *z = p2, *ab = p3, *y = p4;
            matvec(&mt[M_QKV], n, qkv);
            matvec(&mt[M_Z], n, z);
            matvec(&mt[M_A], n, ab);
            matvec(&mt[M_B], n, ab + VH);
            double *cs = m->conv + di * qkvn * (W - 1);
            const float *cw = vc[V_CONV];
            for (size_t c = 0; c < qkvn; ++c) {
                double s = qkv[c] * (double)cw[c * W + W - 1];
                for (uint32_t k = 0; k + 1 < W; ++k) s += cs[c * (W - 1) + k] * (double)cw[c * W + k];
                for (uint32_t k = 0; k + 2 < W; ++k) cs[c * (W - 1) + k] = cs[c * (W - 1) + k + 1];
                if (W > 1) cs[c * (W - 1) + W - 2] = qkv[c];
                qkv[c] = silu64d(s);
            }
            for (uint32_t h = 0; h < KH; ++h) {
                double *q = qkv + (size_t)h * K, *k = qkv + (size_t)KH * K + (size_t)h * K;
                double qs = 0, ks = 0;
                for (uint32_t i = 0; i < K; ++i) {
                    qs += q[i] * q[i];
                    ks += k[i] * k[i];
                }
                const double qn = sqrt(qs + 1e-6) * sqrt((double)K), kn = sqrt(ks + 1e-6);
                for (uint32_t i = 0; i < K; ++i) {
                    q[i] /= qn;
                    k[i] /= kn;
                }
            }
            double *st = m->dstate + di * (size_t)VH * V * K;
            for (uint32_t h = 0; h < VH; ++h) {
                const uint32_t kh = h / (VH / KH);
                const double *q = qkv + (size_t)kh * K, *k = qkv + (size_t)KH * K + (size_t)kh * K;
                const double *v = qkv + 2 * (size_t)KH * K + (size_t)h * V;
                const double decay = exp(-exp((double)vc[V_ALOG][h]) * softplus64(ab[h] + (double)vc[V_DT][h]));
                const double beta = sigmoid64(ab[VH + h]);
                double ss = 0;
                for (uint32_t i = 0; i < V; ++i) {
                    double *row = st + ((size_t)h * V + i) * K;
                    double pred = 0;
                    for (uint32_t j = 0; j < K; ++j) {
                        row[j] *= decay;
                        pred += row[j] * k[j];
                    }
                    const double delta = beta * (v[i] - pred);
                    double o = 0;
                    for (uint32_t j = 0; j < K; ++j) {
                        row[j] += k[j] * delta;
                        o += row[j] * q[j];
                    }
                    y[(size_t)h * V + i] = o;
                    ss += o * o;
                }
                const double inv = 1.0 / sqrt(ss / V + m->eps);
                for (uint32_t i = 0; i < V; ++i) {
                    const size_t o = (size_t)h * V + i;
                    y[o] = y[o] * inv * (double)vc[V_DNORM][i] * silu64d(z[o]);
                }
            }
            matvec(&mt[M_OUT], y, out);
            ++di;
        } else {
            double *proj = p1, *kk = p2, *vv = p3, *y = p4;
            matvec(&mt[M_Q], n, proj);
            matvec(&mt[M_K], n, kk);
            matvec(&mt[M_V], n, vv);
            const uint32_t RD = m->RD, half = RD / 2;
            /* q heads: rms + rope in place inside proj ([h][2][D]: q then gate) */
            for (uint32_t h = 0; h <= NH; ++h) {
                const int is_k = h == NH;
                for (uint32_t kv = 0; kv < (is_k ? NKV : 1u); ++kv) {
                    double *t = is_k ? kk + (size_t)kv * D : proj + (size_t)h * 2 * D;
                    const float *w = is_k ? vc[V_KNORM] : vc[V_QNORM];
                    double ss = 0;
                    for (uint32_t i = 0; i < D; ++i) ss += t[i] * t[i];
                    const double inv = 1.0 / sqrt(ss / D + m->eps);
                    for (uint32_t i = 0; i < D; ++i) t[i] = t[i] * inv * (double)w[i];
                    for (uint32_t j = 0; j < half; ++j) {
                        const double ang = (double)m->pos * pow(m->theta, -(double)(2 * j) / (double)RD);
                        const double a = t[j], b = t[j + half];
                        t[j] = a * cos(ang) - b * sin(ang);
                        t[j + half] = a * sin(ang) + b * cos(ang);
                    }
                }
            }
            double *kc = m->kc + ai * (size_t)m->context * NKV * D;
            double *vcache = m->vc + ai * (size_t)m->context * NKV * D;
            memcpy(kc + (size_t)m->pos * NKV * D, kk, (size_t)NKV * D * sizeof(double));
            memcpy(vcache + (size_t)m->pos * NKV * D, vv, (size_t)NKV * D * sizeof(double));
            const uint32_t len = m->pos + 1;
            for (uint32_t h = 0; h < NH; ++h) {
                const uint32_t kh = h / (NH / NKV);
                const double *q = proj + (size_t)h * 2 * D, *gate = q + D;
                double mx = -INFINITY;
                for (uint32_t t = 0; t < len; ++t) {
                    const double *kt = kc + ((size_t)t * NKV + kh) * D;
                    double s = 0;
                    for (uint32_t i = 0; i < D; ++i) s += q[i] * kt[i];
                    scores[t] = s / sqrt((double)D);
                    if (scores[t] > mx) mx = scores[t];
                }
                double den = 0;
                for (uint32_t t = 0; t < len; ++t) {
                    scores[t] = exp(scores[t] - mx);
                    den += scores[t];
                }
                for (uint32_t d = 0; d < D; ++d) {
                    double acc = 0;
                    for (uint32_t t = 0; t < len; ++t) acc += scores[t] / den * vcache[((size_t)t * NKV + kh) * D + d];
                    y[(size_t)h * D + d] = acc * sigmoid64(gate[d]);
                }
            }
            matvec(&mt[M_O], y, out);
            ++ai;
        }
        for (uint32_t i = 0; i < H; ++i) x[i] += out[i];
        rms_apply(x, vc[V_POST], H, m->eps, n);
        matvec(&mt[M_GATE], n, p1);
        matvec(&mt[M_UP], n, p2);
        for (uint32_t i = 0; i < F; ++i) p1[i] = silu64d(p1[i]) * p2[i];
        matvec(&mt[M_DOWN], p1, out);
        for (uint32_t i = 0; i < H; ++i) x[i] += out[i];
    }
    if (logits) {
        rms_apply(x, m->final_norm, H, m->eps, n);
        matvec(&m->head, n, logits);
    }
    m->pos += 1;
    free(x);
    free(n);
    free(out);
    free(p1);
    free(p2);
    free(p3);
    free(p4);
    free(scores);
    return 0;
}
