/*
 * CPU oracle for the packed-affine matrix path.  TEST INFRASTRUCTURE ONLY:
 * tests, __graft_entry__.smoke() and the cpu_baseline / --impl reference leg
 * of bench.py call this as the checker or as the timed CPU baseline.  The
 * product (libqmr) never links or calls it.
 *
 * It restates the reference's own scalar arithmetic (rucin93/qwen-mlx-runner
 * v0.7.3):
 *   - element dequantisation float(q)*s+b, q little-endian within each u32
 *     word: kernels/qwen.metal:40-47 (FP32 metadata) and
 *     kernels/affine_bf16.metal:439-451 / :294-296 (BF16 metadata, expanded
 *     by uint(bits)<<16);
 *   - the independent FP64 expansion every matrix test checks against:
 *     tests/quantized.rs:39-51, tests/batch_matrix.rs:35-49 and :263-274,
 *     tests/bf16_metadata.rs:41-47 -- (q*s + b) * x in f64, summed left to
 *     right with sequential f64 adds, then rounded to f32;
 *   - token-major block layout X[b*cols+c], Y[b*rows+r]:
 *     kernels/matmul_block.metal:1-3;
 *   - SwiGLU silu(g)*u with silu(x)=x*(1/(1+exp(-x))): kernels/qwen.metal:32-33,
 *     :91-94;
 *   - greedy argmax, ties to the lowest index, f32 total order:
 *     src/chat.rs:383-390;
 *   - exact BF16 metadata packing: src/gpu/metadata.rs:6-14.
 *
 * Compile with -ffp-contract=off: the reference oracle is Rust, which never
 * fuses a*b+c, and the f64 sums must round exactly as it does.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf16_to_f32(uint16_t bits) {
    uint32_t u = (uint32_t)bits << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

/* Metadata element gi as FP32, either stored FP32 or as the high half of FP32. */
static inline float meta(const void *m, int bf16, size_t gi) {
    return bf16 ? bf16_to_f32(((const uint16_t *)m)[gi]) : ((const float *)m)[gi];
}

static inline uint32_t quant(const uint32_t *w, size_t row, size_t col, uint32_t cols,
                             uint32_t bits) {
    const uint32_t pack = 32u / bits;
    const uint32_t word = w[row * (cols / pack) + col / pack];
    return (word >> ((col % pack) * bits)) & ((1u << bits) - 1u);
}

int or_abi_version(void) { return 1; }

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* FP32 dequantisation of row `row`: y[c] = float(q)*s + b, two roundings
 * (kernels/qwen.metal:40-47).  With BF16 metadata q*s is exact, so this equals
 * the fused form bit for bit. */
void or_embed(const uint32_t *w, const void *s, const void *b, int meta_bf16, uint64_t row,
              uint32_t cols, uint32_t bits, uint32_t group, float *y) {
    for (uint32_t c = 0; c < cols; ++c) {
        const size_t gi = (size_t)row * (cols / group) + c / group;
        volatile float prod = (float)quant(w, row, c, cols, bits) * meta(s, meta_bf16, gi);
        y[c] = prod + meta(b, meta_bf16, gi);
    }
}

/* FP64 expansion of Y[b*rows+r] = sum_c (q*s+b) * X[b*cols+c] for rows
 * [row0, row0+nrows).  absdot (optional) receives sum_c |(q*s+b)*x| in f64,
 * the scale of the per-output tolerance.  Output indices are absolute. */
void or_matmul_f64(const uint32_t *w, const void *s, const void *b, int meta_bf16,
                   const float *x, uint32_t rows, uint32_t cols, uint32_t bits,
                   uint32_t group, uint32_t batch, uint32_t row0, uint32_t nrows, double *y,
                   double *absdot) {
    const long long end = (long long)row0 + nrows;
#pragma omp parallel for schedule(dynamic, 8)
    for (long long r = row0; r < end; ++r) {
        for (uint32_t t = 0; t < batch; ++t) {
            const float *xt = x + (size_t)t * cols;
            double acc = 0.0, mag = 0.0;
            for (uint32_t c = 0; c < cols; ++c) {
                const size_t gi = (size_t)r * (cols / group) + c / group;
                const double v = (double)quant(w, (size_t)r, c, cols, bits) *
                                     (double)meta(s, meta_bf16, gi) +
                                 (double)meta(b, meta_bf16, gi);
                const double term = v * (double)xt[c];
                acc += term;
                mag += fabs(term);
            }
            y[(size_t)t * rows + r] = acc;
            if (absdot) absdot[(size_t)t * rows + r] = mag;
        }
    }
}

/* silu in f64, same formula as kernels/qwen.metal:32-33. */
static inline double silu64(double v) { return v * (1.0 / (1.0 + exp(-v))); }

/* act[b*rows+r] = silu(gate.x_b) * (up.x_b) in f64 for a Q4/Q8 affine pair,
 * with the first-order error scale of act for the tolerance:
 *   absact = |u| * 1.1 * sum|g_j x_j| + |silu(g)| * sum|u_j x_j|
 * (|silu'| <= 1.1 everywhere).  rows = gate/up rows. */
void or_swiglu_f64(const uint32_t *wg, const void *sg, const void *bg, const uint32_t *wu,
                   const void *su, const void *bu, int meta_bf16, const float *x,
                   uint32_t rows, uint32_t cols, uint32_t bits, uint32_t group,
                   uint32_t batch, double *act, double *absact) {
#pragma omp parallel for schedule(dynamic, 8)
    for (long long r = 0; r < (long long)rows; ++r) {
        for (uint32_t t = 0; t < batch; ++t) {
            const float *xt = x + (size_t)t * cols;
            double g = 0, u = 0, mg = 0, mu = 0;
            for (uint32_t c = 0; c < cols; ++c) {
                const size_t gi = (size_t)r * (cols / group) + c / group;
                const double vg = (double)quant(wg, (size_t)r, c, cols, bits) *
                                      (double)meta(sg, meta_bf16, gi) +
                                  (double)meta(bg, meta_bf16, gi);
                const double vu = (double)quant(wu, (size_t)r, c, cols, bits) *
                                      (double)meta(su, meta_bf16, gi) +
                                  (double)meta(bu, meta_bf16, gi);
                g += vg * (double)xt[c];
                u += vu * (double)xt[c];
                mg += fabs(vg * (double)xt[c]);
                mu += fabs(vu * (double)xt[c]);
            }
            const double a = silu64(g) * u;
            act[(size_t)t * rows + r] = a;
            if (absact) absact[(size_t)t * rows + r] = fabs(u) * 1.1 * mg + fabs(silu64(g)) * mu;
        }
    }
}

/* Key that orders f32 like Rust's f32::total_cmp, as an unsigned integer. */
static inline uint32_t total_order_key(float v) {
    const uint32_t u = f32_bits(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/* Greedy argmax over n f32 logits: maximum under total order, ties to the
 * lowest index (src/chat.rs:383-390).  Returns -1 for n == 0. */
long long or_argmax_f32(const float *logits, uint64_t n) {
    if (n == 0) return -1;
    uint64_t best = 0;
    uint32_t key = total_order_key(logits[0]);
    for (uint64_t i = 1; i < n; ++i) {
        const uint32_t k = total_order_key(logits[i]);
        if (k > key) {
            key = k;
            best = i;
        }
    }
    return (long long)best;
}

/* Greedy argmax over f64 values, ties to the lowest index. */
long long or_argmax_f64(const double *v, uint64_t n) {
    if (n == 0) return -1;
    uint64_t best = 0;
    for (uint64_t i = 1; i < n; ++i)
        if (v[i] > v[best]) best = i;
    return (long long)best;
}

/* src/gpu/metadata.rs:6-14: keep the high halves only when every value is
 * finite and has zero low 16 bits.  Returns 1 and fills out, or 0. */
int or_pack_bf16_exact(const float *v, uint64_t n, uint16_t *out) {
    for (uint64_t i = 0; i < n; ++i) {
        const uint32_t u = f32_bits(v[i]);
        if ((u & 0x7f800000u) == 0x7f800000u || (u & 0xffffu) != 0) return 0;
    }
    for (uint64_t i = 0; i < n; ++i) out[i] = (uint16_t)(f32_bits(v[i]) >> 16);
    return 1;
}

/* Round-to-nearest-even FP32 -> BF16 bits for finite values, the rounding of
 * scripts/make_fixture.py:262-267. */
uint16_t or_bf16_rne(float v) {
    const uint32_t u = f32_bits(v);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

/* Maximum relative violation of |got - want| <= atol + rtol * scale over n
 * outputs; returns the worst ratio |err| / (atol + rtol*scale) and its index. */
double or_check_tol(const float *got, const double *want, const double *scale, uint64_t n,
                    double atol, double rtol, long long *worst) {
    double w = 0;
    long long wi = -1;
    for (uint64_t i = 0; i < n; ++i) {
        const double err = fabs((double)got[i] - want[i]);
        const double lim = atol + rtol * (scale ? scale[i] : fabs(want[i]));
        const double ratio = (err == 0) ? 0 : (lim > 0 ? err / lim : INFINITY);
        if (!(ratio <= w)) {
            w = ratio;
            wi = (long long)i;
        }
    }
    if (worst) *worst = wi;
    return w;
}
