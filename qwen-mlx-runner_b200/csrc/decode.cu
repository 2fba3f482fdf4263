// Decode-step kernels of the hybrid Qwen3.5 graph on sm_100a (everything
// outside the packed matrix products, which run in the streaming kernels).
//
// Semantics follow the reference's kernels (rucin93/qwen-mlx-runner v0.7.3,
// kernels/qwen.metal:78-258) as the per-token graph calls them
// (src/engine.rs:607-797); the fusion and the work split are this file's:
//  * delta_mixer_kernel: conv_silu + delta_norm + delta_step + gated_rms of
//    one DeltaNet layer in one launch, one CTA per value head (the state
//    rows of a head are prefetched into registers, so its 64 KiB streams
//    once in each direction);
//  * attention_kernel: split_q_gate + head_rms + rope + kv_append +
//    attn_scores + softmax + attn_values (with the sigmoid gate) in one
//    launch: one CTA per (64-position chunk, KV head) computes the
//    partial softmax of the KV group's query heads over its chunk; the last
//    CTA of each KV head merges the chunks in chunk order;
//  * embed_token_kernel reads the step's token from the control block, so a
//    captured step graph replays for every token; advance_kernel ends a step.
// Reductions use a fixed order (xor shuffles, then warps in order), so a
// step is reproducible run to run.
#include <cuda_runtime.h>

#include <cstdint>

#include "decode.h"
#include "matrix_kernels.cuh"
#include "qmr_internal.h"

namespace qmr {

namespace {

__host__ __device__ __forceinline__ uint64_t sg_mix(uint64_t z) {
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ull;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBull;
    z ^= z >> 31;
    return z;
}

__host__ __device__ __forceinline__ uint64_t sg_key(uint64_t seed, uint64_t mid, uint64_t tag) {
    return sg_mix(seed ^ (mid * 0x9E3779B97F4A7C15ull) ^ (tag * 0xD1B54A32D192ED03ull));
}

__device__ __forceinline__ uint16_t bf16_rne_bits(float v) {
    const uint32_t u = __float_as_uint(v);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

// The synthetic generator of the test oracle, bit for bit: word pairs from a
// counter hash; scale uniform [0.002, 0.02] -> BF16; bias = BF16(-8 scale +
// 1e-3 * Irwin-Hall(4) normal approximation), all in explicitly rounded f64.
__global__ void synth_words_kernel(uint32_t *w, uint64_t key, uint64_t first_pair, uint64_t npairs) {
    for (uint64_t j = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; j < npairs;
         j += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t h = sg_mix(key + (first_pair + j + 1) * 0x9E3779B97F4A7C15ull);
        reinterpret_cast<uint2 *>(w)[j] = make_uint2((uint32_t)h, (uint32_t)(h >> 32));
    }
}

__global__ void synth_meta_kernel(uint16_t *s, uint16_t *b, uint64_t key_m, uint64_t key_n, uint64_t first,
                                  uint64_t n) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t g = first + i;
        const uint64_t h = sg_mix(key_m + (g + 1) * 0x9E3779B97F4A7C15ull);
        const double u = __dmul_rn((double)(h >> 11), 1.0 / 9007199254740992.0);
        const float s32 = __double2float_rn(__dadd_rn(0.002, __dmul_rn(0.018, u)));
        const uint16_t sb = bf16_rne_bits(s32);
        const uint64_t h2 = sg_mix(h ^ key_n);
        double nrm = 0.0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
            nrm = __dadd_rn(nrm, __dmul_rn(__dadd_rn((double)((h2 >> (16 * k)) & 0xffffu), 0.5), 1.0 / 65536.0));
        nrm = __dmul_rn(__dadd_rn(nrm, -2.0), 1.7320508075688772);
        const double sv = (double)__uint_as_float((uint32_t)sb << 16);
        const float b32 = __double2float_rn(__dadd_rn(__dmul_rn(-8.0, sv), __dmul_rn(1e-3, nrm)));
        s[i] = sb;
        b[i] = bf16_rne_bits(b32);
    }
}

// A region of the synthetic matrix (seed-derived keys, full width
// full_cols): rows [r0, r0 + nr), columns [c0, c0 + nc), written row by row
// from destination row dst_row0 with the destination's own word and metadata
// strides (so row shards and column shards of one matrix come from the same
// generator stream as the whole matrix).
__global__ void synth_region_kernel(uint32_t *w, uint16_t *s, uint16_t *b, uint64_t key_w, uint64_t key_m,
                                    uint64_t key_n, uint32_t full_cols, uint32_t r0, uint32_t nr, uint32_t c0,
                                    uint32_t nc, uint32_t dst_wstride, uint32_t dst_mstride, uint32_t dst_row0) {
    const uint64_t wpr = full_cols / 8, gpr = full_cols / 64;
    const uint64_t nw = (uint64_t)nr * (nc / 8), ng = (uint64_t)nr * (nc / 64);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < nw; i += stride) {
        const uint64_t r = i / (nc / 8), j = i % (nc / 8);
        const uint64_t gw = (r0 + r) * wpr + c0 / 8 + j;
        const uint64_t h = sg_mix(key_w + (gw / 2 + 1) * 0x9E3779B97F4A7C15ull);
        w[(dst_row0 + r) * dst_wstride + j] = (gw & 1) ? (uint32_t)(h >> 32) : (uint32_t)h;
    }
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < ng; i += stride) {
        const uint64_t r = i / (nc / 64), g = i % (nc / 64);
        const uint64_t gg = (r0 + r) * gpr + c0 / 64 + g;
        const uint64_t h = sg_mix(key_m + (gg + 1) * 0x9E3779B97F4A7C15ull);
        const double u = __dmul_rn((double)(h >> 11), 1.0 / 9007199254740992.0);
        const float s32 = __double2float_rn(__dadd_rn(0.002, __dmul_rn(0.018, u)));
        const uint16_t sb = bf16_rne_bits(s32);
        const uint64_t h2 = sg_mix(h ^ key_n);
        double nrm = 0.0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
            nrm = __dadd_rn(nrm, __dmul_rn(__dadd_rn((double)((h2 >> (16 * k)) & 0xffffu), 0.5), 1.0 / 65536.0));
        nrm = __dmul_rn(__dadd_rn(nrm, -2.0), 1.7320508075688772);
        const double sv = (double)__uint_as_float((uint32_t)sb << 16);
        const float b32 = __double2float_rn(__dadd_rn(__dmul_rn(-8.0, sv), __dmul_rn(1e-3, nrm)));
        s[(dst_row0 + r) * dst_mstride + g] = sb;
        b[(dst_row0 + r) * dst_mstride + g] = bf16_rne_bits(b32);
    }
}

// Sharded decode: x[t][i] += sum over ranks (in rank order) of the partial
// products the ranks pushed into this rank's slots [t][world][H].
__global__ void partial_sum_kernel(float *x, const float *slots, int world, int H, int nq) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (i >= H || t >= nq) return;
    const float *src = slots + (size_t)t * world * H + i;
    float acc = __ldcg(src);
    for (int r = 1; r < world; ++r) acc = __fadd_rn(acc, __ldcg(src + (size_t)r * H));
    x[(size_t)t * H + i] = __fadd_rn(x[(size_t)t * H + i], acc);
}

__global__ void fill_kernel(float *p, uint64_t n, float v) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        p[i] = v;
}

__device__ __forceinline__ uint32_t step_token(const DecodeCtrl *ctrl, const int32_t *prompt) {
    const uint32_t pos = ctrl->pos;
    return pos < ctrl->n_prompt ? (uint32_t)prompt[pos] : (uint32_t)ctrl->token;
}

// embed_affine of the step's token (kernels/affine_bf16.metal:439-451):
// float(q) * s + b with two roundings, bit-exact with the reference.
template <bool BF16>
__global__ void embed_token_kernel(const uint32_t *__restrict__ w, const void *__restrict__ s,
                                   const void *__restrict__ bias, uint32_t cols, uint32_t bits, uint32_t group,
                                   const DecodeCtrl *ctrl, const int32_t *prompt, float *__restrict__ x) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const uint64_t row = step_token(ctrl, prompt);
    const uint32_t pack = 32u / bits;
    const uint32_t word = __ldg(w + row * (cols / pack) + c / pack);
    const uint32_t q = (word >> ((c % pack) * bits)) & ((1u << bits) - 1u);
    const uint64_t gi = row * (cols / group) + c / group;
    x[c] = __fadd_rn(__fmul_rn((float)q, load_meta<BF16>(s, gi)), load_meta<BF16>(bias, gi));
}

// Fixed-order sum over the block: xor shuffles inside each warp, then the
// warps' sums in warp order by one thread; every thread gets the result.
// `red` holds at least 33 floats.  Every thread of the block must call it.
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < nw; ++i) t = __fadd_rn(t, red[i]);
        red[32] = t;
    }
    __syncthreads();
    return red[32];
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float sigmoid_f32(float x) { return __frcp_rn(__fadd_rn(1.0f, expf(-x))); }

__device__ __forceinline__ float rsqrt_f32(float x) { return __fdiv_rn(1.0f, __fsqrt_rn(x)); }

// rms_norm (kernels/qwen.metal:78-86): y = x * inv * w, one CTA.
__global__ void rms_norm_kernel(const float *x, const float *w, float *y, uint32_t n, float eps) {
    __shared__ float red[33];
    float ss = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss = __fmaf_rn(x[i], x[i], ss);
    const float inv = rsqrt_f32(__fadd_rn(__fdiv_rn(block_sum(ss, red), (float)n), eps));
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

// add (kernels/qwen.metal:87-90) in place: x = x + r.
__global__ void add_kernel(float *x, const float *r, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fadd_rn(x[i], r[i]);
}

constexpr int kDeltaThreads = 256;
constexpr int kDeltaRowsPerWarp = 4;
constexpr int kMaxTokens = 4;   // tokens of one mixer or attention launch
constexpr int kMaxConvHist = 7; // conv width <= 8

// One DeltaNet layer's mixer for nq tokens, CTA blockIdx.x = value head h *
// kDeltaSplit + part; the part owns value rows [part*V/S, (part+1)*V/S).
//  conv_silu (qwen.metal:95-106): y = silu(x*w[W-1] + sum_k hist[k]*w[k])
//    over the channels this CTA reads (its key head's q and k, its own v
//    rows), token after token.  Single tokens double-buffer the live history
//    by position parity (read pos&1, write the other), so CTAs sharing q/k
//    channels never race: part 0 of the first value head of each key group
//    writes them.  A verification block only reads the live history and
//    leaves the history after every prefix in conv_snap.
//  delta_norm (:107-116): q *= rsqrt(|q|^2 + 1e-6) * rsqrt(K),
//    k *= rsqrt(|k|^2 + 1e-6).
//  delta_step / delta_step_block (:117-183): decay = exp(-exp(A_log)
//    softplus(a + dt)), beta = sigmoid(b); per value row S = S*decay,
//    delta = (v - S.k)*beta, S += k*delta, y = S.q; the warp's rows stay in
//    registers across the block's tokens, and a block stores S before each
//    token in state_snap.
//  gated_rms (:184-194): out = y * rsqrt(mean(y^2) + eps) * w * silu(z):
//    every part stores its rows' y and sums of squares; the last part of the
//    head to finish adds the parts' sums in part order and writes the head.
__global__ void __launch_bounds__(kDeltaThreads) delta_mixer_kernel(DeltaArgs a) {
    extern __shared__ float dsm[];
    __shared__ unsigned int last;
    const int K = a.K, V = a.V, W = a.W, KH = a.KH, VH = a.VH, nq = a.nq, P = a.proj_stride;
    const int h = blockIdx.x / kDeltaSplit, part = blockIdx.x % kDeltaSplit;
    const int ratio = VH / KH, kh = h / ratio;
    const bool rep = (h % ratio) == 0 && part == 0;
    const int r_begin = part * V / kDeltaSplit, r_end = (part + 1) * V / kDeltaSplit, nr = r_end - r_begin;
    const int nrp = nr > 0 ? nr : 1;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    float *q = dsm, *k = q + nq * K, *v = k + nq * K, *y = v + nq * nrp, *red = y + nq * nrp;
    const int qkv = 2 * KH * K + VH * V;
    const int H1 = W - 1;
    const int par = (int)(a.ctrl->pos & 1u);
    const float *cs_old = a.conv_state + (size_t)par * qkv * H1;
    float *cs_new = a.conv_state + (size_t)(par ^ 1) * qkv * H1;
    for (int i = tid; i < 2 * K + nr; i += blockDim.x) {
        const int c = i < K ? kh * K + i
                            : (i < 2 * K ? KH * K + kh * K + (i - K) : 2 * KH * K + h * V + r_begin + (i - 2 * K));
        const bool owner = i >= 2 * K || rep;
        const float *w = a.conv_w + (size_t)c * W;
        const float *st = cs_old + (size_t)c * H1;
        float hist[kMaxConvHist];
#pragma unroll
        for (int j = 0; j < kMaxConvHist; ++j) hist[j] = j < H1 ? st[j] : 0.0f;
        if (owner && a.conv_snap != nullptr)
            for (int j = 0; j < H1; ++j) a.conv_snap[(size_t)c * H1 + j] = hist[j];
        for (int t = 0; t < nq; ++t) {
            const float xin = a.proj[(size_t)t * P + c];
            float sum = __fmul_rn(xin, w[W - 1]);
            for (int j = 0; j < H1; ++j) sum = __fadd_rn(sum, __fmul_rn(hist[j], w[j]));
#pragma unroll
            for (int j = 0; j + 1 < kMaxConvHist; ++j)
                if (j + 1 < H1) hist[j] = hist[j + 1];
            if (H1 > 0) {
#pragma unroll
                for (int j = 0; j < kMaxConvHist; ++j)
                    if (j == H1 - 1) hist[j] = xin;
            }
            if (owner && a.conv_snap != nullptr)
                for (int j = 0; j < H1; ++j) a.conv_snap[((size_t)(t + 1) * qkv + c) * H1 + j] = hist[j];
            const float yv = silu_f32(sum);
            if (i < K)
                q[t * K + i] = yv;
            else if (i < 2 * K)
                k[t * K + i - K] = yv;
            else
                v[t * nrp + i - 2 * K] = yv;
        }
        if (owner && a.conv_snap == nullptr) {
            float *sn = cs_new + (size_t)c * H1;
            for (int j = 0; j < H1; ++j) sn[j] = hist[j];
        }
    }
    __syncthreads();
    float qi[kMaxTokens], ki[kMaxTokens], decay[kMaxTokens], beta[kMaxTokens];
    for (int t = 0; t < nq; ++t) {
        float qs = 0.0f, ks = 0.0f;
        for (int i = tid; i < K; i += blockDim.x) {
            qs = __fmaf_rn(q[t * K + i], q[t * K + i], qs);
            ks = __fmaf_rn(k[t * K + i], k[t * K + i], ks);
        }
        qs = block_sum(qs, red);
        ks = block_sum(ks, red);
        qi[t] = __fmul_rn(rsqrt_f32(__fadd_rn(qs, 1e-6f)), rsqrt_f32((float)K));
        ki[t] = rsqrt_f32(__fadd_rn(ks, 1e-6f));
        const float *pa = a.proj + (size_t)t * P + 2 * KH * K + 2 * VH * V;
        const float av = __fadd_rn(pa[h], a.dt[h]);
        const float sp = __fadd_rn(fmaxf(av, 0.0f), log1pf(expf(-fabsf(av))));  // softplus, stable
        decay[t] = expf(-__fmul_rn(expf(a.alog[h]), sp));
        beta[t] = sigmoid_f32(pa[VH + h]);
    }
    // Lane layout over K: column lane + 32*m, m < 4 (K <= 128).
    float *S = a.state + (size_t)h * V * K;
    for (int r0 = r_begin + warp * kDeltaRowsPerWarp; r0 < r_end; r0 += nwarps * kDeltaRowsPerWarp) {
        float sv[kDeltaRowsPerWarp][4];
#pragma unroll
        for (int rr = 0; rr < kDeltaRowsPerWarp; ++rr)
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int r = r0 + rr, j = lane + 32 * m;
                sv[rr][m] = (r < r_end && j < K) ? S[(size_t)r * K + j] : 0.0f;
            }
        for (int t = 0; t < nq; ++t) {
            float kr[4], qr[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int j = lane + 32 * m;
                kr[m] = j < K ? __fmul_rn(k[t * K + j], ki[t]) : 0.0f;
                qr[m] = j < K ? __fmul_rn(q[t * K + j], qi[t]) : 0.0f;
            }
#pragma unroll
            for (int rr = 0; rr < kDeltaRowsPerWarp; ++rr) {
                const int r = r0 + rr;
                if (r >= r_end) break;
                if (a.state_snap != nullptr) {
                    float *sn = a.state_snap + ((size_t)t * VH + h) * V * K + (size_t)r * K;
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const int j = lane + 32 * m;
                        if (j < K) sn[j] = sv[rr][m];
                    }
                }
                float pr = 0.0f;
#pragma unroll
                for (int m = 0; m < 4; ++m) pr = __fmaf_rn(__fmul_rn(sv[rr][m], decay[t]), kr[m], pr);
                pr = warp_sum(pr);
                const float delta = __fmul_rn(__fsub_rn(v[t * nrp + r - r_begin], pr), beta[t]);
                float o = 0.0f;
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const float nx = __fmaf_rn(kr[m], delta, __fmul_rn(sv[rr][m], decay[t]));
                    sv[rr][m] = nx;
                    o = __fmaf_rn(nx, qr[m], o);
                }
                o = warp_sum(o);
                if (lane == 0) y[t * nrp + r - r_begin] = o;
            }
        }
#pragma unroll
        for (int rr = 0; rr < kDeltaRowsPerWarp; ++rr) {
            const int r = r0 + rr;
            if (r >= r_end) break;
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int j = lane + 32 * m;
                if (j < K) S[(size_t)r * K + j] = sv[rr][m];
            }
        }
    }
    __syncthreads();
    for (int t = 0; t < nq; ++t) {
        float ys = 0.0f;
        for (int i = tid; i < nr; i += blockDim.x) {
            const float yy = y[t * nrp + i];
            ys = __fmaf_rn(yy, yy, ys);
            a.ybuf[(size_t)t * VH * V + (size_t)h * V + r_begin + i] = yy;
        }
        ys = block_sum(ys, red);
        if (tid == 0) a.ssq[(h * kDeltaSplit + part) * kMaxTokens + t] = ys;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = (atomicAdd(a.count + h, 1u) == (unsigned)kDeltaSplit - 1u) ? 1u : 0u;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int t = 0; t < nq; ++t) {
        float total = 0.0f;
        for (int p2 = 0; p2 < kDeltaSplit; ++p2)
            total = __fadd_rn(total, __ldcg(a.ssq + (h * kDeltaSplit + p2) * kMaxTokens + t));
        const float inv = rsqrt_f32(__fadd_rn(__fdiv_rn(total, (float)V), a.eps));
        const float *z = a.proj + (size_t)t * P + 2 * KH * K + VH * V + (size_t)h * V;
        const size_t o0 = (size_t)t * VH * V + (size_t)h * V;
        for (int i = tid; i < V; i += blockDim.x)
            a.out[o0 + i] = __fmul_rn(__fmul_rn(__fmul_rn(__ldcg(a.ybuf + o0 + i), inv), a.norm_w[i]), silu_f32(z[i]));
    }
    if (tid == 0) a.count[h] = 0u;
}

constexpr int kAttnThreads = 256;

// head_rms (qwen.metal:204-212) then partial rotate-half RoPE (:213-221) of
// one D-vector, by one warp: src (global) -> t (shared), weight w.
__device__ void warp_rms_rope(const float *src, float *t, const float *w, int D, int RD, float pos, float theta,
                              float eps, int lane) {
    float ss = 0.0f;
    for (int i = lane; i < D; i += 32) {
        const float v = src[i];
        t[i] = v;
        ss = __fmaf_rn(v, v, ss);
    }
    const float inv = rsqrt_f32(__fadd_rn(__fdiv_rn(warp_sum(ss), (float)D), eps));
    for (int i = lane; i < D; i += 32) t[i] = __fmul_rn(t[i], __fmul_rn(inv, w[i]));
    __syncwarp();
    const int half = RD / 2;
    for (int j = lane; j < half; j += 32) {
        const float ang = __fmul_rn(pos, powf(theta, __fdiv_rn(-(float)(2 * j), (float)RD)));
        float sn, cs;
        sincosf(ang, &sn, &cs);
        const float x0 = t[j], x1 = t[j + half];
        t[j] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        t[j + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
    }
    __syncwarp();
}

// Decode attention of one KV head over one 64-position chunk for nq query
// tokens at positions pos + i (see the file comment).  Shared memory:
// q [nq][G][D], new keys and values [nq][D] each, p [nq][G][64].
template <int NQ>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnArgs a) {
    extern __shared__ float asm_[];
    const int D = a.D, NH = a.NH, NKV = a.NKV, G = NH / NKV, P = a.proj_stride;
    constexpr int nq = NQ;
    const int c = blockIdx.x, kh = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    float *qs = asm_, *kn = qs + nq * G * D, *vn = kn + nq * D, *ps = vn + nq * D;
    __shared__ unsigned int last;
    const int pos = (int)a.ctrl->pos, len = pos + nq;  // keys 0 .. pos+nq-1
    const int t0 = c * kAttnChunk, t1 = min(t0 + kAttnChunk, len);
    float *part = a.part + ((size_t)kh * a.nchunks + c) * nq * G * (D + 2);
    if (t0 < len) {
        // One warp per (query token, head) of the group and per new key in
        // this chunk: split, head RMS, RoPE at that token's position.
        const int n0 = max(t0, pos), n1 = min(t0 + kAttnChunk, pos + nq);  // new positions in this chunk
        const int nnew = n1 > n0 ? n1 - n0 : 0;
        for (int job = warp; job < nq * G + nnew; job += nwarps) {
            if (job < nq * G) {
                const int i = job / G, g = job % G;
                warp_rms_rope(a.proj + (size_t)i * P + (size_t)(kh * G + g) * 2 * D, qs + job * D, a.qnorm, D, a.RD,
                              (float)(pos + i), a.theta, a.eps, lane);
            } else {
                const int i = n0 + (job - nq * G) - pos;
                const float *base = a.proj + (size_t)i * P + (size_t)NH * 2 * D;
                warp_rms_rope(base + (size_t)kh * D, kn + i * D, a.knorm, D, a.RD, (float)(pos + i), a.theta, a.eps,
                              lane);
                for (int d = lane; d < D; d += 32) vn[i * D + d] = base[(size_t)NKV * D + (size_t)kh * D + d];
            }
        }
        __syncthreads();
        for (int e = tid; e < nnew * D; e += blockDim.x) {
            const int i = n0 - pos + e / D, d = e % D;
            a.kcache[((size_t)(pos + i) * NKV + kh) * D + d] = kn[i * D + d];
            a.vcache[((size_t)(pos + i) * NKV + kh) * D + d] = vn[i * D + d];
        }
        // Scores q.k / sqrt(D) (attn_scores, qwen.metal:228-238), warps over
        // positions; query i sees positions <= pos + i.
        const float rs = rsqrt_f32((float)D);
        for (int t = t0 + warp; t < t1; t += nwarps) {
            const float *kt = (t >= pos) ? kn + (t - pos) * D : a.kcache + ((size_t)t * NKV + kh) * D;
            float kv[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int d = lane + 32 * m;
                kv[m] = d < D ? kt[d] : 0.0f;
            }
            for (int j = 0; j < nq * G; ++j) {
                float sc = 0.0f;
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    const int d = lane + 32 * m;
                    if (d < D) sc = __fmaf_rn(qs[j * D + d], kv[m], sc);
                }
                sc = warp_sum(sc);
                if (lane == 0) ps[j * kAttnChunk + (t - t0)] = (t <= pos + j / G) ? __fmul_rn(sc, rs) : -INFINITY;
            }
        }
        __syncthreads();
        // Chunk-local softmax per (query, head): warp j, lanes over positions.
        for (int j = warp; j < nq * G; j += nwarps) {
            float mx = -INFINITY;
            for (int t = lane; t < t1 - t0; t += 32) mx = fmaxf(mx, ps[j * kAttnChunk + t]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            float l = 0.0f;
            for (int t = lane; t < t1 - t0; t += 32) {
                const float sc = ps[j * kAttnChunk + t];
                const float e = sc == -INFINITY ? 0.0f : expf(__fsub_rn(sc, mx));
                ps[j * kAttnChunk + t] = e;
                l = __fadd_rn(l, e);
            }
            l = warp_sum(l);
            if (lane == 0) {
                part[(size_t)j * (D + 2) + D] = mx;
                part[(size_t)j * (D + 2) + D + 1] = l;
            }
        }
        __syncthreads();
        // Weighted values over the chunk: thread d, every (query, head).
        // Query heads in groups of 8 accumulators (G <= 8 per token).
        for (int d = tid; d < D; d += blockDim.x) {
#pragma unroll
            for (int i = 0; i < NQ; ++i) {
                float acc[8];
#pragma unroll
                for (int g = 0; g < 8; ++g) acc[g] = 0.0f;
                // Eight positions' value loads in flight before their FMAs (one
                // cache round trip per eight positions); each accumulator still
                // adds the positions in ascending order.
                const int tend = min(t1, pos + i + 1);
                int t = t0;
                for (; t + 8 <= tend; t += 8) {
                    float vv[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int tt = t + u;
                        vv[u] = (tt >= pos) ? vn[(tt - pos) * D + d] : a.vcache[((size_t)tt * NKV + kh) * D + d];
                    }
#pragma unroll
                    for (int u = 0; u < 8; ++u)
#pragma unroll
                        for (int g = 0; g < 8; ++g)
                            if (g < G) acc[g] = __fmaf_rn(ps[(i * G + g) * kAttnChunk + (t + u - t0)], vv[u], acc[g]);
                }
                for (; t < tend; ++t) {
                    const float vv = (t >= pos) ? vn[(t - pos) * D + d] : a.vcache[((size_t)t * NKV + kh) * D + d];
#pragma unroll
                    for (int g = 0; g < 8; ++g)
                        if (g < G) acc[g] = __fmaf_rn(ps[(i * G + g) * kAttnChunk + (t - t0)], vv, acc[g]);
                }
#pragma unroll
                for (int g = 0; g < 8; ++g)
                    if (g < G) part[(size_t)(i * G + g) * (D + 2) + d] = acc[g];
            }
        }
    }
    // The last CTA of this KV head merges, per query, the chunks that hold
    // its positions, in chunk order.
    __threadfence();
    __syncthreads();
    if (tid == 0) last = (atomicAdd(a.count + kh, 1u) == (unsigned)a.nchunks - 1u) ? 1u : 0u;
    __syncthreads();
    if (!last) return;
    __threadfence();
    const size_t cstride = (size_t)nq * G * (D + 2);
    for (int e = tid; e < nq * G * D; e += blockDim.x) {
        const int j = e / D, d = e % D, i = j / G, g = j % G;
        const int used = (pos + i) / kAttnChunk + 1;
        const float *pk = a.part + (size_t)kh * a.nchunks * cstride + (size_t)j * (D + 2);
        float M = -INFINITY;
        for (int cc = 0; cc < used; ++cc) M = fmaxf(M, __ldcg(pk + cc * cstride + D));
        float L = 0.0f, o = 0.0f;
        for (int cc = 0; cc < used; ++cc) {
            const float f = expf(__fsub_rn(__ldcg(pk + cc * cstride + D), M));
            L = __fmaf_rn(__ldcg(pk + cc * cstride + D + 1), f, L);
            o = __fmaf_rn(__ldcg(pk + cc * cstride + d), f, o);
        }
        const int h = kh * G + g;
        const float gate = a.proj[(size_t)i * P + (size_t)h * 2 * D + D + d];
        a.out[(size_t)i * NH * D + (size_t)h * D + d] = __fmul_rn(__fdiv_rn(o, L), sigmoid_f32(gate));
    }
    if (tid == 0) a.count[kh] = 0u;
}

// Embed a block of inputs.  Verification block: input 0 is the anchor (the
// last emitted token), input i >= 1 the draft for position pos + i.
// Prefill block (prompt set): input i is the prompt token at pos + i.
template <bool BF16>
__global__ void embed_block_kernel(const uint32_t *__restrict__ w, const void *__restrict__ s,
                                   const void *__restrict__ bias, uint32_t cols, uint32_t bits, uint32_t group,
                                   const DecodeCtrl *ctrl, const int32_t *drafts, const int32_t *prompt,
                                   BlockCtrl *bctrl, float *__restrict__ x) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y;
    const uint32_t pos = ctrl->pos;
    if (bctrl != nullptr && c == 0 && i == 0) bctrl->pos_base = pos;
    if (c >= cols) return;
    const uint64_t row = prompt != nullptr ? (uint32_t)prompt[pos + i]
                                           : (i == 0 ? (uint32_t)ctrl->token : (uint32_t)drafts[pos + i]);
    const uint32_t pack = 32u / bits;
    const uint32_t word = __ldg(w + row * (cols / pack) + c / pack);
    const uint32_t q = (word >> ((c % pack) * bits)) & ((1u << bits) - 1u);
    const uint64_t gi = row * (cols / group) + c / group;
    x[(size_t)i * cols + c] = __fadd_rn(__fmul_rn((float)q, load_meta<BF16>(s, gi)), load_meta<BF16>(bias, gi));
}

// Greedy verification of one block (one warp; lane 0 decides).
__global__ void verify_kernel(DecodeCtrl *ctrl, BlockCtrl *bctrl, const int32_t *argmax, const int32_t *drafts, int nq,
                              int32_t *out, uint32_t cap) {
    if (threadIdx.x != 0) return;
    const uint32_t pos = bctrl->pos_base;
    int acc = 0;
    while (acc < nq - 1 && drafts[pos + 1 + acc] == argmax[acc]) ++acc;
    uint32_t n = ctrl->n_out;
    for (int j = 0; j < acc; ++j, ++n)
        if (n < cap) out[n] = drafts[pos + 1 + j];
    if (n < cap) out[n] = argmax[acc];
    ctrl->n_out = n + 1;
    ctrl->token = argmax[acc];
    ctrl->pos = pos + (uint32_t)acc + 1u;
    bctrl->consumed = (uint32_t)acc + 1u;
    bctrl->accepted = (uint32_t)acc;
    bctrl->rounds += 1u;
    bctrl->drafts_accepted += (uint32_t)acc;
}

// Roll every DeltaNet layer back to the consumed prefix: the convolution
// history after `consumed` inputs into the live buffer of that position's
// parity, and (when inputs were rejected) the recurrent state before input
// `consumed`.  Grid: (chunks, layers).
__global__ void commit_kernel(const BlockCtrl *bctrl, float *const *layer_ptrs, int nq, size_t conv_elems,
                              size_t state_elems) {
    const int layer = blockIdx.y;
    const uint32_t consumed = bctrl->consumed, pos_next = bctrl->pos_base + consumed;
    float *conv = layer_ptrs[4 * layer + 0], *state = layer_ptrs[4 * layer + 1];
    const float *csnap = layer_ptrs[4 * layer + 2], *ssnap = layer_ptrs[4 * layer + 3];
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    float *live = conv + (size_t)(pos_next & 1u) * conv_elems;
    const float *src = csnap + (size_t)consumed * conv_elems;
    for (size_t i = i0; i < conv_elems; i += stride) live[i] = src[i];
    if ((int)consumed < nq) {
        const float4 *ss = reinterpret_cast<const float4 *>(ssnap + (size_t)consumed * state_elems);
        float4 *sd = reinterpret_cast<float4 *>(state);
        for (size_t i = i0; i < state_elems / 4; i += stride) sd[i] = ss[i];
    }
}

// End of a step: append the greedy token (when the step had a head) and
// advance the position.
__global__ void advance_kernel(DecodeCtrl *ctrl, int32_t *out, uint32_t cap, int record, int step) {
    if (threadIdx.x != 0) return;
    if (record) {
        if (ctrl->n_out < cap) out[ctrl->n_out] = ctrl->token;
        ctrl->n_out += 1;
    }
    ctrl->pos += (uint32_t)step;
}

int launched(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    return QMR_OK;
}

}  // namespace

int launch_synth_q4(uint32_t *w, uint16_t *s, uint16_t *b, uint64_t seed, uint32_t mid, uint32_t rows, uint32_t cols,
                    uint32_t row0, cudaStream_t stream) {
    if (cols % 64 != 0) return fail(QMR_EINVAL, "synthetic matrices need cols divisible by 64");
    const uint64_t wpr = cols / 8, gpr = cols / 64;
    const uint64_t npairs = (uint64_t)rows * wpr / 2;
    synth_words_kernel<<<1184, 256, 0, stream>>>(w + (uint64_t)row0 * wpr, sg_key(seed, mid, 1), 0, npairs);
    int rc = launched("synthetic weights");
    if (rc != QMR_OK) return rc;
    synth_meta_kernel<<<592, 256, 0, stream>>>(s + (uint64_t)row0 * gpr, b + (uint64_t)row0 * gpr,
                                               sg_key(seed, mid, 2), sg_key(seed, mid, 3), 0,
                                               (uint64_t)rows * gpr);
    return launched("synthetic metadata");
}

int launch_synth_region(uint32_t *w, uint16_t *s, uint16_t *b, uint64_t seed, uint32_t mid, uint32_t full_cols,
                        uint32_t r0, uint32_t nr, uint32_t c0, uint32_t nc, uint32_t dst_wstride, uint32_t dst_mstride,
                        uint32_t dst_row0, cudaStream_t stream) {
    if (full_cols % 64 != 0 || c0 % 64 != 0 || nc % 64 != 0 || c0 + nc > full_cols)
        return fail(QMR_EINVAL, "synthetic regions need 64-column alignment");
    synth_region_kernel<<<1184, 256, 0, stream>>>(w, s, b, sg_key(seed, mid, 1), sg_key(seed, mid, 2),
                                                  sg_key(seed, mid, 3), full_cols, r0, nr, c0, nc, dst_wstride,
                                                  dst_mstride, dst_row0);
    return launched("synthetic region");
}

int launch_partial_sum(float *x, const float *slots, int world, int H, int nq, cudaStream_t stream) {
    partial_sum_kernel<<<dim3((unsigned)((H + 255) / 256), (unsigned)nq), 256, 0, stream>>>(x, slots, world, H, nq);
    return launched("partial sum");
}

int launch_fill_f32(float *p, uint64_t n, float v, cudaStream_t stream) {
    fill_kernel<<<296, 256, 0, stream>>>(p, n, v);
    return launched("fill");
}

int launch_embed_token(const void *w, const void *s, const void *b, bool bf16, uint32_t cols, uint32_t bits,
                       uint32_t group, const DecodeCtrl *ctrl, const int32_t *prompt, float *x, cudaStream_t stream) {
    const unsigned grid = (cols + 255) / 256;
    if (bf16)
        embed_token_kernel<true><<<grid, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, cols, bits, group,
                                                           ctrl, prompt, x);
    else
        embed_token_kernel<false><<<grid, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, cols, bits, group,
                                                            ctrl, prompt, x);
    return launched("embed");
}

int launch_rms_norm(const float *x, const float *w, float *y, uint32_t n, float eps, cudaStream_t stream) {
    rms_norm_kernel<<<1, 512, 0, stream>>>(x, w, y, n, eps);
    return launched("rms_norm");
}

int launch_add(float *x, const float *r, uint32_t n, cudaStream_t stream) {
    add_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, r, n);
    return launched("add");
}

int launch_delta_mixer(const DeltaArgs &a, cudaStream_t stream) {
    if (a.K > 128 || a.K < 1 || a.V < 1 || a.KH < 1 || a.VH % a.KH != 0 || a.W < 1 || a.W > kMaxConvHist + 1 ||
        a.nq < 1 || a.nq > kMaxTokens || (a.nq % 2 == 0 && a.conv_snap == nullptr))
        // Without snapshots the block's conv history goes to the ping-pong
        // buffer of parity pos + 1, which the next step reads only after an
        // odd number of tokens.
        return fail(QMR_EUNSUPPORTED,
                    "DeltaNet mixer needs key dim <= 128, value heads a multiple of key heads, conv width <= 8 and "
                    "1..4 tokens (an even number only as a verification block)");
    const int rows = (a.V + kDeltaSplit - 1) / kDeltaSplit;
    const size_t smem = (size_t)(a.nq * (2 * a.K + 2 * rows) + 33) * sizeof(float);
    delta_mixer_kernel<<<a.VH * kDeltaSplit, kDeltaThreads, smem, stream>>>(a);
    return launched("DeltaNet mixer");
}

int launch_attention(const AttnArgs &a, cudaStream_t stream) {
    const int G = a.NH / a.NKV;
    if (a.D > 256 || a.D < 1 || a.NKV < 1 || a.NH % a.NKV != 0 || G > 8 || a.RD > a.D || a.RD % 2 != 0 || a.nq < 1 ||
        a.nq > kMaxTokens)
        return fail(QMR_EUNSUPPORTED,
                    "decode attention needs head_dim <= 256, at most 8 query heads per KV head and 1..4 tokens");
    const size_t smem = (size_t)(a.nq * G * a.D + 2 * a.nq * a.D + a.nq * G * kAttnChunk) * sizeof(float);
    if (smem > 48 * 1024) return fail(QMR_EUNSUPPORTED, "decode attention block needs %zu bytes of shared memory", smem);
    const dim3 grid((unsigned)a.nchunks, (unsigned)a.NKV);
    switch (a.nq) {
        case 1: attention_kernel<1><<<grid, kAttnThreads, smem, stream>>>(a); break;
        case 2: attention_kernel<2><<<grid, kAttnThreads, smem, stream>>>(a); break;
        case 3: attention_kernel<3><<<grid, kAttnThreads, smem, stream>>>(a); break;
        default: attention_kernel<4><<<grid, kAttnThreads, smem, stream>>>(a); break;
    }
    return launched("attention");
}

int launch_embed_block(const void *w, const void *s, const void *b, bool bf16, uint32_t cols, uint32_t bits,
                       uint32_t group, const DecodeCtrl *ctrl, const int32_t *drafts, const int32_t *prompt,
                       BlockCtrl *bctrl, int nq, float *x, cudaStream_t stream) {
    const dim3 grid((cols + 255) / 256, (unsigned)nq);
    if (bf16)
        embed_block_kernel<true><<<grid, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, cols, bits, group,
                                                           ctrl, drafts, prompt, bctrl, x);
    else
        embed_block_kernel<false><<<grid, 256, 0, stream>>>(static_cast<const uint32_t *>(w), s, b, cols, bits, group,
                                                            ctrl, drafts, prompt, bctrl, x);
    return launched("block embed");
}

int launch_verify(DecodeCtrl *ctrl, BlockCtrl *bctrl, const int32_t *argmax, const int32_t *drafts, int nq,
                  int32_t *out, uint32_t out_cap, cudaStream_t stream) {
    verify_kernel<<<1, 32, 0, stream>>>(ctrl, bctrl, argmax, drafts, nq, out, out_cap);
    return launched("verify");
}

int launch_commit(const BlockCtrl *bctrl, float *const *layer_ptrs, int nlayers, int nq, size_t conv_elems,
                  size_t state_elems, cudaStream_t stream) {
    if (nlayers == 0) return QMR_OK;
    commit_kernel<<<dim3(64, (unsigned)nlayers), 256, 0, stream>>>(bctrl, layer_ptrs, nq, conv_elems, state_elems);
    return launched("commit");
}

int launch_advance(DecodeCtrl *ctrl, int32_t *out, uint32_t out_cap, bool record, cudaStream_t stream, int step) {
    advance_kernel<<<1, 32, 0, stream>>>(ctrl, out, out_cap, record ? 1 : 0, step);
    return launched("advance");
}

}  // namespace qmr
