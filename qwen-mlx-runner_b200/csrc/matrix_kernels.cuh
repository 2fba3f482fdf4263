// Packed-affine dequantise-and-multiply kernels for sm_100a.
//
// Semantics follow the reference's matrix kernels (rucin93/qwen-mlx-runner
// v0.7.3): y[b*rows+r] = sum_c (q[r,c]*s[r,g]+b[r,g]) * x[b*cols+c], with
// q little-endian inside each u32 word (kernels/qwen.metal:40-47), f32 or
// bf16-high-half metadata (kernels/affine_bf16.metal:294-296) and token-major
// block operands (kernels/matmul_block.metal:1-3).  The arithmetic schedule
// is this file's own, built for B200:
//
//  * Weights stream once from HBM with 16-byte non-allocating loads; one warp
//    owns R rows and its lane l owns 16-byte chunks l, l+32, ... of each row,
//    so a warp-wide load is 512 contiguous bytes of one row.
//  * Dequantisation costs one LOP3 per element.  A nibble (or byte) masked in
//    place, `w & (0xf << 4k)`, read as an f32 bit pattern is the exact
//    subnormal q * 2^(4k-149).  The activation was pre-scaled by
//    2^(E-4k) (prep kernel), so fma(subnormal, x', acc) accumulates
//    q*x*2^(E-149) with one rounding, exactly like an f32 fma of q*x.  E is
//    chosen per 32-element activation chunk so that no pre-scaled value
//    overflows; the chunk result is scaled back by 2^(149-E) (two exact
//    power-of-two multiplies) before the group scale and bias are applied.
//    IEEE subnormals are required: this file must not be built with -ftz.
//  * Products are accumulated with packed f32x2 FMAs (even/odd elements),
//    every (row, RHS) pair in the same order whatever the block width B or
//    rows-per-warp R, so a B-wide block equals B GEMVs bit for bit.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace qmr {

constexpr int kWarp = 32;

// Elements per 16-byte chunk for a bit width.
template <int BITS>
struct Chunk {
    static constexpr int elems = 128 / BITS;      // 32 for Q4, 16 for Q8
    static constexpr int per_word = 32 / BITS;    // 8 for Q4, 4 for Q8
};

// Pre-scale exponent offset f(k) of element k within its word: the power of
// two the in-place mask leaves on the extracted value.  Q4: nibbles 0..4 are
// masked in place (bits 0..19), nibbles 5..7 after w >> 20.  Q8: bytes 0,1 in
// place, bytes 2,3 after w >> 16.
template <int BITS>
__host__ __device__ constexpr int prescale_shift(int k) {
    return BITS == 4 ? 4 * (k < 5 ? k : k - 5) : 8 * (k & 1);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t v) {
    return __uint_as_float(static_cast<uint32_t>(v) << 16);
}

template <bool BF16>
__device__ __forceinline__ float load_meta(const void *__restrict__ m, size_t i) {
    if constexpr (BF16) {
        return bf16_bits_to_f32(__ldg(static_cast<const unsigned short *>(m) + i));
    } else {
        return __ldg(static_cast<const float *>(m) + i);
    }
}

__device__ __forceinline__ uint4 ldg_stream(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    return __ffma2_rn(a, b, c);
}

// Subnormal view of a masked word.
__device__ __forceinline__ float sub(uint32_t bits) { return __uint_as_float(bits); }

// ---------------------------------------------------------------------------
// Activation prep.  For every RHS b and 16-byte chunk j of a row (32 Q4 or 16
// Q8 elements) writes
//   xp : x[b, c] * 2^(E_j - f(c)) in the lane-interleaved order the streaming
//        kernel reads (see xp_index), and
//   xs : {sum_c x[b,c], 2^a, 2^(149-E_j-a), 0} with both factors normal.
// E_j makes max|x'| < 2^125 inside the chunk.  Also zeroes the argmax
// reduction slots when `keys` is non-null.
// ---------------------------------------------------------------------------

// Position, in float4 units, of the 4 pre-scaled values (j, word m, half h)
// of RHS b: 32 consecutive lanes of a warp read 512 contiguous bytes.
template <int BITS>
__host__ __device__ __forceinline__ size_t xp_index(int b, int nblocks, int j, int m, int h) {
    constexpr int halves = Chunk<BITS>::per_word / 4;  // float4s per word: 2 (Q4) or 1 (Q8)
    const int jb = j >> 5, lane = j & 31;
    return ((((size_t)b * nblocks + jb) * 4 + m) * halves + h) * 32 + lane;
}

template <int BITS>
__global__ void __launch_bounds__(256) prep_kernel(const float *__restrict__ x, int cols, int batch,
                                                  int nchunks, float4 *__restrict__ xp,
                                                  float4 *__restrict__ xs,
                                                  unsigned long long *__restrict__ keys,
                                                  unsigned int *__restrict__ counter) {
    // Let the dependent streaming kernel launch and start its weight loads.
    asm volatile("griddepcontrol.launch_dependents;");
    constexpr int E = Chunk<BITS>::elems;  // lanes per chunk: 32 (Q4) or 16 (Q8)
    constexpr int per_warp = 32 / E;       // chunks per warp pass
    const int lane = threadIdx.x & 31;
    const int sub_lane = lane % E;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int nblocks = (nchunks + 31) >> 5;
    if (keys != nullptr && blockIdx.x == 0 && threadIdx.x < batch) {
        keys[threadIdx.x] = 0ull;
        if (threadIdx.x == 0) *counter = 0u;
    }
    const int total = batch * nchunks;
    for (int t0 = warp * per_warp; t0 < total; t0 += nwarps * per_warp) {
        const int t = t0 + lane / E;  // (b, j) handled by this lane group
        const bool valid = t < total;
        const int b = valid ? t / nchunks : 0;
        const int j = valid ? t % nchunks : 0;
        const float v = valid ? x[(size_t)b * cols + (size_t)j * E + sub_lane] : 0.0f;
        // max |x| and sum x over the chunk, fixed butterfly order.
        float mx = fabsf(v), sm = v;
#pragma unroll
        for (int o = E / 2; o > 0; o >>= 1) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            sm = sm + __shfl_xor_sync(0xffffffffu, sm, o);
        }
        // exponent of max|x|: max|x| < 2^(e+1).  Zero or subnormal chunks use
        // e = -127 (any E works: products are exact or zero).
        const uint32_t mb = __float_as_uint(mx);
        int e = (int)((mb >> 23) & 0xff) - 127;
        if (e < -127) e = -127;
        int Ej = 124 - e;  // max|x| * 2^Ej < 2^125; e <= 128 -> Ej >= -4
        const int k = sub_lane % Chunk<BITS>::per_word;
        const float xv = ldexpf(v, Ej - prescale_shift<BITS>(k));
        if (valid) {
            const int m = sub_lane / Chunk<BITS>::per_word;
            const int within = k;  // element inside the word
            float *dst = reinterpret_cast<float *>(xp + xp_index<BITS>(b, nblocks, j, m, within >> 2));
            dst[within & 3] = xv;
            if (sub_lane == 0) {
                int total_shift = 149 - Ej;  // in [-128, 276]
                int a = total_shift > 120 ? 120 : (total_shift < -120 ? -120 : total_shift);
                xs[(size_t)b * nchunks + j] =
                    make_float4(sm, ldexpf(1.0f, a), ldexpf(1.0f, total_shift - a), 0.0f);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Streaming block kernel.  One warp = R consecutive rows, all B RHS.
// EPI selects the epilogue:
//   0: plain, y[b*ystride + row]
//   1: gate/up SwiGLU: a second matrix (w2,s2,b2) with the same layout;
//      y = silu(gate)*up
//   2: head: y written as plain, plus argmax over rows into keys[b].
// ---------------------------------------------------------------------------
struct StreamArgs {
    const uint4 *w;
    const void *s;
    const void *bias;
    const uint4 *w2;  // EPI 1 (up projection)
    const void *s2;
    const void *bias2;
    const float4 *xp;
    const float4 *xs;
    float *y;
    unsigned long long *keys;  // EPI 2
    unsigned int *counter;     // EPI 2
    int *argmax;               // EPI 2 (may be null)
    unsigned long long *best_key_out;  // EPI 2 (may be null)
    int rows;
    int nchunks;     // 16-byte chunks per row
    int group_shift; // log2(chunks per group)
    int ystride;     // rows of y per RHS
    int row_base;    // added to argmax indices
};

__device__ __forceinline__ float silu_f32(float g) {
    // silu(x) = x * (1 / (1 + exp(-x))), kernels/qwen.metal:32-33.
    return g * __frcp_rn(__fadd_rn(1.0f, expf(-g)));
}

__device__ __forceinline__ uint32_t total_order_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Extract the 8 (Q4) or 4 (Q8) elements of one word as exact subnormals,
// pairwise, in the element order of the pre-scaled activations.
template <int BITS>
__device__ __forceinline__ void extract(uint32_t w, float2 (&d)[Chunk<BITS>::per_word / 2]) {
    if constexpr (BITS == 4) {
        const uint32_t h = w >> 20;
        d[0] = make_float2(sub(w & 0xfu), sub(w & 0xf0u));
        d[1] = make_float2(sub(w & 0xf00u), sub(w & 0xf000u));
        d[2] = make_float2(sub(w & 0xf0000u), sub(h & 0xfu));
        d[3] = make_float2(sub(h & 0xf0u), sub(h & 0xf00u));
    } else {
        const uint32_t h = w >> 16;
        d[0] = make_float2(sub(w & 0xffu), sub(w & 0xff00u));
        d[1] = make_float2(sub(h & 0xffu), sub(h & 0xff00u));
    }
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int m) {
    return m == 0 ? v.x : (m == 1 ? v.y : (m == 2 ? v.z : v.w));
}

// Fold one chunk's partial into the row accumulator:
//   acc += s * (p * 2^(149-E)) + bias * xsum.
__device__ __forceinline__ float fold(float acc, float2 p, float4 xsc, float s, float bias) {
    const float t = __fmul_rn(__fmul_rn(__fadd_rn(p.x, p.y), xsc.y), xsc.z);
    acc = __fmaf_rn(s, t, acc);
    return __fmaf_rn(bias, xsc.x, acc);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int BITS, int B, int R, bool BF16, int EPI>
__global__ void __launch_bounds__(256, 2) stream_kernel(const StreamArgs a) {
    constexpr int XW = Chunk<BITS>::per_word / 2;  // float2 pairs per word
    constexpr int NM = (EPI == 1) ? 2 : 1;          // matrices streamed
    const int lane = threadIdx.x & 31;
    const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int row0 = gwarp * R;
    const int nchunks = a.nchunks;
    const int nblocks = (nchunks + 31) >> 5;
    const int groups = nchunks >> a.group_shift;

    float acc[NM][B][R];
#pragma unroll
    for (int q = 0; q < NM; ++q)
#pragma unroll
        for (int b = 0; b < B; ++b)
#pragma unroll
            for (int r = 0; r < R; ++r) acc[q][b][r] = 0.0f;

    const bool warp_live = row0 < a.rows;
    bool waited = false;
    if (warp_live) {
        for (int jb = 0; jb < nblocks; ++jb) {
            const int j = jb * 32 + lane;
            const bool valid = j < nchunks;
            uint4 wv[NM][R];
            float sc[NM][R], bi[NM][R];
#pragma unroll
            for (int q = 0; q < NM; ++q) {
                const uint4 *W = q ? a.w2 : a.w;
                const void *S = q ? a.s2 : a.s;
                const void *Bi = q ? a.bias2 : a.bias;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int row = row0 + r;
                    if (valid && row < a.rows) {
                        wv[q][r] = ldg_stream(W + (size_t)row * nchunks + j);
                        const size_t gi = (size_t)row * groups + (j >> a.group_shift);
                        sc[q][r] = load_meta<BF16>(S, gi);
                        bi[q][r] = load_meta<BF16>(Bi, gi);
                    } else {
                        wv[q][r] = make_uint4(0, 0, 0, 0);
                        sc[q][r] = 0.0f;
                        bi[q][r] = 0.0f;
                    }
                }
            }
            if (!waited) {
                // The first weights are in flight; wait for the prep kernel.
                asm volatile("griddepcontrol.wait;" ::: "memory");
                waited = true;
            }
            float4 xsc[B];
#pragma unroll
            for (int b = 0; b < B; ++b)
                xsc[b] = valid ? __ldg(a.xs + (size_t)b * nchunks + j) : make_float4(0.f, 0.f, 0.f, 0.f);
            float2 p[NM][R][B];
#pragma unroll
            for (int q = 0; q < NM; ++q)
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int b = 0; b < B; ++b) p[q][r][b] = make_float2(0.f, 0.f);
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                float2 xv[B][XW];
#pragma unroll
                for (int b = 0; b < B; ++b) {
#pragma unroll
                    for (int h = 0; h < XW / 2; ++h) {
                        const float4 v = valid ? __ldg(a.xp + xp_index<BITS>(b, nblocks, j, m, h))
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
                        xv[b][2 * h] = make_float2(v.x, v.y);
                        xv[b][2 * h + 1] = make_float2(v.z, v.w);
                    }
                }
#pragma unroll
                for (int q = 0; q < NM; ++q) {
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        float2 d[XW];
                        extract<BITS>(word_of(wv[q][r], m), d);
#pragma unroll
                        for (int b = 0; b < B; ++b)
#pragma unroll
                            for (int e = 0; e < XW; ++e) p[q][r][b] = ffma2(d[e], xv[b][e], p[q][r][b]);
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < NM; ++q)
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int b = 0; b < B; ++b)
                        acc[q][b][r] = fold(acc[q][b][r], p[q][r][b], xsc[b], sc[q][r], bi[q][r]);
        }
    }
    if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");

    // Cross-lane reduction, fixed butterfly order: every lane ends with the sum.
#pragma unroll
    for (int q = 0; q < NM; ++q)
#pragma unroll
        for (int b = 0; b < B; ++b)
#pragma unroll
            for (int r = 0; r < R; ++r) acc[q][b][r] = warp_sum(acc[q][b][r]);

    // Lane r stores row row0 + r.
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (warp_live && lane == r && row0 + r < a.rows) {
#pragma unroll
            for (int b = 0; b < B; ++b) {
                float v = acc[0][b][r];
                if constexpr (EPI == 1) v = __fmul_rn(silu_f32(v), acc[NM - 1][b][r]);
                a.y[(size_t)b * a.ystride + row0 + r] = v;
            }
        }
    }

    if constexpr (EPI == 2) {
        // Argmax over this warp's rows, one atomicMax per warp and RHS on a
        // packed (total-order key, ~index) word: the max is order independent.
        __shared__ unsigned int last_block;
#pragma unroll
        for (int b = 0; b < B; ++b) {
            unsigned long long best = 0ull;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = row0 + r;
                if (row < a.rows) {
                    const unsigned long long key =
                        ((unsigned long long)total_order_key(acc[0][b][r]) << 32) |
                        (unsigned long long)(0xffffffffu - (uint32_t)(a.row_base + row));
                    best = key > best ? key : best;
                }
            }
            if (lane == 0 && warp_live) atomicMax(a.keys + b, best);
        }
        // The last block to finish publishes the winners (fence + counter; no waiting).
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last_block = (atomicAdd(a.counter, 1u) == gridDim.x - 1) ? 1u : 0u;
        __syncthreads();
        if (last_block && threadIdx.x < B) {
            __threadfence();
            const unsigned long long k = atomicAdd(a.keys + threadIdx.x, 0ull);
            if (a.argmax) a.argmax[threadIdx.x] = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
            if (a.best_key_out) a.best_key_out[threadIdx.x] = k;
        }
    }
}

// ---------------------------------------------------------------------------
// Generic kernel: the reference's per-element semantics for any layout the
// dispatch ABI accepts (any group dividing cols, 4-byte aligned views, Q4/Q8,
// f32 or bf16 metadata).  One warp per row, lanes stride the columns, every
// element dequantised as float(q)*s + b (kernels/qwen.metal:40-47) and
// multiplied into an f32 fma chain per RHS.
// ---------------------------------------------------------------------------
template <bool BF16>
__global__ void __launch_bounds__(256) generic_kernel(const uint32_t *__restrict__ w,
                                                     const void *__restrict__ s,
                                                     const void *__restrict__ bias,
                                                     const float *__restrict__ x,
                                                     float *__restrict__ y, uint32_t rows,
                                                     uint32_t cols, uint32_t bits, uint32_t group,
                                                     uint32_t batch) {
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t row = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    const uint32_t pack = 32u / bits;
    const uint32_t mask = (1u << bits) - 1u;
    const uint64_t wbase = row * (cols / pack);
    const uint64_t gbase = row * (cols / group);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (uint32_t c = lane; c < cols; c += 32) {
        const uint32_t word = __ldg(w + wbase + c / pack);
        const uint32_t q = (word >> ((c % pack) * bits)) & mask;
        const uint64_t gi = gbase + c / group;
        const float v = __fadd_rn(__fmul_rn((float)q, load_meta<BF16>(s, gi)), load_meta<BF16>(bias, gi));
#pragma unroll
        for (uint32_t b = 0; b < 4; ++b)
            if (b < batch) acc[b] = __fmaf_rn(v, __ldg(x + (uint64_t)b * cols + c), acc[b]);
    }
#pragma unroll
    for (uint32_t b = 0; b < 4; ++b) {
        if (b < batch) {
            const float t = warp_sum(acc[b]);
            if (lane == 0) y[(uint64_t)b * rows + row] = t;
        }
    }
}

// embed_affine[_bf16]: y[c] = float(q)*s + b for one row, two roundings, which
// is bit-exact with the reference (kernels/qwen.metal:73-77,
// kernels/affine_bf16.metal:439-451).
template <bool BF16>
__global__ void embed_kernel(const uint32_t *__restrict__ w, const void *__restrict__ s,
                             const void *__restrict__ bias, float *__restrict__ y, uint64_t row,
                             uint32_t cols, uint32_t bits, uint32_t group) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const uint32_t pack = 32u / bits;
    const uint32_t word = __ldg(w + row * (cols / pack) + c / pack);
    const uint32_t q = (word >> ((c % pack) * bits)) & ((1u << bits) - 1u);
    const uint64_t gi = row * (cols / group) + c / group;
    y[c] = __fadd_rn(__fmul_rn((float)q, load_meta<BF16>(s, gi)), load_meta<BF16>(bias, gi));
}

}  // namespace qmr
