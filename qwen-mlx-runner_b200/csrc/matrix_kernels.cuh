// Packed-affine dequantise-and-multiply kernels for sm_100a: shared helpers,
// the activation prep pass, the register-streaming fallback kernel, the
// generic per-element kernel and the embed kernel.  The default streaming
// kernel is the tensor-core one in mma_stream.cuh; the FP32 TMA pipeline is
// tile.cuh.
//
// Semantics follow the reference's matrix kernels (rucin93/qwen-mlx-runner
// v0.7.3): y[b*rows+r] = sum_c (q[r,c]*s[r,g]+b[r,g]) * x[b*cols+c], with
// q little-endian inside each u32 word (kernels/qwen.metal:40-47), f32 or
// bf16-high-half metadata (kernels/affine_bf16.metal:294-296) and token-major
// block operands (kernels/matmul_block.metal:1-3).  The arithmetic schedule
// is this build's own:
//
//  * Dequantisation costs one LOP3 per element.  A nibble (or byte) masked in
//    place, `w & (0xf << 4k)`, read as an f32 bit pattern is the exact
//    subnormal q * 2^(4k-149).  The activation of RHS b was pre-scaled by
//    2^(E_b - 4k) (prep_kernel), so fma(subnormal, x', acc) accumulates
//    q*x*2^(E_b-149) with one rounding, exactly as an f32 fma of q*x would.
//    E_b is chosen per RHS from max|x| so that no pre-scaled value overflows;
//    outputs are scaled back by 2^(149-E_b) (two exact power-of-two
//    multiplies).  IEEE subnormals are required: never build with -ftz.
//  * Products accumulate in packed f32x2 FMAs (even/odd elements).  Each
//    16-byte chunk (32 Q4 / 16 Q8 elements, inside one group) yields a
//    partial p that is folded as acc += s*p (f32x2) and acc.x += bias*xsum'
//    with xsum' the chunk's activation sum scaled by 2^(E_b-149).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace qmr {

// Elements per 16-byte chunk for a bit width.
template <int BITS>
struct Chunk {
    static constexpr int elems = 128 / BITS;    // 32 for Q4, 16 for Q8
    static constexpr int per_word = 32 / BITS;  // 8 for Q4, 4 for Q8
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

template <bool BF16>
__device__ __forceinline__ float smem_meta(const uint8_t *base, int i) {
    if constexpr (BF16) {
        return bf16_bits_to_f32(reinterpret_cast<const unsigned short *>(base)[i]);
    } else {
        return reinterpret_cast<const float *>(base)[i];
    }
}

__device__ __forceinline__ uint4 ldg_stream(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// Subnormal view of a masked word.
__device__ __forceinline__ float sub(uint32_t bits) { return __uint_as_float(bits); }

// Extract the 8 (Q4) or 4 (Q8) elements of one word as exact subnormals,
// pairwise, in element order.
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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float silu_f32(float g) {
    // silu(x) = x * (1 / (1 + exp(-x))), kernels/qwen.metal:32-33.
    return __fmul_rn(g, __frcp_rn(__fadd_rn(1.0f, expf(-g))));
}

// Key ordering f32 like Rust's f32::total_cmp, as an unsigned integer.
__device__ __forceinline__ uint32_t total_order_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------------------
// Prepared activations ("scratch"), one buffer per call or caller-owned:
//   xp [B][nblocks][BF] f32: per block of 32 chunks, the values
//                   x[b][k] * 2^(E_b - f(k mod per_word)) in lane-interleaved
//                   order (see block_index), then the 32 chunk sums
//                   (sum of x over the chunk) * 2^(E_b - 149); chunks past
//                   the row end are zero
//   cf [B][2]       2^a, 2^(149 - E_b - a): the output factor, split so both
//                   halves are normal
//   keys [4] u64    argmax reduction (zeroed here)
//   done u32        CTAs finished (zeroed here)
//   counters        split-K arrivals per (row range, tile) (zeroed here; the
//                   kernels also leave them at zero)
//   partial         split-K partial sums
// ---------------------------------------------------------------------------
constexpr int kBlockChunks = 32;           // chunks per prepared block (one per lane)
constexpr int kCounterCount = 8192;        // arrival counters of split tiles
constexpr size_t kPartialFloats = 524288;  // 2 MiB of split-K partial sums

template <int BITS>
__host__ __device__ constexpr int prepared_block_floats() {
    return kBlockChunks * Chunk<BITS>::elems + kBlockChunks;
}

// Float index, inside its block, of element k of chunk c (c < 32): the values
// a lane needs for word m of its chunk are 4*H consecutive floats of a
// 512-byte row shared by the 32 lanes.
template <int BITS>
__host__ __device__ constexpr int block_index(int c, int k) {
    constexpr int per_word = Chunk<BITS>::per_word;
    constexpr int H = per_word / 4;  // float4 per word: 2 (Q4) or 1 (Q8)
    return (((k / per_word) * H + (k % per_word) / 4) * kBlockChunks + c) * 4 + (k & 3);
}

struct ScratchView {
    float *xp;
    float *cf;
    unsigned long long *keys;
    unsigned int *done;
    unsigned int *counters;
    float *partial;
};

// One CTA per RHS: global max|x| -> E_b, then the pre-scaled activations and
// the scaled chunk sums in prepared blocks.  Block 0 also zeroes the
// reduction words.
template <int BITS>
__global__ void __launch_bounds__(512) prep_kernel(const float *__restrict__ x, int cols, int nchunks,
                                                  ScratchView sv) {
    // Let the dependent streaming kernel launch and start its weight loads.
    asm volatile("griddepcontrol.launch_dependents;");
    constexpr int CE = Chunk<BITS>::elems;
    constexpr int BF = prepared_block_floats<BITS>();
    const int b = blockIdx.x;
    const float *xb = x + (size_t)b * cols;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int nblocks = (nchunks + kBlockChunks - 1) / kBlockChunks;
    __shared__ float wmax[32];
    __shared__ int s_e;

    if (b == 0) {
        if (tid < 4) sv.keys[tid] = 0ull;
        if (tid == 0) *sv.done = 0u;
        for (int i = tid; i < kCounterCount; i += blockDim.x) sv.counters[i] = 0u;
    }
    float mx = 0.0f;
    bool nonfinite = false;
    for (int i = tid; i < cols; i += blockDim.x) {
        const float a = fabsf(xb[i]);
        nonfinite |= !(a <= 3.402823466e38f);  // inf or NaN
        mx = fmaxf(mx, a);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    nonfinite = __any_sync(0xffffffffu, nonfinite);
    if (lane == 0) wmax[warp] = nonfinite ? __int_as_float(0x7f800000) : mx;
    __syncthreads();
    if (tid == 0) {
        float m = 0.0f;
        for (int w = 0; w < nw; ++w) m = fmaxf(m, wmax[w]);
        int e = (int)((__float_as_uint(m) >> 23) & 0xff) - 127;  // max|x| < 2^(e+1); inf -> 128
        if (e < -127) e = -127;  // zero or subnormal: any E keeps products exact
        s_e = e;
    }
    __syncthreads();
    const int E = 124 - s_e;  // max|x| * 2^E < 2^125
    if (tid == 0) {
        const int t = 149 - E;
        const int a = t > 120 ? 120 : (t < -120 ? -120 : t);
        sv.cf[2 * b] = ldexpf(1.0f, a);
        sv.cf[2 * b + 1] = ldexpf(1.0f, t - a);
    }
    // One chunk per 32 (Q4) or 16 (Q8) lanes; fixed butterfly for the sums.
    constexpr int per_warp = 32 / CE;
    const int k = lane % CE;
    float *out = sv.xp + (size_t)b * nblocks * BF;
    for (int j0 = warp * per_warp; j0 < nblocks * kBlockChunks; j0 += nw * per_warp) {
        const int j = j0 + lane / CE;
        const float v = j < nchunks ? xb[(size_t)j * CE + k] : 0.0f;
        float sm = v;
#pragma unroll
        for (int o = CE / 2; o > 0; o >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, o));
        float *blk = out + (size_t)(j / kBlockChunks) * BF;
        const int c = j % kBlockChunks;
        blk[block_index<BITS>(c, k)] = ldexpf(v, E - prescale_shift<BITS>(k % Chunk<BITS>::per_word));
        if (k == 0) blk[kBlockChunks * CE + c] = ldexpf(sm, E - 149);
    }
}

// ---------------------------------------------------------------------------
// Register-streaming kernel: the fallback for layouts the TMA kernel cannot
// copy (metadata rows that are not 16-byte multiples, unaligned metadata).
// One warp = R consecutive rows; lane l owns chunks l, l+32, ... of each row;
// the lane partials meet in a butterfly reduction.
// EPI: 0 plain, 1 gate/up SwiGLU (second matrix w2/s2/b2), 2 head + argmax.
// ---------------------------------------------------------------------------
struct StreamArgs {
    const uint4 *w;
    const void *s;
    const void *bias;
    const uint4 *w2;
    const void *s2;
    const void *bias2;
    const float *xp;
    const float *cf;
    float *y;
    unsigned long long *keys;
    unsigned int *done;
    int *argmax;
    unsigned long long *best_key_out;
    int rows;
    int nchunks;
    int group_shift;
    int ystride;
    int row_base;
};

template <int BITS, int B, int R, bool BF16, int EPI>
__global__ void __launch_bounds__(256, 2) stream_kernel(const StreamArgs a) {
    constexpr int XW = Chunk<BITS>::per_word / 2;
    constexpr int H = XW / 2;
    constexpr int CE = Chunk<BITS>::elems;
    constexpr int BF = prepared_block_floats<BITS>();
    constexpr int NM = (EPI == 1) ? 2 : 1;
    const int lane = threadIdx.x & 31;
    const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int row0 = gwarp * R;
    const int nchunks = a.nchunks;
    const int groups = nchunks >> a.group_shift;
    const int nblocks = (nchunks + kBlockChunks - 1) / kBlockChunks;

    float2 acc[NM][R][B];
#pragma unroll
    for (int q = 0; q < NM; ++q)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b) acc[q][r][b] = make_float2(0.f, 0.f);

    const bool warp_live = row0 < a.rows;
    bool waited = false;
    if (warp_live) {
        for (int j0 = 0; j0 < nchunks; j0 += 32) {
            const int j = j0 + lane;
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
                // The first weights are in flight; now wait for the prep kernel.
                asm volatile("griddepcontrol.wait;" ::: "memory");
                waited = true;
            }
            float xsv[B];
#pragma unroll
            for (int b = 0; b < B; ++b)
                xsv[b] = __ldcg(a.xp + ((size_t)b * nblocks + j0 / kBlockChunks) * BF + kBlockChunks * CE + lane);
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
                    for (int h = 0; h < H; ++h) {
                        // Chunks past the row end hold zeros in the prepared block.
                        const float4 v = __ldcg(reinterpret_cast<const float4 *>(
                                                    a.xp + ((size_t)b * nblocks + j0 / kBlockChunks) * BF) +
                                                (m * H + h) * kBlockChunks + lane);
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
                for (int r = 0; r < R; ++r) {
                    const float2 ss = make_float2(sc[q][r], sc[q][r]);
#pragma unroll
                    for (int b = 0; b < B; ++b) {
                        acc[q][r][b] = ffma2(ss, p[q][r][b], acc[q][r][b]);
                        acc[q][r][b].x = __fmaf_rn(bi[q][r], xsv[b], acc[q][r][b].x);
                    }
                }
        }
    }
    if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");

    float tot[NM][R][B];
#pragma unroll
    for (int q = 0; q < NM; ++q)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b) tot[q][r][b] = warp_sum(__fadd_rn(acc[q][r][b].x, acc[q][r][b].y));

    unsigned long long best[B];
#pragma unroll
    for (int b = 0; b < B; ++b) best[b] = 0ull;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int row = row0 + r;
        if (warp_live && row < a.rows) {
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float c1 = __ldcg(a.cf + 2 * b), c2 = __ldcg(a.cf + 2 * b + 1);
                float v = __fmul_rn(__fmul_rn(tot[0][r][b], c1), c2);
                if constexpr (EPI == 1) v = __fmul_rn(silu_f32(v), __fmul_rn(__fmul_rn(tot[NM - 1][r][b], c1), c2));
                if (lane == r) a.y[(size_t)b * a.ystride + row] = v;
                if constexpr (EPI == 2) {
                    const unsigned long long key = ((unsigned long long)total_order_key(v) << 32) |
                                                   (unsigned long long)(0xffffffffu - (uint32_t)(a.row_base + row));
                    best[b] = key > best[b] ? key : best[b];
                }
            }
        }
    }
    if constexpr (EPI == 2) {
        __shared__ unsigned int last_block;
#pragma unroll
        for (int b = 0; b < B; ++b)
            if (lane == 0 && warp_live) atomicMax(a.keys + b, best[b]);
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last_block = (atomicAdd(a.done, 1u) == gridDim.x - 1) ? 1u : 0u;
        __syncthreads();
        if (last_block && threadIdx.x == 0) *a.done = 0u;  // ready for the next launch
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
