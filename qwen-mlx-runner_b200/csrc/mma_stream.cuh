// Weight-streaming block matmul on the tensor cores (sm_100a, mma.sync
// m16n8k16, f16 operands, f32 accumulation).
//
// Why tensor cores for M <= 4: on B200 the FP32 formulation needs one LOP3
// plus B fused multiply-adds per weight element, which issue-limits a B3 block
// well below HBM speed.  Here each warp instruction multiplies 16 rows x 16
// columns x 8 RHS columns, so the per-element cost is only the dequantisation
// (about one instruction per element) whatever the block width.
//
// Operands of one 16-row x 16-column MMA:
//  * A (weights): `w & 0x000f000f` (Q4) or `w & 0x00ff00ff` (Q8) read as a
//    half2 is a pair of exact fp16 subnormals q * 2^-24 -- no offset, no
//    conversion.  The k order inside an MMA is a fixed permutation of the
//    group's columns (block_perm); activations are stored in the same order.
//  * B (activations): x[b] * 2^E_b (E_b puts max|x[b]| just below the fp16
//    maximum) split into an fp16 high part and an fp16 low part; the eight
//    MMA columns are (RHS b, part) so each thread's accumulator pair holds
//    both parts of one RHS for two rows.
//  * Per quantisation group the group's MMAs start from zero; the f32 result
//    P (q*x*2^(E_b-24) summed over the group) is folded as
//    acc += s*P + bias*xsum', xsum' = (sum of x over the group)*2^(E_b-24);
//    the output is acc * 2^(24-E_b) (two exact power-of-two factors).
//
// Work split: CTA c owns the rows [c*rows/G, (c+1)*rows/G) in 16-row units
// (one persistent CTA per SM).  Its row tiles are shared by its warps: with T
// tiles and NW warps, KW = NW/T warps split the columns of each tile and add
// their partial sums in warp order through shared memory; with more tiles
// than warps each warp walks whole tiles.  Weights stream straight from HBM
// into registers through a software prefetch ring about 16 words deep per
// lane (no L1 allocation).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "matrix_kernels.cuh"

namespace qmr {

constexpr int kMmaWarps = 16;  // warps per CTA

// Columns each of the 4 lanes of a quad contributes to one group.
template <int G>
__host__ __device__ constexpr int cols_per_lane() {
    return G / 4;
}

// Words of one row a lane loads per group.
template <int BITS, int G>
__host__ __device__ constexpr int words_per_lane() {
    return cols_per_lane<G>() * BITS / 32;
}

// Column (relative to the lane's first column of the group) that feeds half
// `h` (0/1) of A/B register `reg` of the lane.  Register 2j+i (i = 0, 1) is
// used by MMA j as its k-slot pair (2t, 2t+1) for i = 0 and (2t+8, 2t+9) for
// i = 1.  Q4: register m of word w holds nibbles (m, m+4) of that word; Q8:
// register 2w+m holds bytes (m, m+2) of word w.
template <int BITS>
__host__ __device__ constexpr int block_perm(int reg, int h) {
    if (BITS == 4) {
        const int w = reg / 4, m = reg % 4;
        return 8 * w + m + 4 * h;
    } else {
        const int w = reg / 2, m = reg % 2;
        return 4 * w + m + 2 * h;
    }
}

// Prepared activations for the MMA path, per RHS-part n = 2b + {0: high, 1: low}:
//   xh [ngroups][8 n][4 lanes][G/4 halves]   (permuted by block_perm)
//   xs [B][ngroups] f32                       (sum of x over the group) * 2^(E_b - 24)
//   cf [B][2] f32                             2^a, 2^(24 - E_b - a)
struct MmaPrepView {
    __half *xh;
    float *xs;
    float *cf;
};

// One CTA per RHS: E_b from max|x|, then the split activations.
template <int BITS, int G>
__global__ void __launch_bounds__(512) mma_prep_kernel(const float *__restrict__ x, int cols, int batch,
                                                      MmaPrepView v) {
    asm volatile("griddepcontrol.launch_dependents;");
    constexpr int CPL = cols_per_lane<G>();
    const int b = blockIdx.x;
    const float *xb = x + (size_t)b * cols;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int ngroups = cols / G;
    __shared__ float wmax[32];
    __shared__ int s_e;
    float mx = 0.0f;
    bool nonfinite = false;
    for (int i = tid; i < cols; i += blockDim.x) {
        const float a = fabsf(xb[i]);
        nonfinite |= !(a <= 3.402823466e38f);
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
        if (e < -127) e = -127;
        s_e = e;
    }
    __syncthreads();
    const int E = 14 - s_e;  // max|x| * 2^E < 2^15 (fp16 max 65504)
    if (tid == 0) {
        const int t = 24 - E;
        const int a = t > 120 ? 120 : (t < -120 ? -120 : t);
        v.cf[2 * b] = ldexpf(1.0f, a);
        v.cf[2 * b + 1] = ldexpf(1.0f, t - a);
    }
    // Group sums: one warp per group, fixed order (strided lane sums, butterfly).
    for (int g = warp; g < ngroups; g += nw) {
        float s = 0.0f;
        for (int c = lane; c < G; c += 32) s = __fadd_rn(s, xb[(size_t)g * G + c]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (lane == 0) v.xs[(size_t)b * ngroups + g] = ldexpf(s, E - 24);
    }
    // Split halves: element (group g, lane-quad slot t, register r, half h).
    const int per_group = 4 * CPL;  // = G
    for (int i = tid; i < ngroups * per_group; i += blockDim.x) {
        const int g = i / per_group;
        const int rem = i % per_group;
        const int t = rem / CPL;
        const int slot = rem % CPL;  // = 2*reg + h
        const int reg = slot >> 1, h = slot & 1;
        const int col = g * G + t * CPL + block_perm<BITS>(reg, h);
        const float xv = ldexpf(xb[col], E);
        const __half hi = __float2half_rn(xv);
        const __half lo = __float2half_rn(xv - __half2float(hi));
        __half *base = v.xh + (((size_t)g * 8) * 4 + t) * CPL + slot;
        base[(size_t)(2 * b) * 4 * CPL] = hi;
        base[(size_t)(2 * b + 1) * 4 * CPL] = lo;
    }
}

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int N>
__device__ __forceinline__ void ldg_words(uint32_t (&v)[N], const uint32_t *p) {
    if constexpr (N == 1) {
        asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v[0]) : "l"(p));
    } else if constexpr (N == 2) {
        asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v[0]), "=r"(v[1]) : "l"(p));
    } else {
#pragma unroll
        for (int i = 0; i < N; i += 4)
            asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(v[i]), "=r"(v[i + 1]), "=r"(v[i + 2]), "=r"(v[i + 3])
                         : "l"(p + i));
    }
}

// A register `reg` of a lane from its words of one row.
template <int BITS>
__device__ __forceinline__ uint32_t a_reg(const uint32_t *words, int reg) {
    if constexpr (BITS == 4) {
        const uint32_t w = words[reg / 4];
        return (w >> (4 * (reg % 4))) & 0x000f000fu;
    } else {
        const uint32_t w = words[reg / 2];
        return (w >> (8 * (reg % 2))) & 0x00ff00ffu;
    }
}

struct MmaArgs {
    const uint32_t *w, *w2;   // packed rows (gate/up for EPI 1)
    const void *s, *b, *s2, *b2;
    const __half *xh;
    const float *xs, *cf;
    float *y;
    unsigned long long *keys;
    unsigned int *done;
    int *argmax;
    unsigned long long *best_key_out;
    int rows, cols, ystride, row_base, ranges;
};

template <int BITS, int G, int B, bool BF16, int EPI>
__global__ void __launch_bounds__(32 * kMmaWarps, 1) mma_kernel(const MmaArgs a) {
    constexpr int NM = (EPI == 1) ? 2 : 1;
    constexpr int CPL = cols_per_lane<G>();
    constexpr int WPL = words_per_lane<BITS, G>();
    constexpr int NMMA = G / 16;
    // Groups in flight per lane: about 16 words per lane whatever the format.
    constexpr int PF = (16 / (WPL * NM)) < 2 ? 2 : 16 / (WPL * NM);
    __shared__ float red[kMmaWarps][NM][2][B][32];  // per-warp partial sums
    __shared__ unsigned int flag;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int gq = lane >> 2;  // row within the 8-row half tile
    const int t = lane & 3;    // lane within the quad
    const int ngroups = a.cols / G;
    const size_t row_words = (size_t)a.cols * BITS / 32;
    const size_t row_groups = (size_t)ngroups;

    const int units = (a.rows + 15) / 16;
    const int row_begin = (int)(((long long)blockIdx.x * units) / a.ranges) * 16;
    const int row_end = min(a.rows, (int)(((long long)(blockIdx.x + 1) * units) / a.ranges) * 16);
    const int ntiles = row_end > row_begin ? (row_end - row_begin + 15) / 16 : 0;
    // Warps per tile (column split) when tiles are few; otherwise warps walk tiles.
    const int kw = ntiles > 0 && ntiles < kMmaWarps ? kMmaWarps / ntiles : 1;
    const int my_tile0 = warp / kw;
    const int part = warp % kw;
    const int tile_step = ntiles >= kMmaWarps ? kMmaWarps : ntiles;  // loop stride over tiles
    const int g_begin = (part * ngroups) / kw;
    const int g_end = ((part + 1) * ngroups) / kw;
    const int ng = g_end - g_begin;

    // The weights do not depend on the preceding (prep) kernel, so each warp
    // issues its first weight loads before waiting for the activations.
    bool waited = false;

    unsigned long long best[B];
#pragma unroll
    for (int bb = 0; bb < B; ++bb) best[bb] = 0ull;

    // Tiles this warp works on: my_tile0, my_tile0 + tile_step, ... (only
    // my_tile0 when kw > 1).  All warps run the same number of rounds so the
    // block-wide reductions line up.
    const int rounds = ntiles > 0 ? (kw > 1 ? 1 : (ntiles + kMmaWarps - 1) / kMmaWarps) : 0;
    for (int round = 0; round < rounds; ++round) {
        const int tile = my_tile0 + round * tile_step;
        const bool active = tile < ntiles && my_tile0 < ntiles && (kw == 1 || warp < ntiles * kw);
        const int r0 = row_begin + tile * 16;
        const int rowA = r0 + gq, rowB = r0 + gq + 8;
        const bool okA = active && rowA < row_end, okB = active && rowB < row_end;
        float acc[NM][2];
#pragma unroll
        for (int q = 0; q < NM; ++q) acc[q][0] = acc[q][1] = 0.0f;

        if (active && ng > 0) {
            // Base pointers of this lane's words for rows A and B of each matrix.
            const uint32_t *wp[NM][2];
#pragma unroll
            for (int q = 0; q < NM; ++q) {
                const uint32_t *W = q ? a.w2 : a.w;
                wp[q][0] = W + (size_t)(okA ? rowA : r0) * row_words + (size_t)g_begin * (G * BITS / 32) + t * WPL;
                wp[q][1] = W + (size_t)(okB ? rowB : r0) * row_words + (size_t)g_begin * (G * BITS / 32) + t * WPL;
            }
            uint32_t ring[PF][NM][2][WPL];
#pragma unroll
            for (int s = 0; s < PF; ++s) {
                if (s < ng) {
#pragma unroll
                    for (int q = 0; q < NM; ++q)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            ldg_words<WPL>(ring[s][q][h], wp[q][h] + (size_t)s * (G * BITS / 32));
                }
            }
            if (!waited) {
                asm volatile("griddepcontrol.wait;" ::: "memory");
                waited = true;
            }
            const __half *xg = a.xh + ((size_t)g_begin * 8 + gq) * 4 * CPL + (size_t)t * CPL;
            for (int i0 = 0; i0 < ng; i0 += PF) {
#pragma unroll
                for (int s = 0; s < PF; ++s) {
                    const int i = i0 + s;
                    if (i < ng) {
                        const int grp = g_begin + i;
                        // Activation fragments for this lane's RHS-part column gq.
                        uint32_t xb[CPL / 2];
                        const uint4 *xp4 = reinterpret_cast<const uint4 *>(xg + (size_t)i * 8 * 4 * CPL);
#pragma unroll
                        for (int k = 0; k < CPL / 8; ++k) {
                            const uint4 v = __ldcg(xp4 + k);
                            xb[4 * k] = v.x;
                            xb[4 * k + 1] = v.y;
                            xb[4 * k + 2] = v.z;
                            xb[4 * k + 3] = v.w;
                        }
                        const float xsv = t < B ? __ldcg(a.xs + (size_t)t * row_groups + grp) : 0.0f;
#pragma unroll
                        for (int q = 0; q < NM; ++q) {
                            const void *Sx = q ? a.s2 : a.s;
                            const void *Bx = q ? a.b2 : a.b;
                            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                            for (int j = 0; j < NMMA; ++j) {
                                uint32_t af[4];
                                af[0] = a_reg<BITS>(ring[s][q][0], 2 * j);
                                af[1] = a_reg<BITS>(ring[s][q][1], 2 * j);
                                af[2] = a_reg<BITS>(ring[s][q][0], 2 * j + 1);
                                af[3] = a_reg<BITS>(ring[s][q][1], 2 * j + 1);
                                mma_16816(d, af, xb[2 * j], xb[2 * j + 1]);
                            }
                            // d: (row A, part hi/lo of RHS t), (row B, ...).
                            const float pA = __fadd_rn(d[0], d[1]);
                            const float pB = __fadd_rn(d[2], d[3]);
                            const size_t giA = (size_t)(okA ? rowA : r0) * row_groups + grp;
                            const size_t giB = (size_t)(okB ? rowB : r0) * row_groups + grp;
                            acc[q][0] = __fmaf_rn(load_meta<BF16>(Sx, giA), pA, acc[q][0]);
                            acc[q][0] = __fmaf_rn(load_meta<BF16>(Bx, giA), xsv, acc[q][0]);
                            acc[q][1] = __fmaf_rn(load_meta<BF16>(Sx, giB), pB, acc[q][1]);
                            acc[q][1] = __fmaf_rn(load_meta<BF16>(Bx, giB), xsv, acc[q][1]);
                        }
                        // Refill this slot with the group PF ahead.
                        if (i + PF < ng) {
#pragma unroll
                            for (int q = 0; q < NM; ++q)
#pragma unroll
                                for (int h = 0; h < 2; ++h)
                                    ldg_words<WPL>(ring[s][q][h], wp[q][h] + (size_t)(i + PF) * (G * BITS / 32));
                        }
                    }
                }
            }
        }
        // ---- combine the column parts of the tile, in warp order ----
        if (kw > 1) {
#pragma unroll
            for (int q = 0; q < NM; ++q)
#pragma unroll
                for (int bb = 0; bb < B; ++bb) {
                    red[warp][q][0][bb][lane] = (t == bb) ? acc[q][0] : 0.0f;
                    red[warp][q][1][bb][lane] = (t == bb) ? acc[q][1] : 0.0f;
                }
            __syncthreads();
            if (part == 0 && active) {
#pragma unroll
                for (int q = 0; q < NM; ++q)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float v = 0.0f;
                        for (int p = 0; p < kw; ++p) v = __fadd_rn(v, red[warp + p][q][h][t < B ? t : 0][lane]);
                        acc[q][h] = v;
                    }
            }
            __syncthreads();
        }
        if (!waited) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            waited = true;
        }
        if (active && part == 0 && t < B) {
            const float c1 = __ldcg(a.cf + 2 * t), c2 = __ldcg(a.cf + 2 * t + 1);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = h ? rowB : rowA;
                if (row < row_end) {
                    float v = __fmul_rn(__fmul_rn(acc[0][h], c1), c2);
                    if constexpr (EPI == 1)
                        v = __fmul_rn(silu_f32(v), __fmul_rn(__fmul_rn(acc[NM - 1][h], c1), c2));
                    a.y[(size_t)t * a.ystride + row] = v;
                    if constexpr (EPI == 2) {
                        const unsigned long long key = ((unsigned long long)total_order_key(v) << 32) |
                                                       (unsigned long long)(0xffffffffu - (uint32_t)(a.row_base + row));
#pragma unroll
                        for (int bb = 0; bb < B; ++bb)
                            if (bb == t) best[bb] = key > best[bb] ? key : best[bb];
                    }
                }
            }
        }
    }

    if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");
    if constexpr (EPI == 2) {
        // Per-warp maximum per RHS, one atomic per warp, then the last CTA
        // to finish publishes the winners (fence + counter, no waiting).
#pragma unroll
        for (int bb = 0; bb < B; ++bb) {
            unsigned long long k = best[bb];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
                k = other > k ? other : k;
            }
            if (lane == 0 && k != 0ull) atomicMax(a.keys + bb, k);
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) flag = (atomicAdd(a.done, 1u) == gridDim.x - 1) ? 1u : 0u;
        __syncthreads();
        if (flag && threadIdx.x == 0) *a.done = 0u;  // ready for the next launch
        if (flag && threadIdx.x < B) {
            __threadfence();
            const unsigned long long k = atomicAdd(a.keys + threadIdx.x, 0ull);
            if (a.argmax) a.argmax[threadIdx.x] = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
            if (a.best_key_out) a.best_key_out[threadIdx.x] = k;
        }
    }
}

}  // namespace qmr
