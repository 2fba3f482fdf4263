// Warp-specialised, persistent TMA streaming kernel for the packed-affine
// block matmul (sm_100a).
//
// One CTA per SM.  Warp 0 is the producer: it moves row slices of the packed
// weights and of the scale/bias metadata from HBM into a ring of shared-memory
// stages with 1-D bulk copies (cp.async.bulk, TMA; no multicast), completion
// tracked by an mbarrier per stage.  Warps 1..NC are consumers: each owns R
// rows of the current row tile, dequantises from shared memory and
// accumulates against the prepared activations (prep_kernel, read through
// L1).  Memory parallelism comes from the ring (tens of KB per SM in flight,
// independent of registers), not from occupancy.
//
// Work split: CTA c owns the contiguous rows [c*rows/G, (c+1)*rows/G), so
// every CTA streams the same number of bytes; rows are taken TR = NC*R at a
// time, and each tile in slices of SC 16-byte chunks per row.
//
// Arithmetic is identical to stream_kernel (matrix_kernels.cuh): the same
// chunk partials, the same fold, the same butterfly reduction, so both paths
// give the same bits.
//
// Every wait is bounded: on timeout the kernel records an error code in
// g_qmr_device_error, stops issuing copies, waits (bounded) for the copies it
// already issued and returns.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "matrix_kernels.cuh"

namespace qmr {

// Error word written by a kernel whose bounded wait ran out (0 = none).
__device__ unsigned int g_qmr_device_error = 0;

constexpr unsigned int kErrTimeoutFull = 1u;
constexpr unsigned int kErrTimeoutEmpty = 2u;
constexpr unsigned int kErrTimeoutDrain = 3u;
// ~2^27 polls of try_wait (each may suspend briefly): seconds, far beyond any
// legitimate wait of these kernels.
constexpr uint32_t kSpinLimit = 1u << 27;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

struct TmaArgs {
    const uint8_t *w;    // packed weights (gate for EPI 1)
    const uint8_t *s;    // scales
    const uint8_t *b;    // biases
    const uint8_t *w2;   // up projection (EPI 1)
    const uint8_t *s2;
    const uint8_t *b2;
    const float4 *xp;
    const float4 *xs;
    float *y;
    unsigned long long *keys;
    unsigned int *counter;
    int *argmax;
    unsigned long long *best_key_out;
    int rows;
    int nchunks;       // 16-byte chunks per row
    int group_shift;   // log2(chunks per group)
    int meta_bytes;    // 2 (bf16) or 4 (f32) per group value
    int ystride;
    int row_base;
    int slice_chunks;  // SC: chunks per row per stage
    int stages;        // S
};

// Shared-memory layout of one stage for NM matrices and TR rows:
//   [NM][TR][SC] uint4 weights, then [NM][2][TR][SCg*meta] metadata bytes.
struct StageLayout {
    uint32_t w_bytes;     // per matrix per row
    uint32_t m_bytes;     // per matrix per row per array (scales or biases)
    uint32_t stage_bytes;
};

__host__ __device__ inline StageLayout stage_layout(int nm, int tr, int sc, int group_shift, int meta_bytes) {
    StageLayout L;
    L.w_bytes = (uint32_t)sc * 16u;
    L.m_bytes = (uint32_t)(sc >> group_shift) * (uint32_t)meta_bytes;
    L.stage_bytes = (uint32_t)nm * (uint32_t)tr * (L.w_bytes + 2u * L.m_bytes);
    L.stage_bytes = (L.stage_bytes + 127u) & ~127u;
    return L;
}

template <bool BF16>
__device__ __forceinline__ float smem_meta(const uint8_t *base, int i) {
    if constexpr (BF16) {
        return bf16_bits_to_f32(reinterpret_cast<const unsigned short *>(base)[i]);
    } else {
        return reinterpret_cast<const float *>(base)[i];
    }
}

template <int BITS, int B, int R, int NC, bool BF16, int EPI>
__global__ void __launch_bounds__(32 * (NC + 1), 1) tma_stream_kernel(const TmaArgs a) {
    constexpr int XW = Chunk<BITS>::per_word / 2;
    constexpr int NM = (EPI == 1) ? 2 : 1;
    constexpr int TR = NC * R;
    extern __shared__ __align__(128) uint8_t smem[];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int SC = a.slice_chunks;
    const int S = a.stages;
    const StageLayout L = stage_layout(NM, TR, SC, a.group_shift, a.meta_bytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * L.stage_bytes);
    uint64_t *empty = full + S;

    // Rows of this CTA: an equal share of all rows.
    const int G = gridDim.x;
    const int row_begin = (int)(((long long)blockIdx.x * a.rows) / G);
    const int row_end = (int)(((long long)(blockIdx.x + 1) * a.rows) / G);
    const int nslices = (a.nchunks + SC - 1) / SC;
    const int ntiles = (row_end - row_begin + TR - 1) / TR;
    const int nsteps = ntiles * nslices;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NC);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        // ---------------- producer ----------------
        const uint64_t pol = evict_first_policy();
        const size_t row_w = (size_t)a.nchunks * 16u;
        const size_t row_m = (size_t)(a.nchunks >> a.group_shift) * (size_t)a.meta_bytes;
        bool ok = true;
        int issued = 0;
        for (int step = 0; step < nsteps && ok; ++step) {
            const int stage = step % S;
            const int round = step / S;
            if (round > 0) {
                // Wait until every consumer released this stage (phase round-1).
                if (!mbar_wait(&empty[stage], (uint32_t)((round - 1) & 1))) {
                    ok = false;
                    if (lane == 0) atomicCAS(&g_qmr_device_error, 0u, kErrTimeoutEmpty);
                    break;
                }
            }
            const int tile = step / nslices;
            const int slice = step % nslices;
            const int r0 = row_begin + tile * TR;
            const int nr = min(TR, row_end - r0);
            const int c0 = slice * SC;
            const int sc = min(SC, a.nchunks - c0);
            const uint32_t wb = (uint32_t)sc * 16u;
            const uint32_t mb = (uint32_t)(sc >> a.group_shift) * (uint32_t)a.meta_bytes;
            uint8_t *st = smem + (size_t)stage * L.stage_bytes;
            if (lane == 0) mbar_arrive_expect_tx(&full[stage], (uint32_t)(NM * nr) * (wb + 2u * mb));
            __syncwarp();
            for (int r = lane; r < nr; r += 32) {
                const size_t row = (size_t)(r0 + r);
#pragma unroll
                for (int q = 0; q < NM; ++q) {
                    const uint8_t *W = q ? a.w2 : a.w;
                    const uint8_t *Sx = q ? a.s2 : a.s;
                    const uint8_t *Bx = q ? a.b2 : a.b;
                    uint8_t *dw = st + ((size_t)q * TR + r) * L.w_bytes;
                    uint8_t *dm = st + (size_t)NM * TR * L.w_bytes + ((size_t)(q * 2) * TR + r) * L.m_bytes;
                    bulk_g2s(dw, W + row * row_w + (size_t)c0 * 16u, wb, &full[stage], pol);
                    const size_t moff = row * row_m + (size_t)(c0 >> a.group_shift) * (size_t)a.meta_bytes;
                    bulk_g2s(dm, Sx + moff, mb, &full[stage], pol);
                    bulk_g2s(dm + (size_t)TR * L.m_bytes, Bx + moff, mb, &full[stage], pol);
                }
            }
            issued = step + 1;
        }
        // Drain: wait (bounded) until every copy this warp issued has landed,
        // so that no bulk copy targets this CTA's shared memory after exit.
        const int first = issued > S ? issued - S : 0;
        for (int step = first; step < issued; ++step) {
            if (!mbar_wait(&full[step % S], (uint32_t)((step / S) & 1))) {
                if (lane == 0) atomicCAS(&g_qmr_device_error, 0u, kErrTimeoutDrain);
                break;
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int cw = warp - 1;  // consumer index
    asm volatile("griddepcontrol.wait;" ::: "memory");  // prepared activations are ready
    const int nblocks = (a.nchunks + 31) >> 5;
    float acc[NM][B][R];
#pragma unroll
    for (int q = 0; q < NM; ++q)
#pragma unroll
        for (int b = 0; b < B; ++b)
#pragma unroll
            for (int r = 0; r < R; ++r) acc[q][b][r] = 0.0f;

    for (int step = 0; step < nsteps; ++step) {
        const int stage = step % S;
        const int round = step / S;
        const int tile = step / nslices;
        const int slice = step % nslices;
        const int r0 = row_begin + tile * TR;
        const int nr = min(TR, row_end - r0);
        const int c0 = slice * SC;
        const int sc = min(SC, a.nchunks - c0);
        if (!mbar_wait(&full[stage], (uint32_t)(round & 1))) {
            // Give up on the remaining work but still reach the epilogue
            // barrier below, so the other consumers are not left waiting.
            if (lane == 0) atomicCAS(&g_qmr_device_error, 0u, kErrTimeoutFull);
            break;
        }
        const uint8_t *st = smem + (size_t)stage * L.stage_bytes;
        const int my_r0 = cw * R;  // tile-local first row
        if (my_r0 < nr) {
            for (int cl = lane; cl < sc; cl += 32) {
                const int j = c0 + cl;  // chunk index in the row
                const int gl = cl >> a.group_shift;  // slice-local group
                uint4 wv[NM][R];
                float scv[NM][R], biv[NM][R];
#pragma unroll
                for (int q = 0; q < NM; ++q) {
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int rr = my_r0 + r;
                        if (rr < nr) {
                            wv[q][r] = *reinterpret_cast<const uint4 *>(st + ((size_t)q * TR + rr) * L.w_bytes +
                                                                        (size_t)cl * 16u);
                            const uint8_t *mbase = st + (size_t)NM * TR * L.w_bytes;
                            scv[q][r] = smem_meta<BF16>(mbase + ((size_t)(q * 2) * TR + rr) * L.m_bytes, gl);
                            biv[q][r] = smem_meta<BF16>(mbase + ((size_t)(q * 2 + 1) * TR + rr) * L.m_bytes, gl);
                        } else {
                            wv[q][r] = make_uint4(0, 0, 0, 0);
                            scv[q][r] = 0.f;
                            biv[q][r] = 0.f;
                        }
                    }
                }
                float4 xsc[B];
#pragma unroll
                for (int b = 0; b < B; ++b) xsc[b] = __ldg(a.xs + (size_t)b * a.nchunks + j);
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
                            const float4 v = __ldg(a.xp + xp_index<BITS>(b, nblocks, j, m, h));
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
                            acc[q][b][r] = fold(acc[q][b][r], p[q][r][b], xsc[b], scv[q][r], biv[q][r]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);

        if (slice == nslices - 1) {
            // Tile finished: reduce across lanes and store this warp's rows.
#pragma unroll
            for (int q = 0; q < NM; ++q)
#pragma unroll
                for (int b = 0; b < B; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r) acc[q][b][r] = warp_sum(acc[q][b][r]);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = r0 + my_r0 + r;
                if (lane == r && my_r0 + r < nr) {
#pragma unroll
                    for (int b = 0; b < B; ++b) {
                        float v = acc[0][b][r];
                        if constexpr (EPI == 1) v = __fmul_rn(silu_f32(v), acc[NM - 1][b][r]);
                        a.y[(size_t)b * a.ystride + row] = v;
                    }
                }
            }
            if constexpr (EPI == 2) {
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    unsigned long long best = 0ull;
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        if (my_r0 + r < nr) {
                            const unsigned long long key =
                                ((unsigned long long)total_order_key(acc[0][b][r]) << 32) |
                                (unsigned long long)(0xffffffffu - (uint32_t)(a.row_base + r0 + my_r0 + r));
                            best = key > best ? key : best;
                        }
                    }
                    if (lane == 0 && my_r0 < nr) atomicMax(a.keys + b, best);
                }
            }
#pragma unroll
            for (int q = 0; q < NM; ++q)
#pragma unroll
                for (int b = 0; b < B; ++b)
#pragma unroll
                    for (int r = 0; r < R; ++r) acc[q][b][r] = 0.0f;
        }
    }

    if constexpr (EPI == 2) {
        // Consumers of the last CTA to finish publish the winners.
        __shared__ unsigned int last_cta;
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"r"(32 * NC) : "memory");
        if (cw == 0 && lane == 0) last_cta = (atomicAdd(a.counter, 1u) == gridDim.x - 1) ? 1u : 0u;
        asm volatile("bar.sync 1, %0;" ::"r"(32 * NC) : "memory");
        if (last_cta && cw == 0 && lane < B) {
            __threadfence();
            const unsigned long long k = atomicAdd(a.keys + lane, 0ull);
            if (a.argmax) a.argmax[lane] = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
            if (a.best_key_out) a.best_key_out[lane] = k;
        }
    }
}

}  // namespace qmr
