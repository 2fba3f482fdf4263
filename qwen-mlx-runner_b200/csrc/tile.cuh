// Persistent, warp-specialised TMA kernel for the packed-affine block matmul
// on sm_100a.
//
// Grid: `ranges` row ranges x `ksplit` column parts, one CTA per SM.  Warp 0
// produces, warps 1..NC consume.  A stage covers one K-slice of SC = 32
// 16-byte chunks (512 bytes of every weight row):
//
//  * Producer: per consumer warp one 2-D tensor copy (cp.async.bulk.tensor,
//    TMA, no multicast) of its RW rows x 512 bytes of packed weights; one 2-D
//    tensor copy each of the tile's scales and biases for the slice; one 1-D
//    bulk copy per RHS of the slice's prepared activations (pre-scaled values
//    in lane-interleaved order, then the 32 chunk sums).  All complete on the
//    stage's mbarrier.  Out-of-range rows and columns are zero-filled by TMA.
//  * Consumers: warp w owns rows [w*RW, (w+1)*RW) of the CTA's current row
//    tile for the whole K range; lane c owns chunk c of every slice.  Weight
//    rows and activation blocks are read from shared memory with
//    conflict-free 16-byte loads; each activation value is reused for RW rows
//    from registers.
//  * Per output: lane partials accumulate over the slices in order, then a
//    fixed butterfly adds the 32 lanes; with ksplit > 1 the CTAs of a row
//    range publish partial sums and the last one to finish (fence + counter,
//    no waiting) adds them in part order.  The order does not depend on the
//    block width B, so a block of B RHS equals B GEMVs bit for bit.
//  * Every mbarrier wait is bounded by %globaltimer; on timeout the kernel
//    records an error code in g_qmr_device_error, and the producer drains the
//    copies it issued (also bounded) before the CTA exits.
//
// Arithmetic (matrix_kernels.cuh): masked nibbles/bytes read as exact
// subnormals times activations pre-scaled by 2^(E_b - f(k)) accumulate
// q*x*2^(E_b-149); a chunk partial p (even/odd halves) is folded as
// acc += s*p, acc.x += bias*xsum', and the output is (acc.x+acc.y) summed
// over lanes times 2^(149-E_b).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "matrix_kernels.cuh"
#include "pipe.cuh"

namespace qmr {

// Error word written by a kernel whose bounded wait ran out (0 = none).
__device__ unsigned int g_qmr_device_error = 0;

constexpr int kSliceChunks = 32;  // SC: chunks per row per stage (512 bytes)
constexpr int kSliceWords = 128;  // the same in u32 words

__device__ __forceinline__ void consumer_sync(int nthreads) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Floats of one prepared-activation block (32 chunks) of one RHS: the
// pre-scaled values in lane-interleaved order, then the 32 chunk sums.
template <int BITS>
__host__ __device__ constexpr int block_floats() {
    return kSliceChunks * Chunk<BITS>::elems + kSliceChunks;
}

struct TileArgs {
    const float *xp;              // prepared blocks [B][nblocks][block_floats]
    const float *cf;              // output factors [B][2]
    float *y;
    float *partial;               // [ksplit][NM][B][rows] when ksplit > 1
    unsigned int *range_counter;  // [ranges][4] arrivals of the parts of a tile
    unsigned int *done_counter;   // CTAs finished (EPI 2)
    unsigned long long *keys;     // [B] packed argmax (EPI 2)
    int *argmax;
    unsigned long long *best_key_out;
    int rows, nchunks, group_shift, meta_bytes;
    int ystride, row_base;
    int ranges, ksplit;
    int stages;
};

struct TileLayout {
    uint32_t w_box;   // bytes of one weight box (RW rows x 512 bytes)
    uint32_t m_box;   // bytes of one metadata box (TR rows x slice groups)
    uint32_t x_blk;   // bytes of one RHS activation block
    uint32_t w_off, m_off, x_off, stage_bytes;
};

__host__ __device__ inline TileLayout tile_layout(int nm, int nc, int rw, int batch, int group_shift, int meta_bytes,
                                                  int block_floats_) {
    TileLayout L;
    L.w_box = (uint32_t)rw * kSliceChunks * 16u;
    L.m_box = (uint32_t)(nc * rw) * (uint32_t)(kSliceChunks >> group_shift) * (uint32_t)meta_bytes;
    L.x_blk = (uint32_t)block_floats_ * 4u;
    L.w_off = 0;
    L.m_off = L.w_off + (uint32_t)nm * nc * L.w_box;
    L.x_off = L.m_off + (uint32_t)nm * 2u * L.m_box;
    L.stage_bytes = L.x_off + (uint32_t)batch * L.x_blk;
    L.stage_bytes = (L.stage_bytes + 1023u) & ~1023u;
    return L;
}

template <int BITS, int B, int RW, int NC, bool BF16, int EPI>
__global__ void __launch_bounds__(32 * (NC + 1), 1)
    tile_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                const __grid_constant__ CUtensorMap bmap, const __grid_constant__ CUtensorMap wmap2,
                const __grid_constant__ CUtensorMap smap2, const __grid_constant__ CUtensorMap bmap2,
                const TileArgs a) {
    constexpr int XW = Chunk<BITS>::per_word / 2;  // float2 pairs per word
    constexpr int H = XW / 2;                      // float4 loads per word
    constexpr int BF = block_floats<BITS>();
    constexpr int NM = (EPI == 1) ? 2 : 1;
    constexpr int TR = NC * RW;
    constexpr int NCT = 32 * NC;
    extern __shared__ __align__(1024) uint8_t smem[];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int S = a.stages;
    const TileLayout L = tile_layout(NM, NC, RW, B, a.group_shift, a.meta_bytes, BF);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * L.stage_bytes);
    uint64_t *empty = full + S;
    __shared__ unsigned int flag;

    // Rows of this CTA: row ranges balanced in units of RW rows.
    const int range = blockIdx.x / a.ksplit;
    const int part = blockIdx.x % a.ksplit;
    const int units = (a.rows + RW - 1) / RW;
    const int row_begin = (int)(((long long)range * units) / a.ranges) * RW;
    const int row_end = min(a.rows, (int)(((long long)(range + 1) * units) / a.ranges) * RW);
    const int nslices_all = (a.nchunks + kSliceChunks - 1) / kSliceChunks;
    const int s_begin = (part * nslices_all) / a.ksplit;
    const int s_end = ((part + 1) * nslices_all) / a.ksplit;
    const int nslices = s_end - s_begin;
    const int ntiles = row_end > row_begin ? (row_end - row_begin + TR - 1) / TR : 0;
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
        // ------------------------------ producer ------------------------------
        const uint64_t pol_w = evict_first_policy();
        const uint64_t pol_m = evict_normal_policy();
        const int slice_groups = kSliceChunks >> a.group_shift;
        auto issue_weights = [&](int step) {
            const int stage = step % S;
            const int tile = step / nslices;
            const int slice = s_begin + step % nslices;
            const int r0 = row_begin + tile * TR;
            const int nbox = min(NC, (row_end - r0 + RW - 1) / RW);  // warps with rows
            uint8_t *st = smem + (size_t)stage * L.stage_bytes;
            if (lane == 0)
                mbar_arrive_expect_tx(&full[stage],
                                      (uint32_t)NM * ((uint32_t)nbox * L.w_box + 2u * L.m_box) + (uint32_t)B * L.x_blk);
            __syncwarp();
            if (lane < nbox) {
#pragma unroll
                for (int q = 0; q < NM; ++q)
                    tma_load_2d(st + L.w_off + (size_t)(q * NC + lane) * L.w_box, q ? &wmap2 : &wmap,
                                slice * kSliceWords, r0 + lane * RW, &full[stage], pol_w);
            } else if (lane >= 32 - 2 * NM) {
                const int k = lane - (32 - 2 * NM);  // 0..2*NM-1: (q, scales|biases)
                const int q = k >> 1;
                const CUtensorMap *map = (k & 1) ? (q ? &bmap2 : &bmap) : (q ? &smap2 : &smap);
                tma_load_2d(st + L.m_off + (size_t)k * L.m_box, map, slice * slice_groups, r0, &full[stage], pol_m);
            }
        };
        auto issue_acts = [&](int step) {
            const int stage = step % S;
            const int slice = s_begin + step % nslices;
            uint8_t *st = smem + (size_t)stage * L.stage_bytes;
            if (lane < B)
                bulk_g2s(st + L.x_off + (size_t)lane * L.x_blk,
                         a.xp + ((size_t)lane * nslices_all + slice) * BF, L.x_blk, &full[stage], pol_m);
        };
        // With programmatic dependent launch behind the prep kernel, weights and
        // metadata (which that kernel does not write) are requested for the
        // first round of stages before griddepcontrol.wait, the activation
        // blocks it produces only after.  Without that launch attribute the
        // wait returns at once.
        const int first = nsteps < S ? nsteps : S;
        for (int step = 0; step < first; ++step) issue_weights(step);
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int step = 0; step < first; ++step) issue_acts(step);
        int issued = first;
        for (int step = first; step < nsteps; ++step) {
            const int stage = step % S;
            if (!mbar_wait(&empty[stage], (uint32_t)((step / S - 1) & 1))) {
                if (lane == 0) atomicCAS(&g_qmr_device_error, 0u, kErrTimeoutEmpty);
                break;
            }
            issue_weights(step);
            issue_acts(step);
            issued = step + 1;
        }
        // Drain: every copy issued must have landed before this CTA exits.
        for (int step = issued > S ? issued - S : 0; step < issued; ++step) {
            if (!mbar_wait(&full[step % S], (uint32_t)((step / S) & 1))) {
                if (lane == 0) atomicCAS(&g_qmr_device_error, 0u, kErrTimeoutDrain);
                break;
            }
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    const int cw = warp - 1;
    const int tid = threadIdx.x - 32;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    bool alive = true;
    int step = 0;
    for (int tile = 0; tile < ntiles; ++tile) {
        const int r0 = row_begin + tile * TR;
        const int my_r0 = r0 + cw * RW;  // first row of this warp
        float2 acc[NM][RW][B];
#pragma unroll
        for (int q = 0; q < NM; ++q)
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int b = 0; b < B; ++b) acc[q][r][b] = make_float2(0.f, 0.f);

        for (int si = 0; si < nslices; ++si, ++step) {
            const int stage = step % S;
            if (alive && !mbar_wait(&full[stage], (uint32_t)((step / S) & 1))) {
                if (lane == 0) atomicCAS(&g_qmr_device_error, 0u, kErrTimeoutFull);
                alive = false;
            }
            if (alive && my_r0 < row_end) {
                const uint8_t *st = smem + (size_t)stage * L.stage_bytes;
                const int g = lane >> a.group_shift;
                const float *xblk = reinterpret_cast<const float *>(st + L.x_off);
                float xsv[B];
#pragma unroll
                for (int b = 0; b < B; ++b) xsv[b] = xblk[(size_t)b * BF + kSliceChunks * Chunk<BITS>::elems + lane];
                float2 p[NM][RW][B];
#pragma unroll
                for (int q = 0; q < NM; ++q)
#pragma unroll
                    for (int r = 0; r < RW; ++r)
#pragma unroll
                        for (int b = 0; b < B; ++b) p[q][r][b] = make_float2(0.f, 0.f);
                uint4 wv[NM][RW];
#pragma unroll
                for (int q = 0; q < NM; ++q)
#pragma unroll
                    for (int r = 0; r < RW; ++r)
                        wv[q][r] = *reinterpret_cast<const uint4 *>(st + L.w_off + (size_t)(q * NC + cw) * L.w_box +
                                                                    (size_t)r * (kSliceChunks * 16) + (size_t)lane * 16);
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    float2 xv[B][XW];
#pragma unroll
                    for (int b = 0; b < B; ++b) {
#pragma unroll
                        for (int h = 0; h < H; ++h) {
                            const float4 v = reinterpret_cast<const float4 *>(xblk + (size_t)b * BF)[(m * H + h) * 32 + lane];
                            xv[b][2 * h] = make_float2(v.x, v.y);
                            xv[b][2 * h + 1] = make_float2(v.z, v.w);
                        }
                    }
#pragma unroll
                    for (int q = 0; q < NM; ++q) {
#pragma unroll
                        for (int r = 0; r < RW; ++r) {
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
                for (int q = 0; q < NM; ++q) {
                    const uint8_t *ms = st + L.m_off + (size_t)(2 * q) * L.m_box;
                    const uint8_t *mb = ms + L.m_box;
                    const uint32_t mrow = (uint32_t)(kSliceChunks >> a.group_shift) * (uint32_t)a.meta_bytes;
#pragma unroll
                    for (int r = 0; r < RW; ++r) {
                        const int tr = cw * RW + r;  // tile-local row
                        const float sv = smem_meta<BF16>(ms + (size_t)tr * mrow, g);
                        const float bv = smem_meta<BF16>(mb + (size_t)tr * mrow, g);
                        const float2 ss = make_float2(sv, sv);
#pragma unroll
                        for (int b = 0; b < B; ++b) {
                            acc[q][r][b] = ffma2(ss, p[q][r][b], acc[q][r][b]);
                            acc[q][r][b].x = __fmaf_rn(bv, xsv[b], acc[q][r][b].x);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
        }

        // ---- this tile's outputs: butterfly over lanes, then parts in order ----
        float tot[NM][RW][B];
#pragma unroll
        for (int q = 0; q < NM; ++q)
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int b = 0; b < B; ++b) tot[q][r][b] = warp_sum(__fadd_rn(acc[q][r][b].x, acc[q][r][b].y));
        bool have = true;
        if (a.ksplit > 1) {
            // Publish this part's sums; the last part of the range adds them up.
            if (lane == 0) {
#pragma unroll
                for (int q = 0; q < NM; ++q)
#pragma unroll
                    for (int b = 0; b < B; ++b)
#pragma unroll
                        for (int r = 0; r < RW; ++r)
                            if (my_r0 + r < row_end)
                                a.partial[((size_t)(part * NM + q) * B + b) * a.rows + my_r0 + r] = tot[q][r][b];
            }
            __threadfence();
            consumer_sync(NCT);
            if (tid == 0)
                flag = (atomicAdd(&a.range_counter[range * 4 + tile], 1u) == (unsigned)a.ksplit - 1) ? 1u : 0u;
            consumer_sync(NCT);
            have = flag != 0;
            if (have) {
                __threadfence();
                if (tid == 0) a.range_counter[range * 4 + tile] = 0u;  // ready for the next launch
                if (lane == 0) {
#pragma unroll
                    for (int q = 0; q < NM; ++q)
#pragma unroll
                        for (int b = 0; b < B; ++b)
#pragma unroll
                            for (int r = 0; r < RW; ++r) {
                                float v = 0.f;
                                if (my_r0 + r < row_end)
                                    for (int pp = 0; pp < a.ksplit; ++pp)
                                        v = __fadd_rn(v, __ldcg(&a.partial[((size_t)(pp * NM + q) * B + b) * a.rows +
                                                                           my_r0 + r]));
                                tot[q][r][b] = v;
                            }
                }
            }
            consumer_sync(NCT);  // flag is reused by the next tile
        }
        if (have) {
            unsigned long long best[B];
#pragma unroll
            for (int b = 0; b < B; ++b) best[b] = 0ull;
            if (lane == 0) {
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float c1 = __ldcg(a.cf + 2 * b), c2 = __ldcg(a.cf + 2 * b + 1);
#pragma unroll
                    for (int r = 0; r < RW; ++r) {
                        const int row = my_r0 + r;
                        if (row < row_end) {
                            float v = __fmul_rn(__fmul_rn(tot[0][r][b], c1), c2);
                            if constexpr (EPI == 1)
                                v = __fmul_rn(silu_f32(v), __fmul_rn(__fmul_rn(tot[NM - 1][r][b], c1), c2));
                            a.y[(size_t)b * a.ystride + row] = v;
                            if constexpr (EPI == 2) {
                                const unsigned long long key =
                                    ((unsigned long long)total_order_key(v) << 32) |
                                    (unsigned long long)(0xffffffffu - (uint32_t)(a.row_base + row));
                                best[b] = key > best[b] ? key : best[b];
                            }
                        }
                    }
                    if constexpr (EPI == 2)
                        if (best[b] != 0ull) atomicMax(a.keys + b, best[b]);
                }
            }
        }
    }

    if constexpr (EPI == 2) {
        // The last CTA to finish publishes the winners (fence + counter, no waiting).
        __threadfence();
        consumer_sync(NCT);
        if (tid == 0) flag = (atomicAdd(a.done_counter, 1u) == gridDim.x - 1) ? 1u : 0u;
        consumer_sync(NCT);
        if (flag && tid == 0) *a.done_counter = 0u;  // ready for the next launch
        if (flag && tid < B) {
            __threadfence();
            const unsigned long long k = atomicAdd(a.keys + tid, 0ull);
            if (a.argmax) a.argmax[tid] = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
            if (a.best_key_out) a.best_key_out[tid] = k;
        }
    }
}

}  // namespace qmr
