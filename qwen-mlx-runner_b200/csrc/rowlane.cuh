// Persistent, warp-specialised TMA kernel for the packed-affine block matmul
// on sm_100a, "row-lane" layout.
//
// Grid: `ranges` row ranges x `ksplit` column parts, one CTA per SM.  Warp 0
// produces, warps 1..NC consume.
//
//  * Producer: for every stage (TR = 32*R rows x SC 16-byte chunks) it issues
//    1-D bulk copies (cp.async.bulk, TMA; no multicast) of each row's weight
//    slice and scale/bias slices, plus the matching prepared-activation slice
//    and chunk sums of every RHS, all completing on the stage's mbarrier.
//    Weight rows land with a 16-byte pad so row-strided reads are free of
//    bank conflicts.
//  * Consumers: lane l owns rows l, l+32, ... (R of them) of the tile; warp w
//    owns chunks [w*CPW, (w+1)*CPW) of every stage.  The prepared activations
//    of a chunk are the same for all lanes, so they are read as shared-memory
//    broadcasts and reused for R rows from registers.
//  * Reduction: per-warp partial sums meet in shared memory and are added in
//    warp order; with ksplit > 1 the CTAs of a row range write partial sums
//    and the last one to finish (fence + counter, no waiting) adds the parts
//    in part order.  Every output's arithmetic order is fixed, independent of
//    the block width B, of R and of the epilogue, so a block of B RHS equals
//    B GEMVs bit for bit.
//  * Every mbarrier wait is bounded; on timeout the kernel records an error
//    code in g_qmr_device_error and finishes without waiting further, after
//    the producer has drained the copies it issued (bounded too).
//
// Arithmetic (see matrix_kernels.cuh): masked nibbles/bytes read as exact
// subnormals times activations pre-scaled by 2^(E_b - f(k)) give
// q*x*2^(E_b-149) per product; a chunk partial p (two halves, even/odd
// elements) is folded as acc += s*p, acc.x += b*xsum', with xsum' the chunk
// sum scaled by 2^(E_b-149); the output is (acc.x+acc.y) * 2^(149-E_b).
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
// A wait gives up after this many nanoseconds of the global timer: far beyond
// any legitimate wait of these kernels (microseconds), far below a hang.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

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

// Wait for the phase with the given parity, bounded by kWaitLimitNs of
// wall-clock time; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long start = global_ns();
    for (;;) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - start > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ uint64_t evict_normal_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ void consumer_sync(int nthreads) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

struct RowlaneArgs {
    const uint8_t *w, *s, *b;     // matrix (gate for EPI 1)
    const uint8_t *w2, *s2, *b2;  // up projection (EPI 1)
    const float *xp;              // prepared activations [B][K]
    const float *xs;              // scaled chunk sums [B][nchunks]
    const float *cf;              // output factors [B][2]
    float *y;
    float *partial;               // [ksplit][NM][B][rows] when ksplit > 1
    unsigned int *range_counter;  // [ranges] arrivals of the parts of a range
    unsigned int *done_counter;   // CTAs finished (EPI 2)
    unsigned long long *keys;     // [B] packed argmax (EPI 2)
    int *argmax;
    unsigned long long *best_key_out;
    int rows, nchunks, group_shift, meta_bytes;
    int ystride, row_base;
    int ranges, ksplit;
    int slice_chunks;             // SC
    int stages;                   // S
};

// Shared-memory layout of one stage.
struct RowlaneLayout {
    uint32_t wpitch, mpitch;        // bytes per row of weights / of one metadata array
    uint32_t w_off, m_off, x_off, xs_off, stage_bytes;
};

__host__ __device__ inline RowlaneLayout rowlane_layout(int nm, int tr, int sc, int ce, int batch, int group_shift,
                                                        int meta_bytes) {
    RowlaneLayout L;
    L.wpitch = (uint32_t)sc * 16u + 16u;
    L.mpitch = (uint32_t)(sc >> group_shift) * (uint32_t)meta_bytes;
    L.w_off = 0;
    L.m_off = L.w_off + (uint32_t)nm * tr * L.wpitch;
    L.x_off = L.m_off + (uint32_t)nm * 2u * tr * L.mpitch;
    L.xs_off = L.x_off + (uint32_t)batch * sc * ce * 4u;
    L.stage_bytes = L.xs_off + (uint32_t)batch * sc * 4u;
    L.stage_bytes = (L.stage_bytes + 127u) & ~127u;
    return L;
}

template <int BITS, int B, int R, int NC, bool BF16, int EPI>
__global__ void __launch_bounds__(32 * (NC + 1), 1) rowlane_kernel(const RowlaneArgs a) {
    constexpr int XW = Chunk<BITS>::per_word / 2;  // float2 pairs per word
    constexpr int CE = Chunk<BITS>::elems;          // elements per chunk
    constexpr int NM = (EPI == 1) ? 2 : 1;
    constexpr int TR = 32 * R;
    constexpr int NCT = 32 * NC;                    // consumer threads
    extern __shared__ __align__(128) uint8_t smem[];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int SC = a.slice_chunks;
    const int S = a.stages;
    const RowlaneLayout L = rowlane_layout(NM, TR, SC, CE, B, a.group_shift, a.meta_bytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * L.stage_bytes);
    uint64_t *empty = full + S;
    // Cross-warp reduction area [NC][NM][B][R][32] floats, after the barriers.
    float *red = reinterpret_cast<float *>(empty + S);
    __shared__ unsigned int flag;

    const int range = blockIdx.x / a.ksplit;
    const int part = blockIdx.x % a.ksplit;
    const int row_begin = (int)(((long long)range * a.rows) / a.ranges);
    const int row_end = (int)(((long long)(range + 1) * a.rows) / a.ranges);
    const int nslices_all = (a.nchunks + SC - 1) / SC;
    const int s_begin = (part * nslices_all) / a.ksplit;
    const int s_end = ((part + 1) * nslices_all) / a.ksplit;
    const int nslices = s_end - s_begin;
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
        // ------------------------------ producer ------------------------------
        const uint64_t pol_w = evict_first_policy();
        const uint64_t pol_m = evict_normal_policy();
        const size_t row_w = (size_t)a.nchunks * 16u;
        const size_t row_m = (size_t)(a.nchunks >> a.group_shift) * (size_t)a.meta_bytes;
        const size_t kfloats = (size_t)a.nchunks * CE;
        // With programmatic dependent launch behind the prep kernel, weights and
        // metadata (which that kernel does not write) are copied for the first
        // round of stages before griddepcontrol.wait; the activation slices it
        // produces only after.  Launched without that attribute, the wait
        // returns at once and the order is immaterial.
        auto issue_weights = [&](int step) {
            const int stage = step % S;
            const int tile = step / nslices;
            const int slice = s_begin + step % nslices;
            const int r0 = row_begin + tile * TR;
            const int nr = min(TR, row_end - r0);
            const int c0 = slice * SC;
            const int sc = min(SC, a.nchunks - c0);
            const uint32_t wb = (uint32_t)sc * 16u;
            const uint32_t mb = (uint32_t)(sc >> a.group_shift) * (uint32_t)a.meta_bytes;
            const uint32_t xb = (uint32_t)sc * CE * 4u;
            const uint32_t xsb = (uint32_t)sc * 4u;
            uint8_t *st = smem + (size_t)stage * L.stage_bytes;
            if (lane == 0)
                mbar_arrive_expect_tx(&full[stage], (uint32_t)(NM * nr) * (wb + 2u * mb) + (uint32_t)B * (xb + xsb));
            __syncwarp();
            for (int r = lane; r < nr; r += 32) {
                const size_t row = (size_t)(r0 + r);
                const size_t moff = row * row_m + (size_t)(c0 >> a.group_shift) * (size_t)a.meta_bytes;
#pragma unroll
                for (int q = 0; q < NM; ++q) {
                    const uint8_t *W = q ? a.w2 : a.w;
                    const uint8_t *Sx = q ? a.s2 : a.s;
                    const uint8_t *Bx = q ? a.b2 : a.b;
                    bulk_g2s(st + L.w_off + ((size_t)q * TR + r) * L.wpitch, W + row * row_w + (size_t)c0 * 16u, wb,
                             &full[stage], pol_w);
                    bulk_g2s(st + L.m_off + ((size_t)(2 * q) * TR + r) * L.mpitch, Sx + moff, mb, &full[stage], pol_m);
                    bulk_g2s(st + L.m_off + ((size_t)(2 * q + 1) * TR + r) * L.mpitch, Bx + moff, mb, &full[stage],
                             pol_m);
                }
            }
        };
        auto issue_acts = [&](int step) {
            const int stage = step % S;
            const int slice = s_begin + step % nslices;
            const int c0 = slice * SC;
            const int sc = min(SC, a.nchunks - c0);
            uint8_t *st = smem + (size_t)stage * L.stage_bytes;
            if (lane < B) {
                bulk_g2s(st + L.x_off + (size_t)lane * SC * CE * 4u, a.xp + (size_t)lane * kfloats + (size_t)c0 * CE,
                         (uint32_t)sc * CE * 4u, &full[stage], pol_m);
                bulk_g2s(st + L.xs_off + (size_t)lane * SC * 4u, a.xs + (size_t)lane * a.nchunks + c0,
                         (uint32_t)sc * 4u, &full[stage], pol_m);
            }
        };
        const int first = nsteps < S ? nsteps : S;
        for (int step = 0; step < first; ++step) issue_weights(step);
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int step = 0; step < first; ++step) issue_acts(step);
        int issued = first;
        for (int step = first; step < nsteps; ++step) {
            const int stage = step % S;
            const int round = step / S;
            if (!mbar_wait(&empty[stage], (uint32_t)((round - 1) & 1))) {
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
    const int cpw = SC / NC;  // chunks per warp per stage
    asm volatile("griddepcontrol.wait;" ::: "memory");
    bool alive = true;
    int step = 0;
    for (int tile = 0; tile < ntiles; ++tile) {
        const int r0 = row_begin + tile * TR;
        const int nr = min(TR, row_end - r0);
        float2 acc[NM][R][B];
#pragma unroll
        for (int q = 0; q < NM; ++q)
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < B; ++b) acc[q][r][b] = make_float2(0.f, 0.f);

        for (int si = 0; si < nslices && alive; ++si, ++step) {
            const int stage = step % S;
            const int slice = s_begin + si;
            const int sc = min(SC, a.nchunks - slice * SC);
            if (!mbar_wait(&full[stage], (uint32_t)((step / S) & 1))) {
                if (lane == 0) atomicCAS(&g_qmr_device_error, 0u, kErrTimeoutFull);
                alive = false;
                break;
            }
            const uint8_t *st = smem + (size_t)stage * L.stage_bytes;
            for (int cc = 0; cc < cpw; ++cc) {
                const int c = cw * cpw + cc;  // stage-local chunk, warp-uniform
                if (c >= sc) break;
                const int g = c >> a.group_shift;
                float xsv[B];
#pragma unroll
                for (int b = 0; b < B; ++b)
                    xsv[b] = reinterpret_cast<const float *>(st + L.xs_off)[(size_t)b * SC + c];
                uint4 wv[NM][R];
                float sv[NM][R], bv[NM][R];
#pragma unroll
                for (int q = 0; q < NM; ++q) {
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int rr = lane + 32 * r;
                        if (rr < nr) {
                            wv[q][r] = *reinterpret_cast<const uint4 *>(st + L.w_off + ((size_t)q * TR + rr) * L.wpitch +
                                                                        (size_t)c * 16u);
                            sv[q][r] = smem_meta<BF16>(st + L.m_off + ((size_t)(2 * q) * TR + rr) * L.mpitch, g);
                            bv[q][r] = smem_meta<BF16>(st + L.m_off + ((size_t)(2 * q + 1) * TR + rr) * L.mpitch, g);
                        } else {
                            wv[q][r] = make_uint4(0, 0, 0, 0);
                            sv[q][r] = 0.f;
                            bv[q][r] = 0.f;
                        }
                    }
                }
                float2 p[NM][R][B];
#pragma unroll
                for (int q = 0; q < NM; ++q)
#pragma unroll
                    for (int r = 0; r < R; ++r)
#pragma unroll
                        for (int b = 0; b < B; ++b) p[q][r][b] = make_float2(0.f, 0.f);
                const float4 *xrow = reinterpret_cast<const float4 *>(st + L.x_off) + (size_t)c * (CE / 4);
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    float2 xv[B][XW];
#pragma unroll
                    for (int b = 0; b < B; ++b) {
#pragma unroll
                        for (int h = 0; h < XW / 2; ++h) {
                            const float4 v = xrow[(size_t)b * SC * (CE / 4) + m * (XW / 2) + h];
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
                        const float2 ss = make_float2(sv[q][r], sv[q][r]);
#pragma unroll
                        for (int b = 0; b < B; ++b) {
                            acc[q][r][b] = ffma2(ss, p[q][r][b], acc[q][r][b]);
                            acc[q][r][b].x = __fmaf_rn(bv[q][r], xsv[b], acc[q][r][b].x);
                        }
                    }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
        }

        // ---- reduce this tile: warps in order, then parts in order ----
#pragma unroll
        for (int q = 0; q < NM; ++q)
#pragma unroll
            for (int b = 0; b < B; ++b)
#pragma unroll
                for (int r = 0; r < R; ++r)
                    red[((((size_t)cw * NM + q) * B + b) * R + r) * 32 + lane] = __fadd_rn(acc[q][r][b].x, acc[q][r][b].y);
        consumer_sync(NCT);
        constexpr int NOUT = NM * B * R * 32;  // outputs of the tile (q, b, row slot)
        for (int o = tid; o < NOUT; o += NCT) {
            float v = 0.f;
            for (int w = 0; w < NC; ++w) v = __fadd_rn(v, red[(size_t)w * NOUT + o]);
            red[(size_t)NC * NOUT + o] = v;  // tile sums after the per-warp partials
        }
        consumer_sync(NCT);
        float *sums = red + (size_t)NC * NOUT;
        bool have = true;
        if (a.ksplit > 1) {
            // Publish this part's sums; the last part of the range adds them up.
            for (int o = tid; o < NOUT; o += NCT) {
                const int slot = o % (R * 32);
                const int qb = o / (R * 32);  // q * B + b
                const int rr = (slot % 32) + 32 * (slot / 32);
                if (rr < nr)
                    a.partial[(((size_t)part * NM * B + qb) * a.rows) + r0 + rr] = sums[o];
            }
            __threadfence();
            consumer_sync(NCT);
            if (tid == 0) flag = (atomicAdd(&a.range_counter[range * 64 + tile], 1u) == (unsigned)a.ksplit - 1) ? 1u : 0u;
            consumer_sync(NCT);
            have = flag != 0;
            if (have) {
                __threadfence();
                if (tid == 0) a.range_counter[range * 64 + tile] = 0u;  // ready for the next launch
                for (int o = tid; o < NOUT; o += NCT) {
                    const int slot = o % (R * 32);
                    const int qb = o / (R * 32);
                    const int rr = (slot % 32) + 32 * (slot / 32);
                    float v = 0.f;
                    if (rr < nr)
                        for (int p = 0; p < a.ksplit; ++p)
                            v = __fadd_rn(v, __ldcg(&a.partial[(((size_t)p * NM * B + qb) * a.rows) + r0 + rr]));
                    sums[o] = v;
                }
            }
            consumer_sync(NCT);
        }
        if (have) {
            // Final scale and epilogue; thread t handles rows t, t+NCT, ... of the tile.
            unsigned long long best[B];
#pragma unroll
            for (int b = 0; b < B; ++b) best[b] = 0ull;
            for (int rr = tid; rr < nr; rr += NCT) {
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float c1 = __ldg(a.cf + 2 * b), c2 = __ldg(a.cf + 2 * b + 1);
                    float v = __fmul_rn(__fmul_rn(sums[(size_t)(0 * B + b) * R * 32 + rr], c1), c2);
                    if constexpr (EPI == 1) {
                        const float u = __fmul_rn(__fmul_rn(sums[(size_t)(1 * B + b) * R * 32 + rr], c1), c2);
                        v = __fmul_rn(silu_f32(v), u);
                    }
                    a.y[(size_t)b * a.ystride + r0 + rr] = v;
                    if constexpr (EPI == 2) {
                        const unsigned long long key =
                            ((unsigned long long)total_order_key(v) << 32) |
                            (unsigned long long)(0xffffffffu - (uint32_t)(a.row_base + r0 + rr));
                        best[b] = key > best[b] ? key : best[b];
                    }
                }
            }
            if constexpr (EPI == 2) {
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    unsigned long long k = best[b];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
                        k = other > k ? other : k;
                    }
                    if (lane == 0 && k != 0ull) atomicMax(a.keys + b, k);
                }
            }
        }
        consumer_sync(NCT);  // red[] is reused by the next tile
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
