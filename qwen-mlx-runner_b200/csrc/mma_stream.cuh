// Weight-streaming block matmul on the tensor cores (sm_100a: mma.sync
// m16n8k16 with f16 operands and f32 accumulation, TMA weight tiles,
// cp.async metadata, mbarrier pipelines).
//
// Why tensor cores for a batch of at most 4 right-hand sides: on B200 the FP32
// formulation needs one LOP3 plus B fused multiply-adds per weight element,
// which issue-limits a B3 block well below HBM speed.  Here one warp
// instruction multiplies 16 rows x 16 columns x 8 RHS columns, so the cost per
// element is the dequantisation alone (5 logic ops per 8 nibbles), whatever B.
//
// Operands of one 16-row x 16-column MMA:
//  * A (weights): `w & 0x000f000f` (Q4) or `w & 0x00ff00ff` (Q8) read as a
//    half2 is a pair of exact fp16 subnormals q * 2^-24.  For Q4 the nibbles
//    at bits 4..7 are used in place as `w & 0x00f000f0` = 16q * 2^-24, and
//    the activations paired with them carry a compensating 2^-4; nibbles at
//    bits 8..15 come from `w >> 8` the same way.  The k order inside an MMA
//    is a fixed permutation of the group's columns (block_perm); the
//    activation image is stored in that order.
//  * B (activations): x * 2^E_g, with one exponent per group and RHS that
//    puts the group's largest |x| just below the fp16 maximum, split into an
//    fp16 high part and an fp16 low part; the MMA columns are n = 2b + part,
//    so each thread's accumulator pair holds both parts of one RHS for two
//    rows.
//  * Per quantisation group the group's MMAs start from zero; the f32 result
//    P = (q*x summed over the group) * 2^(E_g-24) is folded as
//    acc += (s * 2^(24-E_g)) * P (both parts) and acc.hi += bias * sum(x);
//    the output is acc.hi + acc.lo.
//
// Work split: the CTAs form clusters of kc CTAs (kc = 1, 2 or 4 column
// slices).  Cluster i owns the 16-row tiles [i*T/C, (i+1)*T/C) of the matrix
// and its CTA of rank h owns the 512/1024-column windows of slice h.  A CTA's
// (tile, window) units, tile-major, are divided into equal contiguous segments,
// one per warp.  A warp accumulates each tile piece of its segment in
// registers; a piece covering a whole tile (kc = 1) is written directly, the
// others go to shared memory and are added in warp order after the loop; with
// kc > 1 the CTAs' per-tile sums are then added in rank order through
// distributed shared memory.  No partial sum leaves the chip and nothing
// waits on another CTA outside the cluster barrier.  The split depends only
// on the matrix shape and the SM count, never on B, so a block of B RHS equals
// B single-RHS calls bit for bit.
//
// Data movement per warp: a private ring of `stages` slots; slot = one unit:
// the tile's 16 rows x window bytes of packed weights as 2-D TMA boxes of
// 16 rows x 128 bytes with the 128-byte swizzle (conflict-free 8-row reads),
// completing on the slot's mbarrier, plus the tile's scales and biases for
// the window's groups by 16-byte cp.async (zero-filled out of range) in one
// commit group per unit, waited for with cp.async.wait_group and a warp
// barrier.  The CTA's activation image (its slice of the image plus the
// table of group sums) is built by the CTA itself from x in its prologue, or
// (argmax and exchange epilogues, host-resident x, the prepared-activation
// API) arrives once by bulk copy from the prep kernel's image.  Weight loads
// are issued before `griddepcontrol.wait`, so they overlap the producer of
// the activations under programmatic dependent launch.  Every wait is bounded by
// %globaltimer; on timeout the kernel records an error code and drains the
// copies it issued (also bounded) before exiting.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "matrix_kernels.cuh"
#include "pipe.cuh"

namespace qmr {

constexpr int kMmaWarps = 8;     // warps per CTA, each with its own copy ring
constexpr int kMmaWarpsLong = 12;  // warps per CTA for Q4 g32/g64 (shallower rings, more issue slots)
constexpr int kTileRows = 16;    // rows of one MMA tile
constexpr int kMaxPieces = 4;    // tile pieces one warp may leave in shared memory
constexpr int kMmaMaxStages = 6;
constexpr int kMaxRanks = 8;     // ranks of an output exchange over peer memory

template <int BITS, int G>
struct MmaShape {
    static constexpr int CPL = G / 4;                               // columns per lane per group
    static constexpr int WPL = CPL * BITS / 32;                     // words per lane per group and row
    static constexpr int NMMA = G / 16;                             // MMAs per group
    static constexpr int NREG = G / 8;                              // half2 registers per lane, row and group
    static constexpr int NCH = G / 32;                              // 16-byte activation chunks per lane and group
    static constexpr int WIN_COLS = 8 * G > 512 ? 8 * G : 512;      // columns of one window
    static constexpr int WG = WIN_COLS / G;                         // groups per window (8 or 16)
    static constexpr int ROW_BYTES = WIN_COLS * BITS / 8;           // bytes of one row in a window
    static constexpr int ROW_WORDS = ROW_BYTES / 4;
    static constexpr int NBOX = ROW_BYTES / 128;                    // 128-byte TMA boxes per window
    static constexpr int GROUP_BYTES = G * BITS / 8;
    static constexpr int W_BYTES = kTileRows * ROW_BYTES;           // weights of one unit
};

// Bytes of one ring slot: the weights of NM matrices (a multiple of 2 KiB, so
// every slot stays 1024-byte aligned for the swizzle) and, in a separate
// region, their metadata: per matrix a scale box then a bias box, each
// [16 rows][the window's groups].
__host__ __device__ constexpr int mma_slot_weight_bytes(int bits, int group, int nm) {
    return nm * kTileRows * (8 * group > 512 ? 8 * group : 512) * bits / 8;
}
__host__ __device__ constexpr int mma_slot_meta_bytes(int group, int nm, int meta_size) {
    return nm * 32 * ((8 * group > 512 ? 8 * group : 512) / group) * meta_size;
}

// Column (relative to the lane's first column of the group) that feeds half
// `h` (0/1) of A/B register `reg` of the lane.  Register 2j+i (i = 0, 1) is
// used by MMA j as its k-slot pair (2t, 2t+1) for i = 0 and (2t+8, 2t+9) for
// i = 1.  Q4: register m of word w holds nibbles (m, m+4) of that word
// (m odd: scaled by 16); Q8: register 2w+m holds bytes (m, m+2) of word w.
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

// The prepared activation image, shared by the prep kernel (writer) and the
// streaming kernel (reader, copied into shared memory verbatim):
//   image [ngroups_pad][NCH][NB = 2B][4 lanes][8 halves]  (block_perm order;
//          x * 2^E_g with the group's own exponent; Q4 odd registers scaled
//          by a further 2^-4; padding groups are zero)
//   table [4][ngroups_pad][2] f32  2^(24 - E_g), sum of x over the group
struct MmaImageView {
    __half *image;
    float *table;
    unsigned long long *keys;  // argmax keys, cleared by the prep
    unsigned int *done;        // CTA counter, cleared by the prep
    // Fused RMSNorm (optional): the image holds x * norm_w, and the prep
    // writes row_scale[b] = 1 / sqrt(mean(x_b^2) + eps), which the streaming
    // kernel multiplies into every output of RHS b.  Needs one prep CTA per
    // RHS (ngroups_pad <= kPrepGroupsPerCta).
    const float *norm_w;
    float eps;
    float *row_scale;
    // An all-reduce of partial sums folded in front of the prep (red_slots
    // null: none): wait, bounded, until every one of red_world ranks has
    // published epoch *red_epoch in red_flags, then x_new[b] = x[b] +
    // (slots[b][0] + slots[b][1] + ...) in rank order (slots
    // [batch][red_world][cols]), written to red_x (may be x itself) and used
    // by the prep in place of x.
    const float *red_slots;
    float *red_x;
    const unsigned int *red_flags;
    const unsigned int *red_epoch;
    unsigned int *red_err;
    int red_world;
};

// ---- activation image arithmetic (the prep kernel's) ----

// E from the largest |x| bit pattern of a group (>= 0x7f800000: not
// finite): max|x| * 2^E < 2^15, just below the fp16 maximum.
__device__ __forceinline__ int act_exponent(uint32_t max_abs_bits) {
    int e = max_abs_bits >= 0x7f800000u ? 128 : (int)(max_abs_bits >> 23) - 127;
    if (e < -127) e = -127;
    return 14 - e;
}

// 2^e as a float: exact for e in [-149, 127], 0 below, +inf above (the
// values ldexpf(1, e) gives).
__device__ __forceinline__ float pow2f(int e) {
    if (e > 127) return __int_as_float(0x7f800000);
    if (e >= -126) return __int_as_float((e + 127) << 23);
    if (e >= -149) return __int_as_float(1 << (e + 149));
    return 0.0f;
}

// v * 2^n: one rounding while 2^n is a normal float; beyond that (groups
// whose largest |x| is below 2^-112 or above 2^126) two power-of-two
// products, 2^(n/2) and the rest, both normal for the exponents act_exponent
// produces.  Short and branch-light: this runs once per activation in every
// CTA's prologue.
__device__ __forceinline__ float pow2_scale(float v, int n) {
    if (n >= -126 && n <= 127) return __fmul_rn(v, __int_as_float((n + 127) << 23));
    const int h = n / 2;
    return __fmul_rn(__fmul_rn(v, __int_as_float((h + 127) << 23)), __int_as_float((n - h + 127) << 23));
}

// High and low fp16 parts of (x0, x1) * 2^n as two half2 words.
__device__ __forceinline__ void act_split2(float x0, float x1, int n, uint32_t *hi2, uint32_t *lo2) {
    const float v0 = pow2_scale(x0, n), v1 = pow2_scale(x1, n);
    const __half2 h = __floats2half2_rn(v0, v1);
    const float2 back = __half22float2(h);
    const __half2 l = __floats2half2_rn(__fsub_rn(v0, back.x), __fsub_rn(v1, back.y));
    *hi2 = *reinterpret_cast<const uint32_t *>(&h);
    *lo2 = *reinterpret_cast<const uint32_t *>(&l);
}

// One quarter of one group of one RHS into the activation image.  The four
// threads of an aligned quad (lanes 4k..4k+3 of one warp, t = lane & 3) take
// one (group, RHS) together: thread t holds the group's columns t*CPL ..
// t*CPL+CPL-1 (exactly the columns MMA lane t reads) in v; the quad shares
// its largest |x| and adds its four partial sums as (s0 + s1) + (s2 + s3).
// Every lane of the warp must call act_quad_stats (it shuffles with the full
// mask); quads with nothing to do pass zeros.  The group's exponent E puts
// its largest |x| just below the fp16 maximum.
template <int CPL>
__device__ __forceinline__ void act_quad_stats(const float (&v)[CPL], int *E, float *sum) {
    float s = 0.0f;
    uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
        s = __fadd_rn(s, v[k]);
        m = max(m, __float_as_uint(v[k]) & 0x7fffffffu);
    }
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
    s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));  // s0 + s1 | s2 + s3 (addition commutes)
    s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
    *E = act_exponent(m);
    *sum = s;
}

// Thread t's part of the group's image block: dst points at the block
// [NCH][NB][4 lanes][8 halves], n0 is the RHS's high-part column (2b).
// Registers of lane t: pair (reg, h = 0/1) holds columns block_perm(reg,
// 0/1); 4 registers (8 halves) per 16-byte chunk jj, high parts at column n0
// and low parts at n0 + 1 (the next 64 bytes).  zero: a padding group past
// the matrix (zeros).
template <int BITS, int G>
__device__ __forceinline__ void act_quad_store(const float (&v)[G / 4], int E, bool zero, uint32_t *dst, int NB, int n0,
                                               int t) {
    using S = MmaShape<BITS, G>;
#pragma unroll
    for (int jj = 0; jj < S::NCH; ++jj) {
        uint32_t hi[4] = {0u, 0u, 0u, 0u}, lo[4] = {0u, 0u, 0u, 0u};
        if (!zero) {
#pragma unroll
            for (int r4 = 0; r4 < 4; ++r4) {
                const int reg = jj * 4 + r4;
                const int shift = (BITS == 4 && (reg & 1)) ? 4 : 0;
                act_split2(v[block_perm<BITS>(reg, 0)], v[block_perm<BITS>(reg, 1)], E - shift, &hi[r4], &lo[r4]);
            }
        }
        uint4 *blk = reinterpret_cast<uint4 *>(dst + ((jj * NB + n0) * 4 + t) * 4);
        blk[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        blk[4] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// Table entry of a group: (2^(24 - E), group sum); zero for padding groups.
__device__ __forceinline__ float2 act_table_entry(int E, float sum, bool zero) {
    return zero ? make_float2(0.0f, 0.0f) : make_float2(pow2f(24 - E), sum);
}

// Prep kernel of the prepared-activation API: CTA (c, b) writes groups
// [128 c, 128 c + 128) of RHS b into the global image and table that the
// streaming kernel then copies, four threads per group (one round: every
// load of the CTA is in flight at once).
constexpr int kPrepGroupsPerCta = 128;

// Threads 0..world-1 of the calling warp wait, bounded, until every rank has
// published this rank's current epoch in `flags` (acquire); after a wait has
// run out anywhere (the error word is set), later waits return at once.
__device__ __forceinline__ void wait_rank_epochs(const unsigned int *flags, const unsigned int *epoch, int world,
                                                 unsigned int *err) {
    const int lane = threadIdx.x & 31;
    if (*(volatile unsigned int *)err != 0u) return;
    const unsigned int e = *epoch;
    if (lane >= world) return;
    const unsigned long long start = global_ns();
    for (;;) {
        unsigned int f;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(flags + lane) : "memory");
        if ((int)(f - e) >= 0) return;
        if (global_ns() - start > kWaitLimitNs) {
            atomicCAS(err, 0u, kErrTimeoutPeer);
            return;
        }
        __nanosleep(100);
    }
}

// x[b][c] plus the ranks' partial sums of that entry, added in rank order:
// the all-reduced residual stream (slots [batch][world][cols]).
__device__ __forceinline__ float reduced_x(const float *x, const float *slots, int world, int cols, int b, int c) {
    const float *sl = slots + (size_t)b * world * cols + c;
    float acc = __ldcg(sl);
    for (int r = 1; r < world; ++r) acc = __fadd_rn(acc, __ldcg(sl + (size_t)r * cols));
    return __fadd_rn(__ldcg(x + (size_t)b * cols + c), acc);
}

// J entries of row b at columns c0, c0 + step, ... (zero past the row), each
// all-reduced as reduced_x does when slots is set: every load of the J
// entries is issued before any of them is used (one round trip, not J).
template <int J>
__device__ __forceinline__ void load_row_entries(float (&v)[J], const float *x, const float *slots, int world, int cols,
                                                 int b, int c0, int step) {
    const float *xb = x + (size_t)b * cols;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int c = c0 + j * step;
        v[j] = c < cols ? __ldcg(xb + c) : 0.0f;
    }
    if (slots == nullptr) return;
    const float *sb = slots + (size_t)b * world * cols;
    float acc[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int c = c0 + j * step;
        acc[j] = c < cols ? __ldcg(sb + c) : 0.0f;
    }
    for (int r = 1; r < world; ++r) {
        float t[J];
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int c = c0 + j * step;
            t[j] = c < cols ? __ldcg(sb + (size_t)r * cols + c) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < J; ++j) acc[j] = __fadd_rn(acc[j], t[j]);
    }
#pragma unroll
    for (int j = 0; j < J; ++j) v[j] = __fadd_rn(v[j], acc[j]);
}

template <int BITS, int G>
__global__ void __launch_bounds__(4 * kPrepGroupsPerCta) mma_prep_kernel(const float *x, int cols, int batch,
                                                                         int ngroups_pad, MmaImageView v) {
    // Launched behind the previous kernel (programmatic dependent launch): let
    // the streaming kernel launch now, then wait for x and for the previous
    // user of this scratch before touching either.
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    using S = MmaShape<BITS, G>;
    constexpr int CPL = S::CPL;
    const int b = blockIdx.y;
    const float *xb = x + (size_t)b * cols;  // the all-reduced x when red_slots is set
    const int tid = threadIdx.x;
    const int ngroups = cols / G;
    const int NB = 2 * batch;
    if (blockIdx.x == 0 && b == 0) {
        // Every call starts with clear argmax state, even after a launch that
        // stopped early on a device error.
        if (tid < 4) v.keys[tid] = 0ull;
        if (tid == 0) *v.done = 0u;
    }
    uint32_t *img = reinterpret_cast<uint32_t *>(v.image);
    float2 *tab = reinterpret_cast<float2 *>(v.table);
    // Every lane takes part in the quad shuffles of act_quad_stats.
    const int g = blockIdx.x * kPrepGroupsPerCta + (tid >> 2), t = tid & 3;
    const bool here = g < ngroups_pad, real = g < ngroups;
    if (v.red_slots != nullptr) {
        // The ranks' epochs: the first warp acquires them, the CTA barrier
        // then orders every thread's slot reads after the acquire.
        if (tid < 32) wait_rank_epochs(v.red_flags, v.red_epoch, v.red_world, v.red_err);
        __syncthreads();
        if (real) {
            const int c0 = g * G + t * CPL;
#pragma unroll
            for (int k = 0; k < CPL; ++k)
                v.red_x[(size_t)b * cols + c0 + k] = reduced_x(x, v.red_slots, v.red_world, cols, b, c0 + k);
        }
        xb = v.red_x + (size_t)b * cols;  // this thread reads back only its own columns
    }
    float v_[CPL];
#pragma unroll
    for (int k = 0; k < CPL; ++k) v_[k] = 0.0f;
    float ss = 0.0f;  // sum of x^2 over this thread's columns (fused RMSNorm)
    if (real) {
        const float *xl = xb + (size_t)g * G + t * CPL;
        if ((reinterpret_cast<uintptr_t>(xl) & 15) == 0) {
#pragma unroll
            for (int k = 0; k < CPL / 4; ++k) {
                const float4 q = __ldcg(reinterpret_cast<const float4 *>(xl) + k);
                v_[4 * k] = q.x;
                v_[4 * k + 1] = q.y;
                v_[4 * k + 2] = q.z;
                v_[4 * k + 3] = q.w;
            }
        } else {
#pragma unroll
            for (int k = 0; k < CPL; ++k) v_[k] = __ldcg(xl + k);
        }
        if (v.norm_w != nullptr) {
            const float *wl = v.norm_w + (size_t)g * G + t * CPL;
#pragma unroll
            for (int k = 0; k < CPL; ++k) {
                ss = __fmaf_rn(v_[k], v_[k], ss);
                v_[k] = __fmul_rn(v_[k], __ldg(wl + k));
            }
        }
    }
    if (v.norm_w != nullptr) {
        // 1 / rms of the whole row: this CTA holds every group of RHS b.
        // Fixed-order reduction: lanes by xor shuffle, then warps in order.
        __shared__ float warp_ss[4 * kPrepGroupsPerCta / 32];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        if ((tid & 31) == 0) warp_ss[tid >> 5] = ss;
        __syncthreads();
        if (tid == 0) {
            float total = 0.0f;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) total = __fadd_rn(total, warp_ss[w]);
            v.row_scale[b] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)cols), v.eps)));
        }
    }
    int E;
    float sum;
    act_quad_stats<CPL>(v_, &E, &sum);
    if (here) {
        act_quad_store<BITS, G>(v_, E, !real, img + (size_t)g * S::NCH * NB * 16, NB, 2 * b, t);
        if (t == 0) tab[(size_t)b * ngroups_pad + g] = act_table_entry(E, sum, !real);
    }
}

// The same image built by a streaming CTA in its own prologue, for the
// groups of its column slice [g0, g0 + ng) and RHS 0..B-1, straight into its
// shared memory (image blocks from the slice's first group; table rows
// [B][ngroups_pad] at the global group index), with the functions the prep
// kernel uses, so the image bits are the prep's.  The quads of the CTA take
// the (group, RHS) items in turn.  norm_w (optional): the image holds
// x * norm_w and rs[b] receives 1 / sqrt(mean(x_b^2) + eps), summed over the
// whole row in an order that does not depend on the slice, so every CTA of a
// call gets the same factor.  slots (optional): x is first all-reduced with
// the ranks' partial sums (reduced_x; the caller has waited for the ranks'
// epochs) and CTA 0 stores the reduced row into x_out.  Every thread of the
// CTA calls this; the caller synchronises the CTA afterwards.
template <int BITS, int G, int B, int NW>
__device__ __forceinline__ void mma_build_image(const float *x, const float *norm_w, float eps, int ngroups,
                                                int ngroups_pad, int g0, int ng, unsigned char *img_s,
                                                unsigned char *tab_s, float *red, float *rs, const float *slots,
                                                int world, float *x_out) {
    using S = MmaShape<BITS, G>;
    constexpr int CPL = S::CPL;
    constexpr int NB = 2 * B;
    constexpr int NQ = NW * 8;
    const int tid = threadIdx.x, t = tid & 3, quad = tid >> 2;
    const int cols = ngroups * G;
    const int items = ng * B;
    uint32_t *img = reinterpret_cast<uint32_t *>(img_s);
    float2 *tab = reinterpret_cast<float2 *>(tab_s);
    float ss[B];
    for (int base = 0; base < items; base += NQ) {  // the same trip count in every warp
        const int i = base + quad;
        const bool here = i < items;
        const int gl = here ? i / B : 0, b = here ? i % B : 0;
        const int g = g0 + gl;
        const bool real = here && g < ngroups;
        float v[CPL];
#pragma unroll
        for (int k = 0; k < CPL; ++k) v[k] = 0.0f;
        if (real && slots != nullptr) {
            load_row_entries<CPL>(v, x, slots, world, cols, b, g * G + t * CPL, 1);
        } else if (real) {
            const float *xl = x + (size_t)b * cols + (size_t)g * G + t * CPL;
            if ((reinterpret_cast<uintptr_t>(xl) & 15) == 0) {
#pragma unroll
                for (int k = 0; k < CPL / 4; ++k) {
                    const float4 q = __ldcg(reinterpret_cast<const float4 *>(xl) + k);
                    v[4 * k] = q.x;
                    v[4 * k + 1] = q.y;
                    v[4 * k + 2] = q.z;
                    v[4 * k + 3] = q.w;
                }
            } else {
#pragma unroll
                for (int k = 0; k < CPL; ++k) v[k] = __ldcg(xl + k);
            }
        }
        if (real && norm_w != nullptr) {
            const float *wl = norm_w + (size_t)g * G + t * CPL;
#pragma unroll
            for (int k = 0; k < CPL; ++k) v[k] = __fmul_rn(v[k], __ldg(wl + k));
        }
        int E;
        float sum;
        act_quad_stats<CPL>(v, &E, &sum);
        if (here) {
            act_quad_store<BITS, G>(v, E, !real, img + (size_t)gl * S::NCH * NB * 16, NB, 2 * b, t);
            if (t == 0) tab[(size_t)b * ngroups_pad + g] = act_table_entry(E, sum, !real);
        }
    }
    if (norm_w != nullptr || x_out != nullptr) {
        // The whole row: thread i takes columns i, i + NT, ... in order; the
        // first CTA stores the all-reduced x (x_out), and the sum of squares
        // for the RMSNorm factor goes lanes by xor shuffle, then warps in
        // order.
        constexpr int NT = NW * 32;
        const bool store = x_out != nullptr && blockIdx.x == 0;
        constexpr int J = 8;  // columns per thread whose loads are in flight together
#pragma unroll
        for (int k = 0; k < B; ++k) {
            float sq = 0.0f;
            for (int c0 = tid; c0 < cols; c0 += J * NT) {
                float xv[J];
                load_row_entries<J>(xv, x, slots, world, cols, k, c0, NT);
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    const int c = c0 + j * NT;
                    if (c < cols) {
                        if (store) x_out[(size_t)k * cols + c] = xv[j];
                        sq = __fmaf_rn(xv[j], xv[j], sq);
                    }
                }
            }
            ss[k] = sq;
        }
    }
    if (norm_w != nullptr) {
        const int warp = tid >> 5;
#pragma unroll
        for (int k = 0; k < B; ++k) {
            float r = ss[k];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, o));
            if ((tid & 31) == 0) red[warp * 4 + k] = r;
        }
        __syncthreads();
        if (tid < B) {
            float total = 0.0f;
            for (int w = 0; w < NW; ++w) total = __fadd_rn(total, red[w * 4 + tid]);
            rs[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)cols), eps)));
        }
    }
}

// D = A * B + D and D = A * B (zero accumulator) for m16n8k16 f16 -> f32.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

// Shared-memory loads at 32-bit shared addresses.  Volatile keeps them after
// the mbarrier wait that publishes the data.
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}

// The N = 1, 2 or 4 words a lane reads from one row of a group.
template <int N>
__device__ __forceinline__ void lds_words(uint32_t (&w)[N], uint32_t a) {
    if constexpr (N == 1) {
        w[0] = lds32(a);
    } else if constexpr (N == 2) {
        const uint2 v = lds64(a);
        w[0] = v.x;
        w[1] = v.y;
    } else {
        const uint4 v = lds128(a);
        w[0] = v.x;
        w[1] = v.y;
        w[2] = v.z;
        w[3] = v.w;
    }
}

// A-operand register `r` of a row from its words (see the file comment).
template <int BITS>
__device__ __forceinline__ uint32_t a_reg(const uint32_t *w, int r) {
    if constexpr (BITS == 4) {
        const uint32_t v = (r & 2) ? (w[r >> 2] >> 8) : w[r >> 2];
        return v & ((r & 1) ? 0x00f000f0u : 0x000f000fu);
    } else {
        const uint32_t v = (r & 1) ? (w[r >> 1] >> 8) : w[r >> 1];
        return v & 0x00ff00ffu;
    }
}

// Scales or biases of groups (g, g+1) of one row from the metadata ring.
template <bool BF16>
__device__ __forceinline__ float2 meta_pair(uint32_t a) {
    if constexpr (BF16) {
        const uint32_t v = lds32(a);
        return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
    } else {
        const uint2 v = lds64(a);
        return make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
    }
}

// Distributed shared memory of the cluster: map a local shared address to
// rank `rank`'s copy, load from or store to it, and the full cluster barrier.
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

struct MmaArgs {
    const unsigned char *s, *b, *s2, *b2;  // metadata [rows][ngroups] (f32 or bf16 bits)
    const __half *image;                   // prepared activation image
    const float *table;                    // [4][ngroups_pad] x (2^(24 - E_g), group sum)
    // build != 0: no prepared image; every CTA builds its slice of the image
    // in its prologue from x [B][cols] (mma_build_image), with the fused
    // RMSNorm weight norm_w (optional; every CTA computes the whole row's
    // output factor and keeps it in shared memory).
    const float *x;
    const float *norm_w;
    float eps;
    int build;
    // With build: x is first all-reduced with the ranks' partial sums
    // (red_slots [B][red_world][cols], after waiting for every rank's epoch
    // *red_epoch in red_flags) and CTA 0 stores the reduced x into x_out.
    const float *red_slots;
    const unsigned int *red_flags;
    const unsigned int *red_epoch;
    int red_world;
    float *x_out;
    float *y;
    unsigned long long *keys;              // [B] packed argmax (EPI 2)
    unsigned int *done;                    // CTAs finished (EPI 2)
    int *argmax;
    unsigned long long *best_key_out;
    unsigned int *err;                     // device error word
    int rows, ngroups, ngroups_pad, ystride, row_base;
    int tiles, nwin, kc, clusters, pieces, stages;
    uint32_t zero;                         // always 0 (an opaque operand, see the slot refill)
    const float *row_scale;                // per-RHS output factor (fused RMSNorm), or null
    const float *resid;                    // residual added to every output (same index as y), or null
    uint32_t off_image, off_table, off_pieces, off_part, off_bars;  // offsets into the 1024-aligned dynamic smem
    // Output exchange over peer memory (xworld > 1): rows also go to every
    // rank's output (peer_y, same index as y; not for EPI 2, whose keys go to
    // xkeys instead), then the last CTA publishes ++*xepoch to every rank's
    // flag array at index xrank.
    float *peer_y[kMaxRanks];
    unsigned int *xflags[kMaxRanks];
    unsigned long long *xkeys[kMaxRanks];  // [world][4] per rank
    unsigned int *xepoch;
    int xworld, xrank;
};

// Tensor maps of the (up to two) matrices of a call: packed weights (boxes
// of 32 words x 16 rows, 128-byte swizzle), scales and biases (boxes of one
// window's groups x 16 rows).
struct MmaMaps {
    CUtensorMap w[2], s[2], b[2];
};

template <int BITS, int G, int B, bool BF16, int EPI, int NW>
__global__ void __launch_bounds__(32 * NW, 1)
    mma_kernel(const __grid_constant__ MmaMaps maps, const MmaArgs a) {
    using S = MmaShape<BITS, G>;
    constexpr int NM = (EPI == 1) ? 2 : 1;
    constexpr int NB = 2 * B;
    constexpr int MSZ = BF16 ? 2 : 4;
    constexpr int META_ROW = S::WG * MSZ;  // bytes of one row of a scale or bias box
    constexpr int META_BYTES = 32 * META_ROW;
    constexpr int SLOT_W = mma_slot_weight_bytes(BITS, G, NM);
    constexpr int SLOT_M = mma_slot_meta_bytes(G, NM, MSZ);
    constexpr int GPB = 128 / S::GROUP_BYTES;  // groups per 128-byte line of a box
    constexpr int LANE_BYTES = S::WPL * 4;      // bytes of one row a lane reads per group
    constexpr int XG = S::NCH * NB * 64;        // activation image bytes per group
    constexpr int PIECE = NM * 64 * 4;          // bytes of one tile piece (64 values per matrix)
    static_assert(LANE_BYTES <= 16 && GPB >= 1, "one 16-byte unit per lane and row");
    extern __shared__ unsigned char smem_raw[];
    __shared__ unsigned int flag;
    const uint32_t sraw = smem_u32(smem_raw);
    const uint32_t sbase = (sraw + 1023u) & ~1023u;
    unsigned char *smem = smem_raw + (sbase - sraw);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, t = lane & 3;
    if (threadIdx.x == 0) {
#pragma unroll
        for (int q = 0; q < NM; ++q) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.w[q])) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.s[q])) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.b[q])) : "memory");
        }
    }
    const int nst = a.stages;
    const uint32_t ring_w = sbase + (uint32_t)(warp * nst * SLOT_W);
    const uint32_t ring_m = sbase + (uint32_t)(NW * nst * SLOT_W + warp * nst * SLOT_M);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + a.off_bars);
    uint64_t *full = bars + warp * nst;
    uint64_t *ibar = bars + NW * nst;  // one per window of the slice

    // Cluster tiles, this CTA's column slice and this warp's segment of
    // (tile, window) units.
    const int rank = (int)(blockIdx.x % (unsigned)a.kc), ci = (int)(blockIdx.x / (unsigned)a.kc);
    const int win0 = rank * a.nwin / a.kc;
    const int nh = (rank + 1) * a.nwin / a.kc - win0;
    const int t0 = ci * a.tiles / a.clusters;
    const int ntl = (ci + 1) * a.tiles / a.clusters - t0;
    const uint32_t U = (uint32_t)(ntl * nh);
    const uint32_t ua = U * (uint32_t)warp / NW, ub = U * (uint32_t)(warp + 1) / NW;
    const int tfirst = nh > 0 ? (int)(ua / (uint32_t)nh) : 0;

    if (lane == 0)
        for (int i = 0; i < nst; ++i) mbar_init(&full[i], 1);  // the expect_tx arrival; TMA bytes complete it
    if (threadIdx.x == 0)
        for (int i = 0; i < nh; ++i) mbar_init(&ibar[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();

    const uint64_t pol_stream = evict_first_policy();
    const uint64_t pol_keep = evict_normal_policy();

    // Issue unit (local tile tl, window wi of the slice) into ring slot sl:
    // one elected lane copies the weight boxes and the scale and bias boxes
    // [16 rows][window groups] of every matrix, all completing on the slot's
    // barrier.  Rows past the matrix and groups past the row arrive as zeros.
    auto issue = [&](int tl, int wi, int sl) {
        if (lane == 0) {
            const int T = t0 + tl;
            const uint32_t slot = ring_w + (uint32_t)(sl * SLOT_W);
            const uint32_t mslot = ring_m + (uint32_t)(sl * SLOT_M);
            uint64_t *bar = &full[sl];
            mbar_arrive_expect_tx(bar, SLOT_W + SLOT_M);
#pragma unroll
            for (int q = 0; q < NM; ++q) {
#pragma unroll
                for (int c = 0; c < S::NBOX; ++c)
                    tma_load_2d_s(slot + q * S::W_BYTES + c * 2048, &maps.w[q], (win0 + wi) * S::ROW_WORDS + c * 32,
                                  T * kTileRows, bar, pol_stream);
                tma_load_2d_s(mslot + q * META_BYTES, &maps.s[q], (win0 + wi) * S::WG, T * kTileRows, bar,
                              pol_stream);
                tma_load_2d_s(mslot + q * META_BYTES + 16 * META_ROW, &maps.b[q], (win0 + wi) * S::WG,
                              T * kTileRows, bar, pol_stream);
            }
        }
        __syncwarp();
    };

    // Issue cursor: unit `issued` = (local tile it, window iw), ring slot is_.
    uint32_t issued = ua;
    int it = tfirst, iw = nh > 0 ? (int)(ua % (uint32_t)nh) : 0, is_ = 0;
    auto issue_next = [&]() {
        issue(it, iw, is_);
        ++issued;
        if (++iw == nh) iw = 0, ++it;
        if (++is_ == nst) is_ = 0;
    };
    for (int i = 0; i < nst && issued < ub; ++i) issue_next();

    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // The activation image: built here from x (the weights keep streaming
    // into the rings meanwhile), or copied window by window from the
    // prepared image (the group-sum table with the first window), so each
    // warp starts as soon as its first window is in.
    bool ok = true;
    __shared__ float build_red[NW * 4];
    __shared__ float build_rs[4];
    // Windows of the image this warp has waited for (bit 0 also covers the
    // table); all of them when the CTA built the image itself.
    uint32_t img_ready = 0u;
    if (a.build) {
        // CTA 0 stores the all-reduced x even when it has no units of its own.
        if (U > 0 || (a.red_slots != nullptr && blockIdx.x == 0)) {  // CTA-uniform
            if (a.red_slots != nullptr) {
                // The ranks' epochs: the first warp acquires them, the CTA
                // barrier orders every thread's slot reads after the acquire.
                if (warp == 0) wait_rank_epochs(a.red_flags, a.red_epoch, a.red_world, a.err);
                __syncthreads();
            }
            mma_build_image<BITS, G, B, NW>(a.x, a.norm_w, a.eps, a.ngroups, a.ngroups_pad, win0 * S::WG,
                                            nh * S::WG, smem + a.off_image, smem + a.off_table, build_red, build_rs,
                                            a.red_slots, a.red_world, a.x_out);
            fence_proxy_async();  // generic-proxy image writes before any later async-proxy use of shared memory
            __syncthreads();
        }
        img_ready = ~0u;
    } else if (U > 0 && threadIdx.x == 0) {
        const uint32_t chunk = (uint32_t)S::WG * XG;
        const uint32_t tab_bytes = 4u * (uint32_t)a.ngroups_pad * 8u;  // [4][ngroups_pad] float2
        const unsigned char *src = reinterpret_cast<const unsigned char *>(a.image) + (size_t)win0 * chunk;
        for (int i = 0; i < nh; ++i) {
            mbar_arrive_expect_tx(&ibar[i], chunk + (i == 0 ? tab_bytes : 0u));
            if (i == 0) bulk_g2s(smem + a.off_table, a.table, tab_bytes, &ibar[0], pol_keep);
            bulk_g2s(smem + a.off_image + (size_t)i * chunk, src + (size_t)i * chunk, chunk, &ibar[i], pol_keep);
        }
    }
    // The output factor of the fused RMSNorm, per RHS (null: none).
    const float *row_scale = a.build ? (a.norm_w != nullptr ? build_rs : nullptr) : a.row_scale;

    // Per-lane byte offsets: A words of row gq for the GPB groups of a box
    // line (128-byte swizzle: 16-byte unit u of row r at u ^ (r & 7)), the
    // activation column this lane reads, its RHS row of the group-sum table
    // and its rows' metadata.
    uint32_t a_off[GPB];
#pragma unroll
    for (int m = 0; m < GPB; ++m) {
        const int byte = m * S::GROUP_BYTES + t * LANE_BYTES;
        a_off[m] = (uint32_t)(gq * 128 + ((((byte >> 4) ^ gq) & 7) << 4) + (byte & 15));
    }
    const int n = gq < NB ? gq : NB - 1;
    const uint32_t x_lane = sbase + a.off_image + (uint32_t)((n * 4 + t) * 16);
    const uint32_t t_lane = sbase + a.off_table + (uint32_t)(t * a.ngroups_pad * 8);
    const uint32_t m_lane = (uint32_t)(gq * META_ROW);  // row gq of the scale box
    const uint32_t piece_base = sbase + a.off_pieces + (uint32_t)(warp * a.pieces * PIECE);

    unsigned long long best = 0ull;
    // The epilogue of one finished tile: scale, activation, store, argmax key.
    auto finish_tile = [&](int T, const float (&v)[NM][2]) {
        if (t < B) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = T * kTileRows + gq + 8 * h;
                if (row < a.rows) {
                    float val = v[0][h];
                    float up = v[NM - 1][h];
                    if (row_scale != nullptr) {
                        const float rs = row_scale[t];
                        val = __fmul_rn(val, rs);
                        up = __fmul_rn(up, rs);
                    }
                    if constexpr (EPI == 1) val = __fmul_rn(silu_f32(val), up);
                    const size_t yi = (size_t)t * a.ystride + row;
                    if (a.resid != nullptr) val = __fadd_rn(a.resid[yi], val);
                    a.y[yi] = val;
                    if constexpr (EPI != 2) {
                        for (int p = 0; p < a.xworld; ++p)  // xworld is 0 without an exchange
                            if (p != a.xrank) a.peer_y[p][yi] = val;
                    }
                    if constexpr (EPI == 2) {
                        const unsigned long long key = ((unsigned long long)total_order_key(val) << 32) |
                                                       (unsigned long long)(0xffffffffu - (uint32_t)(a.row_base + row));
                        best = key > best ? key : best;
                    }
                }
            }
        }
    };

    float acc[NM][2][2];  // [matrix][row A|B][part hi|lo]
    bool piece_whole = false;  // the current piece started at window 0 of its tile
    uint32_t u = ua;
    int tl = tfirst, wi = nh > 0 ? (int)(ua % (uint32_t)nh) : 0, sl = 0;
    uint32_t phase = 0;
    while (ok && u < ub) {
        if (u == ua || wi == 0) {
#pragma unroll
            for (int q = 0; q < NM; ++q) acc[q][0][0] = acc[q][0][1] = acc[q][1][0] = acc[q][1][1] = 0.0f;
            piece_whole = wi == 0;
        }
        const int cur = sl;
        const uint32_t cur_phase = phase;
        if (++sl == nst) {
            sl = 0;
            phase ^= 1u;
        }
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(&full[cur], cur_phase))) {  // warp-uniform outcome
            ok = false;
            if (lane == 0) atomicCAS(a.err, 0u, kErrTimeoutFull);
            break;
        }
        const uint32_t wslot = ring_w + (uint32_t)(cur * SLOT_W);
        const uint32_t mw = ring_m + (uint32_t)(cur * SLOT_M) + m_lane;
        // Stage the unit's weight words and metadata in registers, then hand
        // the slot straight back to the copy engine: every slot but the one
        // being read stays in flight, which is what keeps HBM busy.
        uint32_t wr[NM][S::WG][2][S::WPL];
        uint32_t mr[NM][S::WG / 2][4][BF16 ? 1 : 2];
#pragma unroll
        for (int q = 0; q < NM; ++q) {
#pragma unroll
            for (int gi = 0; gi < S::WG; ++gi) {
                const uint32_t aa = wslot + (uint32_t)(q * S::W_BYTES + (gi / GPB) * 2048) + a_off[gi % GPB];
                lds_words<S::WPL>(wr[q][gi][0], aa);
                lds_words<S::WPL>(wr[q][gi][1], aa + 1024u);
            }
#pragma unroll
            for (int pr = 0; pr < S::WG / 2; ++pr) {
                const uint32_t mq = mw + (uint32_t)(q * META_BYTES + 2 * pr * MSZ);
                // scale and bias of row gq, scale and bias of row gq + 8
                const uint32_t offs[4] = {0u, (uint32_t)(16 * META_ROW), (uint32_t)(8 * META_ROW),
                                          (uint32_t)(24 * META_ROW)};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if constexpr (BF16) {
                        mr[q][pr][k][0] = lds32(mq + offs[k]);
                    } else {
                        const uint2 v = lds64(mq + offs[k]);
                        mr[q][pr][k][0] = v.x;
                        mr[q][pr][k][BF16 ? 0 : 1] = v.y;
                    }
                }
            }
        }
        // The slot is refilled next, by TMA and cp.async.  Every staged load
        // must have returned first: fold one word of each load into a value
        // the warp barrier's mask depends on (a.zero is 0, but opaque to the
        // compiler), so each lane passes the barrier only with all its loads
        // complete.
        uint32_t dep = 0;
#pragma unroll
        for (int q = 0; q < NM; ++q) {
#pragma unroll
            for (int gi = 0; gi < S::WG; ++gi) dep ^= wr[q][gi][0][0] ^ wr[q][gi][1][0];
#pragma unroll
            for (int pr = 0; pr < S::WG / 2; ++pr)
                dep ^= mr[q][pr][0][0] ^ mr[q][pr][1][0] ^ mr[q][pr][2][0] ^ mr[q][pr][3][0];
        }
        __syncwarp(0xffffffffu | (dep & a.zero));
        if (issued < ub) issue_next();  // refills the slot just staged

        if (!((img_ready >> wi) & 1u) || !(img_ready & 1u)) {
            const bool got = __all_sync(0xffffffffu, mbar_wait_sleep(&ibar[0], 0) && mbar_wait_sleep(&ibar[wi], 0));
            if (!got) {
                ok = false;
                if (lane == 0) atomicCAS(a.err, 0u, kErrTimeoutFull);
                break;
            }
            img_ready |= 1u | (1u << wi);
        }
        const uint32_t xw = x_lane + (uint32_t)(wi * S::WG * XG);
        const uint32_t tw = t_lane + (uint32_t)((win0 + wi) * S::WG * 8);
#pragma unroll
        for (int gl = 0; gl < S::WG; gl += 2) {
            uint32_t xb[2][S::NREG];
#pragma unroll
            for (int e = 0; e < 2; ++e)
#pragma unroll
                for (int jj = 0; jj < S::NCH; ++jj) {
                    const uint4 v = lds128(xw + (uint32_t)((gl + e) * XG + jj * NB * 64));
                    xb[e][4 * jj] = v.x;
                    xb[e][4 * jj + 1] = v.y;
                    xb[e][4 * jj + 2] = v.z;
                    xb[e][4 * jj + 3] = v.w;
                }
            // Table entries of groups gl, gl+1 for this lane's RHS: 2^(24 - E_g)
            // and the group sum.
            const uint4 tv = lds128(tw + (uint32_t)(gl * 8));
            const float fg[2] = {__uint_as_float(tv.x), __uint_as_float(tv.z)};
            const float xs[2] = {__uint_as_float(tv.y), __uint_as_float(tv.w)};
#pragma unroll
            for (int q = 0; q < NM; ++q) {
                float d[2][4];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const uint32_t *wa = wr[q][gl + e][0];
                    const uint32_t *wb = wr[q][gl + e][1];
                    mma_16816_z(d[e], a_reg<BITS>(wa, 0), a_reg<BITS>(wb, 0), a_reg<BITS>(wa, 1), a_reg<BITS>(wb, 1),
                                xb[e][0], xb[e][1]);
#pragma unroll
                    for (int mj = 1; mj < S::NMMA; ++mj)
                        mma_16816(d[e], a_reg<BITS>(wa, 2 * mj), a_reg<BITS>(wb, 2 * mj), a_reg<BITS>(wa, 2 * mj + 1),
                                  a_reg<BITS>(wb, 2 * mj + 1), xb[e][2 * mj], xb[e][2 * mj + 1]);
                }
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float m4[4];  // scale A, bias A, scale B, bias B of group gl + e
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if constexpr (BF16) {
                            const uint32_t v = mr[q][gl / 2][k][0];
                            m4[k] = __uint_as_float(e ? (v & 0xffff0000u) : (v << 16));
                        } else {
                            m4[k] = __uint_as_float(mr[q][gl / 2][k][e]);
                        }
                    }
                    const float sa = __fmul_rn(m4[0], fg[e]), sb = __fmul_rn(m4[2], fg[e]);
                    acc[q][0][0] = __fmaf_rn(sa, d[e][0], acc[q][0][0]);
                    acc[q][0][1] = __fmaf_rn(sa, d[e][1], acc[q][0][1]);
                    acc[q][0][0] = __fmaf_rn(m4[1], xs[e], acc[q][0][0]);
                    acc[q][1][0] = __fmaf_rn(sb, d[e][2], acc[q][1][0]);
                    acc[q][1][1] = __fmaf_rn(sb, d[e][3], acc[q][1][1]);
                    acc[q][1][0] = __fmaf_rn(m4[3], xs[e], acc[q][1][0]);
                }
            }
        }

        const bool piece_end = wi == nh - 1 || u + 1 == ub;
        if (piece_end) {
            float v[NM][2];
#pragma unroll
            for (int q = 0; q < NM; ++q) {
                v[q][0] = __fadd_rn(acc[q][0][0], acc[q][0][1]);
                v[q][1] = __fadd_rn(acc[q][1][0], acc[q][1][1]);
            }
            if (a.kc == 1 && piece_whole && wi == nh - 1) {
                finish_tile(t0 + tl, v);
            } else {
                // kc = 1: only a segment's first and last pieces can be split.
                const int slot_i = a.kc == 1 ? (tl == tfirst ? 0 : 1) : tl - tfirst;
                const uint32_t pb = piece_base + (uint32_t)(slot_i * PIECE);
#pragma unroll
                for (int q = 0; q < NM; ++q) {
                    asm volatile("st.shared.f32 [%0], %1;" ::"r"(pb + (uint32_t)(q * 256 + lane * 4)), "f"(v[q][0]) : "memory");
                    asm volatile("st.shared.f32 [%0], %1;" ::"r"(pb + (uint32_t)(q * 256 + 128 + lane * 4)), "f"(v[q][1])
                                 : "memory");
                }
            }
        }
        ++u;
        if (++wi == nh) wi = 0, ++tl;
    }
    // Drain copies issued but not consumed (only after a failed wait).
    for (uint32_t d = u; d < issued; ++d) {
        const uint32_t j = d - ua;
        if (!mbar_wait(&full[(int)(j % (uint32_t)nst)], (j / (uint32_t)nst) & 1u)) {
            if (lane == 0) atomicCAS(a.err, 0u, kErrTimeoutDrain);
            break;
        }
    }

    // Every image copy has landed before the CTA can exit (normally already
    // waited for by the warps that read the window).  A CTA that built its
    // image issued none.
    if (U > 0 && threadIdx.x == 0 && !a.build)
        for (int i = 0; i < nh; ++i)
            if (!mbar_wait(&ibar[i], 0)) {
                atomicCAS(a.err, 0u, kErrTimeoutDrain);
                break;
            }

    // Tiles split between warps: add the pieces in warp order.  With column
    // slices the CTA's sum of a tile goes to its part buffer for the cluster.
    __syncthreads();
    for (int T = warp; T < ntl; T += NW) {
        const uint32_t uf = (uint32_t)(T * nh), ul = uf + (uint32_t)nh - 1u;
        const int wf = (int)(((uf + 1u) * NW - 1u) / U), wl = (int)(((ul + 1u) * NW - 1u) / U);
        if (a.kc == 1 && wf == wl) continue;  // one warp held the whole tile and wrote it
        float v[NM][2];
#pragma unroll
        for (int q = 0; q < NM; ++q) v[q][0] = v[q][1] = 0.0f;
        for (int w = wf; w <= wl; ++w) {
            const uint32_t wa = U * (uint32_t)w / NW, wb = U * (uint32_t)(w + 1) / NW;
            if (wb == wa) continue;  // empty segment
            const int tf = (int)(wa / (uint32_t)nh);
            const int slot_i = a.kc == 1 ? (T == tf ? 0 : 1) : T - tf;
            const uint32_t pb = sbase + a.off_pieces + (uint32_t)((w * a.pieces + slot_i) * PIECE);
#pragma unroll
            for (int q = 0; q < NM; ++q) {
                v[q][0] = __fadd_rn(v[q][0], __uint_as_float(lds32(pb + (uint32_t)(q * 256 + lane * 4))));
                v[q][1] = __fadd_rn(v[q][1], __uint_as_float(lds32(pb + (uint32_t)(q * 256 + 128 + lane * 4))));
            }
        }
        if (a.kc == 1) {
            finish_tile(t0 + T, v);
        } else {
            // Tile T belongs to rank T % kc: store this slice's sum into the
            // owner's part buffer, row T / kc, column = this rank.
            const uint32_t pp = sbase + a.off_part + (uint32_t)(((T / a.kc) * a.kc + rank) * PIECE);
            const uint32_t owner = (uint32_t)(T % a.kc);
#pragma unroll
            for (int q = 0; q < NM; ++q) {
                st_cluster_f32(cluster_map(pp + (uint32_t)(q * 256 + lane * 4), owner), v[q][0]);
                st_cluster_f32(cluster_map(pp + (uint32_t)(q * 256 + 128 + lane * 4), owner), v[q][1]);
            }
        }
    }
    if (a.kc > 1) {
        // One cluster barrier publishes the remote stores; each rank then adds
        // the slices of its own tiles in rank order from local shared memory.
        cluster_sync();
        for (int T = rank + warp * a.kc; T < ntl; T += NW * a.kc) {
            float v[NM][2];
#pragma unroll
            for (int q = 0; q < NM; ++q) v[q][0] = v[q][1] = 0.0f;
            for (int r = 0; r < a.kc; ++r) {
                const uint32_t pp = sbase + a.off_part + (uint32_t)(((T / a.kc) * a.kc + r) * PIECE);
#pragma unroll
                for (int q = 0; q < NM; ++q) {
                    v[q][0] = __fadd_rn(v[q][0], __uint_as_float(lds32(pp + (uint32_t)(q * 256 + lane * 4))));
                    v[q][1] = __fadd_rn(v[q][1], __uint_as_float(lds32(pp + (uint32_t)(q * 256 + 128 + lane * 4))));
                }
            }
            finish_tile(t0 + T, v);
        }
    }

    if constexpr (EPI == 2) {
        // Maximum per RHS over the lanes that share it, one atomic per RHS and
        // warp; the last CTA publishes the winners and clears the keys.
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane < B && best != 0ull) atomicMax(a.keys + lane, best);
    }
    const bool xchg = a.xworld > 1;
    if (EPI == 2 || xchg) {
        // Last CTA: this CTA's stores (peer stores included) are ordered
        // before its count by a GPU-scope fence, the last CTA's epilogue after
        // all counts.  With an exchange, the last CTA alone then fences at
        // system scope before it releases the epoch: fences are cumulative, so
        // that one fence orders every store the counts made visible to it
        // before the flag a peer acquires.  (No CTA waits for its own NVLink
        // stores to be acknowledged before counting.)
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) flag = (atomicAdd(a.done, 1u) == gridDim.x - 1) ? 1u : 0u;
        __syncthreads();
        if (flag) {
            __threadfence();
            if (EPI == 2 && threadIdx.x < B) {
                const unsigned long long k = atomicExch(a.keys + threadIdx.x, 0ull);
                if (a.argmax) a.argmax[threadIdx.x] = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
                if (a.best_key_out) a.best_key_out[threadIdx.x] = k;
                if (xchg)
                    for (int p = 0; p < a.xworld; ++p) a.xkeys[p][a.xrank * 4 + threadIdx.x] = k;
            }
            if (xchg) {
                __syncthreads();  // the key stores above (flag is the same for the whole CTA)
                if (threadIdx.x == 0) {
                    // One system-scope fence, after the CTA barrier and the
                    // counter that observed every other CTA's stores: it is
                    // cumulative over all of them, and a fence followed by
                    // strong (relaxed) stores is a release, so the flag
                    // stores carry no fence of their own.
                    __threadfence_system();
                    const unsigned int e = *a.xepoch + 1u;
                    *a.xepoch = e;
                    for (int p = 0; p < a.xworld; ++p)
                        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(a.xflags[p] + a.xrank), "r"(e)
                                     : "memory");
                }
            }
            if (threadIdx.x == 0) *a.done = 0u;
        }
    }
    (void)best;
}

}  // namespace qmr
