// Launchers for the packed-affine kernels: kernel choice and launch shape for
// B200, the prepared-activation scratch, and programmatic dependent launch of
// the streaming kernel behind its prep pass.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "matrix_kernels.cuh"
#include "qmr_internal.h"
#include "launch.h"

namespace qmr {


namespace {

struct Scratch {
    void *base = nullptr;
    size_t bytes = 0;
};

std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }



size_t prepared_floats(int bits, uint32_t cols, uint32_t batch) {
    const size_t nchunks = (size_t)cols * bits / 128;
    const size_t nblocks = (nchunks + kBlockChunks - 1) / kBlockChunks;
    const size_t bf = bits == 4 ? prepared_block_floats<4>() : prepared_block_floats<8>();
    return batch * nblocks * bf;
}

// Bytes of the tensor-core activation image and its table (two floats per
// group and RHS), sized for the widest window (1024 columns) and the
// smallest group (32).
size_t mma_prepared_bytes(uint32_t cols, uint32_t batch) {
    const size_t padded = ((size_t)cols + 1023) / 1024 * 1024;
    return align_up(padded * 4 * batch) + align_up(padded);
}

// The activation region holds either path's layout.
size_t prepared_region(int bits, uint32_t cols, uint32_t batch) {
    const size_t a = align_up(prepared_floats(bits, cols, batch) * sizeof(float));
    const size_t b = mma_prepared_bytes(cols, batch);
    return a > b ? a : b;
}

// Fixed part of every scratch buffer, at the same offsets whatever the shape
// of the call: the output factors, the argmax keys and CTA counter (which
// must read zero between calls), the split-tile counters and partial sums.
// The shape-dependent prepared activations follow it.
size_t fixed_region() {
    return align_up(8 * sizeof(float)) + align_up(4 * sizeof(unsigned long long) + sizeof(unsigned int)) +
           align_up(kCounterCount * sizeof(unsigned int)) + align_up(kPartialFloats * sizeof(float)) +
           align_up(4 * sizeof(float));
}

void scratch_layout(void *base, int bits, uint32_t cols, uint32_t batch, ScratchView *v, MmaImageView *mv = nullptr) {
    (void)bits;
    char *p = static_cast<char *>(base);
    v->cf = reinterpret_cast<float *>(p);
    p += align_up(8 * sizeof(float));
    v->keys = reinterpret_cast<unsigned long long *>(p);
    v->done = reinterpret_cast<unsigned int *>(p + 4 * sizeof(unsigned long long));
    p += align_up(4 * sizeof(unsigned long long) + sizeof(unsigned int));
    v->counters = reinterpret_cast<unsigned int *>(p);
    p += align_up(kCounterCount * sizeof(unsigned int));
    v->partial = reinterpret_cast<float *>(p);
    p += align_up(kPartialFloats * sizeof(float));
    float *row_scale = reinterpret_cast<float *>(p);  // fused RMSNorm factors, one per RHS
    p += align_up(4 * sizeof(float));
    v->xp = reinterpret_cast<float *>(p);
    if (mv != nullptr) {
        mv->norm_w = nullptr;
        mv->eps = 0.0f;
        mv->row_scale = row_scale;
        mv->red_slots = nullptr;
        mv->red_x = nullptr;
        mv->red_flags = nullptr;
        mv->red_epoch = nullptr;
        mv->red_err = nullptr;
        mv->red_world = 0;
        const size_t padded = ((size_t)cols + 1023) / 1024 * 1024;
        mv->image = reinterpret_cast<__half *>(p);
        mv->table = reinterpret_cast<float *>(p + align_up(padded * 4 * batch));
        mv->keys = v->keys;
        mv->done = v->done;
    }
}

// Largest opt-in shared memory of one block on the current device.
int smem_optin() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cached[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) v = 0;
        cached[dev] = v;
    }
    return cached[dev];
}

bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace

size_t scratch_bytes(int bits, uint32_t cols, uint32_t batch) {
    return fixed_region() + prepared_region(bits, cols, batch);
}

// Per (device, stream) scratch.  The first call on a stream reserves enough
// for cols <= 65536 at batch 4; larger shapes grow it after draining the
// stream, which is not allowed while the stream is being captured.
int acquire_scratch(cudaStream_t stream, size_t need, void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(QMR_ECUDA, "cudaGetDevice failed");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    Scratch &s = g_scratch[{dev, stream}];
    if (s.bytes >= need) {
        *out = s.base;
        return QMR_OK;
    }
    const size_t floor_bytes = scratch_bytes(4, 65536, 4);
    const size_t want = need > floor_bytes ? need : floor_bytes;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(stream, &cs);
    if (cs != cudaStreamCaptureStatusNone)
        return fail(QMR_EUNSUPPORTED,
                    "activation scratch must be allocated or grown, which cannot happen during stream capture; "
                    "make one call with the largest shape on this stream before capturing");
    if (s.base != nullptr) {
        if (cudaStreamSynchronize(stream) != cudaSuccess) return fail(QMR_ECUDA, "stream synchronize failed");
        cudaFree(s.base);
        s.base = nullptr;
        s.bytes = 0;
    }
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaMalloc of activation scratch failed: %s", cudaGetErrorString(e));
    e = cudaMemset(p, 0, want);  // counters start at zero
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaMemset of activation scratch failed: %s", cudaGetErrorString(e));
    // The clear runs on the legacy stream, which does not order against a
    // non-blocking caller stream: finish it before any kernel uses the
    // buffer (cudaMalloc above has synchronised the device already).
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail(QMR_ECUDA, "waiting for the scratch clear failed: %s", cudaGetErrorString(e));
    s.base = p;
    s.bytes = want;
    *out = p;
    return QMR_OK;
}

bool fast_eligible(const void *w, uint32_t cols, uint32_t bits, uint32_t group) {
    if (bits != 4 && bits != 8) return false;
    if (group != 32 && group != 64 && group != 128) return false;
    if (cols % group != 0) return false;
    if (((uint64_t)cols * bits / 8) % 16 != 0) return false;
    if (reinterpret_cast<uintptr_t>(w) % 16 != 0) return false;
    return true;
}


// Activation image of one column slice, worst case B = 4, stays within this
// budget (5120 columns take one slice, 17408 columns 4).
constexpr size_t kMmaImageBudget = 96 * 1024;

namespace {

bool mma_plan_b(uint32_t bits, uint32_t group, uint32_t rows, uint32_t cols, uint32_t batch, int epi, bool bf16,
                int only_kc, int only_warps, MmaPlan *p, uint32_t meta_stride);

}  // namespace

// The launch plan for this call.  Whether the kernel takes a shape is decided
// at B = 4, and the column slicing does not depend on B, so every block width
// of one matrix runs the same kernel with the same summation order.
bool mma_plan(uint32_t bits, uint32_t group, uint32_t rows, uint32_t cols, uint32_t batch, int epi, bool bf16,
              MmaPlan *p, uint32_t meta_stride) {
    MmaPlan widest;
    if (!mma_plan_b(bits, group, rows, cols, 4, epi, bf16, 0, 0, &widest, meta_stride)) return false;
    return mma_plan_b(bits, group, rows, cols, batch, epi, bf16, widest.kc, widest.warps, p, meta_stride);
}

namespace {

// only_kc / only_warps: 0 searches the slice count / warps per CTA,
// otherwise the plan must use that one.
bool mma_plan_b(uint32_t bits, uint32_t group, uint32_t rows, uint32_t cols, uint32_t batch, int epi, bool bf16,
                int only_kc, int only_warps, MmaPlan *p, uint32_t meta_stride) {
    if (bits != 4 && bits != 8) return false;
    if (group != 32 && group != 64 && group != 128) return false;
    if (bits == 8 && group == 128) return false;
    if (rows == 0 || cols == 0 || cols % group != 0 || batch < 1 || batch > 4) return false;
    const uint32_t ngroups = cols / group;
    const uint32_t mstride = meta_stride != 0 ? meta_stride : ngroups;
    if (mstride % 8 != 0 || mstride < ngroups) return false;  // 16-byte metadata rows for the tensor maps
    const uint32_t win_cols = 8 * group > 512 ? 8 * group : 512;
    const uint32_t wg = win_cols / group;
    const int nwin = (int)((cols + win_cols - 1) / win_cols);
    const int tiles = (int)((rows + kTileRows - 1) / kTileRows);
    const int nm = epi == 1 ? 2 : 1;
    const int sms = sm_count();
    // Warps per CTA: 12 for Q4 streams with groups of 32 or 64, where the
    // per-unit instruction latency of 8 warps (2 per scheduler) limits the
    // rate at every size (measured on dependent B1 chains, 1.5 to 50 MB per
    // call); 8 for the gate/up pair (twice the registers per thread) and for
    // Q8 and g128, whose deeper rings matter more.  Chosen from the shape only.
    for (int warps : {kMmaWarpsLong, kMmaWarps}) {
        if (only_warps != 0 && warps != only_warps) continue;
        if (only_warps == 0 && warps == kMmaWarpsLong && (epi == 1 || bits != 4 || group > 64)) continue;
        // Column slices (= cluster size): the smallest kc whose activation slice
        // fits the image budget and whose whole plan (rings of at least two
        // stages, image, table, pieces) fits the shared memory of one SM.  Two
        // matrices per unit (the gate/up epilogue) double the ring slots, which
        // can push a wide matrix from one slice to two.
        const uint32_t piece_bytes = (uint32_t)nm * 64 * 4;
        const uint32_t slot = (uint32_t)(mma_slot_weight_bytes((int)bits, (int)group, nm) +
                                         mma_slot_meta_bytes((int)group, nm, bf16 ? 2 : 4));
        const uint32_t ngroups_pad = (uint32_t)nwin * wg;
        const uint32_t table = 32 * ngroups_pad;
        const int limit = smem_optin() - 512;  // room for the kernel's static shared variables (under 300 bytes)
        for (int kc : {1, 2, 4}) {
            if (only_kc != 0 && kc != only_kc) continue;
            const int nh_min = nwin / kc, nh_max = (nwin + kc - 1) / kc;
            if (nwin < kc || sms < kc || (size_t)nh_max * win_cols * 16 > kMmaImageBudget) continue;
            if (nh_max > 32) continue;  // image-window barriers and the per-warp ready mask
            // One wave: no more clusters than can be resident together.
            int clusters = sms / kc;
            if (kc > 1) {
                const int cap = mma_cluster_capacity(kc);
                if (cap > 0 && cap < clusters) clusters = cap;
            }
            const int ctas = clusters * kc;
            const int tmax = (tiles + clusters - 1) / clusters;
            if ((long long)tmax * nh_max * warps >= (1ll << 31)) continue;  // 32-bit unit arithmetic
            int pieces = 2;
            if (kc > 1) {
                const int lmax = (tmax * nh_max + warps - 1) / warps;
                pieces = (lmax + nh_min - 1) / nh_min + 1;
                if (pieces > kMaxPieces) continue;
            }
            const uint32_t image = (uint32_t)nh_max * win_cols * 4 * batch;
            const uint32_t pieces_bytes = (uint32_t)warps * pieces * piece_bytes;
            const uint32_t part_bytes = kc > 1 ? (uint32_t)((tmax + kc - 1) / kc * kc) * piece_bytes : 0u;
            for (int st = kMmaMaxStages; st >= 2; --st) {
                const uint32_t off_image = (uint32_t)warps * st * slot;
                const uint32_t off_table = off_image + (image + 127) / 128 * 128;
                const uint32_t off_pieces = off_table + (table + 127) / 128 * 128;
                const uint32_t off_part = off_pieces + pieces_bytes;
                const uint32_t off_bars = off_part + part_bytes;
                const uint32_t total = 1024 + off_bars + (uint32_t)(warps * st + nh_max) * 8;
                if ((int)total <= limit) {
                    p->kc = kc;
                    p->clusters = clusters;
                    p->ctas = ctas;
                    p->stages = st;
                    p->pieces = pieces;
                    p->nwin = nwin;
                    p->ngroups_pad = (int)ngroups_pad;
                    p->tiles = tiles;
                    p->warps = warps;
                    p->smem = total;
                    p->off_image = off_image;
                    p->off_table = off_table;
                    p->off_pieces = off_pieces;
                    p->off_part = off_part;
                    p->off_bars = off_bars;
                    return true;
                }
            }
        }
    }
    return false;
}

}  // namespace

int log2i(uint32_t v) {
    int r = 0;
    while ((1u << r) < v) ++r;
    return r;
}

int sm_count() {
    static std::atomic<int> cached[64] = {};
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    n = cached[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
    return n;
}

cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    return attr;
}

int launch_mma_prep_bits(int bits, const float *x, uint32_t cols, uint32_t group, uint32_t batch, int ngroups_pad,
                         const MmaImageView &v, cudaStream_t stream) {
    return bits == 4 ? launch_mma_prep4(x, cols, group, batch, ngroups_pad, v, stream)
                     : launch_mma_prep8(x, cols, group, batch, ngroups_pad, v, stream);
}

namespace {

// The activation layout the tensor-core kernel would read for this shape
// (independent of the matrix): its padded group count, or 0 when the shape
// goes to the FP32 paths.
int mma_layout_groups(uint32_t bits, uint32_t group, uint32_t cols, uint32_t batch) {
    MmaPlan p;
    if (!mma_plan(bits, group, kTileRows, cols, batch, 0, true, &p)) return 0;
    return p.ngroups_pad;
}

// The tensor-core kernel takes this call: a launch plan and 16-byte aligned
// weights and metadata (TMA and cp.async sources).
bool mma_takes(const FastCall &c, MmaPlan *p) {
    if (!mma_plan(c.bits, c.group, c.rows, c.cols, c.batch, c.epilogue, c.bf16, p, c.meta_stride)) return false;
    if (!aligned16(c.w) || !aligned16(c.s) || !aligned16(c.b)) return false;
    if (c.epilogue == 1 && (!aligned16(c.w2) || !aligned16(c.s2) || !aligned16(c.b2))) return false;
    // The fused RMSNorm needs the whole row in one prep CTA per RHS.
    if (c.norm_w != nullptr && p->ngroups_pad > kPrepGroupsPerCta) return false;
    return true;
}

}  // namespace

bool fused_supported(const FastCall &c) {
    if (!fast_eligible(c.w, c.cols, c.bits, c.group)) return false;
    MmaPlan p;
    return mma_takes(c, &p);
}

int run_prepare(const float *x, uint32_t cols, uint32_t bits, uint32_t group, uint32_t batch, void *base, int path,
                cudaStream_t stream) {
    ScratchView sv;
    MmaImageView mv;
    scratch_layout(base, (int)bits, cols, batch, &sv, &mv);
    if (path == kPathMma) {
        const int ngroups_pad = mma_layout_groups(bits, group, cols, batch);
        if (ngroups_pad > 0) return launch_mma_prep_bits((int)bits, x, cols, group, batch, ngroups_pad, mv, stream);
    }
    return launch_prep_fp32(x, cols, bits, batch, sv, stream);
}

int run_stream(const FastCall &c, void *base, cudaStream_t stream) {
    ScratchView sv;
    MmaImageView mv;
    scratch_layout(base, (int)c.bits, c.cols, c.batch, &sv, &mv);
    const int ce = 128 / (int)c.bits;
    const int gpc = (int)c.group / ce;
    const int nchunks = (int)((uint64_t)c.cols * c.bits / 128);
    if (c.path == kPathMma && mma_layout_groups(c.bits, c.group, c.cols, c.batch) > 0) {
        // The activations were prepared in the tensor-core layout.
        MmaPlan p;
        if (!mma_takes(c, &p))
            return fail(QMR_EUNSUPPORTED,
                        "activations prepared for the tensor-core kernel, which does not take this matrix "
                        "(unaligned weights or metadata, or no launch plan)");
        return c.bits == 4 ? launch_mma4(c, p, sv, mv, stream) : launch_mma8(c, p, sv, mv, stream);
    }
    if (c.path != kPathRegisters && tile_eligible(c)) return launch_tile_call(c, sv, stream);
    StreamArgs a = {};
    a.w = static_cast<const uint4 *>(c.w);
    a.s = c.s;
    a.bias = c.b;
    a.w2 = static_cast<const uint4 *>(c.w2);
    a.s2 = c.s2;
    a.bias2 = c.b2;
    a.xp = sv.xp;
    a.cf = sv.cf;
    a.y = c.y;
    a.keys = sv.keys;
    a.done = sv.done;
    a.argmax = c.argmax;
    a.best_key_out = reinterpret_cast<unsigned long long *>(c.best_key);
    a.rows = (int)c.rows;
    a.nchunks = nchunks;
    a.group_shift = log2i((uint32_t)gpc);
    a.ystride = (int)c.rows;
    a.row_base = (int)c.row_base;
    return launch_reg(a, (int)c.bits, c.bf16, c.batch, c.epilogue, c.overlap, stream);
}

// x in device memory (every streaming CTA may read it); pinned host
// activations are read once, by the prep kernel.
bool device_resident(const void *p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

int run_fast(const FastCall &c, cudaStream_t stream) {
    const size_t need = scratch_bytes((int)c.bits, c.cols, c.batch);
    void *base = c.scratch;
    if (base == nullptr) {
        const int rc = acquire_scratch(stream, need, &base);
        if (rc != QMR_OK) return rc;
    } else if (c.scratch_bytes < need) {
        return fail(QMR_ERANGE, "scratch of %zu bytes is smaller than the %zu required", c.scratch_bytes, need);
    }
    FastCall call = c;
    MmaPlan plan;
    if (call.ex != nullptr) {
        // The output exchange lives in the tensor-core kernel's epilogue.
        call.path = kPathMma;
        if (!mma_takes(call, &plan))
            return fail(QMR_EUNSUPPORTED, "the exchange calls need a shape the tensor-core kernel takes");
    }
    const bool fused = call.norm_w != nullptr || call.resid != nullptr || call.meta_stride != 0 || call.reduce != nullptr;
    if (fused && !mma_takes(call, &plan))
        return fail(QMR_EUNSUPPORTED, "the fused RMSNorm/residual epilogue needs a shape the tensor-core kernel takes");
    if (fused) call.path = kPathMma;
    if (call.path == kPathMma && !mma_takes(call, &plan)) call.path = kPathTile;  // FP32 kernels take the rest
    if (call.path == kPathMma) {
        ScratchView sv;
        MmaImageView mv;
        scratch_layout(base, (int)call.bits, call.cols, call.batch, &sv, &mv);
        if (call.reduce != nullptr) {
            const QmrExchange &r = *call.reduce;
            if (r.total_rows != r.world * call.cols || call.batch > 4 || call.x_out == nullptr)
                return fail(QMR_EINVAL, "the folded all-reduce needs slots of [batch][world][cols] and an x output");
        }
        // Device-resident x: the streaming CTAs build the image themselves,
        // one launch behind the producer of x.  The argmax and exchange
        // epilogues count CTAs on scratch words that the prep clears at the
        // start of a call; they build in-kernel only for a caller that clears
        // its scratch after any failed call (counted_build).
        call.build = (call.epilogue != 2 && call.ex == nullptr) || call.counted_build;
        call.build = call.build && device_resident(call.x);
        if (call.reduce != nullptr && call.x_out == call.x) call.build = false;  // its CTAs read x while CTA 0 writes
        if (call.build) {
            call.overlap = true;
            if (call.launch_count != nullptr) *call.launch_count += 1;
            return call.bits == 4 ? launch_mma4(call, plan, sv, mv, stream) : launch_mma8(call, plan, sv, mv, stream);
        }
        if (call.launch_count != nullptr) *call.launch_count += 2;
        // Prep kernel, then the streaming kernel behind it (programmatic
        // dependent launch: the prep writes no weights), one plan for both.
        mv.norm_w = call.norm_w;
        mv.eps = call.eps;
        if (call.reduce != nullptr) {
            const QmrExchange &r = *call.reduce;
            mv.red_slots = r.out[r.rank];
            mv.red_x = call.x_out;
            mv.red_flags = r.flags[r.rank];
            mv.red_epoch = r.epoch;
            mv.red_err = device_error_word();
            mv.red_world = (int)r.world;
            if (mv.red_err == nullptr) return fail(QMR_ECUDA, "device error word is unavailable");
        }
        const int rc = launch_mma_prep_bits((int)call.bits, call.x, call.cols, call.group, call.batch,
                                            plan.ngroups_pad, mv, stream);
        if (rc != QMR_OK) return rc;
        call.overlap = true;
        return call.bits == 4 ? launch_mma4(call, plan, sv, mv, stream) : launch_mma8(call, plan, sv, mv, stream);
    }
    if (call.launch_count != nullptr) *call.launch_count += 2;
    const int rc = run_prepare(call.x, call.cols, call.bits, call.group, call.batch, base, call.path, stream);
    if (rc != QMR_OK) return rc;
    call.overlap = true;  // the preceding kernel is our prep, which writes no weights
    return run_stream(call, base, stream);
}

}  // namespace qmr
