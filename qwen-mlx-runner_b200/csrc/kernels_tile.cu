// The FP32 warp-specialised TMA tile kernel: tensor maps, launch shape.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "launch.h"
#include "tile.cuh"

namespace qmr {

namespace {

constexpr int kConsumers = 8;  // consumer warps of the tile kernel
constexpr int kSmemBudget = 220 * 1024;


PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Encoded maps cached by (address, kind, shape, box): the engine and the
// benchmarks reuse a handful of matrices, so encoding happens once each.
using MapKey = std::tuple<const void *, int, uint64_t, uint64_t, uint32_t, uint32_t, bool, uint64_t>;
std::mutex g_map_mu;
std::map<MapKey, CUtensorMap> g_maps;

}  // namespace

// 2-D map over a row-major array of `rows` rows of `row_elems` elements of
// `esize` bytes, box = box_x elements x box_y rows, zero fill out of range,
// optionally with the 128-byte shared-memory swizzle.
int tensor_map_2d(CUtensorMap *out, const void *base, int esize, uint64_t row_elems, uint64_t rows, uint32_t box_x,
                  uint32_t box_y, bool swizzle128, uint64_t row_stride_elems) {
    if (row_stride_elems == 0) row_stride_elems = row_elems;
    const MapKey key{base, esize, row_elems, rows, box_x, box_y, swizzle128, row_stride_elems};
    {
        std::lock_guard<std::mutex> lock(g_map_mu);
        auto it = g_maps.find(key);
        if (it != g_maps.end()) {
            *out = it->second;
            return QMR_OK;
        }
    }
    auto fn = encode_fn();
    if (fn == nullptr) return fail(QMR_ECUDA, "cuTensorMapEncodeTiled is unavailable");
    const CUtensorMapDataType dt = esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
    const cuuint64_t dims[2] = {row_elems, rows};
    const cuuint64_t strides[1] = {row_stride_elems * (uint64_t)esize};
    const cuuint32_t box[2] = {box_x, box_y};
    const cuuint32_t es[2] = {1, 1};
    CUtensorMap m;
    const CUresult r = fn(&m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(QMR_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    std::lock_guard<std::mutex> lock(g_map_mu);
    if (g_maps.size() > 4096) g_maps.clear();
    g_maps[key] = m;
    *out = m;
    return QMR_OK;
}

namespace {

int tensor_map(CUtensorMap *out, const void *base, int esize, uint64_t row_elems, uint64_t rows, uint32_t box_x,
               uint32_t box_y) {
    return tensor_map_2d(out, base, esize, row_elems, rows, box_x, box_y, false);
}

// ---- tile kernel -------------------------------------------------------------

struct TileMaps {
    CUtensorMap w, s, b, w2, s2, b2;
};

template <int BITS, int B, int RW, bool BF16, int EPI>
int launch_tile_t(const TileMaps &m, TileArgs a, bool overlap, cudaStream_t stream) {
    constexpr int NM = (EPI == 1) ? 2 : 1;
    constexpr int TR = kConsumers * RW;
    const TileLayout L = tile_layout(NM, kConsumers, RW, B, a.group_shift, a.meta_bytes, block_floats<BITS>());
    int stages = (int)((kSmemBudget - 64) / (L.stage_bytes + 2 * sizeof(uint64_t)));
    if (stages > 8) stages = 8;
    if (stages < 2) return fail(QMR_EUNSUPPORTED, "a %u-byte stage does not fit shared memory", L.stage_bytes);
    a.stages = stages;
    const size_t smem = (size_t)stages * L.stage_bytes + (size_t)stages * 2 * sizeof(uint64_t);
    // Split-K bookkeeping: at most 4 tiles per row range use the counters.
    const int units = (a.rows + RW - 1) / RW;
    const int rows_per_range = ((units + a.ranges - 1) / a.ranges) * RW;
    if (a.ksplit > 1 && ((rows_per_range + TR - 1) / TR > 4 || a.ranges > 256))
        return fail(QMR_EUNSUPPORTED, "split-K launch shape exceeds the counter space");
    auto kern = tile_kernel<BITS, B, RW, kConsumers, BF16, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.ranges * a.ksplit, 1, 1);
    cfg.blockDim = dim3(32 * (kConsumers + 1), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = overlap ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, m.w, m.s, m.b, m.w2, m.s2, m.b2, a);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "tile kernel launch failed: %s", cudaGetErrorString(e));
    return QMR_OK;
}

template <int BITS, bool BF16, int EPI>
int launch_tile_b(const TileMaps &m, const TileArgs &a, uint32_t batch, int RW, bool ov, cudaStream_t stream) {
    if constexpr (EPI != 1) {
        if (RW == 8) {
            switch (batch) {
                case 1: return launch_tile_t<BITS, 1, 8, BF16, EPI>(m, a, ov, stream);
                case 2: return launch_tile_t<BITS, 2, 8, BF16, EPI>(m, a, ov, stream);
                case 3: return launch_tile_t<BITS, 3, 8, BF16, EPI>(m, a, ov, stream);
                default: return launch_tile_t<BITS, 4, 8, BF16, EPI>(m, a, ov, stream);
            }
        }
    }
    switch (batch) {
        case 1: return launch_tile_t<BITS, 1, 4, BF16, EPI>(m, a, ov, stream);
        case 2: return launch_tile_t<BITS, 2, 4, BF16, EPI>(m, a, ov, stream);
        case 3: return launch_tile_t<BITS, 3, 4, BF16, EPI>(m, a, ov, stream);
        default: return launch_tile_t<BITS, 4, 4, BF16, EPI>(m, a, ov, stream);
    }
}

template <int EPI>
int launch_tile(const TileMaps &m, const TileArgs &a, int bits, bool bf16, uint32_t batch, int RW, bool ov,
                cudaStream_t stream) {
    if (bits == 4)
        return bf16 ? launch_tile_b<4, true, EPI>(m, a, batch, RW, ov, stream)
                    : launch_tile_b<4, false, EPI>(m, a, batch, RW, ov, stream);
    return bf16 ? launch_tile_b<8, true, EPI>(m, a, batch, RW, ov, stream)
                : launch_tile_b<8, false, EPI>(m, a, batch, RW, ov, stream);
}

}  // namespace

bool tile_eligible(const FastCall &c) {
    const uint32_t gpc = c.group / (128 / c.bits);
    const uint64_t meta = c.bf16 ? 2 : 4;
    const uint64_t nchunks = (uint64_t)c.cols * c.bits / 128;
    if ((nchunks / gpc) * meta % 16 != 0) return false;                    // metadata row stride
    if (((uint64_t)kSliceChunks / gpc) * meta % 16 != 0) return false;     // metadata box width
    auto al = [](const void *p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
    return al(c.w) && al(c.s) && al(c.b) && al(c.w2) && al(c.s2) && al(c.b2);
}

namespace {

// Column split across CTAs: the share of SM time doing useful rows for
// ksplit = 1..4, on tiles of 64 rows; the smallest split within 5% of the best.
int choose_ksplit(int rows, int nslices, int sms, int nm, uint32_t batch) {
    const int units = (rows + 7) / 8;
    double best = -1.0;
    int best_ks = 1;
    for (int ks = 1; ks <= 4 && ks <= nslices; ++ks) {
        if ((size_t)ks * nm * batch * rows > kPartialFloats && ks > 1) break;
        int ranges = sms / ks;
        if (ranges > units) ranges = units;
        if (ranges < 1) ranges = 1;
        const int rpr = ((units + ranges - 1) / ranges) * 8;
        const int tiles = (rpr + 63) / 64;
        if (ks > 1 && (tiles > 4 || ranges > 256)) continue;
        const double eff = (double)rows / ((double)ranges * tiles * 64) * ((double)ranges * ks / sms);
        if (eff > best * 1.05) {
            best = eff;
            best_ks = ks;
        }
    }
    return best_ks;
}

}  // namespace

int launch_tile_call(const FastCall &c, const ScratchView &sv, cudaStream_t stream) {
    const int ce = 128 / (int)c.bits;
    const int gpc = (int)c.group / ce;
    const int meta = c.bf16 ? 2 : 4;
    const int nchunks = (int)((uint64_t)c.cols * c.bits / 128);
        const int NM = c.epilogue == 1 ? 2 : 1;
        const int RW = (c.r2 || c.epilogue == 1) ? 4 : 8;
        const int sms = sm_count();
        const int nslices = (nchunks + kSliceChunks - 1) / kSliceChunks;
        const int ksplit = choose_ksplit((int)c.rows, nslices, sms, NM, c.batch);
        const int units = ((int)c.rows + RW - 1) / RW;
        int ranges = sms / ksplit;
        if (ranges > units) ranges = units;
        if (ranges < 1) ranges = 1;
        const int groups = nchunks / gpc;
        const uint32_t slice_groups = (uint32_t)(kSliceChunks / gpc);
        const uint32_t tr = (uint32_t)(kConsumers * RW);
        TileMaps maps;
        memset(&maps, 0, sizeof maps);
        int rc = tensor_map(&maps.w, c.w, 4, (uint64_t)nchunks * 4, c.rows, kSliceWords, (uint32_t)RW);
        if (rc == QMR_OK) rc = tensor_map(&maps.s, c.s, meta, (uint64_t)groups, c.rows, slice_groups, tr);
        if (rc == QMR_OK) rc = tensor_map(&maps.b, c.b, meta, (uint64_t)groups, c.rows, slice_groups, tr);
        if (rc == QMR_OK && NM == 2) {
            rc = tensor_map(&maps.w2, c.w2, 4, (uint64_t)nchunks * 4, c.rows, kSliceWords, (uint32_t)RW);
            if (rc == QMR_OK) rc = tensor_map(&maps.s2, c.s2, meta, (uint64_t)groups, c.rows, slice_groups, tr);
            if (rc == QMR_OK) rc = tensor_map(&maps.b2, c.b2, meta, (uint64_t)groups, c.rows, slice_groups, tr);
        }
        if (rc != QMR_OK) return rc;
        TileArgs a = {};
        a.xp = sv.xp;
        a.cf = sv.cf;
        a.y = c.y;
        a.partial = sv.partial;
        a.range_counter = sv.counters;
        a.done_counter = sv.done;
        a.keys = sv.keys;
        a.argmax = c.argmax;
        a.best_key_out = reinterpret_cast<unsigned long long *>(c.best_key);
        a.rows = (int)c.rows;
        a.nchunks = nchunks;
        a.group_shift = log2i((uint32_t)gpc);
        a.meta_bytes = meta;
        a.ystride = (int)c.rows;
        a.row_base = (int)c.row_base;
        a.ranges = ranges;
        a.ksplit = ksplit;
        switch (c.epilogue) {
            case 0: return launch_tile<0>(maps, a, (int)c.bits, c.bf16, c.batch, RW, c.overlap, stream);
            case 1: return launch_tile<1>(maps, a, (int)c.bits, c.bf16, c.batch, RW, c.overlap, stream);
            default: return launch_tile<2>(maps, a, (int)c.bits, c.bf16, c.batch, RW, c.overlap, stream);
        }
    }

// Device address of the shared error word on the current device.
unsigned int *device_error_word() {
    static std::mutex mu;
    static void *addr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr && cudaGetSymbolAddress(&addr[dev], g_qmr_device_error) != cudaSuccess) addr[dev] = nullptr;
    return static_cast<unsigned int *>(addr[dev]);
}

int device_error(int *code, bool clear) {
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_qmr_device_error, sizeof v);
    if (e != cudaSuccess) return fail(QMR_ECUDA, "reading the device error word: %s", cudaGetErrorString(e));
    if (clear && v != 0) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_qmr_device_error, &zero, sizeof zero);
        if (e != cudaSuccess) return fail(QMR_ECUDA, "clearing the device error word: %s", cudaGetErrorString(e));
    }
    *code = (int)v;
    return QMR_OK;
}

}  // namespace qmr
