// Internal launch interfaces of the kernel families, one translation unit
// each (they compile in parallel): FP32 prep + register streaming + generic
// + embed (kernels_reg.cu), the FP32 TMA tile kernel (kernels_tile.cu) and
// the tensor-core kernel (kernels_mma.cu, built once per bit width).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "matrix_kernels.cuh"
#include "mma_stream.cuh"
#include "qmr_internal.h"

namespace qmr {

cudaLaunchAttribute pdl_attr();
int sm_count();
// Clusters of kc CTAs (one CTA per SM) that fit on the device at once; 0 if
// the occupancy query failed.
int mma_cluster_capacity(int kc);
int log2i(uint32_t v);

// kernels_reg.cu
int launch_prep_fp32(const float *x, uint32_t cols, uint32_t bits, uint32_t batch, const ScratchView &sv,
                     cudaStream_t stream);
int launch_reg(const StreamArgs &a, int bits, bool bf16, uint32_t batch, int epi, bool overlap, cudaStream_t stream);

// kernels_tile.cu
bool tile_eligible(const FastCall &c);
int launch_tile_call(const FastCall &c, const ScratchView &sv, cudaStream_t stream);
// row_stride_elems: elements from one row to the next (0: row_elems).
int tensor_map_2d(CUtensorMap *out, const void *base, int esize, uint64_t row_elems, uint64_t rows, uint32_t box_x,
                  uint32_t box_y, bool swizzle128, uint64_t row_stride_elems = 0);
unsigned int *device_error_word();

// Launch shape of the tensor-core kernel for one call (matrix.cu).
struct MmaPlan {
    int kc;           // column slices = CTAs per cluster
    int clusters;
    int ctas;
    int stages;       // ring slots per warp
    int pieces;       // shared-memory piece slots per warp
    int nwin;         // 512/1024-column windows of the matrix
    int ngroups_pad;  // groups of the padded activation image
    int tiles;        // 16-row tiles
    int warps;        // warps per CTA
    uint32_t smem, off_image, off_table, off_pieces, off_part, off_bars;
};
// meta_stride: metadata elements per row (0: cols / group); it must be a
// multiple of 8 (16-byte rows for the metadata tensor maps).
bool mma_plan(uint32_t bits, uint32_t group, uint32_t rows, uint32_t cols, uint32_t batch, int epi, bool bf16,
              MmaPlan *p, uint32_t meta_stride = 0);

// kernels_mma.cu (one translation unit per bit width)
int launch_mma_prep_bits(int bits, const float *x, uint32_t cols, uint32_t group, uint32_t batch, int ngroups_pad,
                         const MmaImageView &v, cudaStream_t stream);
int launch_mma4(const FastCall &c, const MmaPlan &p, const ScratchView &sv, const MmaImageView &v,
                cudaStream_t stream);
int launch_mma8(const FastCall &c, const MmaPlan &p, const ScratchView &sv, const MmaImageView &v,
                cudaStream_t stream);
int launch_mma_prep4(const float *x, uint32_t cols, uint32_t group, uint32_t batch, int ngroups_pad,
                     const MmaImageView &v, cudaStream_t stream);
int launch_mma_prep8(const float *x, uint32_t cols, uint32_t group, uint32_t batch, int ngroups_pad,
                     const MmaImageView &v, cudaStream_t stream);

}  // namespace qmr
