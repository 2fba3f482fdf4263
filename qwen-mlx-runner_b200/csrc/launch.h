// Internal launch interfaces of the kernel families, one translation unit
// each (they compile in parallel): FP32 prep + register streaming + generic
// + embed (kernels_reg.cu), the FP32 TMA tile kernel (kernels_tile.cu) and
// the tensor-core kernel (kernels_mma.cu, built once per bit width).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "matrix_kernels.cuh"
#include "mma_stream.cuh"
#include "qmr_internal.h"

namespace qmr {

cudaLaunchAttribute pdl_attr();
int sm_count();
int log2i(uint32_t v);

// kernels_reg.cu
int launch_prep_fp32(const float *x, uint32_t cols, uint32_t bits, uint32_t batch, const ScratchView &sv,
                     cudaStream_t stream);
int launch_reg(const StreamArgs &a, int bits, bool bf16, uint32_t batch, int epi, bool overlap, cudaStream_t stream);

// kernels_tile.cu
bool tile_eligible(const FastCall &c);
int launch_tile_call(const FastCall &c, const ScratchView &sv, cudaStream_t stream);

// kernels_mma.cu
int launch_mma_prep_bits(int bits, const float *x, uint32_t cols, uint32_t group, uint32_t batch,
                         const MmaPrepView &v, cudaStream_t stream);
int launch_mma_bits(int bits, const MmaArgs &a, bool bf16, uint32_t group, uint32_t batch, int epi, bool overlap,
                    cudaStream_t stream);
int launch_mma4(const MmaArgs &a, bool bf16, uint32_t group, uint32_t batch, int epi, bool overlap,
                cudaStream_t stream);
int launch_mma8(const MmaArgs &a, bool bf16, uint32_t group, uint32_t batch, int epi, bool overlap,
                cudaStream_t stream);
int launch_mma_prep4(const float *x, uint32_t cols, uint32_t group, uint32_t batch, const MmaPrepView &v,
                     cudaStream_t stream);
int launch_mma_prep8(const float *x, uint32_t cols, uint32_t group, uint32_t batch, const MmaPrepView &v,
                     cudaStream_t stream);

}  // namespace qmr
