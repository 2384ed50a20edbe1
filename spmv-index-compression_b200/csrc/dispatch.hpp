// dispatch.hpp — host entry points into the kernel instantiations (one translation unit per value type).
#pragma once

#include <cuda_runtime.h>

#include "kernels.cuh"

namespace spmvb200 {

// The kernel family of an operator: its dtype (SPMV_F64, SPMV_F32, SPMV_F16), or kKernelHalfSums for
// FP16 values summed in FP16 (SPMV_ACCUMULATE_HALF).
constexpr int kKernelHalfSums = 3;

// Physical threads per row the tile kernel is built for: P = T / S with S in {1, 2, 4, 8, 16}.
inline bool tile_variant_exists(int tpr, int physical_tpr) {
  if (physical_tpr < 1 || physical_tpr > tpr || tpr % physical_tpr != 0) return false;
  const int slots = tpr / physical_tpr;
  return slots == 1 || slots == 2 || slots == 4 || slots == 8 || slots == 16;
}

// k_spmv_tiles over a.vector_blocks + a.tile_ctas CTAs with the shared memory of the tile plan.
cudaError_t launch_tiles_f64(int layout, int tpr, int physical_tpr, const KernelArgs& a, cudaStream_t stream);
cudaError_t launch_tiles_f32(int layout, int tpr, int physical_tpr, const KernelArgs& a, cudaStream_t stream);
cudaError_t launch_tiles_f16(int layout, int tpr, int physical_tpr, const KernelArgs& a, cudaStream_t stream);
cudaError_t launch_tiles_f16h(int layout, int tpr, int physical_tpr, const KernelArgs& a, cudaStream_t stream);
// Resident k_spmv_tiles CTAs per multiprocessor with `smem` bytes of dynamic shared memory (0 if the
// variant does not exist); also raises the kernel's shared-memory limit to smem. dense: the dense variant
// (KernelArgs::dense) where P = T.
int tiles_occupancy_f64(int layout, int tpr, int physical_tpr, int smem, bool dense);
int tiles_occupancy_f32(int layout, int tpr, int physical_tpr, int smem, bool dense);
int tiles_occupancy_f16(int layout, int tpr, int physical_tpr, int smem, bool dense);
int tiles_occupancy_f16h(int layout, int tpr, int physical_tpr, int smem, bool dense);
// k_spmv_vector over `blocks` CTAs of kVectorBlock threads.
cudaError_t launch_vector_f64(int layout, int tpr, const KernelArgs& a, int64_t blocks, cudaStream_t stream);
cudaError_t launch_vector_f32(int layout, int tpr, const KernelArgs& a, int64_t blocks, cudaStream_t stream);
cudaError_t launch_vector_f16(int layout, int tpr, const KernelArgs& a, int64_t blocks, cudaStream_t stream);
cudaError_t launch_vector_f16h(int layout, int tpr, const KernelArgs& a, int64_t blocks, cudaStream_t stream);

// k_spmv_classes over `blocks` CTAs of kTileBlock threads with `smem` bytes of dynamic shared memory; the
// prepare functions raise the kernel's shared-memory limit to smem.
cudaError_t launch_classes_f64(int layout, int tpr, const KernelArgs& a, int64_t blocks, int smem, cudaStream_t stream);
cudaError_t launch_classes_f32(int layout, int tpr, const KernelArgs& a, int64_t blocks, int smem, cudaStream_t stream);
cudaError_t launch_classes_f16(int layout, int tpr, const KernelArgs& a, int64_t blocks, int smem, cudaStream_t stream);
cudaError_t launch_classes_f16h(int layout, int tpr, const KernelArgs& a, int64_t blocks, int smem, cudaStream_t stream);
cudaError_t prepare_classes_f64(int layout, int tpr, int smem);
cudaError_t prepare_classes_f32(int layout, int tpr, int smem);
cudaError_t prepare_classes_f16(int layout, int tpr, int smem);
cudaError_t prepare_classes_f16h(int layout, int tpr, int smem);

inline cudaError_t launch_classes(int dtype, int layout, int tpr, const KernelArgs& a, int64_t blocks, int smem, cudaStream_t stream) {
  switch (dtype) {
    case SPMV_F64: return launch_classes_f64(layout, tpr, a, blocks, smem, stream);
    case SPMV_F32: return launch_classes_f32(layout, tpr, a, blocks, smem, stream);
    case kKernelHalfSums: return launch_classes_f16h(layout, tpr, a, blocks, smem, stream);
    default:       return launch_classes_f16(layout, tpr, a, blocks, smem, stream);
  }
}

inline cudaError_t prepare_classes(int dtype, int layout, int tpr, int smem) {
  switch (dtype) {
    case SPMV_F64: return prepare_classes_f64(layout, tpr, smem);
    case SPMV_F32: return prepare_classes_f32(layout, tpr, smem);
    case kKernelHalfSums: return prepare_classes_f16h(layout, tpr, smem);
    default:       return prepare_classes_f16(layout, tpr, smem);
  }
}

inline cudaError_t launch_tiles(int dtype, int layout, int tpr, int physical_tpr, const KernelArgs& a, cudaStream_t stream) {
  switch (dtype) {
    case SPMV_F64: return launch_tiles_f64(layout, tpr, physical_tpr, a, stream);
    case SPMV_F32: return launch_tiles_f32(layout, tpr, physical_tpr, a, stream);
    case kKernelHalfSums: return launch_tiles_f16h(layout, tpr, physical_tpr, a, stream);
    default:       return launch_tiles_f16(layout, tpr, physical_tpr, a, stream);
  }
}

inline int tiles_occupancy(int dtype, int layout, int tpr, int physical_tpr, int smem, bool dense) {
  switch (dtype) {
    case SPMV_F64: return tiles_occupancy_f64(layout, tpr, physical_tpr, smem, dense);
    case SPMV_F32: return tiles_occupancy_f32(layout, tpr, physical_tpr, smem, dense);
    case kKernelHalfSums: return tiles_occupancy_f16h(layout, tpr, physical_tpr, smem, dense);
    default:       return tiles_occupancy_f16(layout, tpr, physical_tpr, smem, dense);
  }
}

inline cudaError_t launch_vector(int dtype, int layout, int tpr, const KernelArgs& a, int64_t blocks, cudaStream_t stream) {
  switch (dtype) {
    case SPMV_F64: return launch_vector_f64(layout, tpr, a, blocks, stream);
    case SPMV_F32: return launch_vector_f32(layout, tpr, a, blocks, stream);
    case kKernelHalfSums: return launch_vector_f16h(layout, tpr, a, blocks, stream);
    default:       return launch_vector_f16(layout, tpr, a, blocks, stream);
  }
}

}  // namespace spmvb200
