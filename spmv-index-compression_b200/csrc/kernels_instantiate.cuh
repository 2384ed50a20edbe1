// kernels_instantiate.cuh — the switch from runtime (layout, T, P) to a kernel instantiation for the
// value type VALUE_TYPE, included by kernels_f64.cu, kernels_f32.cu and kernels_f16.cu.
#include "dispatch.hpp"

namespace spmvb200 {
namespace {

// A product kernel launched so that it may start while the previous kernel of the stream finishes (it
// waits for that kernel before it reads x or writes y; see allow_next_grid / wait_for_previous_grid).
template <class Kernel>
cudaError_t launch_product(Kernel kernel, int64_t blocks, int smem, cudaStream_t stream, const KernelArgs& a) {
  cudaLaunchConfig_t config{};
  config.gridDim = dim3((unsigned)blocks);
  config.blockDim = dim3(kTileBlock);
  config.dynamicSmemBytes = (size_t)smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, a);
}

template <class V, int L, int T, int P, int W>
cudaError_t run_tiles(const KernelArgs& a, cudaStream_t stream) {
  const int smem = a.smem_bytes;
  const int64_t blocks = a.vector_blocks + a.tile_ctas;
  if (blocks <= 0) return cudaSuccess;
  return launch_product(k_spmv_tiles<V, L, T, P, W>, blocks, smem, stream, a);
}

// Sets the shared-memory limit of the variant to smem and returns its resident CTAs per multiprocessor.
template <class V, int L, int T, int P, int W>
cudaError_t occupancy_of(int smem, int* blocks) {
  cudaError_t status = cudaFuncSetAttribute(k_spmv_tiles<V, L, T, P, W>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (status != cudaSuccess) return status;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, k_spmv_tiles<V, L, T, P, W>, kTileBlock, smem);
}

// mode 0: launch; mode 1: occupancy query into *blocks
template <class V, int L, int T, int P, int W = 2>
cudaError_t tiles_variant(int mode, const KernelArgs& a, cudaStream_t stream, int smem, int* blocks) {
  return mode == 0 ? run_tiles<V, L, T, P, W>(a, stream) : occupancy_of<V, L, T, P, W>(smem, blocks);
}

template <class V, int L, int T>
cudaError_t tiles_for_tpr(int physical_tpr, int mode, const KernelArgs& a, cudaStream_t stream, int smem, int* blocks) {
  switch (T / physical_tpr) {
    case 1:
      if (a.dense) return tiles_variant<V, L, T, T, DenseResidency<V>::value>(mode, a, stream, smem, blocks);
      return tiles_variant<V, L, T, T>(mode, a, stream, smem, blocks);
    case 2: if constexpr (T >= 2) return tiles_variant<V, L, T, T / 2>(mode, a, stream, smem, blocks); break;
    case 4: if constexpr (T >= 4) return tiles_variant<V, L, T, T / 4>(mode, a, stream, smem, blocks); break;
    case 8: if constexpr (T >= 8) return tiles_variant<V, L, T, T / 8>(mode, a, stream, smem, blocks); break;
    case 16: if constexpr (T >= 16) return tiles_variant<V, L, T, T / 16>(mode, a, stream, smem, blocks); break;
    default: break;
  }
  return cudaErrorInvalidValue;
}

template <class V, int L>
cudaError_t tiles_for_layout(int tpr, int physical_tpr, int mode, const KernelArgs& a, cudaStream_t stream, int smem, int* blocks) {
  if (!tile_variant_exists(tpr, physical_tpr)) return cudaErrorInvalidValue;
  switch (tpr) {
    case 2: return tiles_for_tpr<V, L, 2>(physical_tpr, mode, a, stream, smem, blocks);
    case 4: return tiles_for_tpr<V, L, 4>(physical_tpr, mode, a, stream, smem, blocks);
    case 8: return tiles_for_tpr<V, L, 8>(physical_tpr, mode, a, stream, smem, blocks);
    case 16: return tiles_for_tpr<V, L, 16>(physical_tpr, mode, a, stream, smem, blocks);
    case 32: return tiles_for_tpr<V, L, 32>(physical_tpr, mode, a, stream, smem, blocks);
    default: return cudaErrorInvalidValue;
  }
}

template <class V>
cudaError_t tiles_for_value(int layout, int tpr, int physical_tpr, int mode, const KernelArgs& a, cudaStream_t stream, int smem,
                            int* blocks) {
  switch (layout) {
    case SPMV_LAYOUT_I32: return tiles_for_layout<V, SPMV_LAYOUT_I32>(tpr, physical_tpr, mode, a, stream, smem, blocks);
    case SPMV_LAYOUT_I16: return tiles_for_layout<V, SPMV_LAYOUT_I16>(tpr, physical_tpr, mode, a, stream, smem, blocks);
    case SPMV_LAYOUT_R16: return tiles_for_layout<V, SPMV_LAYOUT_R16>(tpr, physical_tpr, mode, a, stream, smem, blocks);
    case SPMV_LAYOUT_LP:  return tiles_for_layout<V, SPMV_LAYOUT_LP>(tpr, physical_tpr, mode, a, stream, smem, blocks);
    case SPMV_LAYOUT_I8:  return tiles_for_layout<V, SPMV_LAYOUT_I8>(tpr, physical_tpr, mode, a, stream, smem, blocks);
    case SPMV_LAYOUT_R8:  return tiles_for_layout<V, SPMV_LAYOUT_R8>(tpr, physical_tpr, mode, a, stream, smem, blocks);
    default: return cudaErrorInvalidValue;
  }
}

template <class V, int L, int T>
cudaError_t run_vector(const KernelArgs& a, int64_t blocks, cudaStream_t stream) {
  if (blocks <= 0) return cudaSuccess;
  k_spmv_vector<V, L, T><<<(unsigned)blocks, kVectorBlock, 0, stream>>>(a);
  return cudaGetLastError();
}

template <class V, int L>
cudaError_t vector_for_layout(int tpr, const KernelArgs& a, int64_t blocks, cudaStream_t stream) {
  switch (tpr) {
    case 2: return run_vector<V, L, 2>(a, blocks, stream);
    case 4: return run_vector<V, L, 4>(a, blocks, stream);
    case 8: return run_vector<V, L, 8>(a, blocks, stream);
    case 16: return run_vector<V, L, 16>(a, blocks, stream);
    case 32: return run_vector<V, L, 32>(a, blocks, stream);
    default: return cudaErrorInvalidValue;
  }
}

// mode 0: launch k_spmv_classes over `blocks` CTAs; mode 1: raise its shared-memory limit to smem
template <class V, int L, int T>
cudaError_t classes_variant(int mode, const KernelArgs& a, int64_t blocks, int smem, cudaStream_t stream) {
  if (mode == 1) return cudaFuncSetAttribute(k_spmv_classes<V, L, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (blocks <= 0) return cudaSuccess;
  return launch_product(k_spmv_classes<V, L, T>, blocks, smem, stream, a);
}

template <class V, int L>
cudaError_t classes_for_layout(int tpr, int mode, const KernelArgs& a, int64_t blocks, int smem, cudaStream_t stream) {
  switch (tpr) {
    case 2: return classes_variant<V, L, 2>(mode, a, blocks, smem, stream);
    case 4: return classes_variant<V, L, 4>(mode, a, blocks, smem, stream);
    case 8: return classes_variant<V, L, 8>(mode, a, blocks, smem, stream);
    case 16: return classes_variant<V, L, 16>(mode, a, blocks, smem, stream);
    case 32: return classes_variant<V, L, 32>(mode, a, blocks, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <class V>
cudaError_t classes_for_value(int layout, int tpr, int mode, const KernelArgs& a, int64_t blocks, int smem, cudaStream_t stream) {
  switch (layout) {
    case SPMV_LAYOUT_I32: return classes_for_layout<V, SPMV_LAYOUT_I32>(tpr, mode, a, blocks, smem, stream);
    case SPMV_LAYOUT_I16: return classes_for_layout<V, SPMV_LAYOUT_I16>(tpr, mode, a, blocks, smem, stream);
    case SPMV_LAYOUT_R16: return classes_for_layout<V, SPMV_LAYOUT_R16>(tpr, mode, a, blocks, smem, stream);
    case SPMV_LAYOUT_LP:  return classes_for_layout<V, SPMV_LAYOUT_LP>(tpr, mode, a, blocks, smem, stream);
    case SPMV_LAYOUT_I8:  return classes_for_layout<V, SPMV_LAYOUT_I8>(tpr, mode, a, blocks, smem, stream);
    case SPMV_LAYOUT_R8:  return classes_for_layout<V, SPMV_LAYOUT_R8>(tpr, mode, a, blocks, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t LAUNCH_CLASSES_NAME(int layout, int tpr, const KernelArgs& a, int64_t blocks, int smem, cudaStream_t stream) {
  return classes_for_value<VALUE_TYPE>(layout, tpr, 0, a, blocks, smem, stream);
}

cudaError_t PREPARE_CLASSES_NAME(int layout, int tpr, int smem) {
  const KernelArgs unused{};
  return classes_for_value<VALUE_TYPE>(layout, tpr, 1, unused, 0, smem, nullptr);
}

cudaError_t LAUNCH_TILES_NAME(int layout, int tpr, int physical_tpr, const KernelArgs& a, cudaStream_t stream) {
  return tiles_for_value<VALUE_TYPE>(layout, tpr, physical_tpr, 0, a, stream, 0, nullptr);
}

int TILES_OCCUPANCY_NAME(int layout, int tpr, int physical_tpr, int smem, bool dense) {
  int blocks = 0;
  KernelArgs variant{};
  variant.dense = dense ? 1 : 0;
  if (tiles_for_value<VALUE_TYPE>(layout, tpr, physical_tpr, 1, variant, nullptr, smem, &blocks) != cudaSuccess) return 0;
  return blocks;
}

cudaError_t LAUNCH_VECTOR_NAME(int layout, int tpr, const KernelArgs& a, int64_t blocks, cudaStream_t stream) {
  switch (layout) {
    case SPMV_LAYOUT_I32: return vector_for_layout<VALUE_TYPE, SPMV_LAYOUT_I32>(tpr, a, blocks, stream);
    case SPMV_LAYOUT_I16: return vector_for_layout<VALUE_TYPE, SPMV_LAYOUT_I16>(tpr, a, blocks, stream);
    case SPMV_LAYOUT_R16: return vector_for_layout<VALUE_TYPE, SPMV_LAYOUT_R16>(tpr, a, blocks, stream);
    case SPMV_LAYOUT_LP:  return vector_for_layout<VALUE_TYPE, SPMV_LAYOUT_LP>(tpr, a, blocks, stream);
    case SPMV_LAYOUT_I8:  return vector_for_layout<VALUE_TYPE, SPMV_LAYOUT_I8>(tpr, a, blocks, stream);
    case SPMV_LAYOUT_R8:  return vector_for_layout<VALUE_TYPE, SPMV_LAYOUT_R8>(tpr, a, blocks, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace spmvb200
