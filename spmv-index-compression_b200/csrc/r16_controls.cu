// r16_controls.cu — the reference's control builds of CSR-r16 (bench_csr_width.cu:34-42, :343-432), each
// changing only how the row-relative offsets reach the global-memory kernel (one group of T threads per row,
// the raw launch's mapping): LANE reads the offsets laid out lane by lane (16-bit loads), PAIR the same stream
// two offsets to a 32-bit load, WIDE 32-bit offsets, UNROLL16 the 16-bit offsets with the loop unrolled 16
// times at FP16. The summation order is the reference's, so every control gives CSR-i32's bits.
#include <cuda_runtime.h>

#include "capi_internal.hpp"
#include "dispatch.hpp"

namespace spmvb200 {
namespace {

// Lane L of a row's group reads its offsets from position L * quotient + min(L, remainder) of the row's
// place in the lane-major stream; PAIR loads the 32-bit word holding two of them, which may straddle two
// lanes (the stream is padded to whole words).
template <class V, int T, bool PAIR>
__global__ void __launch_bounds__(kVectorBlock) k_r16_lane(const KernelArgs a) {
  using VT = ValueTraits<V>;
  using Acc = typename VT::Acc;
  const V* values = static_cast<const V*>(a.values);
  const V* x = static_cast<const V*>(a.x);
  V* y = static_cast<V*>(a.y);
  const uint16_t* offsets = static_cast<const uint16_t*>(a.columns);
  const int lane = threadIdx.x & (T - 1);
  const int64_t group = ((int64_t)blockIdx.x * kVectorBlock + threadIdx.x) / T;
  const int64_t groups = ((int64_t)gridDim.x * kVectorBlock) / T;
  for (int64_t first = 0; first < a.rows; first += groups) {   // the same trip count on every thread
    const int64_t row = first + group;
    Acc sum = Acc(0);
    if (row < a.rows) {
      const int begin = load_readonly(a.row_ptr + row), length = load_readonly(a.row_ptr + row + 1) - begin;
      const int base = load_readonly(a.row_base + row);
      const int quotient = length / T, remainder = length - quotient * T;
      const int count = quotient + (lane < remainder ? 1 : 0);
      int position = begin + lane * quotient + (lane < remainder ? lane : remainder);
      int entry = begin + lane;
      if constexpr (PAIR) {
        const uint32_t* words = reinterpret_cast<const uint32_t*>(offsets);
        uint32_t word = count > 0 ? load_readonly(words + (position >> 1)) : 0u;
        for (int k = 0; k < count; ++k, ++position, entry += T) {
          if (k > 0 && (position & 1) == 0) word = load_readonly(words + (position >> 1));
          const int offset = (int)((position & 1) ? (word >> 16) : (word & 0xffffu));
          sum = VT::fma(VT::widen(load_readonly(values + entry)), VT::widen(load_readonly(x + base + offset)), sum);
        }
      } else {
        for (int k = 0; k < count; ++k, ++position, entry += T)
          sum = VT::fma(VT::widen(load_readonly(values + entry)),
                        VT::widen(load_readonly(x + base + (int)load_readonly(offsets + position))), sum);
      }
    }
#pragma unroll
    for (int offset = T / 2; offset > 0; offset >>= 1) sum = VT::add(sum, __shfl_down_sync(0xffffffffu, sum, offset, T));
    if (lane == 0 && row < a.rows) y[row] = VT::narrow(sum);
  }
}

// WIDE: the vector path over 32-bit offsets; UNROLL16: over 16-bit offsets, unrolled 16 times at FP16 (the
// other value types keep the raw launch's unroll, as the control build keeps theirs).
template <class V, int LAYOUT, int T, int UNROLL>
__global__ void __launch_bounds__(kVectorBlock) k_r16_vector(const KernelArgs a) {
  vector_rows<V, LAYOUT, T, kVectorBlock, UNROLL>(a, blockIdx.x, gridDim.x);
}

template <class V, int T>
cudaError_t launch_control(int control, const KernelArgs& a, int64_t blocks, cudaStream_t stream) {
  if (blocks <= 0) return cudaSuccess;
  constexpr int kUnroll16 = std::is_same<V, __half>::value ? 16 : 4;
  switch (control) {
    case SPMV_R16_CONTROL_LANE: k_r16_lane<V, T, false><<<(unsigned)blocks, kVectorBlock, 0, stream>>>(a); break;
    case SPMV_R16_CONTROL_PAIR: k_r16_lane<V, T, true><<<(unsigned)blocks, kVectorBlock, 0, stream>>>(a); break;
    case SPMV_R16_CONTROL_WIDE: k_r16_vector<V, kLayoutR16Wide, T, 4><<<(unsigned)blocks, kVectorBlock, 0, stream>>>(a); break;
    case SPMV_R16_CONTROL_UNROLL16:
      k_r16_vector<V, SPMV_LAYOUT_R16, T, kUnroll16><<<(unsigned)blocks, kVectorBlock, 0, stream>>>(a);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <class V>
cudaError_t launch_for_tpr(int control, int tpr, const KernelArgs& a, int64_t blocks, cudaStream_t stream) {
  switch (tpr) {
    case 2: return launch_control<V, 2>(control, a, blocks, stream);
    case 4: return launch_control<V, 4>(control, a, blocks, stream);
    case 8: return launch_control<V, 8>(control, a, blocks, stream);
    case 16: return launch_control<V, 16>(control, a, blocks, stream);
    case 32: return launch_control<V, 32>(control, a, blocks, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace
}  // namespace spmvb200

using namespace spmvb200;

extern "C" int spmv_launch_r16_control(int control, int dtype, int tpr, const spmv_device_matrix* matrix, void* stream) {
  return guarded([&] {
    require(control >= SPMV_R16_CONTROL_LANE && control <= SPMV_R16_CONTROL_UNROLL16, "unknown CSR-r16 control");
    require(matrix, "matrix is required");
    value_bytes_of(dtype);
    require(valid_tpr(tpr), "threads per row must be 2, 4, 8, 16 or 32");
    require(matrix->rows >= 0 && matrix->row_ptr && matrix->row_base && matrix->columns && matrix->values && matrix->x &&
                matrix->y,
            "missing arrays");
    if (control == SPMV_R16_CONTROL_PAIR)
      require(reinterpret_cast<uintptr_t>(matrix->columns) % 4 == 0, "the lane-major stream must be 4-byte aligned");
    KernelArgs a{};
    a.rows = matrix->rows;
    a.cols = matrix->cols;
    a.row_ptr = matrix->row_ptr;
    a.columns = matrix->columns;
    a.row_base = matrix->row_base;
    a.values = matrix->values;
    a.x = matrix->x;
    a.y = matrix->y;
    a.row_list = nullptr;
    a.row_count = matrix->rows;
    // one vector of T threads per row, as the reference launches (bench_csr_width.cu:575-577)
    const int64_t blocks = ((int64_t)matrix->rows * tpr + kVectorBlock - 1) / kVectorBlock;
    require(blocks <= 0x7fffffff, "too many rows for one launch");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t status = cudaErrorInvalidValue;
    switch (dtype) {
      case SPMV_F64: status = launch_for_tpr<double>(control, tpr, a, blocks, s); break;
      case SPMV_F32: status = launch_for_tpr<float>(control, tpr, a, blocks, s); break;
      default: status = launch_for_tpr<__half>(control, tpr, a, blocks, s); break;
    }
    if (status != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("CSR-r16 control launch: ") + cudaGetErrorString(status));
  });
}
