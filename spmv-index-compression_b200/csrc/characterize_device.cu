// characterize_device.cu — the characterization CSV of src/characterize_matrix.cpp with its row-parallel
// metrics computed on the GPU: per row (one thread each) the span, the distance to the diagonal, the
// 8/16-bit fit counts, the lane iterations at every T, the windowed segments and the distinct consecutive
// sectors of x at each value size, summed by warp reductions; the span percentiles by a radix select over
// the spans held on the device (four 8-bit digit histograms per percentile). The FIFO gather model replays
// one ordered stream of sector accesses through each cache, which is sequential by definition: its twelve
// replays (3 value sizes x 4 capacities) run as twelve host threads while the GPU works. The output is
// byte for byte the host characterization's (and so the reference tool's).
#include <cuda_runtime.h>

#include <cstring>
#include <thread>

#include "capi_internal.hpp"
#include "characterize.hpp"

namespace spmvb200 {
namespace {

struct RowTotals {
  unsigned long long empty_rows, rows8, rows16, nnz8, nnz16, span_sum, segments8, segments16, bandwidth, span_max;
  unsigned long long occupied[5], iterations[5], longest[5];
  unsigned long long sectors[3];
};

__device__ __forceinline__ unsigned long long warp_sum(unsigned long long value) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) value += __shfl_down_sync(0xffffffffu, value, offset);
  return value;
}

__device__ __forceinline__ unsigned long long warp_max(unsigned long long value) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) value = max(value, __shfl_down_sync(0xffffffffu, value, offset));
  return value;
}

// One thread per row, grid-stride; every thread of the grid reaches the warp reductions.
__global__ void __launch_bounds__(256) k_characterize_rows(const int* __restrict__ row_ptr, const int* __restrict__ col,
                                                           int rows, int* __restrict__ spans, RowTotals* totals) {
  unsigned long long empty = 0, rows8 = 0, rows16 = 0, nnz8 = 0, nnz16 = 0, span_sum = 0, segments8 = 0,
                     segments16 = 0, bandwidth = 0, span_max = 0;
  unsigned long long occupied[5] = {0, 0, 0, 0, 0}, iterations[5] = {0, 0, 0, 0, 0}, longest[5] = {0, 0, 0, 0, 0};
  unsigned long long sectors[3] = {0, 0, 0};
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += stride) {
    const int row = (int)r;
    const int begin = row_ptr[row], end = row_ptr[row + 1], length = end - begin;
    int span = 0;
    if (length == 0) {
      ++empty;
    } else {
      const int first = col[begin], last = col[end - 1];
      span = last - first;
      const long long to_first = llabs((long long)row - first), to_last = llabs((long long)row - last);
      bandwidth = max(bandwidth, (unsigned long long)max(to_first, to_last));
    }
    spans[row] = span;
    span_sum += (unsigned long long)span;
    span_max = max(span_max, (unsigned long long)span);
    if (span < 256) { ++rows8; nnz8 += (unsigned long long)length; }
    if (span < 65536) { ++rows16; nnz16 += (unsigned long long)length; }
#pragma unroll
    for (int t = 0; t < 5; ++t) {
      const unsigned long long threads = 2ull << t;
      const unsigned long long row_iterations = ((unsigned long long)length + threads - 1) / threads;
      occupied[t] += row_iterations * threads;
      iterations[t] += row_iterations;
      longest[t] = max(longest[t], row_iterations);
    }
    // a segment starts at the row's first entry and wherever a column lies a window or more past the
    // segment's base (count_windowed_segments, characterize_matrix.cpp:167); a sector of x counts when it
    // differs from the previous entry's (measure_gather_traffic, :92)
    int base8 = 0, base16 = 0;
    long long previous[3] = {-1, -1, -1};
    for (int entry = begin; entry < end; ++entry) {
      const int column = col[entry];
      if (entry == begin || (long long)column - base8 >= 256) { base8 = column; ++segments8; }
      if (entry == begin || (long long)column - base16 >= 65536) { base16 = column; ++segments16; }
#pragma unroll
      for (int v = 0; v < 3; ++v) {
        const long long sector = (long long)column * (8 >> v) / 32;
        if (sector != previous[v]) ++sectors[v];
        previous[v] = sector;
      }
    }
  }
  const bool lead = (threadIdx.x & 31) == 0;
  auto add = [&](unsigned long long* target, unsigned long long value) {
    value = warp_sum(value);
    if (lead && value) atomicAdd(target, value);
  };
  auto keep_max = [&](unsigned long long* target, unsigned long long value) {
    value = warp_max(value);
    if (lead && value) atomicMax(target, value);
  };
  add(&totals->empty_rows, empty);
  add(&totals->rows8, rows8);
  add(&totals->rows16, rows16);
  add(&totals->nnz8, nnz8);
  add(&totals->nnz16, nnz16);
  add(&totals->span_sum, span_sum);
  add(&totals->segments8, segments8);
  add(&totals->segments16, segments16);
  keep_max(&totals->bandwidth, bandwidth);
  keep_max(&totals->span_max, span_max);
#pragma unroll
  for (int t = 0; t < 5; ++t) {
    add(&totals->occupied[t], occupied[t]);
    add(&totals->iterations[t], iterations[t]);
    keep_max(&totals->longest[t], longest[t]);
  }
#pragma unroll
  for (int v = 0; v < 3; ++v) add(&totals->sectors[v], sectors[v]);
}

// Histogram of the 8-bit digit at `shift` of the spans whose bits under `mask` equal `prefix`.
__global__ void __launch_bounds__(256) k_span_digits(const int* __restrict__ spans, int rows, unsigned prefix,
                                                     unsigned mask, int shift, unsigned long long* histogram) {
  __shared__ unsigned counts[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) counts[i] = 0;
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += stride) {
    const unsigned key = (unsigned)spans[r];
    if ((key & mask) == prefix) atomicAdd(&counts[(key >> shift) & 255u], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    if (counts[i]) atomicAdd(&histogram[i], (unsigned long long)counts[i]);
}

void check(cudaError_t status, const char* what) {
  if (status != cudaSuccess)
    fail(status == cudaErrorMemoryAllocation ? SPMV_ERR_OUT_OF_MEMORY : SPMV_ERR_CUDA,
         std::string(what) + ": " + cudaGetErrorString(status));
}

template <class T>
struct Device {
  T* data = nullptr;
  explicit Device(size_t count) { check(cudaMalloc(reinterpret_cast<void**>(&data), sizeof(T) * std::max<size_t>(count, 1)), "cudaMalloc"); }
  ~Device() {
    if (data) cudaFree(data);
  }
  Device(const Device&) = delete;
  Device& operator=(const Device&) = delete;
};

// The k-th smallest span (0-based): four passes over 8-bit digits, most significant first.
int select_span(const int* spans, int rows, unsigned long long k, unsigned long long* histogram, int blocks) {
  unsigned prefix = 0, mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    check(cudaMemset(histogram, 0, 256 * sizeof(unsigned long long)), "cudaMemset");
    k_span_digits<<<blocks, 256>>>(spans, rows, prefix, mask, shift, histogram);
    check(cudaGetLastError(), "span histogram");
    unsigned long long counts[256];
    check(cudaMemcpy(counts, histogram, sizeof(counts), cudaMemcpyDeviceToHost), "span histogram copy");
    unsigned digit = 0;
    for (; digit < 255; ++digit) {
      if (k < counts[digit]) break;
      k -= counts[digit];
    }
    prefix |= digit << shift;
    mask |= 255u << shift;
  }
  return (int)prefix;
}

}  // namespace

std::string characterize_device(const Csr& matrix, const std::string& ordering, double ordering_seconds) {
  if (matrix.rows != matrix.cols || matrix.nnz() == 0) fail(SPMV_ERR_INVALID_ARGUMENT, "not square or empty");
  if (ordering != "original" && ordering != "rcm") fail(SPMV_ERR_INVALID_ARGUMENT, "ordering must be original or rcm");
  Characterization result;
  // the FIFO replays on host threads, beside the GPU
  int64_t misses[3][5] = {{0}};
  std::vector<std::thread> replays;
  for (int value_index = 0; value_index < 3; ++value_index)
    for (int level = 1; level < 5; ++level)
      replays.emplace_back([&, value_index, level] { misses[value_index][level] = fifo_gather_misses(matrix, value_index, level); });
  struct Join {
    std::vector<std::thread>& threads;
    ~Join() {
      for (std::thread& thread : threads)
        if (thread.joinable()) thread.join();
    }
  } join{replays};

  const int rows = matrix.rows;
  Device<int> row_ptr((size_t)rows + 1), col((size_t)matrix.nnz()), spans((size_t)rows);
  Device<RowTotals> totals(1);
  Device<unsigned long long> histogram(256);
  check(cudaMemcpy(row_ptr.data, matrix.row_ptr.data(), sizeof(int) * ((size_t)rows + 1), cudaMemcpyHostToDevice), "upload");
  check(cudaMemcpy(col.data, matrix.col_ind.data(), sizeof(int) * (size_t)matrix.nnz(), cudaMemcpyHostToDevice), "upload");
  check(cudaMemset(totals.data, 0, sizeof(RowTotals)), "cudaMemset");
  int device = 0, multiprocessors = 0;
  check(cudaGetDevice(&device), "cudaGetDevice");
  check(cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device), "device attribute");
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(((int64_t)rows + 255) / 256, (int64_t)multiprocessors * 8));
  k_characterize_rows<<<blocks, 256>>>(row_ptr.data, col.data, rows, spans.data, totals.data);
  check(cudaGetLastError(), "row metrics");
  RowTotals t;
  check(cudaMemcpy(&t, totals.data, sizeof(t), cudaMemcpyDeviceToHost), "row metrics copy");
  const int p50 = select_span(spans.data, rows, (unsigned long long)(0.50 * (rows - 1)), histogram.data, blocks);
  const int p90 = select_span(spans.data, rows, (unsigned long long)(0.90 * (rows - 1)), histogram.data, blocks);

  const double nnz = (double)matrix.nnz();
  result.empty_rows = (int64_t)t.empty_rows;
  result.bandwidth = (int64_t)t.bandwidth;
  result.row_span_max = (int)t.span_max;
  result.row_span_mean = (double)t.span_sum / rows;   // an exact integer sum (below 2^53), as the host's
  result.row_span_p50 = p50;
  result.row_span_p90 = p90;
  result.rows_fitting_8bit = (double)t.rows8 / rows;
  result.rows_fitting_16bit = (double)t.rows16 / rows;
  result.nnz_in_rows_fitting_8bit = (double)t.nnz8 / nnz;
  result.nnz_in_rows_fitting_16bit = (double)t.nnz16 / nnz;
  result.segments_8bit = (int64_t)t.segments8;
  result.segments_16bit = (int64_t)t.segments16;
  for (int index = 0; index < 5; ++index) {
    result.lane_occupancy[index] = t.occupied[index] > 0 ? nnz / (double)t.occupied[index] : 0.0;
    result.tail_ratio[index] =
        t.iterations[index] > 0 ? (double)t.longest[index] * (double)rows / (double)t.iterations[index] : 0.0;
  }
  for (int value_index = 0; value_index < 3; ++value_index)
    result.gather_bytes[value_index][0] = (double)t.sectors[value_index] * kCharacterizeSectorBytes / nnz;
  for (std::thread& thread : replays) thread.join();
  for (int value_index = 0; value_index < 3; ++value_index)
    for (int level = 1; level < 5; ++level)
      result.gather_bytes[value_index][level] = (double)misses[value_index][level] * kCharacterizeSectorBytes / nnz;
  byte_model(matrix, result);
  return characterization_csv(matrix, result, ordering, ordering_seconds);
}

}  // namespace spmvb200

using namespace spmvb200;

extern "C" int spmv_characterize_device(const spmv_csr* matrix, const char* ordering, double ordering_seconds, int device,
                                        char* csv, size_t cap, size_t* needed) {
  return guarded([&] {
    require(matrix && ordering, "matrix and ordering are required");
    DeviceScope scope(device);
    const std::string text = characterize_device(matrix->m, ordering, ordering_seconds);
    if (needed) *needed = text.size() + 1;
    if (!csv || cap < text.size() + 1) fail(SPMV_ERR_TOO_LARGE, "output buffer too small");
    std::memcpy(csv, text.c_str(), text.size() + 1);
  });
}
