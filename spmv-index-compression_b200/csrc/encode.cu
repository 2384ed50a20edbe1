// encode.cu — the CSR-lp encoder on the GPU: the same streams as encode_lane_packed (layouts.cpp), which
// restates the reference's build_packed_deltas (bench_csr_width.cu:861-917), built from device-resident
// row_ptr and col_ind.
//
//   1. k_lp_widths   one warp per row: the widest lane delta (from the entry T positions earlier, or from
//                    the row's first column for the first T entries), its bit width, and the row's words;
//   2. a scan of the words per row into row_word (block scans, a scan of the block sums, an add);
//   3. k_lp_pack     one warp per row: every delta OR-ed into its words at bit
//                    width * (lane * quotient + min(lane, remainder) + step), lane-major.
#include <cuda.h>   // CUcontext and CUresult (types only: the driver calls come through the runtime's entry points)
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <utility>

#include "capi_internal.hpp"

namespace spmvb200 {
namespace {

constexpr int kScanBlock = 1024;

__global__ void k_lp_widths(const int* __restrict__ row_ptr, const int* __restrict__ col, int rows, int tpr,
                            uint8_t* __restrict__ row_width, long long* __restrict__ row_words) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) / 32;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; row < rows; row += warps) {
    const int begin = row_ptr[row], end = row_ptr[row + 1];
    unsigned widest = 0;
    for (int entry = begin + lane; entry < end; entry += 32) {
      const int delta = entry - begin < tpr ? col[entry] - col[begin] : col[entry] - col[entry - tpr];
      widest = max(widest, (unsigned)delta);
    }
    widest = __reduce_max_sync(0xffffffffu, widest);
    if (lane == 0) {
      const int width = widest == 0 ? 0 : 32 - __clz((int)widest);
      row_width[row] = (uint8_t)width;
      row_words[row] = ((long long)(end - begin) * width + 31) / 32;
    }
  }
}

// Exclusive scan of kScanBlock values per block; the block's total goes to sums[block].
__global__ void __launch_bounds__(kScanBlock) k_scan_blocks(const long long* __restrict__ values, int64_t count,
                                                          long long* __restrict__ scanned, long long* __restrict__ sums) {
  __shared__ long long warp_totals[kScanBlock / 32];
  const int64_t index = (int64_t)blockIdx.x * kScanBlock + threadIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x / 32;
  const long long value = index < count ? values[index] : 0;
  long long inclusive = value;
#pragma unroll
  for (int offset = 1; offset < 32; offset <<= 1) {
    const long long other = __shfl_up_sync(0xffffffffu, inclusive, offset);
    if (lane >= offset) inclusive += other;
  }
  if (lane == 31) warp_totals[warp] = inclusive;
  __syncthreads();
  if (warp == 0) {
    long long total = warp_totals[lane];
#pragma unroll
    for (int offset = 1; offset < 32; offset <<= 1) {
      const long long other = __shfl_up_sync(0xffffffffu, total, offset);
      if (lane >= offset) total += other;
    }
    warp_totals[lane] = total;   // inclusive over warps
  }
  __syncthreads();
  const long long before = warp == 0 ? 0 : warp_totals[warp - 1];
  if (index < count) scanned[index] = before + inclusive - value;
  if (threadIdx.x == kScanBlock - 1) sums[blockIdx.x] = before + inclusive;
}

// One block: the exclusive scan of `count` block sums in place, chunk by chunk with a carry, and the
// grand total in *total.
__global__ void __launch_bounds__(kScanBlock) k_scan_sums(long long* __restrict__ sums, int64_t count,
                                                        long long* __restrict__ total) {
  __shared__ long long warp_totals[kScanBlock / 32];
  __shared__ long long carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x / 32;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t first = 0; first < count; first += kScanBlock) {
    const int64_t index = first + threadIdx.x;
    const long long value = index < count ? sums[index] : 0;
    long long inclusive = value;
#pragma unroll
    for (int offset = 1; offset < 32; offset <<= 1) {
      const long long other = __shfl_up_sync(0xffffffffu, inclusive, offset);
      if (lane >= offset) inclusive += other;
    }
    if (lane == 31) warp_totals[warp] = inclusive;
    __syncthreads();
    if (warp == 0) {
      long long sum = warp_totals[lane];
#pragma unroll
      for (int offset = 1; offset < 32; offset <<= 1) {
        const long long other = __shfl_up_sync(0xffffffffu, sum, offset);
        if (lane >= offset) sum += other;
      }
      warp_totals[lane] = sum;
    }
    __syncthreads();
    const long long before = warp == 0 ? 0 : warp_totals[warp - 1];
    if (index < count) sums[index] = carry + before + inclusive - value;
    __syncthreads();
    if (threadIdx.x == kScanBlock - 1) carry += before + inclusive;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = carry;
}

__global__ void k_scan_add(const long long* __restrict__ scanned, const long long* __restrict__ sums, int64_t count,
                           int* __restrict__ row_word) {
  const int64_t index = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (index < count) row_word[index] = (int)(scanned[index] + sums[index / kScanBlock]);
}

__global__ void k_lp_pack(const int* __restrict__ row_ptr, const int* __restrict__ col, int rows, int tpr,
                          const uint8_t* __restrict__ row_width, const int* __restrict__ row_word,
                          uint32_t* __restrict__ words) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) / 32;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; row < rows; row += warps) {
    const int width = row_width[row];
    if (width == 0) continue;
    const int begin = row_ptr[row], length = row_ptr[row + 1] - begin;
    const int quotient = length / tpr, remainder = length - quotient * tpr;
    uint32_t* stream = words + row_word[row];
    for (int offset = lane; offset < length; offset += 32) {
      const int entry = begin + offset;
      const uint32_t delta = (uint32_t)(offset < tpr ? col[entry] - col[begin] : col[entry] - col[entry - tpr]);
      const int lane_of = offset % tpr, step = offset / tpr;
      const int64_t bit = (int64_t)width * ((int64_t)lane_of * quotient + min(lane_of, remainder) + step);
      const int shift = (int)(bit & 31);
      if (delta != 0) {
        atomicOr(stream + (bit >> 5), delta << shift);
        if (shift + width > 32) atomicOr(stream + (bit >> 5) + 1, delta >> (32 - shift));
      }
    }
  }
}

unsigned warp_blocks(int rows) {
  const int64_t blocks = ((int64_t)rows * 32 + 255) / 256;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks, 148 * 64));
}

}  // namespace

// Row widths and row_word on the device; returns the word count including the 2 spare words. The
// scratch (words per row, block sums, total) is allocated here.
int64_t device_lane_packed_layout(const int* row_ptr, const int* col_ind, int rows, int tpr, int* row_word,
                                  uint8_t* row_width, cudaStream_t stream) {
  if (rows == 0) return 2;
  const int64_t blocks = ((int64_t)rows + kScanBlock - 1) / kScanBlock;
  long long* scratch = nullptr;
  const size_t scratch_count = 2 * (size_t)rows + (size_t)blocks + 1;
  cudaError_t status = cudaMalloc(&scratch, scratch_count * sizeof(long long));
  if (status != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("cudaMalloc: ") + cudaGetErrorString(status));
  long long* row_words = scratch;
  long long* scanned = scratch + rows;
  long long* sums = scanned + rows;
  long long* total = sums + blocks;
  k_lp_widths<<<warp_blocks(rows), 256, 0, stream>>>(row_ptr, col_ind, rows, tpr, row_width, row_words);
  k_scan_blocks<<<(unsigned)blocks, kScanBlock, 0, stream>>>(row_words, rows, scanned, sums);
  k_scan_sums<<<1, kScanBlock, 0, stream>>>(sums, blocks, total);
  k_scan_add<<<(unsigned)(((int64_t)rows + 255) / 256), 256, 0, stream>>>(scanned, sums, rows, row_word);
  long long host_total = 0;
  status = cudaGetLastError();
  if (status == cudaSuccess) status = cudaMemcpyAsync(&host_total, total, sizeof(long long), cudaMemcpyDeviceToHost, stream);
  if (status == cudaSuccess) status = cudaStreamSynchronize(stream);
  cudaFree(scratch);
  if (status != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("CSR-lp layout on the device: ") + cudaGetErrorString(status));
  return host_total + 2;
}

void device_lane_packed_pack(const int* row_ptr, const int* col_ind, int rows, int tpr, const int* row_word,
                             const uint8_t* row_width, uint32_t* words, int64_t word_count, cudaStream_t stream) {
  cudaError_t status = cudaMemsetAsync(words, 0, sizeof(uint32_t) * (size_t)word_count, stream);
  if (status == cudaSuccess && rows > 0) {
    k_lp_pack<<<warp_blocks(rows), 256, 0, stream>>>(row_ptr, col_ind, rows, tpr, row_width, row_word, words);
    status = cudaGetLastError();
  }
  if (status != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("CSR-lp packing on the device: ") + cudaGetErrorString(status));
}

}  // namespace spmvb200

using namespace spmvb200;

extern "C" int spmv_encode_lane_packed_device(const int* row_ptr, const int* col_ind, int rows, int tpr, int* row_word,
                                              uint8_t* row_width, uint32_t* words, int64_t word_capacity,
                                              int64_t* word_count, void* stream) {
  return guarded([&] {
    require(row_ptr && (col_ind || rows == 0) && row_word && row_width && word_count && rows >= 0, "bad arguments");
    require(valid_tpr(tpr), "threads per row must be 2, 4, 8, 16 or 32");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t count = device_lane_packed_layout(row_ptr, col_ind, rows, tpr, row_word, row_width, s);
    *word_count = count;
    if (count - 2 > INT32_MAX) fail(SPMV_ERR_NOT_ADMISSIBLE, "CSR-lp stream exceeds 2^31 words");
    if (words == nullptr) return;
    require(word_capacity >= count, "words holds fewer than word_count words");
    device_lane_packed_pack(row_ptr, col_ind, rows, tpr, row_word, row_width, words, count, s);
    const cudaError_t status = cudaStreamSynchronize(s);
    if (status != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("CSR-lp packing on the device: ") + cudaGetErrorString(status));
  });
}

// ---- the CSR-lp layout without allocating --------------------------------------------------------------
// For callers that must not allocate device memory while they encode: a framework whose own caching
// allocator owns every device byte (a cudaMalloc behind its back can fail or fragment its pool), code that
// reserves all its memory up front under a fixed budget, and loops that cannot stall on cudaMalloc/cudaFree,
// which may synchronise the device. The scan's scratch (one 64-bit sum per block of 1024 rows, and the
// grand total) lives in this file-scope device array instead of a cudaMalloc'd buffer; the word count of
// each row goes through the caller's own row_word.
namespace spmvb200 {
namespace {

constexpr int64_t kNoAllocMaxBlocks = 65536;                          // rows up to 65536 * 1024 = 2^26
static __device__ __align__(256) long long g_encode_scratch[kNoAllocMaxBlocks + 1];   // 512 KiB + 8 B

// Widths, and each row's word count written to row_word (a row of fewer than 2^31 entries has fewer than
// 2^31 words).
__global__ void k_lp_widths_into(const int* __restrict__ row_ptr, const int* __restrict__ col, int rows, int tpr,
                                 uint8_t* __restrict__ row_width, int* __restrict__ row_words) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) / 32;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; row < rows; row += warps) {
    const int begin = row_ptr[row], end = row_ptr[row + 1];
    unsigned widest = 0;
    for (int entry = begin + lane; entry < end; entry += 32) {
      const int delta = entry - begin < tpr ? col[entry] - col[begin] : col[entry] - col[entry - tpr];
      widest = max(widest, (unsigned)delta);
    }
    widest = __reduce_max_sync(0xffffffffu, widest);
    if (lane == 0) {
      const int width = widest == 0 ? 0 : 32 - __clz((int)widest);
      row_width[row] = (uint8_t)width;
      row_words[row] = (int)(((long long)(end - begin) * width + 31) / 32);
    }
  }
}

// In place over row_word: the exclusive scan within each block of 1024 rows (64-bit sums, stored as int;
// a block whose prefix does not fit makes a total above 2^31 words, which the caller rejects), and the
// block's total into sums[block].
__global__ void __launch_bounds__(kScanBlock) k_scan_blocks_in_place(int* __restrict__ row_word, int64_t count,
                                                                   long long* __restrict__ sums) {
  __shared__ long long warp_totals[kScanBlock / 32];
  const int64_t index = (int64_t)blockIdx.x * kScanBlock + threadIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x / 32;
  const long long value = index < count ? row_word[index] : 0;
  long long inclusive = value;
#pragma unroll
  for (int offset = 1; offset < 32; offset <<= 1) {
    const long long other = __shfl_up_sync(0xffffffffu, inclusive, offset);
    if (lane >= offset) inclusive += other;
  }
  if (lane == 31) warp_totals[warp] = inclusive;
  __syncthreads();
  if (warp == 0) {
    long long total = warp_totals[lane];
#pragma unroll
    for (int offset = 1; offset < 32; offset <<= 1) {
      const long long other = __shfl_up_sync(0xffffffffu, total, offset);
      if (lane >= offset) total += other;
    }
    warp_totals[lane] = total;
  }
  __syncthreads();
  const long long before = warp == 0 ? 0 : warp_totals[warp - 1];
  if (index < count) row_word[index] = (int)(before + inclusive - value);
  if (threadIdx.x == kScanBlock - 1) sums[blockIdx.x] = before + inclusive;
}

__global__ void k_scan_add_in_place(const long long* __restrict__ sums, int64_t count, int* __restrict__ row_word) {
  const int64_t index = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (index < count) row_word[index] = (int)(row_word[index] + sums[index / kScanBlock]);
}

// The unique ID of the context current on this thread (0 when none is): the driver's cuCtxGetCurrent and
// cuCtxGetId, reached through the runtime's driver entry points, so the library does not link libcuda.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static const std::pair<GetCurrent, GetId> driver = [] {
    void* current = nullptr;
    void* id = nullptr;
    cudaDriverEntryPointQueryResult found_current = cudaDriverEntryPointSymbolNotFound, found_id = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &current, cudaEnableDefault, &found_current) != cudaSuccess ||
        found_current != cudaDriverEntryPointSuccess)
      current = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &id, cudaEnableDefault, &found_id) != cudaSuccess ||
        found_id != cudaDriverEntryPointSuccess)
      id = nullptr;
    return std::make_pair(reinterpret_cast<GetCurrent>(current), reinterpret_cast<GetId>(id));
  }();
  CUcontext context = nullptr;
  unsigned long long id = 0;
  if (!driver.first || !driver.second || driver.first(&context) != CUDA_SUCCESS || !context ||
      driver.second(context, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// The address of g_encode_scratch on the current device, taken with that device current: once per device,
// and again when the device's context is not the one the address was taken in (cudaDeviceReset, or a
// framework that tears the primary context down, gives the device a new context and the array a new
// address).
long long* encode_scratch_address() {
  static std::mutex guard;
  static long long* address[64] = {};
  static unsigned long long context[64] = {};
  int device = 0;
  const cudaError_t status = cudaGetDevice(&device);
  if (status != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(status));
  if (device < 0 || device >= 64) fail(SPMV_ERR_UNSUPPORTED, "device ordinal above 63");
  std::lock_guard<std::mutex> lock(guard);
  const unsigned long long id = current_context_id();
  if (!address[device] || id == 0 || id != context[device]) {
    void* pointer = nullptr;
    const cudaError_t found = cudaGetSymbolAddress(&pointer, g_encode_scratch);   // makes the context current
    if (found != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(found));
    address[device] = static_cast<long long*>(pointer);
    context[device] = current_context_id();
  }
  return address[device];
}

}  // namespace
}  // namespace spmvb200

extern "C" int spmv_encode_lane_packed_device_noalloc(const int* row_ptr, const int* col_ind, int rows, int tpr,
                                                      int* row_word, uint8_t* row_width, uint32_t* words,
                                                      int64_t word_capacity, int64_t* word_count, void* stream) {
  return guarded([&] {
    require(row_ptr && (col_ind || rows == 0) && row_word && row_width && word_count && rows >= 0, "bad arguments");
    require(valid_tpr(tpr), "threads per row must be 2, 4, 8, 16 or 32");
    const int64_t blocks = ((int64_t)rows + kScanBlock - 1) / kScanBlock;
    if (blocks > kNoAllocMaxBlocks)
      fail(SPMV_ERR_TOO_LARGE, "the allocation-free encoder takes at most " + std::to_string(kNoAllocMaxBlocks * kScanBlock) +
                                   " rows (its fixed scratch holds one sum per 1024 rows); use spmv_encode_lane_packed_device");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    long long* scratch = encode_scratch_address();   // sums[0..blocks), then the total at [kNoAllocMaxBlocks]
    long long total = 0;
    cudaError_t status = cudaSuccess;
    if (rows > 0) {
      // every scratch entry this call reads is written by it first: nothing needs clearing
      k_lp_widths_into<<<warp_blocks(rows), 256, 0, s>>>(row_ptr, col_ind, rows, tpr, row_width, row_word);
      k_scan_blocks_in_place<<<(unsigned)blocks, kScanBlock, 0, s>>>(row_word, rows, scratch);
      k_scan_sums<<<1, kScanBlock, 0, s>>>(scratch, blocks, scratch + kNoAllocMaxBlocks);
      k_scan_add_in_place<<<(unsigned)(((int64_t)rows + 255) / 256), 256, 0, s>>>(scratch, rows, row_word);
      status = cudaGetLastError();
      if (status == cudaSuccess)
        status = cudaMemcpyAsync(&total, scratch + kNoAllocMaxBlocks, sizeof(long long), cudaMemcpyDeviceToHost, s);
      if (status == cudaSuccess) status = cudaStreamSynchronize(s);
      if (status != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("CSR-lp layout on the device: ") + cudaGetErrorString(status));
    }
    *word_count = total + 2;
    if (total > INT32_MAX) fail(SPMV_ERR_NOT_ADMISSIBLE, "CSR-lp stream exceeds 2^31 words");
    if (words == nullptr) return;
    require(word_capacity >= total + 2, "words holds fewer than word_count words");
    device_lane_packed_pack(row_ptr, col_ind, rows, tpr, row_word, row_width, words, total + 2, s);
    status = cudaStreamSynchronize(s);
    if (status != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("CSR-lp packing on the device: ") + cudaGetErrorString(status));
  });
}
