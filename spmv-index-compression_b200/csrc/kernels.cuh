// kernels.cuh — sm_100a SpMV kernels for CSR with compressed column indices.
//
// Summation contract (bit-parity with the reference, src/bench_csr_width.cu:291-517): for threads per
// row T, logical lane L of a row sums the entries L, L+T, L+2T, ... in order, one correctly rounded fused
// multiply-add each, in the accumulator type (FP64, or FP32 for FP32 and FP16, value_types.cuh:9-13);
// the T lane sums s_0..s_{T-1} are then combined in the order of the __shfl_down_sync tree: for
// offset o = T/2, ..., 1, s_i += s_{i+o}; lane 0 narrows s_0 into y.
//
// Which hardware thread runs which logical lane is free. These kernels run a row on P threads (P divides
// T): thread p owns the logical lanes p, p+P, p+2P, ... (S = T/P "slots"), so it walks the entries p, p+P,
// p+2P, ... of the row and adds entry e into slot ((e - row_begin) mod T) / P. The tree levels with
// o >= P pair two lanes of the same thread and run in registers; the last log2(P) levels are shuffles.
// Lane sums start at +0.0 and an FMA chain or a sum never produces -0.0 from it, so the zero sums of
// empty lanes are exact no-ops, as they are in the reference.
//
// Kernels
//   k_spmv_tiles   persistent CTAs over the tiles of the operator's plan (runs of consecutive rows whose
//                  nonzeros fit in shared memory). Each CTA owns tiles cta, cta + ctas, ... and keeps a
//                  ring of `stages` shared-memory buffers: thread 0 streams upcoming tiles into free
//                  buffers with cp.async.bulk (the 1-D TMA engine), completing on the buffer's "full"
//                  mbarrier. On a resident tile every thread decodes its entries' columns, gathers x at
//                  up to 32 of them at once into registers and adds them into its lane chains, reading
//                  values from shared memory; the last warp to
//                  finish with a buffer refills it with a later tile. The operator
//                  pads every stream by 16 bytes, so each bulk copy is the 16-byte-aligned superset of a
//                  tile's range. Its leading `vector_blocks` CTAs run the vector path over rows longer
//                  than a tile.
//   k_spmv_vector  one group of T threads per row straight from global memory (the reference's
//                  mapping): the raw launch over caller arrays, which carry no plan and no padding.
#pragma once

#include <cuda_fp16.h>
#include <climits>
#include <cstdint>
#include <type_traits>

#include "spmvb200.h"

namespace spmvb200 {

constexpr int kTileBlock = 256;            // threads of a tile CTA
constexpr int kVectorBlock = 128;          // threads of a vector CTA
constexpr int kMaxStages = 4;              // shared-memory buffers of a tile CTA at most
constexpr int kStreamPadding = 16;         // bytes every operator stream carries past its end
constexpr unsigned kStatusTimeout = 1u;    // bit of the status word: a bounded wait gave up
constexpr unsigned kStatusSmem = 2u;       // bit: a long-row chunk did not fit the launch's shared memory
constexpr int kMaxPeers = 15;              // other GPUs' copies of y a product may also store its rows into

// ---- value types --------------------------------------------------------------------------------
template <class V> struct ValueTraits;
template <> struct ValueTraits<double> {
  using Acc = double;
  __device__ static __forceinline__ double widen(double v) { return v; }
  __device__ static __forceinline__ double narrow(double a) { return a; }
  __device__ static __forceinline__ double fma(double a, double b, double c) { return __fma_rn(a, b, c); }
  __device__ static __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
};
template <> struct ValueTraits<float> {
  using Acc = float;
  __device__ static __forceinline__ float widen(float v) { return v; }
  __device__ static __forceinline__ float narrow(float a) { return a; }
  __device__ static __forceinline__ float fma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
  __device__ static __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
};
template <> struct ValueTraits<__half> {
  using Acc = float;
  __device__ static __forceinline__ float widen(__half v) { return __half2float(v); }
  __device__ static __forceinline__ __half narrow(float a) { return __float2half_rn(a); }
  __device__ static __forceinline__ float fma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
  __device__ static __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
};

// FP16 values summed in FP16 (the reference's SPMV_HALF_ACCUMULATE control build, value_types.cuh:7-33):
// every product-add one __hfma, every step of the tree one __hadd, the result stored as it is. The
// storage is __half's under a type of its own, so that the kernels instantiate a family for it.
struct __align__(2) half16 {
  __half h;
};
template <> struct ValueTraits<half16> {
  using Acc = __half;
  __device__ static __forceinline__ __half widen(half16 v) { return v.h; }
  __device__ static __forceinline__ half16 narrow(__half a) { return half16{a}; }
  __device__ static __forceinline__ __half fma(__half a, __half b, __half c) { return __hfma(a, b, c); }
  __device__ static __forceinline__ __half add(__half a, __half b) { return __hadd(a, b); }
};

// ---- column layouts -----------------------------------------------------------------------------
template <int LAYOUT> struct LayoutTraits;
template <> struct LayoutTraits<SPMV_LAYOUT_I32> { using Index = int;      static constexpr bool kBase = false; };
template <> struct LayoutTraits<SPMV_LAYOUT_I16> { using Index = uint16_t; static constexpr bool kBase = false; };
template <> struct LayoutTraits<SPMV_LAYOUT_I8>  { using Index = uint8_t;  static constexpr bool kBase = false; };
template <> struct LayoutTraits<SPMV_LAYOUT_R16> { using Index = uint16_t; static constexpr bool kBase = true; };
template <> struct LayoutTraits<SPMV_LAYOUT_R8>  { using Index = uint8_t;  static constexpr bool kBase = true; };
template <> struct LayoutTraits<SPMV_LAYOUT_LP>  { using Index = uint32_t; static constexpr bool kBase = true; };
// Row-relative offsets in 32 bits: the CSR-r16 control build SPMV_R16_WIDE (bench_csr_width.cu:38-39, :944),
// raw launch only.
constexpr int kLayoutR16Wide = 100;
template <> struct LayoutTraits<kLayoutR16Wide> { using Index = uint32_t; static constexpr bool kBase = true; };

// Arguments of every kernel (device pointers).
struct KernelArgs {
  int rows;
  int cols;
  const int* row_ptr;
  const void* columns;       // absolute / row-base index stream
  const int* row_base;
  const int* row_word;
  const uint8_t* row_width;
  const uint32_t* words;     // CSR-lp stream
  const void* values;
  const void* x;
  void* y;
  const int4* tiles;         // [tile_count] {row_begin, row_end, entry_begin, entry_end}
  const int2* tile_words;    // CSR-lp: [tile_count] {first word, last word + 1} of the tile's stream
  int64_t tile_count;
  int tile_nnz;              // nonzeros a tile holds at most
  int tile_rows;             // rows a tile holds at most
  int tile_index_words;      // CSR-lp: stream words a tile's image holds at most
  const int2* tile_windows;  // [tile_count] {first column, end column} of the x window a tile stages (first ==
                             // end: none); null: no windows in this launch (x not 16-byte aligned)
  int window_elements;       // x elements a tile's window holds at most
  int stages;                // shared-memory buffers of a tile CTA (1..kMaxStages)
  const int* row_list;       // rows of the vector path (nullptr: rows 0..row_count-1)
  // CSR-lp long rows: lane L's column after each kLaneMarkEvery of its deltas, [(j - 1) * T + L] for the
  // j-th mark of the row_list item's row, from lane_mark_first[item] on
  const int* lane_marks;
  const int64_t* lane_mark_first;
  int64_t row_count;         // entries of row_list, or rows
  int64_t vector_blocks;     // k_spmv_tiles: its first vector_blocks CTAs take the rows of row_list
  int long_chunk;            // k_spmv_tiles: entries per chunk of a long row (a multiple of kTileBlock)
  int smem_bytes;            // k_spmv_tiles: dynamic shared memory of the launch
  int64_t tile_ctas;         // k_spmv_tiles: persistent CTAs over the tiles after the vector blocks
  int dense;                 // k_spmv_tiles with one thread per lane (P = T): the variant budgeted for more
                             // CTAs per multiprocessor (kDenseResidency)
  unsigned* status;          // device status word (may be null)
  // copies of y in other GPUs' memory (peer pointers, indexed by the same rows as y): every row's result is
  // stored there too, by the thread that stores it into y, so that a chained product's all-gather happens
  // inside the product
  void* peers[kMaxPeers];
  int peer_count;
  // k_spmv_classes (rows by length): long-row blocks, then the blocks of each segment of listed rows
  // (P = 32, 16, ..., 1 threads per row), then the short-row blocks
  const int4* row_items;     // {row, first entry, end entry, row base} of the listed rows, by segment
  int64_t long_blocks;       // one CTA per row of row_list
  int64_t segment_first[6];  // segment s (P = 2^s): its first item,
  int64_t segment_items[6];  // its items
  int64_t segment_blocks[6]; // and its blocks of 256 / P items
};

// ---- shared-memory plan of a tile CTA (host and device compute it alike) ----------------------------
// [0, 64): full[kMaxStages] mbarriers; then `stages` buffers, each a header (the
// tile's rows and image origins) and 16-byte-aligned images of the tile's row_ptr, row_base, row_word and
// row_width slices and of its value and index (or CSR-lp word) ranges. An image starts at the 16-byte
// boundary at or below its first element, so it holds up to 16 bytes before and after the range.
struct StagePlan {
  int header, row_ptr, row_base, row_word, row_width, values, index, window, bytes;
};

__host__ __device__ inline int round16(int bytes) { return (bytes + 15) & ~15; }

// index_words: CSR-lp, the words a tile's stream image holds at most (the longest tile's word range plus
// the word a delta may read past it); ignored by the other layouts, whose index image holds tile_nnz.
// window_elements: the x elements a tile's window of x holds at most (0: no window).
__host__ __device__ inline StagePlan stage_plan(int tile_nnz, int tile_rows, int value_bytes, int layout, int index_words,
                                                int window_elements) {
  const bool base = layout == SPMV_LAYOUT_R16 || layout == SPMV_LAYOUT_R8 || layout == SPMV_LAYOUT_LP;
  const bool packed = layout == SPMV_LAYOUT_LP;
  const int index_bytes = packed ? 4 : (layout == SPMV_LAYOUT_I32 ? 4 : ((layout == SPMV_LAYOUT_I16 || layout == SPMV_LAYOUT_R16) ? 2 : 1));
  StagePlan plan;
  int offset = 0;
  plan.header = offset;    offset += 32;   // row_begin, rows, 5 image origins
  plan.row_ptr = offset;   offset += round16(4 * (tile_rows + 1)) + 16;
  plan.row_base = offset;  if (base) offset += round16(4 * tile_rows) + 16;
  plan.row_word = offset;  if (packed) offset += round16(4 * tile_rows) + 16;
  plan.row_width = offset; if (packed) offset += round16(tile_rows) + 16;
  plan.values = offset;    offset += round16(value_bytes * tile_nnz) + 16;
  plan.index = offset;     offset += packed ? round16(4 * index_words) + 16 : round16(index_bytes * tile_nnz) + 16;
  plan.window = offset;    if (window_elements > 0) offset += round16(value_bytes * window_elements) + 32;
  plan.bytes = offset;
  return plan;
}

__host__ __device__ inline int tile_smem_bytes(int tile_nnz, int tile_rows, int value_bytes, int layout, int stages,
                                               int index_words, int window_elements) {
  return 64 + stages * stage_plan(tile_nnz, tile_rows, value_bytes, layout, index_words, window_elements).bytes;
}

// ---- small device helpers -----------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_address(const void* pointer) {
  return (uint32_t)__cvta_generic_to_shared(pointer);
}

__device__ __forceinline__ void mbarrier_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbarrier_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbarrier_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbarrier_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbarrier_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t now;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
  return now;
}

// Waits for phase `parity` of an mbarrier for at most about limit_ns (and a bounded number of polls).
// Returns false when it gave up.
__device__ __forceinline__ bool mbarrier_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbarrier_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 0; spin < (1u << 26); ++spin) {
    if (mbarrier_try_wait(bar, parity)) return true;
    if ((spin & 63) == 0 && global_timer_ns() - start > limit_ns) return false;
  }
  return false;
}

// 1-D bulk copy global -> shared (TMA), completing on the mbarrier with its byte count.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

template <class T>
__device__ __forceinline__ T load_readonly(const T* pointer) {
  return __ldg(pointer);
}
template <>
__device__ __forceinline__ uint8_t load_readonly<uint8_t>(const uint8_t* pointer) {
  return (uint8_t)__ldg(reinterpret_cast<const unsigned char*>(pointer));
}
template <>
__device__ __forceinline__ half16 load_readonly<half16>(const half16* pointer) {
  return half16{__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(pointer)))};
}

// L2 policies: x, gathered at random and reused across rows, is kept (evict_last); the matrix streams, read
// once per product, leave L2 first (evict_first), so that they do not push x out.
__device__ __forceinline__ uint64_t l2_keep_policy() {
  uint64_t policy;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}
__device__ __forceinline__ uint64_t l2_stream_policy() {
  uint64_t policy;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// A read-only load of x with an L2 cache policy.
template <class T> __device__ __forceinline__ T load_x(const T* pointer, uint64_t policy);
template <>
__device__ __forceinline__ double load_x<double>(const double* pointer, uint64_t policy) {
  double value;
  asm("ld.global.nc.L2::cache_hint.f64 %0, [%1], %2;" : "=d"(value) : "l"(pointer), "l"(policy));
  return value;
}
template <>
__device__ __forceinline__ float load_x<float>(const float* pointer, uint64_t policy) {
  float value;
  asm("ld.global.nc.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(value) : "l"(pointer), "l"(policy));
  return value;
}
template <>
__device__ __forceinline__ __half load_x<__half>(const __half* pointer, uint64_t policy) {
  unsigned short bits;
  asm("ld.global.nc.L2::cache_hint.b16 %0, [%1], %2;" : "=h"(bits) : "l"(pointer), "l"(policy));
  return __ushort_as_half(bits);
}

template <>
__device__ __forceinline__ half16 load_x<half16>(const half16* pointer, uint64_t policy) {
  unsigned short bits;
  asm("ld.global.nc.L2::cache_hint.b16 %0, [%1], %2;" : "=h"(bits) : "l"(pointer), "l"(policy));
  return half16{__ushort_as_half(bits)};
}

// A read-only load of a matrix stream element with an L2 cache policy (values and column indices).
template <class T> __device__ __forceinline__ T load_stream(const T* pointer, uint64_t policy) {
  return load_x(pointer, policy);
}
template <>
__device__ __forceinline__ int load_stream<int>(const int* pointer, uint64_t policy) {
  int value;
  asm("ld.global.nc.L2::cache_hint.b32 %0, [%1], %2;" : "=r"(value) : "l"(pointer), "l"(policy));
  return value;
}
template <>
__device__ __forceinline__ uint32_t load_stream<uint32_t>(const uint32_t* pointer, uint64_t policy) {
  uint32_t value;
  asm("ld.global.nc.L2::cache_hint.b32 %0, [%1], %2;" : "=r"(value) : "l"(pointer), "l"(policy));
  return value;
}
template <>
__device__ __forceinline__ uint16_t load_stream<uint16_t>(const uint16_t* pointer, uint64_t policy) {
  unsigned short value;
  asm("ld.global.nc.L2::cache_hint.b16 %0, [%1], %2;" : "=h"(value) : "l"(pointer), "l"(policy));
  return value;
}
template <>
__device__ __forceinline__ uint8_t load_stream<uint8_t>(const uint8_t* pointer, uint64_t policy) {
  unsigned int value;
  asm("ld.global.nc.L2::cache_hint.u8 %0, [%1], %2;" : "=r"(value) : "l"(pointer), "l"(policy));
  return (uint8_t)value;
}

// ---- results into other GPUs' memory ---------------------------------------------------------------------
template <int BYTES> struct BitsOf;
template <> struct BitsOf<2> { using type = unsigned short; };
template <> struct BitsOf<4> { using type = unsigned; };
template <> struct BitsOf<8> { using type = unsigned long long; };

// Row `row` of y (already stored in y by this thread) into every peer's copy.
template <class V>
__device__ __forceinline__ void mirror_row(const KernelArgs& a, int row, V value) {
  using B = typename BitsOf<sizeof(V)>::type;
  const B bits = *reinterpret_cast<const B*>(&value);
  for (int d = 0; d < a.peer_count; ++d) reinterpret_cast<B*>(a.peers[d])[row] = bits;
}

// Every peer copy of y is visible to the other GPUs before the kernel counts as done: after the CTA's
// barrier one thread fences at system scope (cumulative over the CTA's stores it synchronised with).
__device__ __forceinline__ void publish_peer_rows(const KernelArgs& a) {
  if (a.peer_count > 0) {
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
  }
}

// The 16-byte-aligned superset of elements [first, last) of a padded stream: its global start, bytes, and
// the element index sitting at image byte 0.
template <class E>
struct AlignedRange {
  uintptr_t begin;
  uint32_t bytes;
  int64_t origin;
  __device__ __forceinline__ AlignedRange(const E* base, int64_t first, int64_t last) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(base + first);
    const uintptr_t b = reinterpret_cast<uintptr_t>(base + last);
    begin = a & ~(uintptr_t)15;
    bytes = (uint32_t)(((b + 15) & ~(uintptr_t)15) - begin);
    origin = first - (int64_t)((a - begin) / sizeof(E));
  }
};

// ---- the reduction over the T logical lanes -----------------------------------------------------------
// acc[j] holds logical lane p + j*P. Levels with offset >= P add two slots of this thread; the last
// log2(P) levels add across the P threads of the row (segments of width P within the warp).
template <class VT, class Acc, int T, int P>
__device__ __forceinline__ Acc reduce_lanes(Acc (&acc)[T / P]) {
#pragma unroll
  for (int offset = T / 2; offset >= P; offset >>= 1) {
#pragma unroll
    for (int j = 0; j < offset / P; ++j) acc[j] = VT::add(acc[j], acc[j + offset / P]);
  }
  Acc sum = acc[0];
#pragma unroll
  for (int offset = P / 2; offset > 0; offset >>= 1) sum = VT::add(sum, __shfl_down_sync(0xffffffffu, sum, offset, P));
  return sum;
}

// ---- rows on groups of P threads ----------------------------------------------------------------------
// Where a row's data is read from: the shifted images of a resident tile in shared memory, or the
// operator's arrays in global memory (read-only path). Both are indexed by absolute row, entry and word.
template <class V, int LAYOUT>
struct TileView {
  using Index = typename LayoutTraits<LAYOUT>::Index;
  int row_begin, rows;
  const int* row_ptr_;
  const int* row_base_;
  const int* row_word_;
  const uint8_t* row_width_;
  const V* values_;
  const Index* index_;
  const V* window_;   // x by absolute column, when the tile staged a window of x
  bool windowed;
  __device__ __forceinline__ TileView(const unsigned char* stage, const StagePlan& plan) {
    const int* header = reinterpret_cast<const int*>(stage + plan.header);
    row_begin = header[0];
    rows = header[1];
    row_ptr_ = reinterpret_cast<const int*>(stage + plan.row_ptr) - header[2];
    row_base_ = reinterpret_cast<const int*>(stage + plan.row_base) - header[3];
    row_word_ = reinterpret_cast<const int*>(stage + plan.row_word) - header[3];
    row_width_ = reinterpret_cast<const uint8_t*>(stage + plan.row_width) - header[4];
    values_ = reinterpret_cast<const V*>(stage + plan.values) - header[5];
    index_ = reinterpret_cast<const Index*>(stage + plan.index) - header[6];
    if constexpr (LAYOUT != SPMV_LAYOUT_LP) {
      windowed = header[7] != INT_MIN;
      window_ = reinterpret_cast<const V*>(stage + plan.window) - (windowed ? header[7] : 0);
    } else {
      // CSR-lp tiles never stage a window: a run-time choice on every gather of the decode measured slower
      // on B200 (27-point stencil T = 8: 0.362 ms against 0.268 ms; random band T = 8 with windows: 0.109 ms
      // against 0.097 ms without)
      windowed = false;
      window_ = nullptr;
    }
  }
  __device__ __forceinline__ int row_ptr(int row) const { return row_ptr_[row]; }
  __device__ __forceinline__ int row_base(int row) const { return row_base_[row]; }
  __device__ __forceinline__ int row_word(int row) const { return row_word_[row]; }
  __device__ __forceinline__ uint32_t row_width(int row) const { return row_width_[row]; }
  __device__ __forceinline__ V value(int entry) const { return values_[entry]; }
  __device__ __forceinline__ Index index(int entry) const { return index_[entry]; }
  __device__ __forceinline__ uint32_t word(int64_t w) const { return reinterpret_cast<const uint32_t*>(index_)[w]; }
};

template <class V, int LAYOUT>
struct GlobalView {
  using Index = typename LayoutTraits<LAYOUT>::Index;
  const KernelArgs& a;
  uint64_t stream;
  static constexpr bool windowed = false;
  const V* window_ = nullptr;
  __device__ __forceinline__ explicit GlobalView(const KernelArgs& args) : a(args), stream(l2_stream_policy()) {}
  __device__ __forceinline__ int row_ptr(int row) const { return load_readonly(a.row_ptr + row); }
  __device__ __forceinline__ int row_base(int row) const { return load_readonly(a.row_base + row); }
  __device__ __forceinline__ int row_word(int row) const { return load_readonly(a.row_word + row); }
  __device__ __forceinline__ uint32_t row_width(int row) const { return load_readonly(a.row_width + row); }
  __device__ __forceinline__ V value(int entry) const { return load_stream(static_cast<const V*>(a.values) + entry, stream); }
  __device__ __forceinline__ Index index(int entry) const { return load_stream(static_cast<const Index*>(a.columns) + entry, stream); }
  __device__ __forceinline__ uint32_t word(int64_t w) const { return load_readonly(a.words + w); }
};

// Delta of a CSR-lp lane at bit `bit` of the row's stream starting at word w0 (bit width * (lane *
// quotient + min(lane, remainder) + k) for its k-th delta, lane_major_bit of the reference): the two
// 32-bit words around it always hold it (a width never exceeds 32 bits).
template <class View, class Bit>
__device__ __forceinline__ uint32_t packed_delta(const View& view, int64_t w0, Bit bit, uint32_t mask) {
  const int64_t w = w0 + (int64_t)(bit >> 5);
  return __funnelshift_r(view.word(w), view.word(w + 1), (uint32_t)(bit & 31)) & mask;
}

// ---- the vector path -----------------------------------------------------------------------------------
// One group of T threads per row, each thread one logical lane, straight from global memory. CTA `block`
// of `blocks` (of BLOCK threads each) takes the rows item = group, group + groups, ... of the row list.
template <class V, int LAYOUT, int T, int BLOCK, int UNROLL = 4>
__device__ __forceinline__ void vector_rows(const KernelArgs& a, int64_t block, int64_t blocks) {
  using VT = ValueTraits<V>;
  using Acc = typename VT::Acc;
  using Index = typename LayoutTraits<LAYOUT>::Index;
  constexpr bool kPacked = LAYOUT == SPMV_LAYOUT_LP;
  constexpr bool kBase = LayoutTraits<LAYOUT>::kBase;
  const V* values = static_cast<const V*>(a.values);
  const V* x = static_cast<const V*>(a.x);
  V* y = static_cast<V*>(a.y);
  const int lane = threadIdx.x & (T - 1);
  const int64_t group = (block * BLOCK + threadIdx.x) / T;
  const int64_t groups = (blocks * BLOCK) / T;

  for (int64_t first = 0; first < a.row_count; first += groups) {   // the same trip count on every thread
    const int64_t item = first + group;
    const int row = item < a.row_count ? (a.row_list ? a.row_list[item] : (int)item) : 0;
    Acc sum = Acc(0);
    if (item < a.row_count) {
      const int64_t entry_begin = a.row_ptr[row], entry_end = a.row_ptr[row + 1];
      if constexpr (!kPacked) {
        const Index* columns = static_cast<const Index*>(a.columns);
        const int base = kBase ? a.row_base[row] : 0;
#pragma unroll UNROLL
        for (int64_t entry = entry_begin + lane; entry < entry_end; entry += T)
          sum = VT::fma(VT::widen(load_readonly(values + entry)),
                        VT::widen(load_readonly(x + base + (int)load_readonly(columns + entry))), sum);
      } else {
        // logical lane `lane` owns the row's deltas lane * quotient + min(lane, remainder) + k, k < its count
        // (lane-major order); each is a funnel shift of the two words around its bit offset, which may pass
        // 2^32 bits in a long row
        const GlobalView<V, LAYOUT> view(a);
        const int64_t length = entry_end - entry_begin;
        const int64_t quotient = length / T, remainder = length - quotient * T;
        const int64_t count = quotient + (lane < remainder ? 1 : 0);
        const uint32_t width = view.row_width(row);
        const uint32_t mask = width == 0 ? 0u : (0xffffffffu >> (32 - width));
        const int64_t w0 = view.row_word(row);
        uint64_t bit = (uint64_t)width * (uint64_t)(lane * quotient + (lane < remainder ? lane : remainder));
        int column = view.row_base(row);
        int64_t entry = entry_begin + lane;
        for (int64_t k = 0; k < count; ++k, entry += T, bit += width) {
          column += (int)packed_delta(view, w0, bit, mask);
          sum = VT::fma(VT::widen(load_readonly(values + entry)), VT::widen(load_readonly(x + column)), sum);
        }
      }
    }
#pragma unroll
    for (int offset = T / 2; offset > 0; offset >>= 1) sum = VT::add(sum, __shfl_down_sync(0xffffffffu, sum, offset, T));
    if (lane == 0 && item < a.row_count) {
      const V result = VT::narrow(sum);
      y[row] = result;
      mirror_row(a, row, result);
    }
  }
}

// x at a column: from the tile's window of x in shared memory when the tile staged one, else from global
// memory (kept in L2).
template <class View, class V>
__device__ __forceinline__ V gather_x(const View& view, const V* __restrict__ x, int column, uint64_t keep) {
  return view.windowed ? view.window_[column] : load_x(x + column, keep);
}

// The lane sums of one row (entries [entry_begin, entry_end), column base `base` for the row-relative and
// CSR-lp layouts) on its P threads (thread p of the group) into acc[j], the sum of logical lane p + j*P.
// A thread gathers x for up to kBatch of its entries at once (R rounds of its S lanes) into registers, then
// adds them into its lane chains in order.
template <class V, int LAYOUT, int T, int P, int kBatch, class View>
__device__ __forceinline__ void row_lane_sums(const View& view, const V* __restrict__ x, int row, int entry_begin,
                                              int entry_end, int base, int p,
                                              typename ValueTraits<V>::Acc (&acc)[T / P]) {
  using VT = ValueTraits<V>;
  constexpr bool kPacked = LAYOUT == SPMV_LAYOUT_LP;
  constexpr bool kBase = LayoutTraits<LAYOUT>::kBase;
  constexpr int S = T / P;
  constexpr int R = S >= kBatch ? 1 : kBatch / S;
  const uint64_t keep = l2_keep_policy();
  if constexpr (!kPacked) {
    if constexpr (!kBase) base = 0;   // absolute columns
    for (int entry = entry_begin + p; entry < entry_end; entry += T * R) {
      V xv[R][S];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int j = 0; j < S; ++j) {
          const int e = entry + r * T + j * P;
          if (e < entry_end) xv[r][j] = load_x(x + base + (int)view.index(e), keep);
        }
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int j = 0; j < S; ++j) {
          const int e = entry + r * T + j * P;
          if (e < entry_end) acc[j] = VT::fma(VT::widen(view.value(e)), VT::widen(xv[r][j]), acc[j]);
        }
    }
  } else {
    // lane p + j*P owns quotient (+1 below remainder) deltas from bit width * (lane * quotient +
    // min(lane, remainder)); both are recomputed where used, so only the running columns stay live
    const int length = entry_end - entry_begin;
    const int quotient = length / T, remainder = length - quotient * T;
    const uint32_t width = view.row_width(row);
    const uint32_t mask = width == 0 ? 0u : (0xffffffffu >> (32 - width));
    const int64_t w0 = view.row_word(row);
    int column[S];
#pragma unroll
    for (int j = 0; j < S; ++j) column[j] = base;
    const int rounds = quotient + (remainder > 0 ? 1 : 0);
    for (int round = 0; round < rounds; round += R) {
      V xv[R][S];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int j = 0; j < S; ++j) {
          const int lane = p + j * P;
          if (round + r < quotient + (lane < remainder ? 1 : 0)) {
            const uint32_t delta = (uint32_t)(lane * quotient + (lane < remainder ? lane : remainder) + round + r);
            column[j] += (int)packed_delta(view, w0, delta * width, mask);
            xv[r][j] = gather_x(view, x, column[j], keep);
          }
        }
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int j = 0; j < S; ++j) {
          const int lane = p + j * P;
          if (round + r < quotient + (lane < remainder ? 1 : 0))
            acc[j] = VT::fma(VT::widen(view.value(entry_begin + lane + (round + r) * T)), VT::widen(xv[r][j]), acc[j]);
        }
    }
  }
}

// CSR-lp rows of at most R rounds (R * T entries) on P threads, R = kBatch / S: the thread decodes its S
// lanes G at a time, each lane from its first delta with its own running column (a lane's deltas are
// contiguous in the lane-major stream, and the lanes' chains are independent), so that every gather of the
// row is in flight at once while only G running columns stay live; the G interleaved chains give the
// decode its parallelism. The products are then added in lane order.
// lanes decoded side by side (2, 4 and 8 measured alike on B200: 27-point stencil T = 32, power law T = 32)
constexpr int kDecodeGroup = 4;
template <class V, int T, int P, int kBatch, class View>
__device__ __forceinline__ void packed_short_row(const View& view, const V* __restrict__ x, int row, int entry_begin,
                                                 int length, int base, int p,
                                                 typename ValueTraits<V>::Acc (&acc)[T / P]) {
  using VT = ValueTraits<V>;
  constexpr int S = T / P;
  constexpr int R = S >= kBatch ? 1 : kBatch / S;
  constexpr int G = S < kDecodeGroup ? S : kDecodeGroup;
  const uint64_t keep = l2_keep_policy();
  const int quotient = length / T, remainder = length - quotient * T;
  const uint32_t width = view.row_width(row);
  const uint32_t mask = width == 0 ? 0u : (0xffffffffu >> (32 - width));
  const int64_t w0 = view.row_word(row);
  V xv[R][S];
#pragma unroll
  for (int j0 = 0; j0 < S; j0 += G) {
    int column[G];
#pragma unroll
    for (int g = 0; g < G; ++g) column[g] = base;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int lane = p + (j0 + g) * P;
        if (r < quotient + (lane < remainder ? 1 : 0)) {
          const uint32_t delta = (uint32_t)(lane * quotient + (lane < remainder ? lane : remainder) + r);
          column[g] += (int)packed_delta(view, w0, delta * width, mask);
          xv[r][j0 + g] = gather_x(view, x, column[g], keep);
        }
      }
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int j = 0; j < S; ++j) {
      const int lane = p + j * P;
      if (r < quotient + (lane < remainder ? 1 : 0))
        acc[j] = VT::fma(VT::widen(view.value(entry_begin + lane + r * T)), VT::widen(xv[r][j]), acc[j]);
    }
}

// CSR-lp rows longer than the lane-by-lane batch (rare in tiles): lane by lane as well, four deltas of the
// lane gathered at a time, so that no column per lane stays live and the registers stay those of
// packed_short_row.
template <class V, int T, int P, class View>
__device__ __forceinline__ void packed_lanes_in_turn(const View& view, const V* __restrict__ x, int row, int entry_begin,
                                                     int length, int base, int p,
                                                     typename ValueTraits<V>::Acc (&acc)[T / P]) {
  using VT = ValueTraits<V>;
  constexpr int S = T / P;
  constexpr int kDepth = 4;
  const uint64_t keep = l2_keep_policy();
  const int quotient = length / T, remainder = length - quotient * T;
  const uint32_t width = view.row_width(row);
  const uint32_t mask = width == 0 ? 0u : (0xffffffffu >> (32 - width));
  const int64_t w0 = view.row_word(row);
#pragma unroll
  for (int j = 0; j < S; ++j) {
    const int lane = p + j * P;
    const int count = quotient + (lane < remainder ? 1 : 0);
    const uint32_t first = (uint32_t)(lane * quotient + (lane < remainder ? lane : remainder));
    int column = base;
    for (int k = 0; k < count; k += kDepth) {
      V xv[kDepth];
#pragma unroll
      for (int r = 0; r < kDepth; ++r)
        if (k + r < count) {
          column += (int)packed_delta(view, w0, (first + k + r) * width, mask);
          xv[r] = gather_x(view, x, column, keep);
        }
#pragma unroll
      for (int r = 0; r < kDepth; ++r)
        if (k + r < count)
          acc[j] = VT::fma(VT::widen(view.value(entry_begin + lane + (k + r) * T)), VT::widen(xv[r]), acc[j]);
    }
  }
}

// The product of one row on its P threads: the lane sums and the reduction tree. Every thread of the warp
// must call it (the tree shuffles); rows of inactive groups contribute nothing.
template <class V, int LAYOUT, int T, int P, int kBatch, class View>
__device__ __forceinline__ typename ValueTraits<V>::Acc row_product(const View& view, const V* __restrict__ x, int row,
                                                                    int entry_begin, int entry_end, int base, bool active,
                                                                    int p) {
  using VT = ValueTraits<V>;
  using Acc = typename VT::Acc;
  constexpr int S = T / P;
  Acc acc[S];
#pragma unroll
  for (int j = 0; j < S; ++j) acc[j] = Acc(0);
  if (active) row_lane_sums<V, LAYOUT, T, P, kBatch>(view, x, row, entry_begin, entry_end, base, p, acc);
  return reduce_lanes<VT, Acc, T, P>(acc);
}

// ---- a resident tile, from one shared-memory buffer -------------------------------------------------
// Rows go to groups of P threads in passes; every thread runs every pass, so the shuffles of the
// reduction always see the full warp; a row of up to R*T entries costs one round trip to memory.
#ifndef SPMV_TILE_GATHERS
#define SPMV_TILE_GATHERS 32
#endif
constexpr int kGathers = SPMV_TILE_GATHERS;

// CTAs per multiprocessor whose registers a tile variant is built for: 2, or for the dense variants of one
// thread per lane (P = T) 4 with 4-byte or narrower values and 3 with FP64 ones. A thread of a dense
// variant gathers 8 x values at once (the lane's entries of a row up to 8*T long in one round trip).
// Measured on B200 (block FEM slice, 64 nonzeros a row in runs of 8, FP32, T = 8): 208 us a product
// against 321 us at 2 CTAs (CSR-lp: 236 us against 365 us with P = 4); rows with x windows (random band)
// lose their window room and run slower.
template <class V>
struct DenseResidency { static constexpr int value = sizeof(V) == 8 ? 3 : 4; };

// Rows go to the groups of P threads from group `rotation` on (row i of the tile to group (rotation + i) mod
// groups, a pass of `groups` rows at a time); returns the tile's rows. The caller advances the rotation by
// each tile's rows, so that a tile with fewer rows than groups leaves different warps idle each time and
// every warp takes its share of the rows (otherwise the last warps of the CTA would never get a row and
// sit idle for the whole launch, e.g. 27-point stencil T = 8 on one thread per row: about 189 rows a tile
// for 256 groups).
template <class V, int LAYOUT, int T, int P, int W>
__device__ __forceinline__ int process_tile(const KernelArgs& a, const unsigned char* stage, const StagePlan& plan,
                                            int rotation) {
  using VT = ValueTraits<V>;
  constexpr bool kPacked = LAYOUT == SPMV_LAYOUT_LP;
  constexpr int S = T / P;
  // x values gathered at once per thread: 32, or 16 for FP64 when 16 lane sums already hold many of the 128
  // registers two CTAs of 256 threads leave a thread
  constexpr int kBatch = W > 2 ? 8 : ((sizeof(V) == 8 && S >= 16) ? kGathers / 2 : kGathers);
  constexpr int kGroups = kTileBlock / P;
  const TileView<V, LAYOUT> tile(stage, plan);
  const V* x = static_cast<const V*>(a.x);
  V* y = static_cast<V*>(a.y);
  const uint64_t keep = l2_keep_policy();
  const int group = threadIdx.x / P, p = threadIdx.x % P;
  const int slot = group >= rotation ? group - rotation : group - rotation + kGroups;

  for (int first = 0; first < tile.rows; first += kGroups) {
    const int local = first + slot;
    const int row = tile.row_begin + local;
    const bool active = local < tile.rows;
    if constexpr (!kPacked) {
      // the entries' loop written out here rather than through row_product: measured faster for the
      // absolute and row-relative layouts (27-point stencil, FP64, T = 8: 257 us against 303 us)
      using Acc = typename VT::Acc;
      constexpr int R = S >= kBatch ? 1 : kBatch / S;
      Acc acc[S];
#pragma unroll
      for (int j = 0; j < S; ++j) acc[j] = Acc(0);
      if (active) {
        const int entry_begin = tile.row_ptr(row), entry_end = tile.row_ptr(row + 1);
        const int base = LayoutTraits<LAYOUT>::kBase ? tile.row_base(row) : 0;
        for (int entry = entry_begin + p; entry < entry_end; entry += T * R) {
          V xv[R][S];
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int j = 0; j < S; ++j) {
              const int e = entry + r * T + j * P;
              if (e < entry_end) {
                const int column = base + (int)tile.index(e);
                xv[r][j] = tile.windowed ? tile.window_[column] : load_x(x + column, keep);
              }
            }
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int j = 0; j < S; ++j) {
              const int e = entry + r * T + j * P;
              if (e < entry_end) acc[j] = VT::fma(VT::widen(tile.value(e)), VT::widen(xv[r][j]), acc[j]);
            }
        }
      }
      const Acc sum = reduce_lanes<VT, Acc, T, P>(acc);
      if (p == 0 && active) {
        const V result = VT::narrow(sum);
        y[row] = result;
        mirror_row(a, row, result);
      }
    } else {
      // CSR-lp: a row of at most R rounds decoded lane by lane with all its gathers at once, a longer row
      // round by round
      using Acc = typename VT::Acc;
      constexpr int R = S >= kBatch ? 1 : kBatch / S;
      Acc acc[S];
#pragma unroll
      for (int j = 0; j < S; ++j) acc[j] = Acc(0);
      if (active) {
        const int begin = tile.row_ptr(row), end = tile.row_ptr(row + 1);
        const int base = tile.row_base(row);
        // FP64 with at most 8 lanes a thread: round by round, 16 gathers at a time (the lanes' running
        // columns interleave the decode chains); measured on B200, 27-point stencil T = 8: 0.270 ms a product
        // against 0.329-0.335 ms decoding 2, 4 or 8 lanes side by side with all 27 gathers at once
        if constexpr (S <= 8 && sizeof(V) == 8) {
          row_lane_sums<V, LAYOUT, T, P, kBatch / 2>(tile, x, row, begin, end, base, p, acc);
        } else if (end - begin <= R * T)
          packed_short_row<V, T, P, kBatch>(tile, x, row, begin, end - begin, base, p, acc);
        else
          packed_lanes_in_turn<V, T, P>(tile, x, row, begin, end - begin, base, p, acc);
      }
      const Acc sum = reduce_lanes<VT, Acc, T, P>(acc);
      if (p == 0 && active) {
        const V result = VT::narrow(sum);
        y[row] = result;
        mirror_row(a, row, result);
      }
    }
  }
  return tile.rows;
}

// Thread 0: streams tile `tile_id` into a stage and arms its full barrier with the byte count.
template <class V, int LAYOUT>
__device__ __forceinline__ void issue_tile(const KernelArgs& a, int64_t tile_id, unsigned char* stage, const StagePlan& plan,
                                           uint32_t full) {
  using Index = typename LayoutTraits<LAYOUT>::Index;
  constexpr bool kPacked = LAYOUT == SPMV_LAYOUT_LP;
  constexpr bool kBase = LayoutTraits<LAYOUT>::kBase;
  const int4 tile = a.tiles[tile_id];
  const AlignedRange<int> row_ptr(a.row_ptr, tile.x, (int64_t)tile.y + 1);
  const AlignedRange<int> row_base(kBase ? a.row_base : a.row_ptr, tile.x, tile.y);
  const AlignedRange<uint8_t> row_width(kPacked ? a.row_width : reinterpret_cast<const uint8_t*>(a.row_ptr), tile.x, tile.y);
  const AlignedRange<V> values(static_cast<const V*>(a.values), tile.z, tile.w);
  const Index* index_base = kPacked ? reinterpret_cast<const Index*>(a.words) : static_cast<const Index*>(a.columns);
  int64_t index_first = tile.z, index_last = tile.w;
  if (kPacked) {
    const int2 words = a.tile_words[tile_id];
    index_first = words.x;
    index_last = (int64_t)words.y + 1;    // a window reads one word past the row's last
  }
  const AlignedRange<Index> index(index_base, index_first, index_last);
  const uint64_t stream = l2_stream_policy();
  int* header = reinterpret_cast<int*>(stage + plan.header);
  header[0] = tile.x;
  header[1] = tile.y - tile.x;
  header[2] = (int)row_ptr.origin;
  header[3] = (int)row_base.origin;
  header[4] = (int)row_width.origin;
  header[5] = (int)values.origin;
  header[6] = (int)index.origin;
  uint32_t bytes = row_ptr.bytes + values.bytes + index.bytes;
  if (kBase) bytes += row_base.bytes;
  if (kPacked) bytes += row_base.bytes + row_width.bytes;   // row_word has the extent of row_base
  // the tile's window of x (columns [window.x, window.y)), when the plan gave it one: its gathers then read
  // shared memory. x is 16-byte aligned whenever windows are on, and the plan keeps every window's 16-byte
  // superset inside x.
  const int2 window = !kPacked && a.tile_windows ? a.tile_windows[tile_id] : make_int2(0, 0);
  const AlignedRange<V> x_window(static_cast<const V*>(a.x), window.x, window.y > window.x ? window.y : window.x);
  const bool windowed = window.y > window.x;
  header[7] = windowed ? (int)x_window.origin : INT_MIN;
  if (windowed) bytes += x_window.bytes;
  mbarrier_arrive_expect_tx(full, bytes);
  // a range may be empty (a tile of empty rows has no values): no copy is issued for 0 bytes
  if (row_ptr.bytes)
    bulk_copy_g2s(smem_address(stage + plan.row_ptr), reinterpret_cast<const void*>(row_ptr.begin), row_ptr.bytes, full, stream);
  if (kBase && row_base.bytes)
    bulk_copy_g2s(smem_address(stage + plan.row_base), reinterpret_cast<const void*>(row_base.begin), row_base.bytes, full, stream);
  if (kPacked && row_base.bytes) {
    const AlignedRange<int> row_word(a.row_word, tile.x, tile.y);
    bulk_copy_g2s(smem_address(stage + plan.row_word), reinterpret_cast<const void*>(row_word.begin), row_word.bytes, full, stream);
  }
  if (kPacked && row_width.bytes)
    bulk_copy_g2s(smem_address(stage + plan.row_width), reinterpret_cast<const void*>(row_width.begin), row_width.bytes, full, stream);
  if (values.bytes)
    bulk_copy_g2s(smem_address(stage + plan.values), reinterpret_cast<const void*>(values.begin), values.bytes, full, stream);
  if (index.bytes)
    bulk_copy_g2s(smem_address(stage + plan.index), reinterpret_cast<const void*>(index.begin), index.bytes, full, stream);
  if (windowed)
    bulk_copy_g2s(smem_address(stage + plan.window), reinterpret_cast<const void*>(x_window.begin), x_window.bytes, full,
                  l2_keep_policy());
}

// ---- rows longer than a tile ----------------------------------------------------------------------------
// A row of the long-row list takes a whole CTA, chunk by chunk (a chunk starts at a multiple of T within
// the row, so an entry keeps its lane), with the warps specialised. Warp 0 consumes: its T lane owners
// add a chunk into their lane sums in order. The gatherers (warps 1..7) fill one of two shared-memory
// buffers per chunk with the chunk's values and x gathered at its columns. For CSR-lp each gatherer decodes
// the columns it gathers: a segment of kLaneMarkEvery deltas of one lane from that lane's column mark, the
// lanes of a segment on neighbouring threads (so that their values are read together). Named barriers hand
// the buffers over (ids 1..4, see below); every thread walks the same rows and chunks, so every barrier
// completes. The lane sums finish in the width-T shuffle tree of warp 0.
__host__ __device__ inline int long_smem_bytes(int chunk, int value_bytes) { return 4 * chunk * value_bytes; }

// CSR-lp long rows: a lane's deltas in segments of this many, each decoded on its own from the lane's
// column mark before it (the marks come from the matrix's columns when the operator is created). A chunk
// holds whole segments of every lane: its entries are a multiple of kLaneMarkEvery * T.
constexpr int kLaneMarkEvery = 16;

// Named barriers with immediate ids, so that the kernel reserves only the barriers it uses.
template <int ID, int THREADS>
__device__ __forceinline__ void named_barrier_sync() {
  asm volatile("barrier.sync %0, %1;" ::"n"(ID), "n"(THREADS) : "memory");
}
template <int ID, int THREADS>
__device__ __forceinline__ void named_barrier_arrive() {
  asm volatile("barrier.arrive %0, %1;" ::"n"(ID), "n"(THREADS) : "memory");
}
// A pair of named barriers (ids ID0 for buffer 0, ID0 + 1 for buffer 1) between THREADS threads.
template <int ID0, int THREADS>
struct BarrierPair {
  __device__ static __forceinline__ void sync(int b) {
    if (b == 0) named_barrier_sync<ID0, THREADS>(); else named_barrier_sync<ID0 + 1, THREADS>();
  }
  __device__ static __forceinline__ void arrive(int b) {
    if (b == 0) named_barrier_arrive<ID0, THREADS>(); else named_barrier_arrive<ID0 + 1, THREADS>();
  }
};

template <class V, int LAYOUT, int T>
__device__ __forceinline__ void long_rows(const KernelArgs& a, unsigned char* smem, int64_t block, int64_t blocks) {
  using VT = ValueTraits<V>;
  using Acc = typename VT::Acc;
  using Index = typename LayoutTraits<LAYOUT>::Index;
  constexpr bool kPacked = LAYOUT == SPMV_LAYOUT_LP;
  constexpr bool kBase = LayoutTraits<LAYOUT>::kBase;
  constexpr int kFirstGatherer = 32;
  constexpr int kGatherers = kTileBlock - kFirstGatherer;
  using Full = BarrierPair<1, kGatherers + 32>;              // gatherers arrive, the consumer waits
  using Free = BarrierPair<3, kGatherers + 32>;              // the consumer arrives, gatherers wait
  // entries per chunk: a multiple of kTileBlock (and so of T), for CSR-lp of kLaneMarkEvery * T as well
  const int chunk = a.long_chunk;
  if (long_smem_bytes(chunk, (int)sizeof(V)) > a.smem_bytes ||
      (kPacked && chunk % (kLaneMarkEvery * T) != 0)) {   // never by construction
    if (threadIdx.x == 0 && a.status) atomicOr(a.status, kStatusSmem);
    return;
  }
  V* const s_values = reinterpret_cast<V*>(smem);                    // [2][chunk]
  V* const s_x = s_values + 2 * chunk;                                // [2][chunk]
  const V* values = static_cast<const V*>(a.values);
  const V* x = static_cast<const V*>(a.x);
  const Index* index = static_cast<const Index*>(a.columns);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  for (int64_t item = block; item < a.row_count; item += blocks) {
    const int row = a.row_list[item];
    const int64_t begin = a.row_ptr[row], length = a.row_ptr[row + 1] - begin;
    const int chunks = (int)((length + chunk - 1) / chunk);
    auto count_of = [&](int k) {
      return (int)(length - (int64_t)k * chunk < chunk ? length - (int64_t)k * chunk : chunk);
    };
    if (warp == 0) {   // consumer
      Acc sum = Acc(0);
      for (int k = 0; k < chunks; ++k) {
        const int b = k & 1, count = count_of(k);
        Full::sync(b);
        if (lane < T) {
          const V* v = s_values + b * chunk;
          const V* g = s_x + b * chunk;
#pragma unroll 8
          for (int i = lane; i < count; i += T) sum = VT::fma(VT::widen(v[i]), VT::widen(g[i]), sum);
        }
        Free::arrive(b);
      }
#pragma unroll
      for (int offset = T / 2; offset > 0; offset >>= 1) sum = VT::add(sum, __shfl_down_sync(0xffffffffu, sum, offset, T));
      if (lane == 0) {
        const V result = VT::narrow(sum);
        static_cast<V*>(a.y)[row] = result;
        mirror_row(a, row, result);
      }
    } else {   // gatherers
      const int gatherer = (int)threadIdx.x - kFirstGatherer;
      const int base = kBase ? a.row_base[row] : 0;
      const uint64_t keep = l2_keep_policy(), stream = l2_stream_policy();
      for (int k = 0; k < chunks; ++k) {
        const int b = k & 1, count = count_of(k);
        if (k >= 2) Free::sync(b);   // the consumer is done with chunk k - 2
        const int64_t first = begin + (int64_t)k * chunk;
        V* v = s_values + b * chunk;
        V* g = s_x + b * chunk;
        if constexpr (kPacked) {
          // task t: lane t % T, segment t / T of the chunk's segments (deltas d0 .. d0 + K - 1 of the lane)
          constexpr int K = kLaneMarkEvery;
          const int quotient = (int)(length / T), remainder = (int)(length - (int64_t)quotient * T);
          const uint32_t width = a.row_width[row];
          const uint32_t mask = width == 0 ? 0u : (0xffffffffu >> (32 - width));
          const uint32_t* words = a.words + a.row_word[row];
          const int* marks = a.lane_marks + a.lane_mark_first[item];
          const int per_lane = chunk / T;
          for (int t = gatherer; t < (per_lane / K) * T; t += kGatherers) {
            const int lane_of = t % T;
            const int d0 = k * per_lane + (t / T) * K;
            const int n = quotient + (lane_of < remainder ? 1 : 0) - d0;   // deltas of the lane from d0 on
            if (n <= 0) continue;
            int column = d0 == 0 ? base : marks[(d0 / K - 1) * T + lane_of];
            const uint64_t bit0 =
                (uint64_t)width * (uint64_t)(lane_of * quotient + (lane_of < remainder ? lane_of : remainder) + d0);
            const int64_t e0 = (int64_t)lane_of + (int64_t)d0 * T - (int64_t)k * chunk;   // chunk entry of d0
#pragma unroll
            for (int h = 0; h < K; h += 8) {
              // the words of 8 deltas first (their positions do not depend on the decode), then the
              // running column, the values and the gathers
              uint32_t delta[8];
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (h + j < n) {
                  const uint64_t at = bit0 + (uint64_t)(h + j) * width;
                  const uint64_t w = at >> 5;
                  delta[j] = __funnelshift_r(load_readonly(words + w), load_readonly(words + w + 1),
                                             (uint32_t)(at & 31)) & mask;
                }
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (h + j < n) {
                  column += (int)delta[j];
                  const int i = (int)(e0 + (int64_t)(h + j) * T);
                  v[i] = load_stream(values + first + i, stream);
                  g[i] = load_x(x + column, keep);
                }
            }
          }
        } else {
#pragma unroll 8
          for (int i = gatherer; i < count; i += kGatherers) {
            const int c = base + (int)load_stream(index + first + i, stream);
            v[i] = load_stream(values + first + i, stream);
            g[i] = load_x(x + c, keep);
          }
        }
        Full::arrive(b);
      }
      // the next row refills the buffers: wait until the consumer has released the last ones
      for (int k = chunks >= 2 ? chunks - 2 : 0; k < chunks; ++k) Free::sync(k & 1);
    }
  }
}

// ---- rows by length (k_spmv_classes) ------------------------------------------------------------------
// For matrices whose nonzeros sit in rows of very different lengths, rows are classed by length and each
// class runs on its own mapping straight from global memory (no tiles): short rows (at most kShortMax
// entries) one per thread, several per thread at once; longer rows from a list, each on P threads with P
// chosen per row (the fewest, with at most 8 lane sums a thread, that leave a thread at most 32 of its
// entries; segments of equal P, longest rows first); rows longer than the long-row threshold one per CTA (long_rows above). The summation order
// is the same in every class.
constexpr int kShortMax = 8;
// x values a thread of a listed row gathers at once (the class kernel runs 4 CTAs of 256 threads per
// multiprocessor, 64 registers a thread)
template <class V> struct ClassGathers { static constexpr int value = sizeof(V) == 8 ? 8 : 16; };

template <class V> struct ShortRowsPerThread { static constexpr int value = sizeof(V) == 8 ? 1 : 2; };

// Rows chunk * 256U + u * 256 + threadIdx.x (u < U) of the matrix; rows longer than kShortMax are left to
// the listed and long rows. Entry j of a short row is entry j / W of logical lane j % W, W = min(T, kShortMax).
// For T > W the lanes W..T-1 are empty (+0): the tree levels with offsets >= W add +0 to each of the first
// W lane sums (which only turns a -0 into +0, once), and the levels below W are the tree of W lanes.
template <class V, int LAYOUT, int T>
__device__ __forceinline__ void short_rows(const KernelArgs& a, int64_t chunk) {
  using VT = ValueTraits<V>;
  using Acc = typename VT::Acc;
  constexpr int U = ShortRowsPerThread<V>::value;
  constexpr int W = T < kShortMax ? T : kShortMax;
  constexpr bool kPacked = LAYOUT == SPMV_LAYOUT_LP;
  constexpr bool kBase = LayoutTraits<LAYOUT>::kBase;
  const GlobalView<V, LAYOUT> g(a);
  const V* x = static_cast<const V*>(a.x);
  V* y = static_cast<V*>(a.y);
  const uint64_t keep = l2_keep_policy();
  int row[U], begin[U], length[U];
  bool mine[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int64_t r = chunk * (int64_t)(kTileBlock * U) + u * kTileBlock + threadIdx.x;
    row[u] = (int)r;
    mine[u] = r < a.rows;
    begin[u] = mine[u] ? g.row_ptr(row[u]) : 0;
    length[u] = mine[u] ? g.row_ptr(row[u] + 1) - begin[u] : 0;
    mine[u] = mine[u] && length[u] <= kShortMax;
  }
  V xv[U][kShortMax];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if constexpr (!kPacked) {
      const int base = kBase && mine[u] ? g.row_base(row[u]) : 0;
#pragma unroll
      for (int j = 0; j < kShortMax; ++j)
        if (mine[u] && j < length[u]) xv[u][j] = load_x(x + base + (int)g.index(begin[u] + j), keep);
    } else {
      if (mine[u] && length[u] > 0) {
        const int quotient = length[u] / T, remainder = length[u] - quotient * T;
        const uint32_t width = g.row_width(row[u]);
        const uint32_t mask = width == 0 ? 0u : (0xffffffffu >> (32 - width));
        const int64_t w0 = g.row_word(row[u]);
        int column[W];
        const int base = g.row_base(row[u]);
#pragma unroll
        for (int l = 0; l < W; ++l) column[l] = base;
#pragma unroll
        for (int j = 0; j < kShortMax; ++j) {
          const int lane = j % W, k = j / W;
          if (j < length[u]) {
            const uint32_t delta = (uint32_t)(lane * quotient + (lane < remainder ? lane : remainder) + k);
            column[lane] += (int)packed_delta(g, w0, delta * width, mask);
            xv[u][j] = load_x(x + column[lane], keep);
          }
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    Acc acc[W];
#pragma unroll
    for (int l = 0; l < W; ++l) acc[l] = Acc(0);
#pragma unroll
    for (int j = 0; j < kShortMax; ++j)
      if (mine[u] && j < length[u]) acc[j % W] = VT::fma(VT::widen(g.value(begin[u] + j)), VT::widen(xv[u][j]), acc[j % W]);
    if constexpr (T > W) {
#pragma unroll
      for (int l = 0; l < W; ++l) acc[l] = VT::add(acc[l], Acc(0));
    }
#pragma unroll
    for (int offset = W / 2; offset > 0; offset >>= 1)
#pragma unroll
      for (int l = 0; l < offset; ++l) acc[l] = VT::add(acc[l], acc[l + offset]);
    if (mine[u]) {
      const V result = VT::narrow(acc[0]);
      y[row[u]] = result;
      mirror_row(a, row[u], result);
    }
  }
}

// Items chunk * (256 / P) + group of segment `segment` of the row items, one row per group of P threads.
template <class V, int LAYOUT, int T, int P>
__device__ __forceinline__ void listed_rows(const KernelArgs& a, int segment, int64_t chunk) {
  using VT = ValueTraits<V>;
  const int group = threadIdx.x / P, p = threadIdx.x % P;
  const int64_t index = chunk * (kTileBlock / P) + group;
  const bool active = index < a.segment_items[segment];
  const int4 item = active ? __ldg(a.row_items + a.segment_first[segment] + index) : make_int4(0, 0, 0, 0);
  const GlobalView<V, LAYOUT> g(a);
  // CSR-lp gathers half as deep: its decode state and the 16-deep batch spill at the class kernel's 64
  // registers (44 bytes a thread for FP16 at T = 32)
  constexpr int kBatch = LAYOUT == SPMV_LAYOUT_LP ? ClassGathers<V>::value / 2 : ClassGathers<V>::value;
  if constexpr (LAYOUT == SPMV_LAYOUT_LP) {
    // CSR-lp: lane by lane (one running column), all of a row's gathers at once when it has at most R
    // rounds, else four deltas of a lane at a time
    using Acc = typename VT::Acc;
    constexpr int S = T / P;
    constexpr int R = S >= kBatch ? 1 : kBatch / S;
    Acc acc[S];
#pragma unroll
    for (int j = 0; j < S; ++j) acc[j] = Acc(0);
    if (active) {
      const int length = item.z - item.y;
      if (length <= R * T)
        packed_short_row<V, T, P, kBatch>(g, static_cast<const V*>(a.x), item.x, item.y, length, item.w, p, acc);
      else
        packed_lanes_in_turn<V, T, P>(g, static_cast<const V*>(a.x), item.x, item.y, length, item.w, p, acc);
    }
    const Acc sum = reduce_lanes<VT, Acc, T, P>(acc);
    if (p == 0 && active) {
      const V result = VT::narrow(sum);
      static_cast<V*>(a.y)[item.x] = result;
      mirror_row(a, item.x, result);
    }
  } else {
    const auto sum = row_product<V, LAYOUT, T, P, kBatch>(g, static_cast<const V*>(a.x), item.x, item.y, item.z, item.w,
                                                          active, p);
    if (p == 0 && active) {
      const V result = VT::narrow(sum);
      static_cast<V*>(a.y)[item.x] = result;
      mirror_row(a, item.x, result);
    }
  }
}

// The segments that exist for T: P divides T with T / P <= 8 (at most 8 lane sums a thread).
__host__ __device__ constexpr bool segment_exists(int tpr, int segment) {
  return (1 << segment) <= tpr && tpr / (1 << segment) <= 8;
}

template <class V, int LAYOUT, int T, int SEGMENT>
__device__ __forceinline__ bool run_segment(const KernelArgs& a, int64_t& block) {
  if constexpr (segment_exists(T, SEGMENT)) {
    if (block < a.segment_blocks[SEGMENT]) {
      listed_rows<V, LAYOUT, T, (1 << SEGMENT)>(a, SEGMENT, block);
      return true;
    }
    block -= a.segment_blocks[SEGMENT];
  }
  return false;
}

// Blocks [0, long_blocks): one long row each; then the segments from P = 32 down to P = 1; then short rows.
// ---- programmatic dependent launch -------------------------------------------------------------------
// The product kernels are launched with programmatic stream serialization: each CTA lets the next kernel of
// the stream be scheduled as soon as every CTA of this grid has started, and that kernel's CTAs take the
// multiprocessors this grid's CTAs leave while it finishes. Before it reads x or writes y, a CTA waits
// until the previous kernel of the stream has completed and its memory is visible (griddepcontrol.wait
// returns at once when there is no such kernel, or when it never let its dependents start early: every
// other kernel of the library, the copies and the collectives keep the full stream order).
__device__ __forceinline__ void allow_next_grid() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void wait_for_previous_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <class V, int LAYOUT, int T>
__global__ void __launch_bounds__(kTileBlock, 4) k_spmv_classes(const KernelArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  allow_next_grid();
  wait_for_previous_grid();
  int64_t block = blockIdx.x;
  if (block < a.long_blocks) {
    long_rows<V, LAYOUT, T>(a, smem, block, a.long_blocks);
  } else {
    block -= a.long_blocks;
    if (!(run_segment<V, LAYOUT, T, 5>(a, block) || run_segment<V, LAYOUT, T, 4>(a, block) ||
          run_segment<V, LAYOUT, T, 3>(a, block) || run_segment<V, LAYOUT, T, 2>(a, block) ||
          run_segment<V, LAYOUT, T, 1>(a, block) || run_segment<V, LAYOUT, T, 0>(a, block)))
      short_rows<V, LAYOUT, T>(a, block);
  }
  publish_peer_rows(a);
}

// ---- k_spmv_tiles --------------------------------------------------------------------------------------
// Per tile k (buffer s = k mod stages): every thread waits for the buffer's bulk copies and processes its
// rows; each warp then counts itself out of the buffer, and the last warp out refills it at once with
// tile k + stages. No warp ever waits for another, nor for a producer.
// W: the CTAs per multiprocessor the registers are budgeted for (2, or DenseResidency for dense variants).
template <class V, int LAYOUT, int T, int P, int W>
__global__ void __launch_bounds__(kTileBlock, W) k_spmv_tiles(const KernelArgs a) {
  static_assert(T % P == 0 && P >= 1 && P <= 32, "P must divide T");
  constexpr int kWarps = kTileBlock / 32;
  extern __shared__ __align__(128) unsigned char smem[];
  allow_next_grid();
  if ((int64_t)blockIdx.x < a.vector_blocks) {   // rows longer than a tile, scheduled first
    wait_for_previous_grid();
    long_rows<V, LAYOUT, T>(a, smem, blockIdx.x, a.vector_blocks);
    publish_peer_rows(a);
    return;
  }
  __shared__ int s_abort;
  __shared__ int s_released[kMaxStages];   // warps done with the buffer's current tile
  __shared__ int s_fills[kMaxStages];      // bulk fills issued into the buffer so far
  const StagePlan plan = stage_plan(a.tile_nnz, a.tile_rows, (int)sizeof(V), LAYOUT, a.tile_index_words, a.window_elements);
  const int stages = a.stages;
  const int64_t cta = (int64_t)blockIdx.x - a.vector_blocks;
  const int64_t ctas = (int64_t)gridDim.x - a.vector_blocks;
  const int64_t my_tiles = cta < a.tile_count ? (a.tile_count - cta + ctas - 1) / ctas : 0;
  const uint32_t full0 = smem_address(smem);
  unsigned char* buffers = smem + 64;

  // the first buffers' copies read only the matrix, so they are issued before the wait for the previous
  // kernel; a tile that stages a window of x reads x, so with windows the wait comes first
  if (a.tile_windows) wait_for_previous_grid();
  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < stages; ++s) {
      mbarrier_init(full0 + 8 * s, 1);
      s_released[s] = 0;
      s_fills[s] = 0;
    }
    mbarrier_init_fence();
    for (int s = 0; s < stages && s < my_tiles; ++s) {
      issue_tile<V, LAYOUT>(a, cta + s * ctas, buffers + s * plan.bytes, plan, full0 + 8 * s);
      s_fills[s] = 1;
    }
  }
  wait_for_previous_grid();
  __syncthreads();

  int rotation = 0;   // the first group of the next tile's rows
  for (int64_t k = 0; k < my_tiles; ++k) {
    const int s = (int)(k % stages);
    if (!mbarrier_wait_bounded(full0 + 8 * s, (uint32_t)((k / stages) & 1), 2000000000ull)) {
      atomicExch(&s_abort, 1);
      if (a.status) atomicOr(a.status, kStatusTimeout);
    }
    // leave together or not at all: the reduction's shuffles need every lane of the warp
    if (__shfl_sync(0xffffffffu, *(volatile int*)&s_abort, 0)) break;
    const int rows = process_tile<V, LAYOUT, T, P, W>(a, buffers + s * plan.bytes, plan, rotation);
    rotation = (rotation + rows) % (kTileBlock / P);
    __syncwarp();
    if ((threadIdx.x & 31) == 0) {
      __threadfence_block();   // this warp's reads of the buffer happen before its release
      if (atomicAdd(&s_released[s], 1) == kWarps - 1) {
        __threadfence_block();
        s_released[s] = 0;
        if (k + stages < my_tiles) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue_tile<V, LAYOUT>(a, cta + (k + stages) * ctas, buffers + s * plan.bytes, plan, full0 + 8 * s);
          atomicAdd(&s_fills[s], 1);
        }
      }
    }
  }
  publish_peer_rows(a);
  __syncthreads();
  if (threadIdx.x == 0 && s_abort) {
    // after an abort: wait, bounded, for each buffer's last fill before the CTA's shared memory is released
    for (int s = 0; s < stages; ++s)
      if (s_fills[s] > 0) mbarrier_wait_bounded(full0 + 8 * s, (uint32_t)((s_fills[s] - 1) & 1), 100000000ull);
  }
}

// k_spmv_vector: the vector path over every row (row_list null) or a list of rows.
template <class V, int LAYOUT, int T>
__global__ void __launch_bounds__(kVectorBlock) k_spmv_vector(const KernelArgs a) {
  vector_rows<V, LAYOUT, T, kVectorBlock>(a, blockIdx.x, gridDim.x);
}

}  // namespace spmvb200
