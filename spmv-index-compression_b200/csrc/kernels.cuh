// kernels.cuh — sm_100a SpMV kernels for CSR with compressed column indices.
//
// Summation contract (bit-parity with the reference, src/bench_csr_width.cu:291-517): for threads per
// row T, logical lane L of a row sums the entries L, L+T, L+2T, ... in order, one correctly rounded fused
// multiply-add each, in the accumulator type (FP64, or FP32 for FP32 and FP16, value_types.cuh:9-13);
// the T lane sums s_0..s_{T-1} are then combined in the order of the __shfl_down_sync tree: for
// offset o = T/2, ..., 1, s_i += s_{i+o}; lane 0 narrows s_0 into y.
//
// Which hardware thread runs which logical lane is free. These kernels run a row on P threads (P divides
// T): thread p owns the logical lanes p, p+P, p+2P, ... (T/P "slots"), so it walks the entries p, p+P,
// p+2P, ... of the row and adds entry e into slot ((e - row_begin) mod T) / P. The tree levels with
// o >= P pair two lanes of the same thread and run in registers; the last log2(P) levels are shuffles.
// Lane sums start at +0.0 and an FMA chain or a sum never produces -0.0 from it, so the zero sums of
// empty lanes are exact no-ops, as they are in the reference.
//
// Kernels
//   k_spmv_tiles   one CTA per tile: a run of consecutive rows whose nonzeros fit in shared memory.
//                  The tile's value and column (or CSR-lp word) streams are brought in by cp.async.bulk
//                  (the 1-D TMA engine) on an mbarrier, 16-byte-aligned interior by the bulk copy and
//                  ragged ends by plain loads; the row metadata is read with coalesced loads. The
//                  compute phase then reads shared memory and gathers x through the read-only path.
//   k_spmv_vector  one group of T threads per row straight from global memory (the reference's
//                  mapping): rows longer than a tile, and the raw launch over caller arrays.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "spmvb200.h"

namespace spmvb200 {

constexpr int kTileBlock = 256;          // threads of a tile CTA
constexpr int kVectorBlock = 128;        // threads of a vector CTA
constexpr unsigned kStatusTimeout = 1u;  // bit of the status word: a bounded wait gave up
constexpr unsigned kStatusAlignment = 2u;  // bit: a bulk copy was not 16-byte aligned (not issued)

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

// ---- column layouts -----------------------------------------------------------------------------
template <int LAYOUT> struct LayoutTraits;
template <> struct LayoutTraits<SPMV_LAYOUT_I32> { using Index = int;      static constexpr bool kBase = false; };
template <> struct LayoutTraits<SPMV_LAYOUT_I16> { using Index = uint16_t; static constexpr bool kBase = false; };
template <> struct LayoutTraits<SPMV_LAYOUT_I8>  { using Index = uint8_t;  static constexpr bool kBase = false; };
template <> struct LayoutTraits<SPMV_LAYOUT_R16> { using Index = uint16_t; static constexpr bool kBase = true; };
template <> struct LayoutTraits<SPMV_LAYOUT_R8>  { using Index = uint8_t;  static constexpr bool kBase = true; };
template <> struct LayoutTraits<SPMV_LAYOUT_LP>  { using Index = uint32_t; static constexpr bool kBase = true; };

// Arguments of every kernel (device pointers).
struct KernelArgs {
  int rows;
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
  const int2* tile_words;    // CSR-lp: [tile_count] {word_begin, word_end} of the tile's stream
  int64_t tile_count;
  int tile_nnz;              // nonzeros a tile holds at most
  int tile_rows;             // rows a tile holds at most
  const int* row_list;       // rows of the vector path (nullptr: rows 0..row_count-1)
  int64_t row_count;         // entries of row_list, or rows
  int64_t vector_blocks;     // k_spmv_tiles: its first vector_blocks CTAs run the vector path on row_list
  unsigned* status;          // device status word (may be null)
};

// ---- small device helpers -----------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_address(const void* pointer) {
  return (uint32_t)__cvta_generic_to_shared(pointer);
}

__device__ __forceinline__ void mbarrier_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbarrier_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
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

// Waits for phase `parity` of an mbarrier for at most ~limit_ns. Returns false when it gave up.
__device__ __forceinline__ bool mbarrier_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbarrier_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 0; spin < (1u << 26); ++spin) {
    if (mbarrier_try_wait(bar, parity)) return true;
    if ((spin & 63) == 0 && global_timer_ns() - start > limit_ns) return false;
  }
  return false;
}

// 1-D bulk copy global -> shared (TMA), completing on the mbarrier with the byte count.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

template <class T>
__device__ __forceinline__ T load_readonly(const T* pointer) {
  return __ldg(pointer);
}
template <>
__device__ __forceinline__ __half load_readonly<__half>(const __half* pointer) {
  return __ldg(pointer);
}
template <>
__device__ __forceinline__ uint8_t load_readonly<uint8_t>(const uint8_t* pointer) {
  return (uint8_t)__ldg(reinterpret_cast<const unsigned char*>(pointer));
}

// The shared-memory image of a global range [first, last) of elements of type E: it starts at the
// 16-byte boundary at or below element `first`, so element e sits at byte (addr(e) - start) of the
// image. The 16-byte-aligned interior goes through one bulk copy; the head and tail (fewer than 16
// bytes each) are loaded by the threads. Returns the bulk bytes issued by thread 0.
template <class E>
struct StagedRange {
  const E* origin;      // global address of image byte 0 (16-byte aligned, may precede `first`)
  int64_t first;        // first element staged
  int64_t last;         // one past the last element staged

  __device__ __forceinline__ StagedRange(const E* base, int64_t first_, int64_t last_) : first(first_), last(last_) {
    const uintptr_t address = reinterpret_cast<uintptr_t>(base + first_);
    origin = reinterpret_cast<const E*>(address & ~(uintptr_t)15);
  }
  // element index -> position in the shared image (in elements)
  __device__ __forceinline__ int position(int64_t element, const E* base) const {
    return (int)(base + element - origin);
  }
  // bytes of the aligned interior [interior_begin, interior_end)
  __device__ __forceinline__ void interior(const E* base, uintptr_t& begin, uintptr_t& end) const {
    const uintptr_t a = reinterpret_cast<uintptr_t>(base + first);
    const uintptr_t b = reinterpret_cast<uintptr_t>(base + last);
    begin = (a + 15) & ~(uintptr_t)15;
    end = b & ~(uintptr_t)15;
    if (end < begin) end = begin;
  }
};

// Bytes of a range's aligned interior and whether a bulk copy of it into image is well formed (16-byte
// aligned source, destination and size; always true by construction, checked so that a violation
// degrades to plain loads instead of an ill-formed copy).
template <class E>
__device__ __forceinline__ bool interior_copyable(const StagedRange<E>& range, const E* base, const E* image,
                                                  uint32_t& bytes) {
  uintptr_t begin, end;
  range.interior(base, begin, end);
  bytes = (uint32_t)(end - begin);
  const uint32_t dst = smem_address(reinterpret_cast<const char*>(image) + (begin - reinterpret_cast<uintptr_t>(range.origin)));
  return (dst & 15u) == 0 && (begin & 15u) == 0 && (bytes & 15u) == 0;
}

// Issues the bulk copy of a range's interior into image (one thread).
template <class E>
__device__ __forceinline__ void stage_interior(const StagedRange<E>& range, const E* base, E* image, uint32_t bar) {
  uintptr_t begin, end;
  range.interior(base, begin, end);
  if (end <= begin) return;
  const uint32_t dst = smem_address(reinterpret_cast<const char*>(image) + (begin - reinterpret_cast<uintptr_t>(range.origin)));
  bulk_copy_g2s(dst, reinterpret_cast<const void*>(begin), (uint32_t)(end - begin), bar);
}

// Loads the elements of a range outside its bulk interior (head and tail) with plain loads; also used
// for the whole range when the bulk copy was not issued (returns after loading everything then).
template <class E>
__device__ __forceinline__ void stage_edges(const StagedRange<E>& range, const E* base, E* image, bool whole) {
  uintptr_t begin, end;
  range.interior(base, begin, end);
  const int64_t interior_first = whole ? range.last : (int64_t)((const E*)begin - base);
  const int64_t interior_last = whole ? range.last : (int64_t)((const E*)end - base);
  for (int64_t element = range.first + threadIdx.x; element < range.last; element += blockDim.x) {
    if (!whole && element >= interior_first && element < interior_last) continue;
    image[range.position(element, base)] = load_readonly(base + element);
  }
}

// ---- shared-memory plan of a tile CTA (host and device compute it alike) ----------------------------
struct TileSmem {
  int row_ptr, row_base, row_word, row_width, values, index, total;
};

__host__ __device__ inline int round16(int bytes) { return (bytes + 15) & ~15; }

__host__ __device__ inline TileSmem tile_smem(int tile_nnz, int tile_rows, int value_bytes, int layout) {
  const bool base = layout == SPMV_LAYOUT_R16 || layout == SPMV_LAYOUT_R8 || layout == SPMV_LAYOUT_LP;
  const bool packed = layout == SPMV_LAYOUT_LP;
  const int index_bytes = packed ? 4 : (layout == SPMV_LAYOUT_I32 ? 4 : ((layout == SPMV_LAYOUT_I16 || layout == SPMV_LAYOUT_R16) ? 2 : 1));
  TileSmem plan;
  int offset = 16;                                     // [0, 8): the mbarrier
  plan.row_ptr = offset;   offset = round16(offset + 4 * (tile_rows + 1));
  plan.row_base = offset;  if (base) offset = round16(offset + 4 * tile_rows);
  plan.row_word = offset;  if (packed) offset = round16(offset + 4 * tile_rows);
  plan.row_width = offset; if (packed) offset = round16(offset + tile_rows);
  plan.values = offset;    offset = round16(offset + value_bytes * (tile_nnz + 16 / value_bytes));
  plan.index = offset;
  offset = packed ? round16(offset + 4 * (tile_nnz + 8)) : round16(offset + index_bytes * (tile_nnz + 16 / index_bytes));
  plan.total = offset;
  return plan;
}

// ---- the reduction over the T logical lanes ----------------------------------------------------------
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

// ---- the vector path -----------------------------------------------------------------------------------
// One group of T threads per row, each thread one logical lane, straight from global memory. CTA `block`
// of `blocks` (of BLOCK threads each) takes the rows item = group, group + groups, ... of the row list.
template <class V, int LAYOUT, int T, int BLOCK>
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
#pragma unroll 4
        for (int64_t entry = entry_begin + lane; entry < entry_end; entry += T)
          sum = VT::fma(VT::widen(load_readonly(values + entry)),
                        VT::widen(load_readonly(x + base + (int)load_readonly(columns + entry))), sum);
      } else {
        // the reference's decode (bench_csr_width.cu:482-510): a 64-bit window over the lane's run
        const int length = (int)(entry_end - entry_begin);
        const int quotient = length / T, remainder = length - quotient * T;
        const int mine = quotient + (lane < remainder ? 1 : 0);
        const int width = a.row_width[row];
        const uint64_t mask = width == 0 ? 0ull : (~0ull >> (64 - width));
        const int64_t start_bit = (int64_t)width * ((int64_t)lane * quotient + (lane < remainder ? lane : remainder));
        int64_t word = (int64_t)a.row_word[row] + (start_bit >> 5);
        uint64_t window = (((uint64_t)load_readonly(a.words + word + 1) << 32) | load_readonly(a.words + word)) >> (start_bit & 31);
        int available = 64 - (int)(start_bit & 31);
        int64_t next_word = word + 2;
        int column = a.row_base[row];
        int64_t entry = entry_begin + lane;
        for (int taken = 0; taken < mine; ++taken) {
          column += (int)(window & mask);
          sum = VT::fma(VT::widen(load_readonly(values + entry)), VT::widen(load_readonly(x + column)), sum);
          window >>= width;
          available -= width;
          entry += T;
          if (available < width) {
            window |= (uint64_t)load_readonly(a.words + next_word) << available;
            available += 32;
            ++next_word;
          }
        }
      }
    }
#pragma unroll
    for (int offset = T / 2; offset > 0; offset >>= 1) sum = VT::add(sum, __shfl_down_sync(0xffffffffu, sum, offset, T));
    if (lane == 0 && item < a.row_count) y[row] = VT::narrow(sum);
  }
}

// ---- k_spmv_tiles --------------------------------------------------------------------------------------
template <class V, int LAYOUT, int T, int P>
__global__ void __launch_bounds__(kTileBlock) k_spmv_tiles(const KernelArgs a) {
  using VT = ValueTraits<V>;
  using Acc = typename VT::Acc;
  using Index = typename LayoutTraits<LAYOUT>::Index;
  constexpr bool kPacked = LAYOUT == SPMV_LAYOUT_LP;
  constexpr bool kBase = LayoutTraits<LAYOUT>::kBase;
  constexpr int S = T / P;
  static_assert(T % P == 0 && P >= 1 && P <= 32, "P must divide T");

  extern __shared__ __align__(128) unsigned char smem[];
  const TileSmem plan = tile_smem(a.tile_nnz, a.tile_rows, (int)sizeof(V), LAYOUT);
  int* s_row_ptr = reinterpret_cast<int*>(smem + plan.row_ptr);
  int* s_row_base = reinterpret_cast<int*>(smem + plan.row_base);
  int* s_row_word = reinterpret_cast<int*>(smem + plan.row_word);
  uint8_t* s_row_width = reinterpret_cast<uint8_t*>(smem + plan.row_width);
  V* s_values = reinterpret_cast<V*>(smem + plan.values);
  Index* s_index = reinterpret_cast<Index*>(smem + plan.index);
  const uint32_t bar = smem_address(smem);

  if ((int64_t)blockIdx.x < a.vector_blocks) {   // rows longer than a tile, scheduled first
    vector_rows<V, LAYOUT, T, kTileBlock>(a, blockIdx.x, a.vector_blocks);
    return;
  }
  const int64_t tile_id = (int64_t)blockIdx.x - a.vector_blocks;
  const int4 tile = a.tiles[tile_id];
  const int row_begin = tile.x, rows = tile.y - tile.x;
  const V* values = static_cast<const V*>(a.values);
  const Index* index = kPacked ? reinterpret_cast<const Index*>(a.words) : static_cast<const Index*>(a.columns);
  const StagedRange<V> value_range(values, tile.z, tile.w);
  int64_t index_first = tile.z, index_last = tile.w;
  if (kPacked) {
    const int2 words = a.tile_words[tile_id];
    index_first = words.x;
    index_last = (int64_t)words.y + 1;   // the extraction of a row's last delta may read one word further
  }
  const StagedRange<Index> index_range(index, index_first, index_last);

  uint32_t value_bytes = 0, index_bytes = 0;
  const bool bulk = interior_copyable(value_range, values, s_values, value_bytes) &&
                    interior_copyable(index_range, index, s_index, index_bytes);
  if (threadIdx.x == 0) mbarrier_init(bar, 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (bulk) {
      mbarrier_arrive_expect_tx(bar, value_bytes + index_bytes);
      stage_interior(value_range, values, s_values, bar);
      stage_interior(index_range, index, s_index, bar);
    } else {
      if (a.status) atomicOr(a.status, kStatusAlignment);
      mbarrier_arrive_expect_tx(bar, 0);
    }
  }
  // ragged ends of both streams (everything, without the bulk copy) and the row metadata, plain loads
  stage_edges(value_range, values, s_values, !bulk);
  stage_edges(index_range, index, s_index, !bulk);
  for (int local = threadIdx.x; local <= rows; local += kTileBlock) s_row_ptr[local] = a.row_ptr[row_begin + local];
  if (kBase)
    for (int local = threadIdx.x; local < rows; local += kTileBlock) s_row_base[local] = a.row_base[row_begin + local];
  if (kPacked)
    for (int local = threadIdx.x; local < rows; local += kTileBlock) {
      s_row_word[local] = a.row_word[row_begin + local];
      s_row_width[local] = a.row_width[row_begin + local];
    }
  const bool arrived = mbarrier_wait_bounded(bar, 0, 2000000000ull);
  if (__syncthreads_or(!arrived)) {
    if (threadIdx.x == 0 && a.status) atomicOr(a.status, kStatusTimeout);
    mbarrier_wait_bounded(bar, 0, 100000000ull);   // give copies still in flight a last bounded chance
    return;
  }

  const int value_origin = (int)(tile.z - (int64_t)value_range.position(tile.z, values));
  const int index_origin = (int)(index_first - (int64_t)index_range.position(index_first, index));
  const V* x = static_cast<const V*>(a.x);
  V* y = static_cast<V*>(a.y);
  constexpr int kGroups = kTileBlock / P;
  const int group = threadIdx.x / P, p = threadIdx.x % P;

  for (int first = 0; first < rows; first += kGroups) {
    const int local = first + group;
    Acc acc[S];
#pragma unroll
    for (int j = 0; j < S; ++j) acc[j] = Acc(0);
    if (local < rows) {
      const int entry_begin = s_row_ptr[local], entry_end = s_row_ptr[local + 1];
      if constexpr (!kPacked) {
        const int base = kBase ? s_row_base[local] : 0;
        for (int entry = entry_begin + p; entry < entry_end; entry += T) {
#pragma unroll
          for (int j = 0; j < S; ++j) {
            const int e = entry + j * P;
            if (e < entry_end) {
              const int column = base + (int)s_index[e - index_origin];
              acc[j] = VT::fma(VT::widen(s_values[e - value_origin]), VT::widen(load_readonly(x + column)), acc[j]);
            }
          }
        }
      } else {
        const int length = entry_end - entry_begin;
        const int quotient = length / T, remainder = length - quotient * T;
        const int width = s_row_width[local];
        const uint32_t mask = width == 0 ? 0u : (0xffffffffu >> (32 - width));
        const uint32_t* stream = reinterpret_cast<const uint32_t*>(s_index) + (s_row_word[local] - index_origin);
        int column[S];
        uint32_t bit[S];
        int mine[S];
#pragma unroll
        for (int j = 0; j < S; ++j) {
          const int lane = p + j * P;
          mine[j] = quotient + (lane < remainder ? 1 : 0);
          bit[j] = (uint32_t)width * (uint32_t)(lane * quotient + (lane < remainder ? lane : remainder));
          column[j] = s_row_base[local];
        }
        const int rounds = quotient + (remainder > 0 ? 1 : 0);
        for (int round = 0; round < rounds; ++round) {
#pragma unroll
          for (int j = 0; j < S; ++j) {
            if (round < mine[j]) {
              const uint32_t at = bit[j];
              const uint32_t delta = __funnelshift_r(stream[at >> 5], stream[(at >> 5) + 1], at & 31) & mask;
              column[j] += (int)delta;
              bit[j] = at + (uint32_t)width;
              const int e = entry_begin + p + j * P + round * T;
              acc[j] = VT::fma(VT::widen(s_values[e - value_origin]), VT::widen(load_readonly(x + column[j])), acc[j]);
            }
          }
        }
      }
    }
    const Acc sum = reduce_lanes<VT, Acc, T, P>(acc);
    if (p == 0 && local < rows) y[row_begin + local] = VT::narrow(sum);
  }
}

// k_spmv_vector: the vector path over every row (row_list null) or a list of rows.
template <class V, int LAYOUT, int T>
__global__ void __launch_bounds__(kVectorBlock) k_spmv_vector(const KernelArgs a) {
  vector_rows<V, LAYOUT, T, kVectorBlock>(a, blockIdx.x, gridDim.x);
}

}  // namespace spmvb200
