/*
 * spmv_oracle.c — CPU oracle for the CSR SpMV hot path. TEST INFRASTRUCTURE ONLY.
 *
 * Only the tests, __graft_entry__.smoke() and the cpu_baseline / reference arm of bench.py load
 * this file's library, and only as the checker or the timed CPU baseline. The product (the CUDA
 * library in spmv-index-compression_b200/) never links or calls it.
 *
 * It restates, in plain C, the arithmetic of the reference benchmark (HERMES-TorVerLab/
 * spmv-index-compression, src/bench_csr_width.cu and include/value_types.cuh):
 *
 *   - the SpMV of the three kernel families in their exact summation order: lane L of a row sums
 *     the entries L, L+T, L+2T, ... with one fused multiply-add each, in the accumulator type
 *     (FP64 for FP64, FP32 for FP32 and FP16), and the T lane sums are then combined in the order
 *     of the __shfl_down_sync tree (offsets T/2, ..., 1), lane 0 narrowing the result;
 *     With FP16 summed in FP16 (the SPMV_HALF_ACCUMULATE control build, value_types.cuh:7-33) every
 *     multiply-add is one correctly rounded FP16 fma (__hfma) and every step of the tree one FP16 add;
 *   - the layout encoders (16/8-bit absolute columns, row-base offsets, the lane-packed delta
 *     stream), the admissibility tests and the byte model memory_of.
 *
 * Parity is pinned by the tests against the reference itself (oracle/_ref, the reference's
 * encoders and kernels compiled from its sources) and against the published byte counts and the
 * lane-packed worked example committed under tests/golden/.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { O_F64 = 0, O_F32 = 1, O_F16 = 2, O_F16_HALF_SUMS = 3 };
enum { O_I32 = 0, O_I16 = 1, O_R16 = 2, O_LP = 3, O_I8 = 4, O_R8 = 5 };

/* ---------------------------------------------------------------------------------------------
 * Widths (bench_csr_width.cu:153-176)
 * ------------------------------------------------------------------------------------------- */

/* required_bits (bench_csr_width.cu:153): bits of the largest value, at least 1. */
static int required_bits(uint64_t largest) {
  int bits = 0;
  while (bits < 64 && (largest >> bits) != 0) ++bits;
  return bits < 1 ? 1 : bits;
}

/* delta_width_bits (bench_csr_width.cu:166): 0 when every delta of the row is 0. */
static int delta_width_bits(int64_t widest) { return widest == 0 ? 0 : required_bits((uint64_t)widest); }

/* tpr_slot (bench_csr_width.cu:171): log2 of a threads-per-row value in {1..32}. */
int oracle_tpr_slot(int tpr) {
  int slot = 0;
  while ((1 << slot) < tpr && slot < 5) ++slot;
  return slot;
}

/* lane_delta (bench_csr_width.cu:180): delta from the entry T positions earlier in the row, or from
 * the row's first column for the first T entries. */
static int64_t lane_delta(const int* col, int row_begin, int entry, int tpr) {
  return entry - row_begin < tpr ? (int64_t)col[entry] - col[row_begin]
                                 : (int64_t)col[entry] - col[entry - tpr];
}

/* lane_major_bit (bench_csr_width.cu:197): bit of an entry in its row's lane-major stream. */
static int64_t lane_major_bit(int offset, int length, int tpr, int width) {
  const int quotient = length / tpr;
  const int remainder = length - quotient * tpr;
  const int lane = offset % tpr;
  const int step = offset / tpr;
  return (int64_t)width * ((int64_t)lane * quotient + (lane < remainder ? lane : remainder) + step);
}

/* packed_word_count (bench_csr_width.cu:206): 32-bit words of the CSR-lp stream, plus 2 spare. */
int64_t oracle_lane_packed_words(int rows, const int* row_ptr, const int* col, int tpr) {
  int64_t words = 0;
  for (int row = 0; row < rows; ++row) {
    const int begin = row_ptr[row], end = row_ptr[row + 1];
    int64_t widest = 0;
    for (int entry = begin; entry < end; ++entry) {
      const int64_t delta = lane_delta(col, begin, entry, tpr);
      if (delta > widest) widest = delta;
    }
    words += ((int64_t)(end - begin) * delta_width_bits(widest) + 31) / 32;
  }
  return words + 2;
}

/* build_packed_deltas (bench_csr_width.cu:861): per row its first word and bit width, and the
 * deltas laid out lane by lane. words must hold word_count zero-initialised entries. */
int oracle_build_lane_packed(int rows, const int* row_ptr, const int* col, int tpr, int64_t word_count,
                             int* row_word, uint8_t* row_width, uint32_t* words) {
  int64_t cursor = 0;
  memset(words, 0, sizeof(uint32_t) * (size_t)word_count);
  for (int row = 0; row < rows; ++row) {
    const int begin = row_ptr[row], end = row_ptr[row + 1];
    int64_t widest = 0;
    for (int entry = begin; entry < end; ++entry) {
      const int64_t delta = lane_delta(col, begin, entry, tpr);
      if (delta > widest) widest = delta;
    }
    const int width = delta_width_bits(widest);
    row_word[row] = (int)cursor;
    row_width[row] = (uint8_t)width;
    for (int entry = begin; entry < end; ++entry) {
      const uint64_t delta = (uint64_t)lane_delta(col, begin, entry, tpr);
      const int64_t bit = lane_major_bit(entry - begin, end - begin, tpr, width);
      const int64_t word = cursor + (bit >> 5);
      const int shift = (int)(bit & 31);
      if (word >= word_count) return -1;
      words[word] |= (uint32_t)(delta << shift);
      if (shift + width > 32) {
        if (word + 1 >= word_count) return -1;
        words[word + 1] |= (uint32_t)(delta >> (32 - shift));
      }
    }
    cursor += ((int64_t)(end - begin) * width + 31) / 32;
  }
  return 0;
}

/* upload_row_bases (bench_csr_width.cu:807): first column of every row, 0 for an empty row. */
void oracle_row_bases(int rows, const int* row_ptr, const int* col, int* row_base) {
  for (int row = 0; row < rows; ++row)
    row_base[row] = row_ptr[row + 1] > row_ptr[row] ? col[row_ptr[row]] : 0;
}

/* upload_relative_columns (bench_csr_width.cu:820): col - row base, narrowed to 1 or 2 bytes. */
void oracle_relative_columns(int rows, const int* row_ptr, const int* col, int bytes, void* out) {
  for (int row = 0; row < rows; ++row) {
    const int first = row_ptr[row + 1] > row_ptr[row] ? col[row_ptr[row]] : 0;
    for (int entry = row_ptr[row]; entry < row_ptr[row + 1]; ++entry) {
      if (bytes == 2) ((uint16_t*)out)[entry] = (uint16_t)(col[entry] - first);
      else            ((uint8_t*)out)[entry]  = (uint8_t)(col[entry] - first);
    }
  }
}

/* upload_columns<T, I> (bench_csr_width.cu:796): absolute columns narrowed to 1 or 2 bytes. */
void oracle_narrow_columns(int64_t nnz, const int* col, int bytes, void* out) {
  for (int64_t entry = 0; entry < nnz; ++entry) {
    if (bytes == 2) ((uint16_t*)out)[entry] = (uint16_t)col[entry];
    else            ((uint8_t*)out)[entry]  = (uint8_t)col[entry];
  }
}

/* facts_of (bench_csr_width.cu:223): widest row span and the CSR-lp word counts at T = 2..32. */
int oracle_widest_row_span(int rows, const int* row_ptr, const int* col) {
  int widest = 0;
  for (int row = 0; row < rows; ++row)
    if (row_ptr[row + 1] > row_ptr[row]) {
      const int span = col[row_ptr[row + 1] - 1] - col[row_ptr[row]];
      if (span > widest) widest = span;
    }
  return widest;
}

/* configuration_admissible (bench_csr_width.cu:238-253). mode: 0 absolute, 1 row-base, 2 lane-packed. */
int oracle_admissible(int cols, int widest_span, const int64_t* lane_words /* [6] by slot */,
                      int mode, int column_bytes, int fixed_tpr) {
  if (mode == 0) return column_bytes >= 4 || (uint64_t)cols <= ((uint64_t)1 << (8 * column_bytes));
  if (mode == 1) return column_bytes < 4 && (uint64_t)widest_span < ((uint64_t)1 << (8 * column_bytes));
  return lane_words[oracle_tpr_slot(fixed_tpr > 0 ? fixed_tpr : 8)] <= INT32_MAX;
}

/* memory_of (bench_csr_width.cu:258): out = {values, columns, column_bases, row_pointer, vectors, total}. */
void oracle_memory_of(int rows, int cols, int64_t nnz, const int64_t* lane_words, int value_bytes,
                      int column_bytes, int mode, int fixed_tpr, double* out) {
  const int slot = oracle_tpr_slot(fixed_tpr > 0 ? fixed_tpr : 8);
  const double n = (double)nnz;
  out[0] = n * value_bytes;
  out[1] = mode == 2 ? 4.0 * (double)lane_words[slot] : n * column_bytes;
  out[2] = mode == 1 ? 4.0 * rows : (mode == 2 ? 9.0 * rows : 0.0);
  out[3] = (rows + 1.0) * 4;
  out[4] = (double)(cols + rows) * value_bytes;
  out[5] = out[0] + out[1] + out[2] + out[3] + out[4];
}

/* upload_matrix (bench_csr_width.cu:927): device values are (T)(float)val. */
void oracle_convert_values(int dtype, int64_t count, const double* in, void* out) {
  for (int64_t i = 0; i < count; ++i) {
    const float narrowed = (float)in[i];
    if (dtype == O_F64)      ((double*)out)[i] = (double)narrowed;
    else if (dtype == O_F32) ((float*)out)[i] = narrowed;
    else                     ((_Float16*)out)[i] = (_Float16)narrowed;
  }
}

/* Widens typed values to double (result_at_fixed_tpr, bench_csr_width.cu:787). */
void oracle_widen(int dtype, int64_t count, const void* in, double* out) {
  for (int64_t i = 0; i < count; ++i) {
    if (dtype == O_F64)      out[i] = ((const double*)in)[i];
    else if (dtype == O_F32) out[i] = (double)((const float*)in)[i];
    else                     out[i] = (double)(float)((const _Float16*)in)[i];
  }
}

/* ---------------------------------------------------------------------------------------------
 * SpMV in the reference's order (k_csr_cumulative :291, k_csr_row_relative :322,
 * k_csr_lane_packed :449; accumulate_product / narrow_value in value_types.cuh:16-35).
 * ------------------------------------------------------------------------------------------- */

/* Column of one entry for the absolute and row-base layouts. */
static inline int column_of(int layout, const void* columns, int base, int64_t entry) {
  switch (layout) {
    case O_I32: return ((const int*)columns)[entry];
    case O_I16: return (int)((const uint16_t*)columns)[entry];
    case O_I8:  return (int)((const uint8_t*)columns)[entry];
    case O_R16: return base + (int)((const uint16_t*)columns)[entry];
    default:    return base + (int)((const uint8_t*)columns)[entry];   /* O_R8 */
  }
}

#define LANES_MAX 32

/* One row in FP64: lane sums with fma, then the shuffle tree. */
static double row_f64(int layout, int tpr, int row, const int* row_ptr, const void* columns,
                      const int* row_base, const int* row_word, const uint8_t* row_width,
                      const uint32_t* words, const double* values, const double* x) {
  double lane_sum[LANES_MAX];
  const int begin = row_ptr[row], end = row_ptr[row + 1];
  for (int lane = 0; lane < tpr; ++lane) {
    double sum = 0.0;
    if (layout == O_LP) {
      /* k_csr_lane_packed :482-510: a 64-bit window over the lane's run, refilled a word at a time. */
      const int length = end - begin, quotient = length / tpr, remainder = length - quotient * tpr;
      const int mine = quotient + (lane < remainder ? 1 : 0);
      const int width = row_width[row];
      const uint64_t mask = width == 0 ? 0ull : (~0ull >> (64 - width));
      const int64_t start_bit = (int64_t)width * ((int64_t)lane * quotient + (lane < remainder ? lane : remainder));
      int64_t word = row_word[row] + (start_bit >> 5);
      uint64_t window = (((uint64_t)words[word + 1] << 32) | words[word]) >> (start_bit & 31);
      int available = 64 - (int)(start_bit & 31);
      int64_t next_word = word + 2;
      int column = row_base[row];
      int64_t entry = begin + lane;
      for (int taken = 0; taken < mine; ++taken) {
        column += (int)(window & mask);
        sum = fma(values[entry], x[column], sum);
        window >>= width;
        available -= width;
        entry += tpr;
        if (available < width) {
          window |= (uint64_t)words[next_word] << available;
          available += 32;
          ++next_word;
        }
      }
    } else {
      const int base = (layout == O_R16 || layout == O_R8) ? row_base[row] : 0;
      for (int64_t entry = begin + lane; entry < end; entry += tpr)
        sum = fma(values[entry], x[column_of(layout, columns, base, entry)], sum);
    }
    lane_sum[lane] = sum;
  }
  for (int offset = tpr / 2; offset > 0; offset >>= 1)
    for (int lane = 0; lane < offset; ++lane) lane_sum[lane] += lane_sum[lane + offset];
  return lane_sum[0];
}

/* One row in FP32 arithmetic for FP32 and FP16 values (FP16 widens to FP32, AccumulatorOf). */
static float row_f32(int dtype, int layout, int tpr, int row, const int* row_ptr, const void* columns,
                     const int* row_base, const int* row_word, const uint8_t* row_width,
                     const uint32_t* words, const void* values, const void* x) {
  float lane_sum[LANES_MAX];
  const int begin = row_ptr[row], end = row_ptr[row + 1];
  const float* vf = (const float*)values;
  const float* xf = (const float*)x;
  const _Float16* vh = (const _Float16*)values;
  const _Float16* xh = (const _Float16*)x;
#define WIDEN_V(e) (dtype == O_F32 ? vf[e] : (float)vh[e])
#define WIDEN_X(c) (dtype == O_F32 ? xf[c] : (float)xh[c])
  for (int lane = 0; lane < tpr; ++lane) {
    float sum = 0.0f;
    if (layout == O_LP) {
      const int length = end - begin, quotient = length / tpr, remainder = length - quotient * tpr;
      const int mine = quotient + (lane < remainder ? 1 : 0);
      const int width = row_width[row];
      const uint64_t mask = width == 0 ? 0ull : (~0ull >> (64 - width));
      const int64_t start_bit = (int64_t)width * ((int64_t)lane * quotient + (lane < remainder ? lane : remainder));
      int64_t word = row_word[row] + (start_bit >> 5);
      uint64_t window = (((uint64_t)words[word + 1] << 32) | words[word]) >> (start_bit & 31);
      int available = 64 - (int)(start_bit & 31);
      int64_t next_word = word + 2;
      int column = row_base[row];
      int64_t entry = begin + lane;
      for (int taken = 0; taken < mine; ++taken) {
        column += (int)(window & mask);
        sum = fmaf(WIDEN_V(entry), WIDEN_X(column), sum);
        window >>= width;
        available -= width;
        entry += tpr;
        if (available < width) {
          window |= (uint64_t)words[next_word] << available;
          available += 32;
          ++next_word;
        }
      }
    } else {
      const int base = (layout == O_R16 || layout == O_R8) ? row_base[row] : 0;
      for (int64_t entry = begin + lane; entry < end; entry += tpr)
        sum = fmaf(WIDEN_V(entry), WIDEN_X(column_of(layout, columns, base, entry)), sum);
    }
    lane_sum[lane] = sum;
  }
#undef WIDEN_V
#undef WIDEN_X
  for (int offset = tpr / 2; offset > 0; offset >>= 1)
    for (int lane = 0; lane < offset; ++lane) lane_sum[lane] += lane_sum[lane + offset];
  return lane_sum[0];
}

/* ---------------------------------------------------------------------------------------------
 * FP16 arithmetic rounded once, round to nearest even (the IEEE 754 binary16 fma and add that
 * __hfma and __hadd compute), restated from the definition:
 *   - a*b of two FP16 values is exact in FP64 (11-bit significands, exponents from 2^-48 to 2^32);
 *   - s = fl64(a*b + c) and its error e (Knuth's TwoSum, exact: a*b + c = s + e);
 *   - the FP16 rounding of a*b + c is that of s, except where s lies exactly halfway between two
 *     FP16 values and e != 0: the exact value is then on e's side of the midpoint.
 *   (No other double rounding can occur: every FP16 midpoint is an FP64 value, and s is the FP64
 *   value nearest the exact sum, so the exact sum and s are never on different sides of a midpoint
 *   that s does not equal.) The sum of two FP16 values is exact in FP64, so the add rounds once.
 * ------------------------------------------------------------------------------------------- */

/* The FP16 value next to h towards +inf (up) or -inf, by its bit pattern. */
static _Float16 half_step(_Float16 h, int up) {
  uint16_t bits;
  memcpy(&bits, &h, sizeof bits);
  if ((bits & 0x7fffu) == 0) bits = up ? 0x0001u : 0x8001u;
  else if (!(bits & 0x8000u)) bits = (uint16_t)(up ? bits + 1 : bits - 1);
  else bits = (uint16_t)(up ? bits - 1 : bits + 1);
  memcpy(&h, &bits, sizeof bits);
  return h;
}

_Float16 oracle_half_fma(_Float16 a, _Float16 b, _Float16 c) {
  const double p = (double)a * (double)b, q = (double)c;
  const double s = p + q;
  const double t = s - p;
  const double e = (p - (s - t)) + (q - t);
  const _Float16 h = (_Float16)s;
  if (e == 0.0 || (double)h == s || isnan(s)) return h;
  /* the FP16 values around s: h and its neighbour on the other side of s */
  const int h_below = isinf((double)h) ? (s < 0.0) : ((double)h < s);
  const _Float16 other = half_step(h, h_below);
  const double low = h_below ? (double)h : (double)other, high = h_below ? (double)other : (double)h;
  /* the midpoint; the one above 65504 (towards infinity) is 65520 */
  double middle;
  if (isinf(high)) middle = 65520.0;
  else if (isinf(low)) middle = -65520.0;
  else middle = 0.5 * (low + high);
  if (s != middle) return h;
  return e > 0.0 ? (h_below ? other : h) : (h_below ? h : other);
}

_Float16 oracle_half_add(_Float16 a, _Float16 b) { return (_Float16)((double)a + (double)b); }

/* oracle_half_fma over arrays of FP16 bit patterns (for the tests' exact-arithmetic check). */
void oracle_half_fma_array(int64_t count, const _Float16* a, const _Float16* b, const _Float16* c, _Float16* out) {
  for (int64_t i = 0; i < count; ++i) out[i] = oracle_half_fma(a[i], b[i], c[i]);
}

/* One row with FP16 sums (__hfma per entry, __hadd per tree step), CSR-lp or a column array. */
static _Float16 row_f16_half_sums(int layout, int tpr, int row, const int* row_ptr, const void* columns,
                                  const int* row_base, const int* row_word, const uint8_t* row_width,
                                  const uint32_t* words, const _Float16* values, const _Float16* x) {
  _Float16 lane_sum[LANES_MAX];
  const int begin = row_ptr[row], end = row_ptr[row + 1];
  for (int lane = 0; lane < tpr; ++lane) {
    _Float16 sum = (_Float16)0.0f;
    if (layout == O_LP) {
      const int length = end - begin, quotient = length / tpr, remainder = length - quotient * tpr;
      const int mine = quotient + (lane < remainder ? 1 : 0);
      const int width = row_width[row];
      const uint64_t mask = width == 0 ? 0ull : (~0ull >> (64 - width));
      const int64_t start_bit = (int64_t)width * ((int64_t)lane * quotient + (lane < remainder ? lane : remainder));
      int64_t word = row_word[row] + (start_bit >> 5);
      uint64_t window = (((uint64_t)words[word + 1] << 32) | words[word]) >> (start_bit & 31);
      int available = 64 - (int)(start_bit & 31);
      int64_t next_word = word + 2;
      int column = row_base[row];
      int64_t entry = begin + lane;
      for (int taken = 0; taken < mine; ++taken) {
        column += (int)(window & mask);
        sum = oracle_half_fma(values[entry], x[column], sum);
        window >>= width;
        available -= width;
        entry += tpr;
        if (available < width) {
          window |= (uint64_t)words[next_word] << available;
          available += 32;
          ++next_word;
        }
      }
    } else {
      const int base = (layout == O_R16 || layout == O_R8) ? row_base[row] : 0;
      for (int64_t entry = begin + lane; entry < end; entry += tpr)
        sum = oracle_half_fma(values[entry], x[column_of(layout, columns, base, entry)], sum);
    }
    lane_sum[lane] = sum;
  }
  for (int offset = tpr / 2; offset > 0; offset >>= 1)
    for (int lane = 0; lane < offset; ++lane) lane_sum[lane] = oracle_half_add(lane_sum[lane], lane_sum[lane + offset]);
  return lane_sum[0];
}

/*
 * y = A x in the reference order for one layout at one threads-per-row T.
 *   columns: int32 (i32), uint16 (i16, r16 offsets) or uint8 (i8, r8 offsets); unused for lp.
 *   row_base: r16/r8/lp; row_word, row_width, words: lp only.
 * Returns 0, or -1 on a bad argument. threads <= 0 uses every available thread.
 */
int oracle_spmv(int dtype, int layout, int tpr, int rows, const int* row_ptr, const void* columns,
                const int* row_base, const int* row_word, const uint8_t* row_width, const uint32_t* words,
                const void* values, const void* x, void* y, int threads) {
  if (tpr != 1 && tpr != 2 && tpr != 4 && tpr != 8 && tpr != 16 && tpr != 32) return -1;
  if (dtype < 0 || dtype > 3 || layout < 0 || layout > 5 || rows < 0) return -1;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 2048) num_threads(threads)
#endif
  for (int row = 0; row < rows; ++row) {
    if (dtype == O_F64) {
      ((double*)y)[row] = row_f64(layout, tpr, row, row_ptr, columns, row_base, row_word, row_width, words,
                                  (const double*)values, (const double*)x);
    } else if (dtype == O_F16_HALF_SUMS) {
      ((_Float16*)y)[row] = row_f16_half_sums(layout, tpr, row, row_ptr, columns, row_base, row_word, row_width,
                                              words, (const _Float16*)values, (const _Float16*)x);
    } else {
      const float sum = row_f32(dtype, layout, tpr, row, row_ptr, columns, row_base, row_word, row_width,
                                words, values, x);
      if (dtype == O_F32) ((float*)y)[row] = sum;
      else                ((_Float16*)y)[row] = (_Float16)sum;   /* __float2half: round to nearest even */
    }
  }
  (void)threads;
  return 0;
}

/* Sets the number of threads the oracle SpMV uses by default (count >= 1). */
void oracle_set_threads(int count) {
#ifdef _OPENMP
  if (count >= 1) omp_set_num_threads(count);
#else
  (void)count;
#endif
}

/* Number of threads the oracle SpMV uses by default (the host cores OpenMP sees). */
int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
