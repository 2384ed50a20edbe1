// layouts.cpp — column layouts: admissibility, the byte model and the host encoders.
//
// The streams are those of src/bench_csr_width.cu (upload_columns :796, upload_row_bases :807,
// upload_relative_columns :820, build_packed_deltas :861) byte for byte: the kernels' bit-parity with
// CSR-i32 and the byte counts that the study publishes both depend on it. The encoders here run over
// the rows in parallel: the CSR-lp stream is built in two passes, per-row widths and word counts first,
// then an exclusive scan into each row's first word, then every row packed independently.
#include "internal.hpp"

#include <cstring>
#include <mutex>

namespace spmvb200 {

namespace {

int required_bits(uint64_t largest) {
  int bits = 0;
  while (bits < 64 && (largest >> bits) != 0) ++bits;
  return std::max(bits, 1);
}

// Bits of a row's packed deltas (delta_width_bits, :166): 0 when every delta is 0.
int delta_width(int64_t widest) { return widest == 0 ? 0 : required_bits((uint64_t)widest); }

// Widest lane delta of one row (lane_delta, :180): from the entry tpr positions earlier, or from the
// row's first column for the first tpr entries.
int64_t widest_lane_delta(const Csr& matrix, int row, int tpr) {
  const int begin = matrix.row_ptr[row], end = matrix.row_ptr[row + 1];
  const int* col = matrix.col_ind.data();
  int64_t widest = 0;
  for (int entry = begin; entry < end; ++entry) {
    const int64_t delta = entry - begin < tpr ? (int64_t)col[entry] - col[begin] : (int64_t)col[entry] - col[entry - tpr];
    widest = std::max(widest, delta);
  }
  return widest;
}

}  // namespace

int tpr_slot(int tpr) {
  int slot = 0;
  while ((1 << slot) < tpr && slot < 5) ++slot;
  return slot;
}

bool valid_tpr(int tpr) { return tpr == 2 || tpr == 4 || tpr == 8 || tpr == 16 || tpr == 32; }

int value_bytes_of(int dtype) {
  switch (dtype) {
    case SPMV_F64: return 8;
    case SPMV_F32: return 4;
    case SPMV_F16: return 2;
    default: fail(SPMV_ERR_INVALID_ARGUMENT, "unknown value type " + std::to_string(dtype));
  }
}

int column_bytes_of(int layout) {
  switch (layout) {
    case SPMV_LAYOUT_I32: return 4;
    case SPMV_LAYOUT_I16: case SPMV_LAYOUT_R16: return 2;
    case SPMV_LAYOUT_I8: case SPMV_LAYOUT_R8: return 1;
    case SPMV_LAYOUT_LP: return 0;
    default: fail(SPMV_ERR_INVALID_ARGUMENT, "unknown layout " + std::to_string(layout));
  }
}

// packed_word_count (:206): words of the CSR-lp stream for one T, plus 2 spare words.
int64_t lane_packed_word_count(const Csr& matrix, int tpr) {
  std::mutex guard;
  int64_t total = 0;
  parallel_for(matrix.rows, [&](int64_t first, int64_t last) {
    int64_t words = 0;
    for (int64_t row = first; row < last; ++row) {
      const int64_t length = matrix.row_ptr[row + 1] - matrix.row_ptr[row];
      words += (length * delta_width(widest_lane_delta(matrix, (int)row, tpr)) + 31) / 32;
    }
    std::lock_guard<std::mutex> lock(guard);
    total += words;
  });
  return total + 2;
}

// facts_of (:223).
Facts facts_of(const Csr& matrix) {
  Facts facts;
  for (int row = 0; row < matrix.rows; ++row) {
    const int begin = matrix.row_ptr[row], end = matrix.row_ptr[row + 1];
    if (end > begin) facts.widest_row_span = std::max(facts.widest_row_span, matrix.col_ind[end - 1] - matrix.col_ind[begin]);
  }
  for (int slot = 1; slot <= 5; ++slot) facts.lane_packed_words[slot] = lane_packed_word_count(matrix, 1 << slot);
  return facts;
}

// configuration_admissible (:246) with column_width_admissible (:238) and row_base_admissible (:242).
bool admissible(const Csr& matrix, const Facts& facts, int layout, int tpr) {
  const int column_bytes = column_bytes_of(layout);
  switch (layout) {
    case SPMV_LAYOUT_I32: case SPMV_LAYOUT_I16: case SPMV_LAYOUT_I8:
      return column_bytes >= 4 || (uint64_t)matrix.cols <= ((uint64_t)1 << (8 * column_bytes));
    case SPMV_LAYOUT_R16: case SPMV_LAYOUT_R8:
      return (uint64_t)facts.widest_row_span < ((uint64_t)1 << (8 * column_bytes));
    default:
      return facts.lane_packed_words[tpr_slot(tpr > 0 ? tpr : 8)] <= INT32_MAX;
  }
}

// memory_of (:258): values + columns + row metadata + row pointer + x and y.
spmv_memory memory_of(const Csr& matrix, const Facts& facts, int layout, int dtype, int tpr) {
  const int value_bytes = value_bytes_of(dtype);
  const double nnz = (double)matrix.nnz();
  spmv_memory memory{};
  memory.values = nnz * value_bytes;
  memory.columns = nnz * column_bytes_of(layout);
  if (layout == SPMV_LAYOUT_LP) memory.columns = 4.0 * facts.lane_packed_words[tpr_slot(tpr > 0 ? tpr : 8)];
  memory.row_pointer = (matrix.rows + 1.0) * 4;
  memory.vectors = (double)((int64_t)matrix.cols + matrix.rows) * value_bytes;
  memory.column_bases = 0.0;
  if (layout == SPMV_LAYOUT_R16 || layout == SPMV_LAYOUT_R8) memory.column_bases = 4.0 * matrix.rows;
  if (layout == SPMV_LAYOUT_LP) memory.column_bases = 9.0 * matrix.rows;
  memory.total = memory.values + memory.columns + memory.column_bases + memory.row_pointer + memory.vectors;
  return memory;
}

void encode_absolute(const Csr& matrix, int column_bytes, void* out) {
  if (column_bytes != 1 && column_bytes != 2) fail(SPMV_ERR_INVALID_ARGUMENT, "column_bytes must be 1 or 2");
  parallel_for(matrix.nnz(), [&](int64_t first, int64_t last) {
    for (int64_t entry = first; entry < last; ++entry) {
      if (column_bytes == 2) static_cast<uint16_t*>(out)[entry] = (uint16_t)matrix.col_ind[entry];
      else                   static_cast<uint8_t*>(out)[entry] = (uint8_t)matrix.col_ind[entry];
    }
  });
}

void encode_row_base(const Csr& matrix, int* row_base) {
  parallel_for(matrix.rows, [&](int64_t first, int64_t last) {
    for (int64_t row = first; row < last; ++row)
      row_base[row] = matrix.row_ptr[row + 1] > matrix.row_ptr[row] ? matrix.col_ind[matrix.row_ptr[row]] : 0;
  });
}

void encode_relative(const Csr& matrix, int column_bytes, void* out) {
  if (column_bytes != 1 && column_bytes != 2 && column_bytes != 4)
    fail(SPMV_ERR_INVALID_ARGUMENT, "column_bytes must be 1, 2 or 4");
  parallel_for(matrix.rows, [&](int64_t first, int64_t last) {
    for (int64_t row = first; row < last; ++row) {
      const int begin = matrix.row_ptr[row], end = matrix.row_ptr[row + 1];
      const int base = end > begin ? matrix.col_ind[begin] : 0;
      for (int entry = begin; entry < end; ++entry) {
        if (column_bytes == 4)      static_cast<uint32_t*>(out)[entry] = (uint32_t)(matrix.col_ind[entry] - base);
        else if (column_bytes == 2) static_cast<uint16_t*>(out)[entry] = (uint16_t)(matrix.col_ind[entry] - base);
        else                        static_cast<uint8_t*>(out)[entry] = (uint8_t)(matrix.col_ind[entry] - base);
      }
    }
  }, 4096);
}

// The 16-bit row-relative offsets of every row in lane-major order for T (upload_lane_major_offsets,
// bench_csr_width.cu:838): within the row's own positions, logical lane L's offsets (entries L, L+T, ...)
// come next to each other from position L * quotient + min(L, remainder); (nnz + 1) / 2 * 2 entries, the last
// one zero when nnz is odd, so that 32-bit loads of two offsets never read past the stream.
void encode_relative_lane(const Csr& matrix, int tpr, uint16_t* out) {
  const int64_t count = (matrix.nnz() + 1) / 2 * 2;
  if (count > matrix.nnz()) out[count - 1] = 0;
  parallel_for(matrix.rows, [&](int64_t first, int64_t last) {
    for (int64_t row = first; row < last; ++row) {
      const int begin = matrix.row_ptr[row], length = matrix.row_ptr[row + 1] - begin;
      if (length == 0) continue;
      const int base = matrix.col_ind[begin];
      const int quotient = length / tpr, remainder = length - quotient * tpr;
      for (int lane = 0; lane < tpr && lane < length; ++lane) {
        int position = begin + lane * quotient + std::min(lane, remainder);
        for (int entry = begin + lane; entry < begin + length; entry += tpr)
          out[position++] = (uint16_t)(matrix.col_ind[entry] - base);
      }
    }
  }, 4096);
}

// build_packed_deltas (:861) in two parallel passes. Deltas of lane L sit one after the other from bit
// width * (L * quotient + min(L, remainder)) of the row's stream (lane_major_bit, :197).
void encode_lane_packed(const Csr& matrix, int tpr, int64_t word_count, int* row_word, uint8_t* row_width,
                        uint32_t* words) {
  if (!valid_tpr(tpr)) fail(SPMV_ERR_INVALID_ARGUMENT, "threads per row must be 2, 4, 8, 16 or 32");
  const int rows = matrix.rows;
  std::vector<int64_t> row_words((size_t)rows + 1, 0);
  parallel_for(rows, [&](int64_t first, int64_t last) {
    for (int64_t row = first; row < last; ++row) {
      const int width = delta_width(widest_lane_delta(matrix, (int)row, tpr));
      row_width[row] = (uint8_t)width;
      row_words[row + 1] = ((int64_t)(matrix.row_ptr[row + 1] - matrix.row_ptr[row]) * width + 31) / 32;
    }
  }, 4096);
  for (int row = 0; row < rows; ++row) row_words[row + 1] += row_words[row];
  if (row_words[rows] + 2 != word_count) fail(SPMV_ERR_INVALID_ARGUMENT, "word_count does not match the matrix");
  if (row_words[rows] > INT32_MAX) fail(SPMV_ERR_NOT_ADMISSIBLE, "CSR-lp stream exceeds 2^31 words");
  std::memset(words, 0, sizeof(uint32_t) * (size_t)word_count);
  const int* col = matrix.col_ind.data();
  parallel_for(rows, [&](int64_t first, int64_t last) {
    for (int64_t row = first; row < last; ++row) {
      const int begin = matrix.row_ptr[row], end = matrix.row_ptr[row + 1], length = end - begin;
      const int width = row_width[row];
      row_word[row] = (int)row_words[row];
      if (width == 0) continue;
      const int quotient = length / tpr, remainder = length - quotient * tpr;
      uint32_t* row_stream = words + row_words[row];
      for (int offset = 0; offset < length; ++offset) {
        const int entry = begin + offset;
        const uint64_t delta = (uint64_t)(offset < tpr ? (int64_t)col[entry] - col[begin]
                                                       : (int64_t)col[entry] - col[entry - tpr]);
        const int lane = offset % tpr, step = offset / tpr;
        const int64_t bit = (int64_t)width * ((int64_t)lane * quotient + std::min(lane, remainder) + step);
        const int shift = (int)(bit & 31);
        row_stream[bit >> 5] |= (uint32_t)(delta << shift);
        if (shift + width > 32) row_stream[(bit >> 5) + 1] |= (uint32_t)(delta >> (32 - shift));
      }
    }
  }, 4096);
}

}  // namespace spmvb200
