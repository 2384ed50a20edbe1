// characterize.cpp — structural metrics of one matrix and the FP64 byte-model ceilings, as the single
// CSV line (with its header) of src/characterize_matrix.cpp in the reference. The column schema and the
// number formats are that tool's (write_csv, characterize_matrix.cpp:253), so its consumers read this
// output unchanged.
//
// The gather model counts the distinct 32-byte sectors of x each row touches and replays them through
// first-in first-out caches of 0, 8, 32, 128 and 131072 sectors. A FIFO cache holds exactly the last C
// sectors it inserted (a hit inserts nothing), so a sector is resident when its most recent insertion
// is among the last C; one array of last-insertion stamps per capacity replaces the hash sets.
#include "characterize.hpp"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <thread>

namespace spmvb200 {

// measure_gather_traffic (characterize_matrix.cpp:92), one capacity level of one value size.
int64_t fifo_gather_misses(const Csr& matrix, int value_index, int level) {
  const int value_bytes = kCharacterizeValueBytes[value_index];
  const int64_t capacity = kCharacterizeCacheSectors[level];
  const int64_t sector_count = (int64_t)matrix.cols * value_bytes / kCharacterizeSectorBytes + 1;
  std::vector<int64_t> stamp((size_t)sector_count, -1);
  int64_t misses = 0, insertions = 0;
  for (int row = 0; row < matrix.rows; ++row) {
    int64_t previous = -1;
    for (int entry = matrix.row_ptr[row]; entry < matrix.row_ptr[row + 1]; ++entry) {
      const int64_t sector = (int64_t)matrix.col_ind[entry] * value_bytes / kCharacterizeSectorBytes;
      if (sector == previous) continue;
      previous = sector;
      int64_t& last = stamp[sector];
      if (last >= 0 && last >= insertions - capacity) continue;
      ++misses;
      last = insertions++;
    }
  }
  return misses;
}

namespace {

// The sectors a row-by-row gather touches without a cache (gather level 0): distinct sectors in a row's
// run of equal sectors count once.
int64_t uncached_gathers(const Csr& matrix, int value_index) {
  const int value_bytes = kCharacterizeValueBytes[value_index];
  int64_t misses = 0;
  for (int row = 0; row < matrix.rows; ++row) {
    int64_t previous = -1;
    for (int entry = matrix.row_ptr[row]; entry < matrix.row_ptr[row + 1]; ++entry) {
      const int64_t sector = (int64_t)matrix.col_ind[entry] * value_bytes / kCharacterizeSectorBytes;
      if (sector != previous) ++misses;
      previous = sector;
    }
  }
  return misses;
}

// measure_lane_occupancy (characterize_matrix.cpp:139).
void lane_occupancy(const Csr& matrix, Characterization& result) {
  for (int index = 0; index < 5; ++index) {
    const int threads = kCharacterizeThreadsPerRow[index];
    int64_t occupied = 0, iterations = 0, longest = 0;
    for (int row = 0; row < matrix.rows; ++row) {
      const int length = matrix.row_ptr[row + 1] - matrix.row_ptr[row];
      const int64_t row_iterations = (length + threads - 1) / threads;
      occupied += row_iterations * threads;
      iterations += row_iterations;
      longest = std::max(longest, row_iterations);
    }
    result.lane_occupancy[index] = occupied > 0 ? (double)matrix.nnz() / (double)occupied : 0.0;
    result.tail_ratio[index] = iterations > 0 ? (double)longest * (double)matrix.rows / (double)iterations : 0.0;
  }
}

// count_windowed_segments (characterize_matrix.cpp:167).
int64_t windowed_segments(const Csr& matrix, int64_t window) {
  int64_t segments = 0;
  int base = 0;
  for (int row = 0; row < matrix.rows; ++row)
    for (int entry = matrix.row_ptr[row]; entry < matrix.row_ptr[row + 1]; ++entry) {
      const int column = matrix.col_ind[entry];
      if (entry == matrix.row_ptr[row] || (int64_t)column - base >= window) {
        base = column;
        ++segments;
      }
    }
  return segments;
}

// measure_row_spans (characterize_matrix.cpp:185).
void row_spans(const Csr& matrix, Characterization& result) {
  std::vector<int> spans((size_t)matrix.rows, 0);
  int64_t rows8 = 0, rows16 = 0, nnz8 = 0, nnz16 = 0;
  double span_sum = 0.0;
  for (int row = 0; row < matrix.rows; ++row) {
    const int begin = matrix.row_ptr[row], end = matrix.row_ptr[row + 1], length = end - begin;
    if (length == 0) {
      ++result.empty_rows;
    } else {
      spans[row] = matrix.col_ind[end - 1] - matrix.col_ind[begin];
      const int64_t distance = std::max<int64_t>(std::llabs((int64_t)row - matrix.col_ind[begin]),
                                                 std::llabs((int64_t)row - matrix.col_ind[end - 1]));
      result.bandwidth = std::max(result.bandwidth, distance);
    }
    span_sum += spans[row];
    if (spans[row] < 256) { ++rows8; nnz8 += length; }
    if (spans[row] < 65536) { ++rows16; nnz16 += length; }
  }
  result.rows_fitting_8bit = (double)rows8 / matrix.rows;
  result.rows_fitting_16bit = (double)rows16 / matrix.rows;
  result.nnz_in_rows_fitting_8bit = (double)nnz8 / (double)matrix.nnz();
  result.nnz_in_rows_fitting_16bit = (double)nnz16 / (double)matrix.nnz();
  result.row_span_mean = span_sum / matrix.rows;
  std::sort(spans.begin(), spans.end());
  result.row_span_max = spans.back();
  result.row_span_p50 = spans[(size_t)(0.50 * (spans.size() - 1))];
  result.row_span_p90 = spans[(size_t)(0.90 * (spans.size() - 1))];
}

}  // namespace

void characterize_rows(const Csr& matrix, Characterization& result) {
  row_spans(matrix, result);
  lane_occupancy(matrix, result);
  for (int value_index = 0; value_index < 3; ++value_index)
    result.gather_bytes[value_index][0] =
        (double)uncached_gathers(matrix, value_index) * kCharacterizeSectorBytes / (double)matrix.nnz();
  result.segments_8bit = windowed_segments(matrix, 256);
  result.segments_16bit = windowed_segments(matrix, 65536);
}

// apply_byte_model (characterize_matrix.cpp:225): FP64 values, int32 row pointer.
void byte_model(const Csr& matrix, Characterization& result) {
  const double value_bytes = 8.0, pointer_bytes = 4.0, nnz = (double)matrix.nnz();
  const double auxiliary = ((matrix.rows + 1.0) * pointer_bytes + (double)(matrix.cols + matrix.rows) * value_bytes) / nnz;
  const double row_base = 4.0 * matrix.rows / nnz;
  const double segment8 = ((result.segments_8bit + 1.0) * 4.0 + 4.0 * result.segments_8bit) / nnz;
  const double segment16 = ((result.segments_16bit + 1.0) * 4.0 + 4.0 * result.segments_16bit) / nnz;
  result.bytes_per_nnz_csr_i32 = value_bytes + 4.0 + auxiliary;
  result.bytes_per_nnz_index_free = value_bytes + auxiliary;
  result.bytes_per_nnz_windowed_16 = value_bytes + 2.0 + auxiliary + segment16;
  result.bytes_per_nnz_windowed_8 = value_bytes + 1.0 + auxiliary + segment8;
  if (result.rows_fitting_16bit == 1.0) result.bytes_per_nnz_rowbase_16 = value_bytes + 2.0 + auxiliary + row_base;
  if (result.rows_fitting_8bit == 1.0) result.bytes_per_nnz_rowbase_8 = value_bytes + 1.0 + auxiliary + row_base;
  result.gamma_csr_i32 = result.bytes_per_nnz_csr_i32 / (value_bytes + 4.0);
  result.speedup_ceiling = result.bytes_per_nnz_csr_i32 / result.bytes_per_nnz_index_free;
  result.speedup_windowed_16 = result.bytes_per_nnz_csr_i32 / result.bytes_per_nnz_windowed_16;
  result.speedup_windowed_8 = result.bytes_per_nnz_csr_i32 / result.bytes_per_nnz_windowed_8;
  result.speedup_rowbase_16 = result.bytes_per_nnz_csr_i32 / result.bytes_per_nnz_rowbase_16;
  result.speedup_rowbase_8 = result.bytes_per_nnz_csr_i32 / result.bytes_per_nnz_rowbase_8;
  result.working_set_mib_csr_i32 = result.bytes_per_nnz_csr_i32 * nnz / 1048576.0;
}

std::string characterization_csv(const Csr& matrix, const Characterization& r, const std::string& ordering,
                                 double ordering_seconds) {
  const char* header =
      "name,rows,cols,nnz,row_length_mean,row_length_max,row_length_std,empty_rows,bandwidth,"
      "row_span_max,row_span_mean,row_span_p50,row_span_p90,rows_fitting_8bit,rows_fitting_16bit,"
      "nnz_in_rows_fitting_8bit,nnz_in_rows_fitting_16bit,segments_8bit,segments_16bit,"
      "gamma_csr_i32,bytes_per_nnz_csr_i32,bytes_per_nnz_index_free,bytes_per_nnz_rowbase_16,"
      "bytes_per_nnz_rowbase_8,bytes_per_nnz_windowed_16,bytes_per_nnz_windowed_8,speedup_ceiling,"
      "speedup_rowbase_16,speedup_rowbase_8,speedup_windowed_16,speedup_windowed_8,"
      "working_set_mib_csr_i32,dynamic_range,ordering,ordering_seconds,"
      "lane_occupancy_t2,lane_occupancy_t4,lane_occupancy_t8,lane_occupancy_t16,lane_occupancy_t32,"
      "tail_ratio_t2,tail_ratio_t4,tail_ratio_t8,tail_ratio_t16,tail_ratio_t32,"
      "gather_v8_c0,gather_v8_c8,gather_v8_c32,gather_v8_c128,gather_v8_cl2,"
      "gather_v4_c0,gather_v4_c8,gather_v4_c32,gather_v4_c128,gather_v4_cl2,"
      "gather_v2_c0,gather_v2_c8,gather_v2_c32,gather_v2_c128,gather_v2_cl2\n";
  std::vector<char> line(4096 + matrix.name.size() * 2);
  std::snprintf(line.data(), line.size(),
      "%s,%d,%d,%lld,%.4f,%d,%.4f,%lld,%lld,%d,%.2f,%d,%d,%.6f,%.6f,%.6f,%.6f,%lld,%lld,"
      "%.6f,%.6f,%.6f,%.6f,%.6f,%.6f,%.6f,%.6f,%.6f,%.6f,%.6f,%.6f,%.3f,%.6e,%s,%.3f,"
      "%.6f,%.6f,%.6f,%.6f,%.6f,%.4f,%.4f,%.4f,%.4f,%.4f,"
      "%.4f,%.4f,%.4f,%.4f,%.4f,%.4f,%.4f,%.4f,%.4f,%.4f,%.4f,%.4f,%.4f,%.4f,%.4f\n",
      matrix.name.c_str(), matrix.rows, matrix.cols, (long long)matrix.nnz(), matrix.stats.nnz_per_row_mean,
      matrix.stats.nnz_per_row_max, matrix.stats.nnz_per_row_std, (long long)r.empty_rows, (long long)r.bandwidth,
      r.row_span_max, r.row_span_mean, r.row_span_p50, r.row_span_p90, r.rows_fitting_8bit, r.rows_fitting_16bit,
      r.nnz_in_rows_fitting_8bit, r.nnz_in_rows_fitting_16bit, (long long)r.segments_8bit, (long long)r.segments_16bit,
      r.gamma_csr_i32, r.bytes_per_nnz_csr_i32, r.bytes_per_nnz_index_free, r.bytes_per_nnz_rowbase_16,
      r.bytes_per_nnz_rowbase_8, r.bytes_per_nnz_windowed_16, r.bytes_per_nnz_windowed_8, r.speedup_ceiling,
      r.speedup_rowbase_16, r.speedup_rowbase_8, r.speedup_windowed_16, r.speedup_windowed_8,
      r.working_set_mib_csr_i32, matrix.stats.dynamic_range, ordering.c_str(), ordering_seconds,
      r.lane_occupancy[0], r.lane_occupancy[1], r.lane_occupancy[2], r.lane_occupancy[3], r.lane_occupancy[4],
      r.tail_ratio[0], r.tail_ratio[1], r.tail_ratio[2], r.tail_ratio[3], r.tail_ratio[4],
      r.gather_bytes[0][0], r.gather_bytes[0][1], r.gather_bytes[0][2], r.gather_bytes[0][3], r.gather_bytes[0][4],
      r.gather_bytes[1][0], r.gather_bytes[1][1], r.gather_bytes[1][2], r.gather_bytes[1][3], r.gather_bytes[1][4],
      r.gather_bytes[2][0], r.gather_bytes[2][1], r.gather_bytes[2][2], r.gather_bytes[2][3], r.gather_bytes[2][4]);
  return std::string(header) + line.data();
}

std::string characterize(const Csr& matrix, const std::string& ordering, double ordering_seconds) {
  if (matrix.rows != matrix.cols || matrix.nnz() == 0) fail(SPMV_ERR_INVALID_ARGUMENT, "not square or empty");
  if (ordering != "original" && ordering != "rcm") fail(SPMV_ERR_INVALID_ARGUMENT, "ordering must be original or rcm");
  Characterization result;
  characterize_rows(matrix, result);
  for (int value_index = 0; value_index < 3; ++value_index)
    for (int level = 1; level < 5; ++level)
      result.gather_bytes[value_index][level] =
          (double)fifo_gather_misses(matrix, value_index, level) * kCharacterizeSectorBytes / (double)matrix.nnz();
  byte_model(matrix, result);
  return characterization_csv(matrix, result, ordering, ordering_seconds);
}

}  // namespace spmvb200
