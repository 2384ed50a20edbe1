// characterize.hpp — the metrics of the characterization CSV (src/characterize_matrix.cpp in the
// reference) shared by the host version (characterize.cpp) and the GPU version (characterize_device.cu).
#pragma once

#include <cmath>
#include <string>

#include "internal.hpp"

namespace spmvb200 {

constexpr int kCharacterizeValueBytes[3] = {8, 4, 2};
constexpr int kCharacterizeSectorBytes = 32;
constexpr int64_t kCharacterizeCacheSectors[5] = {0, 8, 32, 128, 131072};
constexpr int kCharacterizeThreadsPerRow[5] = {2, 4, 8, 16, 32};

struct Characterization {
  int64_t empty_rows = 0;
  int64_t bandwidth = 0;
  int row_span_max = 0;
  double row_span_mean = 0.0;
  int row_span_p50 = 0;
  int row_span_p90 = 0;
  double rows_fitting_8bit = 0.0, rows_fitting_16bit = 0.0;
  double nnz_in_rows_fitting_8bit = 0.0, nnz_in_rows_fitting_16bit = 0.0;
  int64_t segments_8bit = 0, segments_16bit = 0;
  double gamma_csr_i32 = 0.0, bytes_per_nnz_csr_i32 = 0.0, bytes_per_nnz_index_free = 0.0;
  double bytes_per_nnz_rowbase_16 = NAN, bytes_per_nnz_rowbase_8 = NAN;
  double bytes_per_nnz_windowed_16 = 0.0, bytes_per_nnz_windowed_8 = 0.0;
  double speedup_ceiling = 0.0, speedup_rowbase_16 = NAN, speedup_rowbase_8 = NAN;
  double speedup_windowed_16 = 0.0, speedup_windowed_8 = 0.0, working_set_mib_csr_i32 = 0.0;
  double lane_occupancy[5] = {0, 0, 0, 0, 0};
  double tail_ratio[5] = {0, 0, 0, 0, 0};
  double gather_bytes[3][5] = {{0}};
};

// The row and percentile metrics, lane occupancy, windowed segments and the uncached gather counts
// (gather level 0), on the host.
void characterize_rows(const Csr& matrix, Characterization& result);
// The FIFO gather model at one value size (index into kCharacterizeValueBytes) and one cache capacity level
// 1..4: the sector misses of the replay (measure_gather_traffic, characterize_matrix.cpp:92-131).
int64_t fifo_gather_misses(const Csr& matrix, int value_index, int level);
// apply_byte_model (characterize_matrix.cpp:225), from the metrics above.
void byte_model(const Csr& matrix, Characterization& result);
// The header and value line of write_csv (characterize_matrix.cpp:253).
std::string characterization_csv(const Csr& matrix, const Characterization& result, const std::string& ordering,
                                 double ordering_seconds);

}  // namespace spmvb200
