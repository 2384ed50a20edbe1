// internal.hpp — host-side types of libspmvb200: the CSR container, errors and a thread pool helper.
#pragma once

#include "spmvb200.h"

#include <algorithm>
#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace spmvb200 {

// A failure carrying its C-ABI status; the C entry points turn it into a return code.
struct Error : std::runtime_error {
  int status;
  Error(int status_, const std::string& message) : std::runtime_error(message), status(status_) {}
};

[[noreturn]] inline void fail(int status, const std::string& message) { throw Error(status, message); }

// MatrixStats (include/csr.hpp:22).
struct Stats {
  double nnz_per_row_mean = 0.0;
  int nnz_per_row_max = 0;
  int nnz_per_row_min = 0;
  double nnz_per_row_std = 0.0;
  double dynamic_range = 0.0;
  double norm_inf = 0.0;
  double max_abs = 0.0;
  double min_abs = 0.0;
};

// CsrMatrix (include/csr.hpp:33): int32 row pointer and columns, FP64 values, columns sorted in rows.
struct Csr {
  int rows = 0;
  int cols = 0;
  std::vector<int> row_ptr;
  std::vector<int> col_ind;
  std::vector<double> val;
  Stats stats;
  bool symmetric_expanded = false;
  std::string name;

  int64_t nnz() const { return (int64_t)col_ind.size(); }
  void compute_stats();
};

// Worker count for host loops: the hardware threads, capped so small jobs do not pay for many.
int host_threads();

// Runs body(begin, end) over [0, count) split into contiguous chunks, one per worker thread.
void parallel_for(int64_t count, const std::function<void(int64_t, int64_t)>& body, int64_t min_chunk = 1 << 14);

// csr.cpp
void sort_columns_within_rows(Csr& matrix);
Csr read_matrix_market(const std::string& path);
std::string matrix_name_from_path(const std::string& path);
void validate(const Csr& matrix);

// rcm.cpp
std::vector<int> reverse_cuthill_mckee(const Csr& matrix);
Csr apply_symmetric_permutation(const Csr& matrix, const std::vector<int>& new_to_old);
std::string permutation_path_for(const std::string& matrix_path, const std::string& ordering);
void write_permutation(const std::string& path, const std::vector<int>& new_to_old, double seconds);
bool read_permutation(const std::string& path, int expected_rows, std::vector<int>& new_to_old, double& seconds);
Csr reorder_with_rcm(const std::string& matrix_path, const Csr& matrix, double& seconds);

// characterize.cpp
std::string characterize(const Csr& matrix, const std::string& ordering, double ordering_seconds);
// characterize_device.cu: the same text with the per-row metrics computed on the current GPU
std::string characterize_device(const Csr& matrix, const std::string& ordering, double ordering_seconds);

// layouts.cpp
struct Facts {
  int widest_row_span = 0;
  int64_t lane_packed_words[6] = {0, 0, 0, 0, 0, 0};
};
int tpr_slot(int tpr);
bool valid_tpr(int tpr);
Facts facts_of(const Csr& matrix);
int64_t lane_packed_word_count(const Csr& matrix, int tpr);
bool admissible(const Csr& matrix, const Facts& facts, int layout, int tpr);
spmv_memory memory_of(const Csr& matrix, const Facts& facts, int layout, int dtype, int tpr);
int value_bytes_of(int dtype);
int column_bytes_of(int layout);
void encode_absolute(const Csr& matrix, int column_bytes, void* out);
void encode_row_base(const Csr& matrix, int* row_base);
void encode_relative(const Csr& matrix, int column_bytes, void* out);
void encode_relative_lane(const Csr& matrix, int tpr, uint16_t* out);
void encode_lane_packed(const Csr& matrix, int tpr, int64_t word_count, int* row_word, uint8_t* row_width,
                        uint32_t* words);

// synth.cpp
Csr synth_laplacian2d(int grid);
Csr synth_random_band(int n, int half_bandwidth, double mean, uint64_t seed);
Csr synth_stencil27(int grid);
Csr synth_power_law(int n, double alpha, int max_length, double mean, uint64_t seed);
Csr synth_block_fem(int n, int block, int blocks_per_row, int offset_range, uint64_t seed, int row_begin, int row_end);
void fill_uniform(int dtype, int64_t count, uint64_t seed, void* out);
void fill_reference_x(int dtype, int64_t count, void* out);
void convert_values(int dtype, const double* in, int64_t count, int value_rounding, void* out);

}  // namespace spmvb200

struct spmv_csr {
  spmvb200::Csr m;
};
