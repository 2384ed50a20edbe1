// ref_wrapper.cu — TEST INFRASTRUCTURE ONLY. Builds the reference benchmark's own code
// (src/bench_csr_width.cu of HERMES-TorVerLab/spmv-index-compression, with include/csr.hpp and
// include/rcm.hpp) into oracle/_ref/libspmvref.so and exposes the pieces the tests compare against
// through a C ABI: the CSR reader, RCM, the CSR-lp encoder, facts_of, memory_of, admissibility and the
// reference kernels themselves (launch<T>, :607). The reference source is included from the reference
// tree at build time (oracle/Makefile passes its path); nothing of it is copied into this repository.
//
// Only the tests (and smoke()) load this library, as a checker. The product never does.
#define main spmv_reference_bench_main
#include "src/bench_csr_width.cu"
#undef main

#include <cstring>
#include <new>

namespace {

CsrMatrix matrix_from_arrays(int rows, int cols, const int* row_ptr, const int* col_ind, const double* values) {
  CsrMatrix matrix;
  const int64_t nnz = row_ptr[rows];
  matrix.rows = rows;
  matrix.cols = cols;
  matrix.row_ptr.assign(row_ptr, row_ptr + rows + 1);
  matrix.col_ind.assign(col_ind, col_ind + nnz);
  if (values) matrix.val.assign(values, values + nnz);
  else        matrix.val.assign((size_t)nnz, 1.0);
  return matrix;
}

}  // namespace

extern "C" {

// --- matrices held by the reference's own CsrMatrix -------------------------------------------
void* ref_read_matrix_market(const char* path, char* error, int error_cap) {
  try {
    return new CsrMatrix(read_matrix_market(path));
  } catch (const std::exception& failure) {
    std::snprintf(error, error_cap, "%s", failure.what());
    return nullptr;
  }
}

void* ref_matrix_from_arrays(int rows, int cols, const int* row_ptr, const int* col_ind, const double* values) {
  return new CsrMatrix(matrix_from_arrays(rows, cols, row_ptr, col_ind, values));
}

void ref_matrix_free(void* handle) { delete static_cast<CsrMatrix*>(handle); }

void ref_matrix_shape(void* handle, int* rows, int* cols, long long* nnz) {
  const CsrMatrix& matrix = *static_cast<CsrMatrix*>(handle);
  *rows = matrix.rows;
  *cols = matrix.cols;
  *nnz = (long long)matrix.nnz();
}

void ref_matrix_copy(void* handle, int* row_ptr, int* col_ind, double* values) {
  const CsrMatrix& matrix = *static_cast<CsrMatrix*>(handle);
  std::memcpy(row_ptr, matrix.row_ptr.data(), sizeof(int) * (matrix.rows + 1));
  std::memcpy(col_ind, matrix.col_ind.data(), sizeof(int) * matrix.nnz());
  std::memcpy(values, matrix.val.data(), sizeof(double) * matrix.nnz());
}

// stats: mean, max, min, std, dynamic_range, norm_inf, max_abs, min_abs
void ref_matrix_stats(void* handle, double* stats) {
  const CsrMatrix& matrix = *static_cast<CsrMatrix*>(handle);
  stats[0] = matrix.stats.nnz_per_row_mean;
  stats[1] = matrix.stats.nnz_per_row_max;
  stats[2] = matrix.stats.nnz_per_row_min;
  stats[3] = matrix.stats.nnz_per_row_std;
  stats[4] = matrix.stats.dynamic_range;
  stats[5] = matrix.stats.norm_inf;
  stats[6] = matrix.stats.max_abs;
  stats[7] = matrix.stats.min_abs;
}

// reverse_cuthill_mckee (rcm.hpp:199)
int ref_rcm_order(void* handle, int* new_to_old) {
  try {
    const std::vector<int> order = reverse_cuthill_mckee(*static_cast<CsrMatrix*>(handle));
    std::memcpy(new_to_old, order.data(), sizeof(int) * order.size());
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// apply_symmetric_permutation (rcm.hpp:219)
void* ref_permute(void* handle, const int* new_to_old) {
  const CsrMatrix& matrix = *static_cast<CsrMatrix*>(handle);
  std::vector<int> order(new_to_old, new_to_old + matrix.rows);
  return new CsrMatrix(apply_symmetric_permutation(matrix, order));
}

// reorder_with_rcm (rcm.hpp:306): reads or writes <stem>.rcm.perm next to matrix_path.
void* ref_reorder_with_rcm(const char* matrix_path, void* handle, double* seconds) {
  try {
    return new CsrMatrix(reorder_with_rcm(matrix_path, *static_cast<CsrMatrix*>(handle), *seconds));
  } catch (const std::exception&) {
    return nullptr;
  }
}

// --- encoders and byte model -----------------------------------------------------------------
long long ref_packed_word_count(void* handle, int tpr) {
  return (long long)packed_word_count(*static_cast<CsrMatrix*>(handle), tpr);
}

void ref_build_packed_deltas(void* handle, int tpr, long long word_count, int* row_word, unsigned char* row_width,
                             unsigned int* words) {
  std::vector<int> host_row_word;
  std::vector<uint8_t> host_row_width;
  std::vector<uint32_t> host_words;
  const CsrMatrix& matrix = *static_cast<CsrMatrix*>(handle);
  build_packed_deltas(matrix, tpr, word_count, host_row_word, host_row_width, host_words);
  std::memcpy(row_word, host_row_word.data(), sizeof(int) * host_row_word.size());
  std::memcpy(row_width, host_row_width.data(), host_row_width.size());
  std::memcpy(words, host_words.data(), sizeof(uint32_t) * host_words.size());
}

void ref_facts(void* handle, int* widest_row_span, long long* lane_packed_words /* [6] */) {
  const MatrixFacts facts = facts_of(*static_cast<CsrMatrix*>(handle));
  *widest_row_span = facts.widest_row_span;
  for (int slot = 0; slot < 6; ++slot) lane_packed_words[slot] = facts.lane_packed_words[slot];
}

// mode: 0 absolute, 1 row-base, 2 lane-packed; out = values, columns, column_bases, row_pointer, vectors, total
void ref_memory_of(void* handle, int value_bytes, int column_bytes, int mode, int fixed_tpr, double* out) {
  const CsrMatrix& matrix = *static_cast<CsrMatrix*>(handle);
  const MatrixFacts facts = facts_of(matrix);
  Configuration configuration;
  configuration.value_bytes = value_bytes;
  configuration.column_bytes = column_bytes;
  configuration.column_mode = mode == 0 ? ColumnMode::absolute : (mode == 1 ? ColumnMode::row_base : ColumnMode::lane_packed);
  configuration.fixed_tpr = fixed_tpr;
  const MemoryBreakdown memory = memory_of(matrix, facts, configuration);
  out[0] = memory.values;
  out[1] = memory.columns;
  out[2] = memory.column_bases;
  out[3] = memory.row_pointer;
  out[4] = memory.vectors;
  out[5] = memory.total;
}

int ref_admissible(void* handle, int column_bytes, int mode, int fixed_tpr) {
  const CsrMatrix& matrix = *static_cast<CsrMatrix*>(handle);
  const MatrixFacts facts = facts_of(matrix);
  Configuration configuration;
  configuration.column_bytes = column_bytes;
  configuration.column_mode = mode == 0 ? ColumnMode::absolute : (mode == 1 ? ColumnMode::row_base : ColumnMode::lane_packed);
  configuration.fixed_tpr = fixed_tpr;
  return configuration_admissible(matrix, facts, configuration) ? 1 : 0;
}

// --- the reference kernels rebuilt for sm_100a (launch<T>, :607) ------------------------------
// Device pointers; layout 0 i32, 1 i16, 2 r16, 3 lp, 4 i8, 5 r8; dtype 0 f64, 1 f32, 2 f16.
// Launches on the default stream like the reference and synchronises. Returns the cudaError_t.
static int ref_launch_impl(int dtype, int layout, int tpr, int rows, int cols, long long nnz, const int* row_ptr,
                           const void* columns, const int* row_base, const int* row_word, const unsigned char* row_width,
                           const unsigned int* words, const void* values, const void* x, void* y, int wait) {
  Configuration configuration;
  configuration.column_bytes = layout == 0 ? 4 : ((layout == 1 || layout == 2) ? 2 : (layout == 3 ? 0 : 1));
  configuration.column_mode = (layout == 2 || layout == 5) ? ColumnMode::row_base
                              : (layout == 3 ? ColumnMode::lane_packed : ColumnMode::absolute);
  configuration.fixed_tpr = layout == 3 ? tpr : 0;
  auto fill = [&](auto& device) {
    using T = typename std::remove_reference<decltype(*device.values)>::type;
    device.rows = rows;
    device.cols = cols;
    device.nnz = nnz;
    device.values = const_cast<T*>(static_cast<const T*>(values));
    device.x = const_cast<T*>(static_cast<const T*>(x));
    device.y = static_cast<T*>(y);
    device.row_ptr = const_cast<int*>(row_ptr);
    device.row_base = const_cast<int*>(row_base);
    device.lane_row_word = const_cast<int*>(row_word);
    device.lane_row_width = const_cast<uint8_t*>(row_width);
    device.lane_words = const_cast<uint32_t*>(words);
    if (layout == 0) device.col_ind_32 = const_cast<int*>(static_cast<const int*>(columns));
    if (layout == 1) device.col_ind_16 = const_cast<uint16_t*>(static_cast<const uint16_t*>(columns));
    if (layout == 4) device.col_ind_8 = const_cast<uint8_t*>(static_cast<const uint8_t*>(columns));
    if (layout == 2) device.col_rel_16 = const_cast<uint16_t*>(static_cast<const uint16_t*>(columns));
    if (layout == 5) device.col_rel_8 = const_cast<uint8_t*>(static_cast<const uint8_t*>(columns));
  };
  if (dtype == 0) {
    DeviceMatrix<double> device;
    fill(device);
    configuration.value_bytes = 8;
    launch<double>(tpr, configuration, device);
  } else if (dtype == 1) {
    DeviceMatrix<float> device;
    fill(device);
    configuration.value_bytes = 4;
    launch<float>(tpr, configuration, device);
  } else {
    DeviceMatrix<__half> device;
    fill(device);
    configuration.value_bytes = 2;
    launch<__half>(tpr, configuration, device);
  }
  cudaError_t status = cudaGetLastError();
  if (status == cudaSuccess && wait) status = cudaDeviceSynchronize();
  return (int)status;
}

/* launch<T> on the default stream, then a device synchronize; returns the cudaError_t. */
int ref_launch(int dtype, int layout, int tpr, int rows, int cols, long long nnz, const int* row_ptr,
               const void* columns, const int* row_base, const int* row_word, const unsigned char* row_width,
               const unsigned int* words, const void* values, const void* x, void* y) {
  return ref_launch_impl(dtype, layout, tpr, rows, cols, nnz, row_ptr, columns, row_base, row_word, row_width, words,
                         values, x, y, 1);
}

/* launch<T> on the default stream without waiting (for timing back-to-back launches); returns the launch's
 * cudaError_t. */
int ref_launch_async(int dtype, int layout, int tpr, int rows, int cols, long long nnz, const int* row_ptr,
                     const void* columns, const int* row_base, const int* row_word, const unsigned char* row_width,
                     const unsigned int* words, const void* values, const void* x, void* y) {
  return ref_launch_impl(dtype, layout, tpr, rows, cols, nnz, row_ptr, columns, row_base, row_word, row_width, words,
                         values, x, y, 0);
}

}  // extern "C"
