// capi.cpp — the host-side C entry points of libspmvb200 (matrices, RCM, characterization, layouts,
// synthetic inputs) and the library's error reporting. Each entry point turns exceptions into a status
// and keeps the message for spmv_last_error(); nothing here touches a GPU.
#include "internal.hpp"
#include "capi_internal.hpp"

#include <cstring>
#include <new>

namespace spmvb200 {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string& message) { g_last_error = message; }

int guarded(const std::function<void()>& body) {
  try {
    body();
    return SPMV_OK;
  } catch (const Error& failure) {
    set_last_error(failure.what());
    return failure.status;
  } catch (const std::bad_alloc&) {
    set_last_error("host allocation failed");
    return SPMV_ERR_OUT_OF_MEMORY;
  } catch (const std::length_error& failure) {
    set_last_error(failure.what());
    return SPMV_ERR_OUT_OF_MEMORY;
  } catch (const std::exception& failure) {
    set_last_error(failure.what());
    return SPMV_ERR_INVALID_ARGUMENT;
  }
}

void require(bool condition, const char* message) {
  if (!condition) fail(SPMV_ERR_INVALID_ARGUMENT, message);
}

Facts facts_for(const spmv_csr* matrix, const spmv_facts* facts) {
  Facts result;
  if (facts) {
    result.widest_row_span = facts->widest_row_span;
    for (int slot = 0; slot < 6; ++slot) result.lane_packed_words[slot] = facts->lane_packed_words[slot];
  } else {
    result = facts_of(matrix->m);
  }
  return result;
}

}  // namespace spmvb200

using namespace spmvb200;

extern "C" {

const char* spmv_version(void) { return "spmvb200 0.1.0 (sm_100a)"; }

const char* spmv_status_string(int status) {
  switch (status) {
    case SPMV_OK: return "ok";
    case SPMV_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SPMV_ERR_IO: return "i/o error";
    case SPMV_ERR_FORMAT: return "malformed file";
    case SPMV_ERR_NOT_ADMISSIBLE: return "not admissible";
    case SPMV_ERR_OUT_OF_MEMORY: return "out of memory";
    case SPMV_ERR_CUDA: return "CUDA error";
    case SPMV_ERR_UNSUPPORTED: return "unsupported";
    case SPMV_ERR_NCCL: return "NCCL error";
    case SPMV_ERR_TIMEOUT: return "device wait timed out";
    case SPMV_ERR_TOO_LARGE: return "size limit exceeded";
    default: return "unknown status";
  }
}

const char* spmv_last_error(void) { return g_last_error.c_str(); }

// ---- matrices ---------------------------------------------------------------------------------------
int spmv_csr_read_matrix_market(const char* path, spmv_csr** out) {
  return guarded([&] {
    require(path && out, "path and out are required");
    *out = nullptr;
    spmv_csr* matrix = new spmv_csr{read_matrix_market(path)};
    *out = matrix;
  });
}

int spmv_csr_create(int rows, int cols, const int* row_ptr, const int* col_ind, const double* values, const char* name,
                    spmv_csr** out) {
  return guarded([&] {
    require(out && rows >= 0 && cols >= 0 && row_ptr, "bad arguments");
    *out = nullptr;
    require(row_ptr[0] == 0 && row_ptr[rows] >= 0, "row_ptr must start at 0");
    const int64_t nnz = row_ptr[rows];
    require(nnz == 0 || col_ind, "col_ind is required");
    std::unique_ptr<spmv_csr> matrix(new spmv_csr);
    Csr& m = matrix->m;
    m.rows = rows;
    m.cols = cols;
    m.row_ptr.assign(row_ptr, row_ptr + rows + 1);
    m.col_ind.assign(col_ind, col_ind + nnz);
    if (values) m.val.assign(values, values + nnz);
    else m.val.assign((size_t)nnz, 1.0);
    validate(m);
    sort_columns_within_rows(m);
    m.name = name ? name : "matrix";
    m.compute_stats();
    *out = matrix.release();
  });
}

int spmv_csr_get_info(const spmv_csr* matrix, spmv_csr_info* info) {
  return guarded([&] {
    require(matrix && info, "matrix and info are required");
    const Csr& m = matrix->m;
    info->rows = m.rows;
    info->cols = m.cols;
    info->nnz = m.nnz();
    info->nnz_per_row_mean = m.stats.nnz_per_row_mean;
    info->nnz_per_row_max = m.stats.nnz_per_row_max;
    info->nnz_per_row_min = m.stats.nnz_per_row_min;
    info->nnz_per_row_std = m.stats.nnz_per_row_std;
    info->dynamic_range = m.stats.dynamic_range;
    info->norm_inf = m.stats.norm_inf;
    info->max_abs = m.stats.max_abs;
    info->min_abs = m.stats.min_abs;
    info->symmetric_expanded = m.symmetric_expanded ? 1 : 0;
  });
}

int spmv_csr_get_arrays(const spmv_csr* matrix, const int** row_ptr, const int** col_ind, const double** values) {
  return guarded([&] {
    require(matrix, "matrix is required");
    if (row_ptr) *row_ptr = matrix->m.row_ptr.data();
    if (col_ind) *col_ind = matrix->m.col_ind.data();
    if (values) *values = matrix->m.val.data();
  });
}

const char* spmv_csr_name(const spmv_csr* matrix) { return matrix ? matrix->m.name.c_str() : ""; }

int spmv_csr_set_name(spmv_csr* matrix, const char* name) {
  return guarded([&] {
    require(matrix && name, "matrix and name are required");
    matrix->m.name = name;
  });
}

void spmv_csr_destroy(spmv_csr* matrix) { delete matrix; }

int spmv_csr_slice_rows(const spmv_csr* matrix, int row_begin, int row_end, spmv_csr** out) {
  return guarded([&] {
    require(matrix && out, "matrix and out are required");
    *out = nullptr;
    const Csr& m = matrix->m;
    require(row_begin >= 0 && row_begin <= row_end && row_end <= m.rows, "row range out of bounds");
    std::unique_ptr<spmv_csr> slice(new spmv_csr);
    Csr& s = slice->m;
    s.rows = row_end - row_begin;
    s.cols = m.cols;
    s.symmetric_expanded = m.symmetric_expanded;
    s.name = m.name;
    const int first = m.row_ptr[row_begin], last = m.row_ptr[row_end];
    s.row_ptr.resize((size_t)s.rows + 1);
    for (int row = 0; row <= s.rows; ++row) s.row_ptr[row] = m.row_ptr[row_begin + row] - first;
    s.col_ind.assign(m.col_ind.begin() + first, m.col_ind.begin() + last);
    s.val.assign(m.val.begin() + first, m.val.begin() + last);
    s.compute_stats();
    *out = slice.release();
  });
}

// ---- RCM --------------------------------------------------------------------------------------------
int spmv_rcm_order(const spmv_csr* matrix, int* new_to_old) {
  return guarded([&] {
    require(matrix && new_to_old, "matrix and new_to_old are required");
    const std::vector<int> order = reverse_cuthill_mckee(matrix->m);
    std::memcpy(new_to_old, order.data(), sizeof(int) * order.size());
  });
}

int spmv_csr_permute(const spmv_csr* matrix, const int* new_to_old, spmv_csr** out) {
  return guarded([&] {
    require(matrix && new_to_old && out, "matrix, new_to_old and out are required");
    *out = nullptr;
    const std::vector<int> order(new_to_old, new_to_old + matrix->m.rows);
    *out = new spmv_csr{apply_symmetric_permutation(matrix->m, order)};
  });
}

int spmv_permutation_path(const char* matrix_path, const char* ordering, char* out, size_t cap) {
  return guarded([&] {
    require(matrix_path && ordering && out, "arguments are required");
    const std::string path = permutation_path_for(matrix_path, ordering);
    if (path.size() + 1 > cap) fail(SPMV_ERR_TOO_LARGE, "output buffer too small");
    std::memcpy(out, path.c_str(), path.size() + 1);
  });
}

int spmv_permutation_write(const char* path, const int* new_to_old, int64_t rows, double seconds) {
  return guarded([&] {
    require(path && (new_to_old || rows == 0) && rows >= 0, "bad arguments");
    write_permutation(path, std::vector<int>(new_to_old, new_to_old + rows), seconds);
  });
}

int spmv_permutation_read(const char* path, int expected_rows, int* new_to_old, double* seconds, int* found) {
  return guarded([&] {
    require(path && found, "path and found are required");
    std::vector<int> order;
    double time = 0.0;
    *found = 0;
    if (!read_permutation(path, expected_rows, order, time)) return;
    *found = 1;
    if (new_to_old) std::memcpy(new_to_old, order.data(), sizeof(int) * order.size());
    if (seconds) *seconds = time;
  });
}

int spmv_csr_reorder_rcm(const char* matrix_path, const spmv_csr* matrix, spmv_csr** out, double* seconds) {
  return guarded([&] {
    require(matrix_path && matrix && out, "arguments are required");
    *out = nullptr;
    double time = 0.0;
    *out = new spmv_csr{reorder_with_rcm(matrix_path, matrix->m, time)};
    if (seconds) *seconds = time;
  });
}

// ---- characterization ------------------------------------------------------------------------------
int spmv_characterize(const spmv_csr* matrix, const char* ordering, double ordering_seconds, char* csv, size_t cap,
                      size_t* needed) {
  return guarded([&] {
    require(matrix && ordering, "matrix and ordering are required");
    const std::string text = characterize(matrix->m, ordering, ordering_seconds);
    if (needed) *needed = text.size() + 1;
    if (!csv || cap < text.size() + 1) fail(SPMV_ERR_TOO_LARGE, "output buffer too small");
    std::memcpy(csv, text.c_str(), text.size() + 1);
  });
}

// ---- layouts ----------------------------------------------------------------------------------------
int spmv_matrix_facts(const spmv_csr* matrix, spmv_facts* facts) {
  return guarded([&] {
    require(matrix && facts, "matrix and facts are required");
    const Facts result = facts_of(matrix->m);
    facts->widest_row_span = result.widest_row_span;
    for (int slot = 0; slot < 6; ++slot) facts->lane_packed_words[slot] = result.lane_packed_words[slot];
  });
}

int spmv_admissible(const spmv_csr* matrix, const spmv_facts* facts, int layout, int tpr, int* result) {
  return guarded([&] {
    require(matrix && result, "matrix and result are required");
    column_bytes_of(layout);
    require(tpr == 0 || valid_tpr(tpr), "threads per row must be 0, 2, 4, 8, 16 or 32");
    *result = admissible(matrix->m, facts_for(matrix, facts), layout, tpr) ? 1 : 0;
  });
}

int spmv_memory_of(const spmv_csr* matrix, const spmv_facts* facts, int layout, int dtype, int tpr, spmv_memory* memory) {
  return guarded([&] {
    require(matrix && memory, "matrix and memory are required");
    column_bytes_of(layout);
    require(tpr == 0 || valid_tpr(tpr), "threads per row must be 0, 2, 4, 8, 16 or 32");
    *memory = memory_of(matrix->m, facts_for(matrix, facts), layout, dtype, tpr);
  });
}

int spmv_encode_absolute(const spmv_csr* matrix, int column_bytes, void* columns) {
  return guarded([&] {
    require(matrix && columns, "matrix and columns are required");
    encode_absolute(matrix->m, column_bytes, columns);
  });
}

int spmv_encode_row_base(const spmv_csr* matrix, int* row_base) {
  return guarded([&] {
    require(matrix && row_base, "matrix and row_base are required");
    encode_row_base(matrix->m, row_base);
  });
}

int spmv_encode_relative(const spmv_csr* matrix, int column_bytes, void* offsets) {
  return guarded([&] {
    require(matrix && offsets, "matrix and offsets are required");
    encode_relative(matrix->m, column_bytes, offsets);
  });
}

int spmv_encode_relative_lane(const spmv_csr* matrix, int tpr, uint16_t* offsets) {
  return guarded([&] {
    require(matrix && offsets, "matrix and offsets are required");
    require(valid_tpr(tpr), "threads per row must be 2, 4, 8, 16 or 32");
    encode_relative_lane(matrix->m, tpr, offsets);
  });
}

int spmv_lane_packed_word_count(const spmv_csr* matrix, int tpr, int64_t* word_count) {
  return guarded([&] {
    require(matrix && word_count, "matrix and word_count are required");
    require(valid_tpr(tpr), "threads per row must be 2, 4, 8, 16 or 32");
    *word_count = lane_packed_word_count(matrix->m, tpr);
  });
}

int spmv_encode_lane_packed(const spmv_csr* matrix, int tpr, int64_t word_count, int* row_word, uint8_t* row_width,
                            uint32_t* words) {
  return guarded([&] {
    require(matrix && row_word && row_width && words, "arguments are required");
    encode_lane_packed(matrix->m, tpr, word_count, row_word, row_width, words);
  });
}

// ---- synthetic inputs ---------------------------------------------------------------------------------
int spmv_synth_laplacian2d(int grid, spmv_csr** out) {
  return guarded([&] {
    require(out, "out is required");
    *out = new spmv_csr{synth_laplacian2d(grid)};
  });
}

int spmv_synth_random_band(int n, int half_bandwidth, double mean, uint64_t seed, spmv_csr** out) {
  return guarded([&] {
    require(out, "out is required");
    *out = new spmv_csr{synth_random_band(n, half_bandwidth, mean, seed)};
  });
}

int spmv_synth_stencil27(int grid, spmv_csr** out) {
  return guarded([&] {
    require(out, "out is required");
    *out = new spmv_csr{synth_stencil27(grid)};
  });
}

int spmv_synth_power_law(int n, double alpha, int max_length, double mean, uint64_t seed, spmv_csr** out) {
  return guarded([&] {
    require(out, "out is required");
    *out = new spmv_csr{synth_power_law(n, alpha, max_length, mean, seed)};
  });
}

int spmv_synth_block_fem(int n, int block, int blocks_per_row, int offset_range, uint64_t seed, int row_begin, int row_end,
                         spmv_csr** out) {
  return guarded([&] {
    require(out, "out is required");
    *out = new spmv_csr{synth_block_fem(n, block, blocks_per_row, offset_range, seed, row_begin, row_end)};
  });
}

int spmv_fill_uniform(int dtype, int64_t count, uint64_t seed, void* out) {
  return guarded([&] {
    require(out || count == 0, "out is required");
    fill_uniform(dtype, count, seed, out);
  });
}

int spmv_fill_reference_x(int dtype, int64_t count, void* out) {
  return guarded([&] {
    require(out || count == 0, "out is required");
    fill_reference_x(dtype, count, out);
  });
}

// ---- multi-GPU row shards -------------------------------------------------------------------------------
// Shard s starts at the first row whose starting nonzero is at or past s * nnz / nshards, so every shard
// holds about nnz / nshards nonzeros (rows are never split; an empty shard is possible only with fewer
// rows than shards or a single dominant row).
int spmv_shard_rows(const spmv_csr* matrix, int nshards, int* row_begin) {
  return guarded([&] {
    require(matrix && row_begin && nshards >= 1, "bad arguments");
    const Csr& m = matrix->m;
    const int64_t nnz = m.nnz();
    row_begin[0] = 0;
    for (int shard = 1; shard < nshards; ++shard) {
      const int64_t target = nnz * shard / nshards;
      int row = (int)(std::lower_bound(m.row_ptr.begin(), m.row_ptr.end() - 1, (int)target) - m.row_ptr.begin());
      if (nnz == 0) row = (int)((int64_t)m.rows * shard / nshards);
      row_begin[shard] = std::max(row_begin[shard - 1], std::min(row, m.rows));
    }
    row_begin[nshards] = m.rows;
  });
}

}  // extern "C"
