// csr.cpp — the CSR container, its statistics and the Matrix Market reader.
//
// Follows include/csr.hpp of the reference: the same accepted banners, the same symmetric expansion
// (an off-diagonal (r, c, v) also stores (c, r, v), negated for skew-symmetric), the same out-of-range
// skip, a stable scatter into rows by file order and the same per-row column sort, so the nonzero order
// the summation order depends on is the reference's.
#include "internal.hpp"

#include <cerrno>
#include <sched.h>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <sstream>

namespace spmvb200 {

// The CPUs this process may run on (its affinity mask, which a container or job scheduler narrows),
// or SPMV_HOST_THREADS.
int host_threads() {
  static const int threads = [] {
    const char* forced = std::getenv("SPMV_HOST_THREADS");
    int count = forced ? std::atoi(forced) : 0;
    if (count <= 0) {
      cpu_set_t mask;
      CPU_ZERO(&mask);
      count = sched_getaffinity(0, sizeof(mask), &mask) == 0 ? CPU_COUNT(&mask) : (int)std::thread::hardware_concurrency();
    }
    return std::max(1, std::min(count, 64));
  }();
  return threads;
}

void parallel_for(int64_t count, const std::function<void(int64_t, int64_t)>& body, int64_t min_chunk) {
  if (count <= 0) return;
  const int64_t workers = std::max<int64_t>(1, std::min<int64_t>(host_threads(), (count + min_chunk - 1) / min_chunk));
  if (workers == 1) {
    body(0, count);
    return;
  }
  std::vector<std::thread> threads;
  std::exception_ptr failure;
  std::vector<std::exception_ptr> failures((size_t)workers);
  const int64_t chunk = (count + workers - 1) / workers;
  for (int64_t worker = 0; worker < workers; ++worker) {
    const int64_t begin = worker * chunk, end = std::min(count, begin + chunk);
    if (begin >= end) break;
    threads.emplace_back([&, worker, begin, end] {
      try {
        body(begin, end);
      } catch (...) {
        failures[(size_t)worker] = std::current_exception();
      }
    });
  }
  for (std::thread& thread : threads) thread.join();
  for (std::exception_ptr& caught : failures)
    if (caught) std::rethrow_exception(caught);
}

// CsrMatrix::compute_stats (include/csr.hpp:43): row-length moments, value range and infinity norm.
void Csr::compute_stats() {
  double length_sum = 0.0, length_square_sum = 0.0, largest = 0.0, smallest = 1e308;
  stats = Stats{};
  if (rows == 0) return;
  stats.nnz_per_row_min = INT32_MAX;
  for (int row = 0; row < rows; ++row) {
    const int length = row_ptr[row + 1] - row_ptr[row];
    length_sum += length;
    length_square_sum += (double)length * length;
    stats.nnz_per_row_max = std::max(stats.nnz_per_row_max, length);
    stats.nnz_per_row_min = std::min(stats.nnz_per_row_min, length);
    double row_abs_sum = 0.0;
    for (int entry = row_ptr[row]; entry < row_ptr[row + 1]; ++entry) {
      const double magnitude = std::fabs(val[entry]);
      row_abs_sum += magnitude;
      if (magnitude > 0.0) {
        largest = std::max(largest, magnitude);
        smallest = std::min(smallest, magnitude);
      }
    }
    stats.norm_inf = std::max(stats.norm_inf, row_abs_sum);
  }
  stats.nnz_per_row_mean = length_sum / rows;
  stats.nnz_per_row_std =
      std::sqrt(std::max(0.0, length_square_sum / rows - stats.nnz_per_row_mean * stats.nnz_per_row_mean));
  stats.max_abs = largest;
  stats.min_abs = smallest < 1e308 ? smallest : 0.0;
  stats.dynamic_range = stats.min_abs > 0.0 ? stats.max_abs / stats.min_abs : 0.0;
}

// sort_columns_within_rows (include/csr.hpp:162). A row whose columns are already strictly increasing is
// left as it is (its sorted order is unique); any other row is ordered with std::sort over the entry
// positions keyed by column, the reference's own procedure, so rows with repeated columns end in the
// same order as there.
void sort_columns_within_rows(Csr& matrix) {
  parallel_for(matrix.rows, [&](int64_t first, int64_t last) {
    std::vector<int> order;
    std::vector<int> columns;
    std::vector<double> values;
    for (int64_t row = first; row < last; ++row) {
      const int begin = matrix.row_ptr[row], end = matrix.row_ptr[row + 1];
      bool increasing = true;
      for (int entry = begin + 1; entry < end && increasing; ++entry)
        increasing = matrix.col_ind[entry - 1] < matrix.col_ind[entry];
      if (increasing) continue;
      order.resize(end - begin);
      std::iota(order.begin(), order.end(), 0);
      std::sort(order.begin(), order.end(), [&](int left, int right) {
        return matrix.col_ind[begin + left] < matrix.col_ind[begin + right];
      });
      columns.resize(order.size());
      values.resize(order.size());
      for (size_t position = 0; position < order.size(); ++position) {
        columns[position] = matrix.col_ind[begin + order[position]];
        values[position] = matrix.val[begin + order[position]];
      }
      std::copy(columns.begin(), columns.end(), matrix.col_ind.begin() + begin);
      std::copy(values.begin(), values.end(), matrix.val.begin() + begin);
    }
  }, 4096);
}

// matrix_name_from_path (include/csr.hpp:192): file name without directory and last extension.
std::string matrix_name_from_path(const std::string& path) {
  const size_t separator = path.find_last_of("/\\");
  const std::string file = separator == std::string::npos ? path : path.substr(separator + 1);
  const size_t dot = file.find_last_of('.');
  return dot == std::string::npos ? file : file.substr(0, dot);
}

void validate(const Csr& matrix) {
  if (matrix.rows < 0 || matrix.cols < 0) fail(SPMV_ERR_INVALID_ARGUMENT, "negative dimensions");
  if ((int64_t)matrix.row_ptr.size() != (int64_t)matrix.rows + 1) fail(SPMV_ERR_INVALID_ARGUMENT, "row_ptr size");
  if (matrix.row_ptr[0] != 0) fail(SPMV_ERR_INVALID_ARGUMENT, "row_ptr[0] must be 0");
  for (int row = 0; row < matrix.rows; ++row)
    if (matrix.row_ptr[row + 1] < matrix.row_ptr[row]) fail(SPMV_ERR_INVALID_ARGUMENT, "row_ptr is not monotone");
  if ((int64_t)matrix.row_ptr[matrix.rows] != matrix.nnz()) fail(SPMV_ERR_INVALID_ARGUMENT, "row_ptr[rows] != nnz");
  for (int64_t entry = 0; entry < matrix.nnz(); ++entry)
    if (matrix.col_ind[entry] < 0 || matrix.col_ind[entry] >= matrix.cols)
      fail(SPMV_ERR_INVALID_ARGUMENT, "column index out of range");
}

namespace {

struct Entry {
  int row, col;
  double value;
};

std::string lower(std::string text) {
  std::transform(text.begin(), text.end(), text.begin(), [](unsigned char c) { return (char)std::tolower(c); });
  return text;
}

}  // namespace

// read_matrix_market (include/csr.hpp:232).
Csr read_matrix_market(const std::string& path) {
  std::FILE* file = std::fopen(path.c_str(), "rb");
  if (!file) fail(SPMV_ERR_IO, "cannot open matrix file: " + path);
  std::string text;
  {
    char buffer[1 << 16];
    size_t got = 0;
    while ((got = std::fread(buffer, 1, sizeof(buffer), file)) > 0) text.append(buffer, got);
    std::fclose(file);
  }
  if (text.empty()) fail(SPMV_ERR_FORMAT, "empty matrix file: " + path);

  // banner: the first line, "%%MatrixMarket matrix coordinate <field> <symmetry>"
  size_t line_end = text.find('\n');
  std::string banner_line = text.substr(0, line_end == std::string::npos ? text.size() : line_end);
  if (!banner_line.empty() && banner_line.back() == '\r') banner_line.pop_back();
  if (banner_line.rfind("%%MatrixMarket", 0) != 0) fail(SPMV_ERR_FORMAT, "not a Matrix Market file: " + path);
  std::istringstream banner_stream(banner_line);
  std::string tag, object, format, field, symmetry;
  banner_stream >> tag >> object >> format >> field >> symmetry;
  object = lower(object);
  format = lower(format);
  field = lower(field);
  symmetry = lower(symmetry);
  if (format != "coordinate") fail(SPMV_ERR_FORMAT, "only coordinate format supported (got " + format + ")");
  const bool is_pattern = field == "pattern";
  const bool is_symmetric = symmetry == "symmetric" || symmetry == "skew-symmetric" || symmetry == "hermitian";
  const bool is_skew = symmetry == "skew-symmetric";

  // skip_to_body (csr.hpp:119): the size line is the first non-empty line not starting with '%'.
  size_t cursor = line_end == std::string::npos ? text.size() : line_end + 1;
  std::string size_line;
  while (cursor < text.size()) {
    size_t next = text.find('\n', cursor);
    if (next == std::string::npos) next = text.size();
    std::string line = text.substr(cursor, next - cursor);
    cursor = next + 1;
    if (!line.empty() && line[0] != '%') {
      size_line = line;
      break;
    }
  }
  int rows = 0, cols = 0;
  int64_t declared_nnz = 0;
  {
    std::istringstream size_stream(size_line);
    size_stream >> rows >> cols >> declared_nnz;
  }
  if (rows <= 0 || cols <= 0) fail(SPMV_ERR_FORMAT, "bad dimensions in " + path);
  if (cursor > text.size()) cursor = text.size();

  // parse_body (csr.hpp:131): strtol, strtol, strtod per entry, whitespace skipped between entries.
  std::vector<Entry> entries;
  entries.reserve(is_symmetric ? (size_t)declared_nnz * 2 : (size_t)declared_nnz);
  const char* position = text.c_str() + cursor;
  const char* body_end = text.c_str() + text.size();
  char* stop = nullptr;
  for (int64_t entry = 0; entry < declared_nnz && position < body_end; ++entry) {
    const long row_one_based = std::strtol(position, &stop, 10);
    if (stop == position) break;
    position = stop;
    const long col_one_based = std::strtol(position, &stop, 10);
    position = stop;
    double value = 1.0;
    if (!is_pattern) {
      value = std::strtod(position, &stop);
      position = stop;
    }
    const int row_index = (int)row_one_based - 1;
    const int col_index = (int)col_one_based - 1;
    while (position < body_end && (*position == '\n' || *position == '\r' || *position == ' ' || *position == '\t'))
      ++position;
    if (row_index < 0 || row_index >= rows || col_index < 0 || col_index >= cols) continue;
    entries.push_back({row_index, col_index, value});
    if (is_symmetric && row_index != col_index) entries.push_back({col_index, row_index, is_skew ? -value : value});
  }
  if (entries.size() > (size_t)INT32_MAX) fail(SPMV_ERR_TOO_LARGE, "more than 2^31-1 nonzeros: " + path);
  std::string().swap(text);

  Csr matrix;
  matrix.rows = rows;
  matrix.cols = cols;
  matrix.symmetric_expanded = is_symmetric;
  matrix.row_ptr.assign((size_t)rows + 1, 0);
  for (const Entry& entry : entries) matrix.row_ptr[entry.row + 1]++;
  for (int row = 0; row < rows; ++row) matrix.row_ptr[row + 1] += matrix.row_ptr[row];
  matrix.col_ind.resize(entries.size());
  matrix.val.resize(entries.size());
  {
    // scatter_entries (csr.hpp:153): stable by file order within each row
    std::vector<int> next_slot(matrix.row_ptr.begin(), matrix.row_ptr.end() - 1);
    for (const Entry& entry : entries) {
      const int slot = next_slot[entry.row]++;
      matrix.col_ind[slot] = entry.col;
      matrix.val[slot] = entry.value;
    }
  }
  std::vector<Entry>().swap(entries);
  sort_columns_within_rows(matrix);
  matrix.name = matrix_name_from_path(path);
  matrix.compute_stats();
  return matrix;
}

}  // namespace spmvb200
