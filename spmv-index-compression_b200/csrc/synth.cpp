// synth.cpp — seeded synthetic matrices standing in for the benchmark configurations, and the x vectors.
//
// Every random draw comes from a counter-based stream keyed by (seed, row) — a SplitMix64 sequence
// started from a hash of both — so rows are generated in parallel, and a row range (one GPU's shard)
// comes out identical to the same rows of the whole matrix without building the rest.
#include "internal.hpp"

#include <cmath>
#include <random>

namespace spmvb200 {

namespace {

inline uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// SplitMix64 sequence for one (seed, stream, index) triple.
struct Stream {
  uint64_t state;
  Stream(uint64_t seed, uint64_t stream, uint64_t index) : state(mix64(mix64(seed ^ (stream << 56)) ^ index)) {}
  uint64_t next() {
    state += 0x9e3779b97f4a7c15ull;
    uint64_t z = state;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
  }
  double uniform01() { return (double)(next() >> 11) * 0x1.0p-53; }            // [0, 1)
  double uniform(double low, double high) { return low + (high - low) * uniform01(); }
  uint64_t below(uint64_t bound) { return (uint64_t)(((unsigned __int128)next() * bound) >> 64); }
  double normal() {                                                              // Box-Muller
    const double u1 = 1.0 - uniform01(), u2 = uniform01();
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
  }
  int poisson(double mean) {                                                     // inversion
    const double u = uniform01();
    double probability = std::exp(-mean), cumulative = probability;
    int k = 0;
    while (u > cumulative && k < 100000) {
      ++k;
      probability *= mean / k;
      cumulative += probability;
    }
    return k;
  }
};

enum : uint64_t { kStructure = 1, kValues = 2, kVector = 3 };

// Builds a Csr from per-row column lists produced in parallel: columns(row, out) fills out (sorted,
// unique), value(row, position, columns) gives each value.
template <class Columns, class Values>
Csr build_rows(int rows, int cols, int row_begin, int row_end, const Columns& columns, const Values& values) {
  const int count = row_end - row_begin;
  Csr matrix;
  matrix.rows = count;
  matrix.cols = cols;
  std::vector<int64_t> lengths((size_t)count + 1, 0);
  parallel_for(count, [&](int64_t first, int64_t last) {
    std::vector<int> scratch;
    for (int64_t local = first; local < last; ++local) {
      columns(row_begin + (int)local, scratch);
      lengths[local + 1] = (int64_t)scratch.size();
    }
  }, 1024);
  for (int local = 0; local < count; ++local) lengths[local + 1] += lengths[local];
  if (lengths[count] > INT32_MAX) fail(SPMV_ERR_TOO_LARGE, "more than 2^31-1 nonzeros");
  matrix.row_ptr.resize((size_t)count + 1);
  for (int local = 0; local <= count; ++local) matrix.row_ptr[local] = (int)lengths[local];
  matrix.col_ind.resize((size_t)lengths[count]);
  matrix.val.resize((size_t)lengths[count]);
  parallel_for(count, [&](int64_t first, int64_t last) {
    std::vector<int> scratch;
    for (int64_t local = first; local < last; ++local) {
      const int row = row_begin + (int)local;
      columns(row, scratch);
      const int begin = matrix.row_ptr[local];
      std::copy(scratch.begin(), scratch.end(), matrix.col_ind.begin() + begin);
      values(row, scratch, matrix.val.data() + begin);
    }
  }, 1024);
  (void)rows;
  matrix.compute_stats();
  return matrix;
}

// k distinct integers uniform in [low, high] other than excluded (or all of them when k is too large),
// sorted ascending.
void distinct_in_range(Stream& stream, int64_t low, int64_t high, int64_t excluded, int64_t k, std::vector<int>& out) {
  const int64_t available = high - low + 1 - ((excluded >= low && excluded <= high) ? 1 : 0);
  out.clear();
  if (k >= available) {
    for (int64_t value = low; value <= high; ++value)
      if (value != excluded) out.push_back((int)value);
    return;
  }
  while ((int64_t)out.size() < k) {
    const int64_t missing = k - (int64_t)out.size();
    for (int64_t draw = 0; draw < missing; ++draw) {
      const int64_t value = low + (int64_t)stream.below((uint64_t)(high - low + 1));
      if (value != excluded) out.push_back((int)value);
    }
    // each round draws only what is missing, so the unique count never exceeds k
    std::sort(out.begin(), out.end());
    out.erase(std::unique(out.begin(), out.end()), out.end());
  }
}

}  // namespace

Csr synth_laplacian2d(int grid) {
  if (grid <= 0 || (int64_t)grid * grid > INT32_MAX / 5) fail(SPMV_ERR_INVALID_ARGUMENT, "bad grid size");
  const int n = grid * grid;
  Csr matrix = build_rows(n, n, 0, n,
      [&](int row, std::vector<int>& out) {
        const int r = row / grid, c = row % grid;
        out.clear();
        if (r > 0) out.push_back(row - grid);
        if (c > 0) out.push_back(row - 1);
        out.push_back(row);
        if (c + 1 < grid) out.push_back(row + 1);
        if (r + 1 < grid) out.push_back(row + grid);
      },
      [&](int row, const std::vector<int>& columns, double* values) {
        for (size_t k = 0; k < columns.size(); ++k) values[k] = columns[k] == row ? 4.0 : -1.0;
      });
  matrix.name = "laplacian2d_" + std::to_string(grid);
  return matrix;
}

Csr synth_stencil27(int grid) {
  if (grid <= 0 || (int64_t)grid * grid * grid * 27 > INT32_MAX) fail(SPMV_ERR_INVALID_ARGUMENT, "bad grid size");
  const int n = grid * grid * grid;
  Csr matrix = build_rows(n, n, 0, n,
      [&](int row, std::vector<int>& out) {
        const int x = row % grid, y = (row / grid) % grid, z = row / (grid * grid);
        out.clear();
        for (int dz = -1; dz <= 1; ++dz)
          for (int dy = -1; dy <= 1; ++dy)
            for (int dx = -1; dx <= 1; ++dx) {
              const int xx = x + dx, yy = y + dy, zz = z + dz;
              if (xx < 0 || yy < 0 || zz < 0 || xx >= grid || yy >= grid || zz >= grid) continue;
              out.push_back((zz * grid + yy) * grid + xx);
            }
      },
      [&](int row, const std::vector<int>& columns, double* values) {
        for (size_t k = 0; k < columns.size(); ++k) values[k] = columns[k] == row ? 26.0 : -1.0;
      });
  matrix.name = "stencil27_" + std::to_string(grid);
  return matrix;
}

Csr synth_random_band(int n, int half_bandwidth, double mean, uint64_t seed) {
  if (n <= 0 || half_bandwidth < 0 || mean < 0) fail(SPMV_ERR_INVALID_ARGUMENT, "bad band parameters");
  Csr matrix = build_rows(n, n, 0, n,
      [&](int row, std::vector<int>& out) {
        Stream stream(seed, kStructure, (uint64_t)row);
        const int k = std::max(1, stream.poisson(mean));
        const int64_t low = std::max<int64_t>(0, (int64_t)row - half_bandwidth);
        const int64_t high = std::min<int64_t>(n - 1, (int64_t)row + half_bandwidth);
        distinct_in_range(stream, low, high, row, k, out);
        out.insert(std::lower_bound(out.begin(), out.end(), row), row);
      },
      [&](int row, const std::vector<int>& columns, double* values) {
        Stream stream(seed, kValues, (uint64_t)row);
        for (size_t k = 0; k < columns.size(); ++k) values[k] = stream.normal();
      });
  matrix.name = "random_band_" + std::to_string(n);
  return matrix;
}

Csr synth_power_law(int n, double alpha, int max_length, double mean, uint64_t seed) {
  if (n <= 0 || alpha <= 1.0 || max_length <= 0 || max_length > n || mean < 1.0)
    fail(SPMV_ERR_INVALID_ARGUMENT, "bad power-law parameters");
  // Zipf(alpha) on [1, max_length]: cumulative table for inversion
  std::vector<double> cumulative((size_t)max_length + 1, 0.0);
  for (int k = 1; k <= max_length; ++k) cumulative[k] = cumulative[k - 1] + std::pow((double)k, -alpha);
  const double total = cumulative[max_length];
  for (double& value : cumulative) value /= total;
  // scale c with E[clip(round(c Z), 1, max_length)] = mean, by bisection on the exact distribution
  auto expected = [&](double scale) {
    double sum = 0.0;
    for (int k = 1; k <= max_length; ++k) {
      const double length = std::min<double>(max_length, std::max(1.0, std::nearbyint(scale * k)));
      sum += (cumulative[k] - cumulative[k - 1]) * length;
    }
    return sum;
  };
  double low = 1e-6, high = (double)max_length;
  for (int iteration = 0; iteration < 200; ++iteration) {
    const double middle = 0.5 * (low + high);
    (expected(middle) < mean ? low : high) = middle;
  }
  const double scale = 0.5 * (low + high);
  Csr matrix = build_rows(n, n, 0, n,
      [&](int row, std::vector<int>& out) {
        Stream stream(seed, kStructure, (uint64_t)row);
        const double u = stream.uniform01();
        const int zipf = (int)(std::upper_bound(cumulative.begin() + 1, cumulative.end(), u) - cumulative.begin());
        const int length = (int)std::min<double>(max_length, std::max(1.0, std::nearbyint(scale * std::min(zipf, max_length))));
        distinct_in_range(stream, 0, n - 1, -1, length, out);
      },
      [&](int row, const std::vector<int>& columns, double* values) {
        Stream stream(seed, kValues, (uint64_t)row);
        for (size_t k = 0; k < columns.size(); ++k) values[k] = stream.uniform(-1.0, 1.0);
      });
  matrix.name = "power_law_" + std::to_string(n);
  return matrix;
}

Csr synth_block_fem(int n, int block, int blocks_per_row, int offset_range, uint64_t seed, int row_begin, int row_end) {
  if (n <= 0 || block <= 0 || n % block != 0 || blocks_per_row <= 0 || offset_range < 0 || row_begin < 0 ||
      row_end > n || row_begin > row_end)
    fail(SPMV_ERR_INVALID_ARGUMENT, "bad block-matrix parameters");
  if ((int64_t)(row_end - row_begin) * block * blocks_per_row > INT32_MAX) fail(SPMV_ERR_TOO_LARGE, "shard exceeds 2^31-1 nonzeros");
  const int block_rows = n / block;
  const int block_range = offset_range / block;
  auto block_columns = [&](int block_row, std::vector<int>& out) {
    Stream stream(seed, kStructure, (uint64_t)block_row);
    const int64_t low = std::max<int64_t>(0, (int64_t)block_row - block_range);
    const int64_t high = std::min<int64_t>(block_rows - 1, (int64_t)block_row + block_range);
    distinct_in_range(stream, low, high, block_row, blocks_per_row - 1, out);
    out.insert(std::lower_bound(out.begin(), out.end(), block_row), block_row);
  };
  Csr matrix = build_rows(n, n, row_begin, row_end,
      [&](int row, std::vector<int>& out) {
        std::vector<int> blocks;
        block_columns(row / block, blocks);
        out.clear();
        for (int block_column : blocks)
          for (int k = 0; k < block; ++k) out.push_back(block_column * block + k);
      },
      [&](int row, const std::vector<int>& columns, double* values) {
        Stream stream(seed, kValues, (uint64_t)row);
        double off_diagonal = 0.0;
        size_t diagonal = 0;
        for (size_t k = 0; k < columns.size(); ++k) {
          values[k] = stream.normal();
          if (columns[k] == row) diagonal = k;
          else off_diagonal += std::fabs(values[k]);
        }
        values[diagonal] = 1.0 + off_diagonal;
      });
  matrix.name = "block_fem_" + std::to_string(n);
  return matrix;
}

namespace {

template <class Store>
void fill_values(int dtype, int64_t count, void* out, const Store& value_at) {
  parallel_for(count, [&](int64_t first, int64_t last) {
    for (int64_t index = first; index < last; ++index) {
      const float narrowed = (float)value_at(index);
      if (dtype == SPMV_F64) static_cast<double*>(out)[index] = (double)narrowed;
      else if (dtype == SPMV_F32) static_cast<float*>(out)[index] = narrowed;
      else static_cast<_Float16*>(out)[index] = (_Float16)narrowed;
    }
  });
}

}  // namespace

void fill_uniform(int dtype, int64_t count, uint64_t seed, void* out) {
  value_bytes_of(dtype);
  fill_values(dtype, count, out, [&](int64_t index) {
    Stream stream(seed, kVector, (uint64_t)index);
    return stream.uniform(-1.0, 1.0);
  });
}

void fill_reference_x(int dtype, int64_t count, void* out) {
  value_bytes_of(dtype);
  std::mt19937 generator(7);
  std::uniform_real_distribution<double> uniform(-1.0, 1.0);
  for (int64_t index = 0; index < count; ++index) {
    const float narrowed = (float)uniform(generator);
    if (dtype == SPMV_F64) static_cast<double*>(out)[index] = (double)narrowed;
    else if (dtype == SPMV_F32) static_cast<float*>(out)[index] = narrowed;
    else static_cast<_Float16*>(out)[index] = (_Float16)narrowed;
  }
}

// Device values of a layout: (T)(float)val like upload_matrix (bench_csr_width.cu:927), or (T)val.
void convert_values(int dtype, const double* in, int64_t count, int value_rounding, void* out) {
  value_bytes_of(dtype);
  parallel_for(count, [&](int64_t first, int64_t last) {
    for (int64_t index = first; index < last; ++index) {
      const double value = in[index];
      if (value_rounding == 0) {
        const float narrowed = (float)value;
        if (dtype == SPMV_F64) static_cast<double*>(out)[index] = (double)narrowed;
        else if (dtype == SPMV_F32) static_cast<float*>(out)[index] = narrowed;
        else static_cast<_Float16*>(out)[index] = (_Float16)narrowed;
      } else {
        if (dtype == SPMV_F64) static_cast<double*>(out)[index] = value;
        else if (dtype == SPMV_F32) static_cast<float*>(out)[index] = (float)value;
        else static_cast<_Float16*>(out)[index] = (_Float16)value;
      }
    }
  });
}

}  // namespace spmvb200
