// rcm.cpp — Reverse Cuthill-McKee ordering, the symmetric permutation B = P A P^T and the on-disk
// permutation cache.
//
// The ordering is the one of include/rcm.hpp: the pattern of A + A^T without the diagonal (neighbours
// sorted and unique); per connected component, taken in order of its lowest-index node, a George-Liu
// pseudo-peripheral start found by at most 8 restarts from the lowest-degree node of the last BFS level
// (the first such node in reverse visiting order on ties); then Cuthill-McKee from that start, appending
// each node's unvisited neighbours by increasing degree and index; finally the whole order reversed.
// The same rules give the same permutation, which the tests check against the reference itself.
#include "internal.hpp"

#include <chrono>
#include <cstdio>
#include <cstring>

namespace spmvb200 {

namespace {

constexpr char kPermutationMagic[8] = {'R', 'C', 'M', 'P', 'E', 'R', 'M', '1'};
constexpr int kPseudoPeripheralIterations = 8;

// Adjacency of A + A^T without the diagonal, each list sorted ascending and unique.
struct Graph {
  std::vector<int64_t> offsets;
  std::vector<int> neighbours;
  int64_t degree(int node) const { return offsets[node + 1] - offsets[node]; }
};

Graph symmetric_graph(const Csr& matrix) {
  const int n = matrix.rows;
  // transpose pattern: for every column, the rows holding it, ascending (rows are visited in order)
  std::vector<int64_t> transpose_offsets((size_t)n + 1, 0);
  for (int64_t entry = 0; entry < matrix.nnz(); ++entry) ++transpose_offsets[matrix.col_ind[entry] + 1];
  for (int column = 0; column < n; ++column) transpose_offsets[column + 1] += transpose_offsets[column];
  std::vector<int> transpose_rows((size_t)matrix.nnz());
  {
    std::vector<int64_t> next(transpose_offsets.begin(), transpose_offsets.end() - 1);
    for (int row = 0; row < n; ++row)
      for (int entry = matrix.row_ptr[row]; entry < matrix.row_ptr[row + 1]; ++entry)
        transpose_rows[next[matrix.col_ind[entry]]++] = row;
  }
  // merge row r of A (sorted) with row r of A^T (sorted), dropping r itself and repeats
  auto merge = [&](int row, int* out) -> int64_t {
    int64_t a = matrix.row_ptr[row], a_end = matrix.row_ptr[row + 1];
    int64_t b = transpose_offsets[row], b_end = transpose_offsets[row + 1];
    int64_t written = 0;
    int previous = -1;
    while (a < a_end || b < b_end) {
      int node;
      if (b >= b_end || (a < a_end && matrix.col_ind[a] <= transpose_rows[b])) node = matrix.col_ind[a++];
      else node = transpose_rows[b++];
      if (node == row || node == previous) continue;
      previous = node;
      if (out) out[written] = node;
      ++written;
    }
    return written;
  };
  Graph graph;
  graph.offsets.assign((size_t)n + 1, 0);
  std::vector<int64_t> counts((size_t)n, 0);
  parallel_for(n, [&](int64_t first, int64_t last) {
    for (int64_t row = first; row < last; ++row) counts[row] = merge((int)row, nullptr);
  });
  for (int row = 0; row < n; ++row) graph.offsets[row + 1] = graph.offsets[row] + counts[row];
  graph.neighbours.resize((size_t)graph.offsets[n]);
  parallel_for(n, [&](int64_t first, int64_t last) {
    for (int64_t row = first; row < last; ++row) merge((int)row, graph.neighbours.data() + graph.offsets[row]);
  });
  return graph;
}

// BFS level structure from root inside its component: visiting order in nodes, the nodes of the last
// level (collected from the end of the visiting order) in last_level; returns the eccentricity.
int level_structure(const Graph& graph, int root, std::vector<int>& distance, std::vector<int>& nodes,
                    std::vector<int>& last_level) {
  nodes.clear();
  last_level.clear();
  distance[root] = 0;
  nodes.push_back(root);
  for (size_t head = 0; head < nodes.size(); ++head) {
    const int node = nodes[head];
    for (int64_t slot = graph.offsets[node]; slot < graph.offsets[node + 1]; ++slot) {
      const int next = graph.neighbours[slot];
      if (distance[next] >= 0) continue;
      distance[next] = distance[node] + 1;
      nodes.push_back(next);
    }
  }
  const int eccentricity = distance[nodes.back()];
  for (size_t position = nodes.size(); position-- > 0;) {
    if (distance[nodes[position]] != eccentricity) break;
    last_level.push_back(nodes[position]);
  }
  return eccentricity;
}

void clear_distances(const std::vector<int>& nodes, std::vector<int>& distance) {
  for (int node : nodes) distance[node] = -1;
}

int pseudo_peripheral(const Graph& graph, int seed, std::vector<int>& distance, std::vector<int>& nodes) {
  std::vector<int> last_level, candidate_nodes, candidate_last_level;
  int current = seed;
  int eccentricity = level_structure(graph, current, distance, nodes, last_level);
  for (int iteration = 0; iteration < kPseudoPeripheralIterations; ++iteration) {
    int candidate = last_level.front();
    for (int node : last_level)
      if (graph.degree(node) < graph.degree(candidate)) candidate = node;
    clear_distances(nodes, distance);
    const int candidate_eccentricity = level_structure(graph, candidate, distance, candidate_nodes, candidate_last_level);
    if (candidate_eccentricity <= eccentricity) break;
    current = candidate;
    eccentricity = candidate_eccentricity;
    nodes.swap(candidate_nodes);
    last_level.swap(candidate_last_level);
  }
  return current;
}

void cuthill_mckee(const Graph& graph, int start, std::vector<char>& visited, std::vector<int>& order) {
  std::vector<int> fresh;
  size_t head = order.size();
  visited[start] = 1;
  order.push_back(start);
  while (head < order.size()) {
    const int node = order[head++];
    fresh.clear();
    for (int64_t slot = graph.offsets[node]; slot < graph.offsets[node + 1]; ++slot) {
      const int next = graph.neighbours[slot];
      if (visited[next]) continue;
      visited[next] = 1;
      fresh.push_back(next);
    }
    std::sort(fresh.begin(), fresh.end(), [&](int left, int right) {
      const int64_t left_degree = graph.degree(left), right_degree = graph.degree(right);
      return left_degree != right_degree ? left_degree < right_degree : left < right;
    });
    order.insert(order.end(), fresh.begin(), fresh.end());
  }
}

}  // namespace

std::vector<int> reverse_cuthill_mckee(const Csr& matrix) {
  if (matrix.rows != matrix.cols) fail(SPMV_ERR_INVALID_ARGUMENT, "RCM requires a square matrix");
  const Graph graph = symmetric_graph(matrix);
  std::vector<int> distance((size_t)matrix.rows, -1);
  std::vector<char> visited((size_t)matrix.rows, 0);
  std::vector<int> order, nodes;
  order.reserve((size_t)matrix.rows);
  for (int seed = 0; seed < matrix.rows; ++seed) {
    if (visited[seed]) continue;
    const int start = pseudo_peripheral(graph, seed, distance, nodes);
    clear_distances(nodes, distance);
    cuthill_mckee(graph, start, visited, order);
  }
  std::reverse(order.begin(), order.end());
  return order;
}

// apply_symmetric_permutation (rcm.hpp:219): b_ij = a_{p(i), p(j)}, columns re-sorted, stats recomputed.
Csr apply_symmetric_permutation(const Csr& source, const std::vector<int>& new_to_old) {
  if ((int)new_to_old.size() != source.rows || source.rows != source.cols)
    fail(SPMV_ERR_INVALID_ARGUMENT, "permutation size does not match a square matrix");
  std::vector<int> old_to_new((size_t)source.rows, -1);
  for (int index = 0; index < source.rows; ++index) {
    const int old_index = new_to_old[index];
    if (old_index < 0 || old_index >= source.rows || old_to_new[old_index] >= 0)
      fail(SPMV_ERR_INVALID_ARGUMENT, "not a permutation");
    old_to_new[old_index] = index;
  }
  Csr result;
  result.rows = source.rows;
  result.cols = source.cols;
  result.symmetric_expanded = source.symmetric_expanded;
  result.name = source.name;
  result.row_ptr.assign((size_t)source.rows + 1, 0);
  for (int row = 0; row < source.rows; ++row) {
    const int old_row = new_to_old[row];
    result.row_ptr[row + 1] = result.row_ptr[row] + (source.row_ptr[old_row + 1] - source.row_ptr[old_row]);
  }
  result.col_ind.resize(source.col_ind.size());
  result.val.resize(source.val.size());
  parallel_for(source.rows, [&](int64_t first, int64_t last) {
    for (int64_t row = first; row < last; ++row) {
      const int old_row = new_to_old[row];
      int destination = result.row_ptr[row];
      for (int entry = source.row_ptr[old_row]; entry < source.row_ptr[old_row + 1]; ++entry, ++destination) {
        result.col_ind[destination] = old_to_new[source.col_ind[entry]];
        result.val[destination] = source.val[entry];
      }
    }
  });
  sort_columns_within_rows(result);
  result.compute_stats();
  return result;
}

std::string permutation_path_for(const std::string& matrix_path, const std::string& ordering) {
  const size_t extension = matrix_path.rfind(".mtx");
  const std::string stem = extension == std::string::npos ? matrix_path : matrix_path.substr(0, extension);
  return stem + "." + ordering + ".perm";
}

void write_permutation(const std::string& path, const std::vector<int>& new_to_old, double seconds) {
  const int64_t rows = (int64_t)new_to_old.size();
  const std::string temporary = path + ".partial";
  std::FILE* output = std::fopen(temporary.c_str(), "wb");
  if (!output) fail(SPMV_ERR_IO, "cannot write permutation " + temporary);
  bool written = std::fwrite(kPermutationMagic, 1, sizeof(kPermutationMagic), output) == sizeof(kPermutationMagic) &&
                 std::fwrite(&rows, sizeof(rows), 1, output) == 1 &&
                 std::fwrite(&seconds, sizeof(seconds), 1, output) == 1 &&
                 std::fwrite(new_to_old.data(), sizeof(int), new_to_old.size(), output) == new_to_old.size();
  written = (std::fclose(output) == 0) && written;
  if (!written || std::rename(temporary.c_str(), path.c_str()) != 0) fail(SPMV_ERR_IO, "cannot write permutation " + path);
}

bool read_permutation(const std::string& path, int expected_rows, std::vector<int>& new_to_old, double& seconds) {
  std::FILE* input = std::fopen(path.c_str(), "rb");
  if (!input) return false;
  char magic[8];
  int64_t rows = 0;
  bool valid = std::fread(magic, 1, sizeof(magic), input) == sizeof(magic) &&
               std::memcmp(magic, kPermutationMagic, sizeof(magic)) == 0 &&
               std::fread(&rows, sizeof(rows), 1, input) == 1 && rows == expected_rows &&
               std::fread(&seconds, sizeof(seconds), 1, input) == 1;
  if (valid) {
    new_to_old.resize((size_t)rows);
    valid = std::fread(new_to_old.data(), sizeof(int), new_to_old.size(), input) == new_to_old.size();
  }
  std::fclose(input);
  if (valid) {
    std::vector<char> seen((size_t)rows, 0);
    for (int old_index : new_to_old) {
      if (old_index < 0 || old_index >= expected_rows || seen[old_index]) {
        valid = false;
        break;
      }
      seen[old_index] = 1;
    }
  }
  if (!valid) fail(SPMV_ERR_FORMAT, "invalid permutation file " + path);
  return true;
}

Csr reorder_with_rcm(const std::string& matrix_path, const Csr& matrix, double& seconds) {
  const std::string path = permutation_path_for(matrix_path, "rcm");
  std::vector<int> new_to_old;
  if (!read_permutation(path, matrix.rows, new_to_old, seconds)) {
    const auto start = std::chrono::steady_clock::now();
    new_to_old = reverse_cuthill_mckee(matrix);
    seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
    write_permutation(path, new_to_old, seconds);
  }
  return apply_symmetric_permutation(matrix, new_to_old);
}

}  // namespace spmvb200
