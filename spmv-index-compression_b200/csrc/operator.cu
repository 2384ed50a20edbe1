// operator.cu — the device-resident operator: encode, plan tiles, upload, launch.
//
// Layout in HBM of one operator (one allocation per stream, each 256-byte aligned by cudaMalloc):
//   row_ptr   int32[rows + 1]                     the CSR row pointer (all layouts)
//   values    T[nnz]                              (T)(float)val by default, as upload_matrix (:927)
//   columns   int32 / uint16 / uint8 [nnz]        i32, i16, i8 absolute; r16, r8 offsets from the base
//   row_base  int32[rows]                         r16, r8, lp: the row's first column
//   row_word  int32[rows], row_width uint8[rows]  lp: first word and bit width of the row's stream
//   words     uint32[word_count]                  lp: lane-major packed deltas + 2 spare words
//   tiles     int4[tiles]                         {row_begin, row_end, entry_begin, entry_end}
//   tile_words int2[tiles]                        lp: {first word, last word + 1} of each tile's stream
//   long_rows int32[long_rows]                    rows longer than a tile
//   lane_marks int32[...], lane_mark_first int64[long_rows]
//                                                 lp long rows: each lane's column after every 16 deltas
//   status    uint32                              bit 0: a bounded device wait gave up
// The streams are the reference's (bench_csr_width.cu:795-951), so memory_of counts them exactly; the
// tile plan adds 16 bytes per tile (about 2048 nonzeros) and 4 bytes per long row, and CSR-lp 4 bytes per 16
// entries of its long rows.
#include <cuda_runtime.h>
#include <climits>

#include <cstring>
#include <memory>

#include "capi_internal.hpp"
#include "dispatch.hpp"

namespace spmvb200 {

namespace {

void cuda_check(cudaError_t status, const char* what) {
  if (status == cudaSuccess) return;
  const int code = status == cudaErrorMemoryAllocation ? SPMV_ERR_OUT_OF_MEMORY : SPMV_ERR_CUDA;
  fail(code, std::string(what) + ": " + cudaGetErrorString(status));
}

// A device copy of count elements followed by kStreamPadding zero bytes, so that a tile's bulk copy may
// round its end up to the next 16-byte boundary.
template <class T>
T* device_upload(const void* host, size_t count, int64_t& total_bytes) {
  T* device = nullptr;
  const size_t bytes = sizeof(T) * count + kStreamPadding;
  cuda_check(cudaMalloc(reinterpret_cast<void**>(&device), bytes), "cudaMalloc");
  total_bytes += (int64_t)bytes;
  cudaError_t status = cudaMemset(device, 0, bytes);
  if (status == cudaSuccess && host && count) status = cudaMemcpy(device, host, sizeof(T) * count, cudaMemcpyHostToDevice);
  if (status != cudaSuccess) {
    cudaFree(device);
    cuda_check(status, "device upload");
  }
  return device;
}

// A device buffer owned for the duration of operator creation.
template <class T>
struct DeviceBuffer {
  T* data = nullptr;
  void allocate(size_t count, const T* host) {
    cuda_check(cudaMalloc(reinterpret_cast<void**>(&data), sizeof(T) * std::max<size_t>(count, 1)), "cudaMalloc");
    if (count) cuda_check(cudaMemcpy(data, host, sizeof(T) * count, cudaMemcpyHostToDevice), "upload");
  }
  void release() {
    if (data) cudaFree(data);
    data = nullptr;
  }
  ~DeviceBuffer() { release(); }
};

// CSR-lp matrices with at least this many nonzeros are encoded on the device.
constexpr int64_t kDeviceEncodeNnz = 1 << 20;

}  // namespace

DeviceScope::DeviceScope(int device) {
  cuda_check(cudaGetDevice(&previous), "cudaGetDevice");
  if (device >= 0 && device != previous) cuda_check(cudaSetDevice(device), "cudaSetDevice");
}
DeviceScope::~DeviceScope() {
  if (previous >= 0) cudaSetDevice(previous);
}

// encode.cu
int64_t device_lane_packed_layout(const int* row_ptr, const int* col_ind, int rows, int tpr, int* row_word,
                                  uint8_t* row_width, cudaStream_t stream);
void device_lane_packed_pack(const int* row_ptr, const int* col_ind, int rows, int tpr, const int* row_word,
                             const uint8_t* row_width, uint32_t* words, int64_t word_count, cudaStream_t stream);

// Tile plan: maximal runs of consecutive rows with at most tile_nnz nonzeros and tile_rows rows; a row
// with more than tile_nnz nonzeros is listed as long and processed by the vector path instead.
struct TilePlan {
  std::vector<int4> tiles;
  std::vector<int2> tile_words;
  std::vector<int> long_rows;
  int64_t short_rows = 0;
  int64_t short_nnz = 0;
  int index_words = 0;   // CSR-lp: the longest tile's word range plus one
};

TilePlan plan_tiles(const Csr& matrix, int tile_nnz, int tile_rows, const int* row_word, const uint8_t* row_width) {
  TilePlan plan;
  int begin = -1, count = 0;
  int64_t nnz = 0;
  auto close = [&](int end) {
    if (begin < 0) return;
    plan.tiles.push_back(make_int4(begin, end, matrix.row_ptr[begin], matrix.row_ptr[end]));
    if (row_word) {
      const int last = end - 1;
      const int64_t last_words = ((int64_t)(matrix.row_ptr[last + 1] - matrix.row_ptr[last]) * row_width[last] + 31) / 32;
      plan.tile_words.push_back(make_int2(row_word[begin], (int)(row_word[last] + last_words)));
      plan.index_words = std::max(plan.index_words, (int)(row_word[last] + last_words) + 1 - row_word[begin]);
    }
    begin = -1;
    count = 0;
    nnz = 0;
  };
  for (int row = 0; row < matrix.rows; ++row) {
    const int length = matrix.row_ptr[row + 1] - matrix.row_ptr[row];
    if (length > tile_nnz) {
      close(row);
      plan.long_rows.push_back(row);
      continue;
    }
    if (begin >= 0 && (nnz + length > tile_nnz || count + 1 > tile_rows)) close(row);
    if (begin < 0) begin = row;
    ++count;
    nnz += length;
    ++plan.short_rows;
    plan.short_nnz += length;
  }
  close(matrix.rows);
  return plan;
}

// The x window of each tile: the columns [first column of its rows, last column of its rows] (rows are
// sorted), kept when it holds at most limit elements and its 16-byte-aligned superset stays inside x
// (cols elements of value_bytes, x 16-byte aligned); {0, 0} otherwise.
std::vector<int2> plan_windows(const Csr& matrix, const TilePlan& plan, int limit, int value_bytes) {
  std::vector<int2> windows(plan.tiles.size(), make_int2(0, 0));
  const int64_t x_bytes = (int64_t)matrix.cols * value_bytes;
  for (size_t t = 0; t < plan.tiles.size(); ++t) {
    int first = INT32_MAX, last = -1;
    for (int row = plan.tiles[t].x; row < plan.tiles[t].y; ++row) {
      const int begin = matrix.row_ptr[row], end = matrix.row_ptr[row + 1];
      if (end == begin) continue;
      first = std::min(first, matrix.col_ind[begin]);
      last = std::max(last, matrix.col_ind[end - 1]);
    }
    if (last < first) continue;
    const int64_t end_bytes = ((int64_t)(last + 1) * value_bytes + 15) / 16 * 16;
    if (last - first + 1 <= limit && end_bytes <= x_bytes) windows[t] = make_int2(first, last + 1);
  }
  return windows;
}

// Nonzeros per distinct 32-byte sector of x that a row reads, over the matrix: about 1 when the columns
// of a row are scattered (every gather its own sector), several when they come in runs (stencils, blocks).
double entries_per_x_sector(const Csr& matrix, int value_bytes) {
  int64_t sectors = 0;
  for (int row = 0; row < matrix.rows; ++row) {
    int64_t previous = -1;
    for (int entry = matrix.row_ptr[row]; entry < matrix.row_ptr[row + 1]; ++entry) {
      const int64_t sector = (int64_t)matrix.col_ind[entry] * value_bytes / 32;
      if (sector != previous) ++sectors;
      previous = sector;
    }
  }
  return sectors == 0 ? 0.0 : (double)matrix.nnz() / sectors;
}

// The window capacity worth reserving: the widest kept window when at least half the tiles keep one under
// limit elements, else 0 (no windows).
int window_capacity(const std::vector<int2>& windows) {
  int kept = 0, widest = 0;
  for (const int2& window : windows)
    if (window.y > window.x) {
      ++kept;
      widest = std::max(widest, window.y - window.x);
    }
  return windows.empty() || 2 * kept < (int)windows.size() ? 0 : widest;
}

// Physical threads per row P: the fewest that leave a thread at most 28 entries of an average row (one
// batch of gathers), and at least T/16 (at most 16 lane sums per thread). A tile then holds 256/P rows (at
// least 128), so that one pass of the CTA's 256/P row groups covers it. Measured on B200 (CSR-i32):
// 27-point stencil (27 entries a row) P = 1 at T = 8; random band (33) P = 2; block FEM (64) P = 4.
int choose_physical_tpr(int tpr, int layout, double mean_length) {
  (void)layout;
  int physical = 1;
  while (physical < tpr && mean_length / physical > 28.0) physical *= 2;
  while (tpr / physical > 16) physical *= 2;
  return physical;
}

// Rows by length: the nonzeros of rows longer than 4x the mean + 32 make at least a tenth of the matrix
// (a power-law graph), so that tiles of consecutive rows would mix very short and very long rows.
bool skewed_rows(const Csr& matrix) {
  if (matrix.rows == 0 || matrix.nnz() == 0) return false;
  const double heavy = 4.0 * (double)matrix.nnz() / matrix.rows + 32.0;
  int64_t heavy_nnz = 0;
  for (int row = 0; row < matrix.rows; ++row) {
    const int length = matrix.row_ptr[row + 1] - matrix.row_ptr[row];
    if (length > heavy) heavy_nnz += length;
  }
  return heavy_nnz * 10 >= matrix.nnz();
}

// Rows by length: rows of at most kShortMax entries need no list (their blocks walk all rows); rows up to
// long_threshold are listed as {row, first entry, end entry, row base} items, each in the segment of its
// P (the fewest threads, among the P that divide T with T / P <= 8, that leave a thread at most 32 of
// its entries), longest first within a segment; longer rows are long rows, one CTA each.
struct ClassPlan {
  std::vector<int4> items;
  int64_t segment_first[6] = {0, 0, 0, 0, 0, 0};
  int64_t segment_items[6] = {0, 0, 0, 0, 0, 0};
  std::vector<int> long_rows;
};

// CSR-lp long rows: lane L's column after each kLaneMarkEvery of its deltas, which is the column of its
// entry L + (j * kLaneMarkEvery - 1) * T for the j-th mark (0 where the lane has no such entry), j = 1 ..
// ceil(ceil(length / T) / kLaneMarkEvery) - 1, at [first[item] + (j - 1) * T + L].
void build_lane_marks(const Csr& matrix, const std::vector<int>& long_rows, int tpr, std::vector<int>& marks,
                      std::vector<int64_t>& first) {
  marks.clear();
  first.assign(long_rows.size(), 0);
  for (size_t item = 0; item < long_rows.size(); ++item) {
    const int row = long_rows[item];
    const int64_t begin = matrix.row_ptr[row], length = (int64_t)matrix.row_ptr[row + 1] - begin;
    const int64_t per_lane = (length + tpr - 1) / tpr;
    const int64_t count = (per_lane + kLaneMarkEvery - 1) / kLaneMarkEvery - 1;
    first[item] = (int64_t)marks.size();
    for (int64_t j = 1; j <= count; ++j)
      for (int lane = 0; lane < tpr; ++lane) {
        const int64_t entry = lane + (j * kLaneMarkEvery - 1) * tpr;
        marks.push_back(entry < length ? matrix.col_ind[(size_t)(begin + entry)] : 0);
      }
  }
}

ClassPlan plan_classes(const Csr& matrix, int tpr, int long_threshold) {
  ClassPlan plan;
  std::vector<int4> segments[6];
  for (int row = 0; row < matrix.rows; ++row) {
    const int begin = matrix.row_ptr[row], length = matrix.row_ptr[row + 1] - begin;
    if (length <= kShortMax) continue;
    if (length > long_threshold) {
      plan.long_rows.push_back(row);
      continue;
    }
    int segment = 0;
    while (!segment_exists(tpr, segment)) ++segment;
    while (segment < 5 && segment_exists(tpr, segment + 1) && length > 32 * (1 << segment)) ++segment;
    segments[segment].push_back(make_int4(row, begin, begin + length, matrix.col_ind[begin]));
  }
  for (int segment = 0; segment < 6; ++segment) {
    std::stable_sort(segments[segment].begin(), segments[segment].end(),
                     [](const int4& a, const int4& b) { return a.z - a.y > b.z - b.y; });
    plan.segment_first[segment] = (int64_t)plan.items.size();
    plan.segment_items[segment] = (int64_t)segments[segment].size();
    plan.items.insert(plan.items.end(), segments[segment].begin(), segments[segment].end());
  }
  return plan;
}

}  // namespace spmvb200

struct spmv_operator {
  int device = 0;
  int layout = 0, dtype = 0, tpr = 0, physical_tpr = 0, tile_nnz = 0, tile_rows = 0, stages = 0, tile_index_words = 0;
  int kernel = 0;   // kernel family: dtype, or kKernelHalfSums (FP16 summed in FP16)
  int accumulate = SPMV_ACCUMULATE_WIDE;
  int rows = 0, cols = 0;
  int64_t nnz = 0;
  spmv_memory memory{};
  int* row_ptr = nullptr;
  void* values = nullptr;
  void* columns = nullptr;
  int* row_base = nullptr;
  int* row_word = nullptr;
  uint8_t* row_width = nullptr;
  uint32_t* words = nullptr;
  int4* tiles = nullptr;
  int2* tile_words = nullptr;
  int* long_rows = nullptr;
  int* lane_marks = nullptr;           // CSR-lp long rows (build_lane_marks)
  int64_t* lane_mark_first = nullptr;
  unsigned* status = nullptr;
  int64_t tile_count = 0;
  int64_t tile_ctas = 0;
  int64_t long_count = 0;
  int64_t long_ctas = 0;
  int long_chunk = 0;
  int smem_bytes = 0;
  int64_t device_bytes = 0;
  // rows by length (SPMV_SCHEDULE_CLASSES)
  int schedule = SPMV_SCHEDULE_TILES;
  int4* row_items = nullptr;
  int2* tile_windows = nullptr;   // tiles: the x window each tile stages, {first, end} column (first == end: none)
  int window_elements = 0;
  int resident = 1;   // tiles: persistent CTAs per multiprocessor
  bool dense = false; // tiles: the dense variant (one thread per lane, more CTAs per multiprocessor)
  int64_t segment_first[6] = {0, 0, 0, 0, 0, 0};
  int64_t segment_items[6] = {0, 0, 0, 0, 0, 0};
  int64_t segment_blocks[6] = {0, 0, 0, 0, 0, 0};
  int64_t short_blocks = 0;

  ~spmv_operator() {
    int previous = -1;
    cudaGetDevice(&previous);
    if (previous != device) cudaSetDevice(device);
    for (void* pointer : {(void*)row_ptr, values, columns, (void*)row_base, (void*)row_word, (void*)row_width,
                          (void*)words, (void*)tiles, (void*)tile_words, (void*)long_rows, (void*)lane_marks,
                          (void*)lane_mark_first, (void*)status,
                          (void*)row_items, (void*)tile_windows})
      if (pointer) cudaFree(pointer);
    if (previous >= 0 && previous != device) cudaSetDevice(previous);
  }
};

using namespace spmvb200;

namespace {

void upload_lane_marks(spmv_operator* op, const Csr& m, const std::vector<int>& long_rows, int tpr) {
  std::vector<int> marks;
  std::vector<int64_t> first;
  build_lane_marks(m, long_rows, tpr, marks, first);
  op->lane_marks = device_upload<int>(marks.empty() ? nullptr : marks.data(), std::max<size_t>(marks.size(), 1),
                                      op->device_bytes);
  op->lane_mark_first = device_upload<int64_t>(first.data(), first.size(), op->device_bytes);
}

KernelArgs kernel_args(const spmv_operator* op, const void* x, void* y) {
  KernelArgs a{};
  a.rows = op->rows;
  a.cols = op->cols;
  a.row_ptr = op->row_ptr;
  a.columns = op->columns;
  a.row_base = op->row_base;
  a.row_word = op->row_word;
  a.row_width = op->row_width;
  a.words = op->words;
  a.values = op->values;
  a.x = x;
  a.y = y;
  a.tiles = op->tiles;
  a.tile_words = op->tile_words;
  a.tile_count = op->tile_count;
  a.tile_nnz = op->tile_nnz;
  a.tile_rows = op->tile_rows;
  a.tile_index_words = op->tile_index_words;
  // x windows need x 16-byte aligned (the bulk copies of x start on 16-byte boundaries)
  a.tile_windows = op->window_elements > 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 ? op->tile_windows : nullptr;
  a.window_elements = op->window_elements;
  a.stages = op->stages;
  a.tile_ctas = op->tile_ctas;
  a.dense = op->dense ? 1 : 0;
  a.row_list = op->long_rows;
  a.row_count = op->long_count;
  a.lane_marks = op->lane_marks;
  a.lane_mark_first = op->lane_mark_first;
  a.vector_blocks = op->long_ctas;
  a.long_chunk = op->long_chunk;
  a.smem_bytes = op->smem_bytes;
  a.status = op->status;
  a.row_items = op->row_items;
  a.long_blocks = op->schedule == SPMV_SCHEDULE_CLASSES ? op->long_count : 0;
  for (int segment = 0; segment < 6; ++segment) {
    a.segment_first[segment] = op->segment_first[segment];
    a.segment_items[segment] = op->segment_items[segment];
    a.segment_blocks[segment] = op->segment_blocks[segment];
  }
  return a;
}

int64_t class_blocks(const spmv_operator* op) {
  int64_t blocks = op->long_count + op->short_blocks;
  for (int segment = 0; segment < 6; ++segment) blocks += op->segment_blocks[segment];
  return blocks;
}

cudaError_t launch_product(const spmv_operator* op, const KernelArgs& a, cudaStream_t stream) {
  if (op->schedule == SPMV_SCHEDULE_CLASSES)
    return launch_classes(op->kernel, op->layout, op->tpr, a, class_blocks(op), op->smem_bytes, stream);
  return launch_tiles(op->kernel, op->layout, op->tpr, op->physical_tpr, a, stream);
}

}  // namespace

namespace spmvb200 {
// One product on a stream, the tile kernel's persistent CTAs leaving free_sms multiprocessors idle, so that
// kernels on other streams (a collective) run beside it. The class schedule needs no reservation: its
// CTAs are not persistent.
cudaError_t run_operator_leaving_sms(const spmv_operator* op, const void* x, void* y, cudaStream_t stream, int free_sms) {
  KernelArgs a = kernel_args(op, x, y);
  if (op->schedule == SPMV_SCHEDULE_TILES && free_sms > 0 && a.tile_ctas > 0)
    a.tile_ctas = std::max<int64_t>(1, std::min<int64_t>(a.tile_ctas, a.tile_ctas - (int64_t)free_sms * op->resident));
  return launch_product(op, a, stream);
}
cudaError_t run_operator_with_peers(const spmv_operator* op, const void* x, void* y, void* const* peers, int peer_count,
                                    cudaStream_t stream) {
  if (peer_count < 0 || peer_count > kMaxPeers) return cudaErrorInvalidValue;
  KernelArgs a = kernel_args(op, x, y);
  for (int d = 0; d < peer_count; ++d) a.peers[d] = peers[d];
  a.peer_count = peer_count;
  return launch_product(op, a, stream);
}
}  // namespace spmvb200

extern "C" {

void spmv_operator_config_init(spmv_operator_config* config, int layout, int dtype, int tpr) {
  if (!config) return;
  std::memset(config, 0, sizeof(*config));
  config->layout = layout;
  config->dtype = dtype;
  config->tpr = tpr;
  config->device = -1;
}

int spmv_operator_create(const spmv_csr* matrix, const spmv_operator_config* config, spmv_operator** out) {
  return guarded([&] {
    require(matrix && config && out, "matrix, config and out are required");
    *out = nullptr;
    const Csr& m = matrix->m;
    const int layout = config->layout, dtype = config->dtype, tpr = config->tpr;
    const int value_bytes = value_bytes_of(dtype);
    column_bytes_of(layout);
    require(valid_tpr(tpr), "threads per row must be 2, 4, 8, 16 or 32");
    require(config->physical_tpr == 0 || tile_variant_exists(tpr, config->physical_tpr),
            "physical_tpr must divide T with T / physical_tpr in {1, 2, 4, 8, 16}");
    require(config->tile_nnz == 0 || (config->tile_nnz >= 64 && config->tile_nnz <= 16384),
            "tile_nnz must be 0 or in [64, 16384]");
    require(config->accumulate == SPMV_ACCUMULATE_WIDE || config->accumulate == SPMV_ACCUMULATE_HALF,
            "accumulate must be SPMV_ACCUMULATE_WIDE or SPMV_ACCUMULATE_HALF");
    require(config->accumulate == SPMV_ACCUMULATE_WIDE || dtype == SPMV_F16,
            "SPMV_ACCUMULATE_HALF applies to FP16 values only");
    // the kernel family: FP16 sums in FP16 have their own instantiation
    const int kernel = config->accumulate == SPMV_ACCUMULATE_HALF ? kKernelHalfSums : dtype;
    int device_count = 0;
    if (cudaGetDeviceCount(&device_count) != cudaSuccess || device_count == 0)
      fail(SPMV_ERR_UNSUPPORTED, "no CUDA device");
    DeviceScope scope(config->device);

    // admissibility and byte model need the widest span, and the lp word count at this T
    Facts facts;
    for (int row = 0; row < m.rows; ++row)
      if (m.row_ptr[row + 1] > m.row_ptr[row])
        facts.widest_row_span = std::max(facts.widest_row_span, m.col_ind[m.row_ptr[row + 1] - 1] - m.col_ind[m.row_ptr[row]]);
    // CSR-lp of a large matrix is encoded on the device (encode.cu): the row_ptr and column arrays go up
    // once and the layout (widths, row words, word count) comes from the GPU; smaller ones on the host
    std::unique_ptr<spmv_operator> op(new spmv_operator);
    const bool device_encode = layout == SPMV_LAYOUT_LP && m.nnz() >= kDeviceEncodeNnz;
    DeviceBuffer<int> encode_columns;
    if (device_encode) {
      op->row_ptr = device_upload<int>(m.row_ptr.data(), (size_t)m.rows + 1, op->device_bytes);
      encode_columns.allocate((size_t)m.nnz(), m.col_ind.data());
      op->row_word = device_upload<int>(nullptr, (size_t)m.rows, op->device_bytes);
      op->row_width = device_upload<uint8_t>(nullptr, (size_t)m.rows, op->device_bytes);
      facts.lane_packed_words[tpr_slot(tpr)] =
          device_lane_packed_layout(op->row_ptr, encode_columns.data, m.rows, tpr, op->row_word, op->row_width, nullptr);
    } else if (layout == SPMV_LAYOUT_LP) {
      facts.lane_packed_words[tpr_slot(tpr)] = lane_packed_word_count(m, tpr);
    }
    if (!admissible(m, facts, layout, tpr))
      fail(SPMV_ERR_NOT_ADMISSIBLE, "layout not admissible for this matrix");

    cuda_check(cudaGetDevice(&op->device), "cudaGetDevice");
    op->layout = layout;
    op->dtype = dtype;
    op->kernel = kernel;
    op->accumulate = config->accumulate;
    op->tpr = tpr;
    op->rows = m.rows;
    op->cols = m.cols;
    op->nnz = m.nnz();
    op->memory = memory_of(m, facts, layout, dtype, tpr);
    const double mean_length = m.rows > 0 ? (double)m.nnz() / m.rows : 1.0;
    const double run_length = entries_per_x_sector(m, value_bytes);
    op->physical_tpr = config->physical_tpr > 0 ? config->physical_tpr : choose_physical_tpr(tpr, layout, mean_length);
    op->tile_rows = config->tile_rows > 0 ? config->tile_rows : std::max(128, kTileBlock / op->physical_tpr);
    // long rows of column runs (at least 4 nonzeros per x sector, as in block matrices): one thread per
    // lane up to T = 16 (the dense variant: consecutive lanes read consecutive columns of a run together),
    // else 8 threads a row (not CSR-lp); a tile is at least two passes. Measured on B200 (block-FEM slice,
    // 64 nonzeros a row in runs of 8, FP32, CSR-i32): T = 8 208 us a product (P = 8 dense) against 321 us
    // (P = 8, 2 CTAs an SM) and 0.47 of the peak with P = 4; T = 16 240 us (P = 16) against 321 us (P = 8);
    // T = 32 326 us with P = 8 against 364 us with P = 32.
    const bool column_runs = config->physical_tpr == 0 && config->tile_rows == 0 && run_length >= 4.0 &&
                             mean_length >= 32.0 && tpr >= 8;
    if (column_runs && tpr <= 16) {
      op->physical_tpr = tpr;
      op->tile_rows = std::max(64, 2 * kTileBlock / op->physical_tpr);
    } else if (column_runs && layout != SPMV_LAYOUT_LP) {
      op->physical_tpr = std::max(op->physical_tpr, 8);
      op->tile_rows = 2 * kTileBlock / op->physical_tpr;
    }
    require(op->tile_rows % 16 == 0 && op->tile_rows <= 16384, "tile_rows must be a multiple of 16, at most 16384");
    op->tile_nnz = config->tile_nnz > 0 ? config->tile_nnz : 8192;
    op->stages = config->stages > 0 ? config->stages : 2;
    require(op->stages >= 1 && op->stages <= kMaxStages, "stages must be 0 or 1..4");
    int shared_limit = 0, multiprocessors = 0, per_sm = 0;
    cuda_check(cudaDeviceGetAttribute(&shared_limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, op->device), "device attribute");
    cuda_check(cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, op->device), "device attribute");
    cuda_check(cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, op->device), "device attribute");
    require(config->schedule >= SPMV_SCHEDULE_AUTO && config->schedule <= SPMV_SCHEDULE_CLASSES,
            "schedule must be SPMV_SCHEDULE_AUTO, _TILES or _CLASSES");
    op->schedule = config->schedule != SPMV_SCHEDULE_AUTO ? config->schedule
                                                          : (skewed_rows(m) ? SPMV_SCHEDULE_CLASSES : SPMV_SCHEDULE_TILES);

    // encoded streams
    const size_t nnz = (size_t)m.nnz();
    if (!op->row_ptr) op->row_ptr = device_upload<int>(m.row_ptr.data(), (size_t)m.rows + 1, op->device_bytes);
    {
      std::vector<unsigned char> converted(nnz * value_bytes);
      convert_values(dtype, m.val.data(), (int64_t)nnz, config->value_rounding, converted.data());
      op->values = device_upload<unsigned char>(converted.data(), converted.size(), op->device_bytes);
    }
    std::vector<int> row_word;
    std::vector<uint8_t> row_width;
    switch (layout) {
      case SPMV_LAYOUT_I32:
        op->columns = device_upload<int>(m.col_ind.data(), nnz, op->device_bytes);
        break;
      case SPMV_LAYOUT_I16: case SPMV_LAYOUT_I8: {
        std::vector<unsigned char> narrow(nnz * column_bytes_of(layout));
        encode_absolute(m, column_bytes_of(layout), narrow.data());
        op->columns = device_upload<unsigned char>(narrow.data(), narrow.size(), op->device_bytes);
        break;
      }
      case SPMV_LAYOUT_R16: case SPMV_LAYOUT_R8: {
        std::vector<unsigned char> offsets(nnz * column_bytes_of(layout));
        encode_relative(m, column_bytes_of(layout), offsets.data());
        op->columns = device_upload<unsigned char>(offsets.data(), offsets.size(), op->device_bytes);
        break;
      }
      default: {
        const int64_t word_count = facts.lane_packed_words[tpr_slot(tpr)];
        row_word.resize((size_t)m.rows);
        row_width.resize((size_t)m.rows);
        if (device_encode) {
          op->words = device_upload<uint32_t>(nullptr, (size_t)word_count, op->device_bytes);
          device_lane_packed_pack(op->row_ptr, encode_columns.data, m.rows, tpr, op->row_word, op->row_width, op->words,
                                  word_count, nullptr);
          encode_columns.release();
          cuda_check(cudaMemcpy(row_word.data(), op->row_word, sizeof(int) * row_word.size(), cudaMemcpyDeviceToHost),
                     "row words");
          cuda_check(cudaMemcpy(row_width.data(), op->row_width, row_width.size(), cudaMemcpyDeviceToHost), "row widths");
          break;
        }
        std::vector<uint32_t> words((size_t)word_count);
        encode_lane_packed(m, tpr, word_count, row_word.data(), row_width.data(), words.data());
        op->words = device_upload<uint32_t>(words.data(), words.size(), op->device_bytes);
        op->row_word = device_upload<int>(row_word.data(), row_word.size(), op->device_bytes);
        op->row_width = device_upload<uint8_t>(row_width.data(), row_width.size(), op->device_bytes);
        break;
      }
    }
    if (layout == SPMV_LAYOUT_R16 || layout == SPMV_LAYOUT_R8 || layout == SPMV_LAYOUT_LP) {
      std::vector<int> bases((size_t)m.rows);
      encode_row_base(m, bases.data());
      op->row_base = device_upload<int>(bases.data(), bases.size(), op->device_bytes);
    }

    op->status = device_upload<unsigned>(nullptr, 1, op->device_bytes);
    cuda_check(cudaMemset(op->status, 0, sizeof(unsigned)), "cudaMemset");
    if (op->schedule == SPMV_SCHEDULE_CLASSES) {
      // rows by length; long rows (above 64 T entries) one CTA each, in double-buffered chunks of 2048
      // entries (1024 for FP64) held in shared memory
      const ClassPlan plan = plan_classes(m, tpr, 64 * tpr);
      op->long_count = (int64_t)plan.long_rows.size();
      op->row_items = device_upload<int4>(plan.items.data(), plan.items.size(), op->device_bytes);
      op->long_rows = device_upload<int>(plan.long_rows.data(), plan.long_rows.size(), op->device_bytes);
      // (CSR-lp with 2-byte values: 3584 = 224 * 16, a chunk of exactly one 16-delta segment per gatherer)
      op->long_chunk = value_bytes == 8 ? 1024 : (layout == SPMV_LAYOUT_LP && value_bytes == 2 ? 3584 : 2048);
      op->smem_bytes = op->long_count > 0 ? long_smem_bytes(op->long_chunk, value_bytes) : 0;
      if (layout == SPMV_LAYOUT_LP && op->long_count > 0) upload_lane_marks(op.get(), m, plan.long_rows, tpr);
      int64_t blocks = op->long_count;
      for (int segment = 0; segment < 6; ++segment) {
        const int per_block = kTileBlock >> segment;
        op->segment_first[segment] = plan.segment_first[segment];
        op->segment_items[segment] = plan.segment_items[segment];
        op->segment_blocks[segment] = (plan.segment_items[segment] + per_block - 1) / per_block;
        blocks += op->segment_blocks[segment];
      }
      const int short_rows_per_block = kTileBlock * (dtype == SPMV_F64 ? ShortRowsPerThread<double>::value
                                                                       : ShortRowsPerThread<float>::value);
      op->short_blocks = ((int64_t)m.rows + short_rows_per_block - 1) / short_rows_per_block;
      blocks += op->short_blocks;
      if (blocks > 0x7fffffff)
        fail(SPMV_ERR_TOO_LARGE, "grid exceeds 2^31-1 blocks");
      cuda_check(prepare_classes(kernel, layout, tpr, op->smem_bytes), "class kernel shared memory");
      cuda_check(cudaDeviceSynchronize(), "operator upload");
      *out = op.release();
      return;
    }

    // tile plan. Default tile: at most the nonzeros of tile_rows average rows (+1/8, a multiple of 256, up
    // to 8192; a tile holds at most tile_rows rows), and small enough that the buffers let as many CTAs
    // share a multiprocessor as its registers allow; a CSR-lp buffer holds the longest tile's words, so
    // its size follows the plan.
    const bool packed = layout == SPMV_LAYOUT_LP;
    if (config->tile_nnz == 0) {
      const double row_nnz = (double)op->tile_rows * std::max(1.0, mean_length) * 1.125;
      op->tile_nnz = std::max(256, std::min(8192, ((int)row_nnz + 255) / 256 * 256));
    }
    // the dense variant where one thread holds one lane (P = T) and the gathers come in runs: its x never
    // takes a window, so the shared memory goes to more CTAs per multiprocessor instead
    op->dense = op->physical_tpr == tpr && run_length >= 1.5;
    const int register_ctas = std::max(1, tiles_occupancy(kernel, layout, tpr, op->physical_tpr, 0, op->dense));
    const int budget = per_sm / register_ctas - 1024 - 1024;   // per CTA: minus reserved and static shared memory
    auto plan_for = [&](int tile_nnz) {
      return plan_tiles(m, tile_nnz, op->tile_rows, packed ? row_word.data() : nullptr, packed ? row_width.data() : nullptr);
    };
    auto smem_for = [&](int tile_nnz, const TilePlan* plan, int window_elements) {
      return tile_smem_bytes(tile_nnz, op->tile_rows, value_bytes, layout, op->stages, plan ? plan->index_words : 0,
                             window_elements);
    };
    if (config->tile_nnz == 0 && !packed)
      while (op->tile_nnz > 256 && smem_for(op->tile_nnz, nullptr, 0) > budget) op->tile_nnz -= 256;
    TilePlan plan = plan_for(op->tile_nnz);
    if (config->tile_nnz == 0 && packed)
      while (op->tile_nnz > 256 && smem_for(op->tile_nnz, &plan, 0) > budget) {
        op->tile_nnz -= 256;
        plan = plan_for(op->tile_nnz);
      }
    // windows of x: when the gathers are scattered (under 1.5 nonzeros per x sector a row reads) and most
    // tiles read x within at most 24 KB of columns (a random band), every tile stages that window with its
    // streams and gathers from shared memory; the tiles then shrink to leave room for it. Not for CSR-lp
    // (measured slower: the decode's gathers then choose their source at run time), nor where gathers come
    // in runs (stencils: slower).
    const int window_limit = 24 * 1024 / value_bytes;
    std::vector<int2> windows;
    if (!packed && run_length < 1.5) {
      windows = plan_windows(m, plan, window_limit, value_bytes);
      op->window_elements = window_capacity(windows);
    }
    if (op->window_elements > 0) {
      if (config->tile_nnz == 0)
        while (op->tile_nnz > 256 && smem_for(op->tile_nnz, &plan, op->window_elements) > budget) {
          op->tile_nnz -= 256;
          plan = plan_for(op->tile_nnz);
        }
      windows = plan_windows(m, plan, op->window_elements, value_bytes);
    }
    op->tile_index_words = plan.index_words;
    const int smem = smem_for(op->tile_nnz, &plan, op->window_elements);
    if (smem > shared_limit)
      fail(SPMV_ERR_INVALID_ARGUMENT, "tiles need " + std::to_string(smem) + " bytes of shared memory, above the " +
                                          std::to_string(shared_limit) + " a block may have");
    op->tile_count = (int64_t)plan.tiles.size();
    op->long_count = (int64_t)plan.long_rows.size();
    op->tiles = device_upload<int4>(plan.tiles.data(), plan.tiles.size(), op->device_bytes);
    if (op->window_elements > 0)
      op->tile_windows = device_upload<int2>(windows.data(), windows.size(), op->device_bytes);
    if (layout == SPMV_LAYOUT_LP)
      op->tile_words = device_upload<int2>(plan.tile_words.data(), plan.tile_words.size(), op->device_bytes);
    op->long_rows = device_upload<int>(plan.long_rows.data(), plan.long_rows.size(), op->device_bytes);
    // long rows: one CTA per row at a time; a chunk of a long row (values and gathered x) lives in the
    // CTA's shared memory, at least kTileBlock entries (CSR-lp: and whole lane segments), at most 8192, and
    // the launch gets the larger of the tile buffers and one chunk
    const int chunk_unit = packed ? std::max(kTileBlock, kLaneMarkEvery * tpr) : kTileBlock;
    op->long_chunk = std::max(chunk_unit, std::min(8192, (smem / long_smem_bytes(1, value_bytes)) / chunk_unit * chunk_unit));
    op->smem_bytes = std::max(smem, op->long_count > 0 ? long_smem_bytes(op->long_chunk, value_bytes) : 0);
    if (packed && op->long_count > 0) upload_lane_marks(op.get(), m, plan.long_rows, tpr);
    if (op->smem_bytes > shared_limit) fail(SPMV_ERR_INVALID_ARGUMENT, "long-row chunk exceeds the shared memory of a block");
    // persistent tile CTAs: as many as fit on the device at once, never more than there are tiles
    const int resident = tiles_occupancy(kernel, layout, tpr, op->physical_tpr, op->smem_bytes, op->dense);
    if (resident <= 0 && (op->tile_count > 0 || op->long_count > 0))
      fail(SPMV_ERR_CUDA, "tile kernel cannot be resident with this configuration");
    op->resident = std::max(1, resident);
    op->tile_ctas = std::min<int64_t>(op->tile_count, (int64_t)std::max(1, resident) * multiprocessors);
    op->long_ctas = std::min<int64_t>(op->long_count, (int64_t)std::max(1, resident) * multiprocessors);
    if (op->tile_ctas + op->long_ctas > 0x7fffffff) fail(SPMV_ERR_TOO_LARGE, "grid exceeds 2^31-1 blocks");
    cuda_check(cudaDeviceSynchronize(), "operator upload");
    *out = op.release();
  });
}

int spmv_operator_get_info(const spmv_operator* op, spmv_operator_info* info) {
  return guarded([&] {
    require(op && info, "op and info are required");
    info->rows = op->rows;
    info->cols = op->cols;
    info->nnz = op->nnz;
    info->layout = op->layout;
    info->dtype = op->dtype;
    info->tpr = op->tpr;
    info->physical_tpr = op->physical_tpr;
    info->tile_nnz = op->tile_nnz;
    info->tiles = op->tile_count;
    info->tile_ctas = op->tile_ctas;
    info->stages = op->stages;
    info->tile_rows = op->tile_rows;
    info->long_rows = op->long_count;
    info->device_bytes = op->device_bytes;
    info->memory = op->memory;
    info->schedule = op->schedule;
    info->listed_rows = 0;
    for (int segment = 0; segment < 6; ++segment) info->listed_rows += op->segment_items[segment];
    info->blocks = op->schedule == SPMV_SCHEDULE_CLASSES ? class_blocks(op) : op->long_ctas + op->tile_ctas;
    info->window_elements = op->window_elements;
  });
}

// The tile kernel copies x with 4- or 8-byte asynchronous copies: x must be aligned to its element size,
// and to 4 bytes for FP16.
static void check_vector_alignment(const spmv_operator* op, const void* x, const void* y) {
  const uintptr_t x_alignment = (uintptr_t)std::max(4, value_bytes_of(op->dtype));
  require(((uintptr_t)x % x_alignment) == 0, "x must be aligned to its element size (4 bytes for FP16)");
  require(((uintptr_t)y % (uintptr_t)value_bytes_of(op->dtype)) == 0, "y must be aligned to its element size");
}

int spmv_operator_run(const spmv_operator* op, const void* x, void* y, void* stream) {
  return guarded([&] {
    require(op && x && y, "op, x and y are required");
    check_vector_alignment(op, x, y);
    cuda_check(launch_product(op, kernel_args(op, x, y), static_cast<cudaStream_t>(stream)), "SpMV launch");
  });
}

int spmv_operator_run_host(const spmv_operator* op, const void* x_host, void* y_host, void* x_device, void* y_device,
                           void* stream) {
  return guarded([&] {
    require(op && x_host && y_host && x_device && y_device, "all buffers are required");
    check_vector_alignment(op, x_device, y_device);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t value_bytes = (size_t)value_bytes_of(op->dtype);
    cuda_check(cudaMemcpyAsync(x_device, x_host, value_bytes * op->cols, cudaMemcpyHostToDevice, s), "copy x");
    cuda_check(launch_product(op, kernel_args(op, x_device, y_device), s), "SpMV launch");
    cuda_check(cudaMemcpyAsync(y_host, y_device, value_bytes * op->rows, cudaMemcpyDeviceToHost, s), "copy y");
    cuda_check(cudaStreamSynchronize(s), "stream synchronize");
  });
}

int spmv_operator_run_host_batch(const spmv_operator* op, const void* x_host, int64_t x_stride, void* y_host,
                                 int64_t y_stride, int count, void* x_device, void* y_device, void* stream) {
  return guarded([&] {
    require(op && x_host && y_host && x_device && y_device && count >= 0, "bad arguments");
    const size_t value_bytes = (size_t)value_bytes_of(op->dtype);
    const size_t x_bytes = value_bytes * (size_t)op->cols, y_bytes = value_bytes * (size_t)op->rows;
    // device buffers b = 0, 1: x at x_device + b * x_bytes rounded up to 16 bytes, y likewise
    const size_t x_pitch = (x_bytes + 15) / 16 * 16, y_pitch = (y_bytes + 15) / 16 * 16;
    char* xd = static_cast<char*>(x_device);
    char* yd = static_cast<char*>(y_device);
    check_vector_alignment(op, xd, yd);
    const cudaStream_t copy_in = static_cast<cudaStream_t>(stream);
    cudaStream_t compute = nullptr, copy_out = nullptr;
    cudaEvent_t copied_in[2] = {}, computed[2] = {}, copied_out[2] = {};
    cudaError_t status = cudaStreamCreateWithFlags(&compute, cudaStreamNonBlocking);
    if (status == cudaSuccess) status = cudaStreamCreateWithFlags(&copy_out, cudaStreamNonBlocking);
    for (int b = 0; b < 2 && status == cudaSuccess; ++b) {
      status = cudaEventCreateWithFlags(&copied_in[b], cudaEventDisableTiming);
      if (status == cudaSuccess) status = cudaEventCreateWithFlags(&computed[b], cudaEventDisableTiming);
      if (status == cudaSuccess) status = cudaEventCreateWithFlags(&copied_out[b], cudaEventDisableTiming);
    }
    // vector i uses buffers i mod 2: its copy in waits until the product of vector i - 2 has read x, its
    // product until the copy out of vector i - 2 has read y; the three streams overlap the rest
    for (int i = 0; i < count && status == cudaSuccess; ++i) {
      const int b = i & 1;
      const char* xh = static_cast<const char*>(x_host) + (int64_t)i * x_stride;
      char* yh = static_cast<char*>(y_host) + (int64_t)i * y_stride;
      if (i >= 2) status = cudaStreamWaitEvent(copy_in, computed[b], 0);
      if (status == cudaSuccess) status = cudaMemcpyAsync(xd + b * x_pitch, xh, x_bytes, cudaMemcpyHostToDevice, copy_in);
      if (status == cudaSuccess) status = cudaEventRecord(copied_in[b], copy_in);
      if (status == cudaSuccess) status = cudaStreamWaitEvent(compute, copied_in[b], 0);
      if (status == cudaSuccess && i >= 2) status = cudaStreamWaitEvent(compute, copied_out[b], 0);
      if (status == cudaSuccess) status = launch_product(op, kernel_args(op, xd + b * x_pitch, yd + b * y_pitch), compute);
      if (status == cudaSuccess) status = cudaEventRecord(computed[b], compute);
      if (status == cudaSuccess) status = cudaStreamWaitEvent(copy_out, computed[b], 0);
      if (status == cudaSuccess) status = cudaMemcpyAsync(yh, yd + b * y_pitch, y_bytes, cudaMemcpyDeviceToHost, copy_out);
      if (status == cudaSuccess) status = cudaEventRecord(copied_out[b], copy_out);
    }
    if (status == cudaSuccess && count > 0) status = cudaStreamWaitEvent(copy_in, copied_out[(count - 1) & 1], 0);
    // every stream drains before the call returns, after an error too: no copy into the caller's buffers
    // may still run once it has returned (the first error is the one reported)
    for (cudaStream_t drained : {copy_in, compute, copy_out}) {
      if (!drained) continue;
      const cudaError_t synchronized = cudaStreamSynchronize(drained);
      if (status == cudaSuccess) status = synchronized;
    }
    for (int b = 0; b < 2; ++b)
      for (cudaEvent_t event : {copied_in[b], computed[b], copied_out[b]})
        if (event) cudaEventDestroy(event);
    if (compute) cudaStreamDestroy(compute);
    if (copy_out) cudaStreamDestroy(copy_out);
    cuda_check(status, "batched product through host buffers");
  });
}

int spmv_operator_check(const spmv_operator* op) {
  int timed_out = 0;
  const int status = guarded([&] {
    require(op, "op is required");
    DeviceScope scope(op->device);
    cuda_check(cudaDeviceSynchronize(), "device synchronize");
    unsigned word = 0;
    cuda_check(cudaMemcpy(&word, op->status, sizeof(word), cudaMemcpyDeviceToHost), "read status");
    cuda_check(cudaMemset(op->status, 0, sizeof(unsigned)), "clear status");
    if (word & kStatusTimeout) {
      timed_out = 1;
      set_last_error("a bounded device-side wait gave up");
    }
    if (word & kStatusSmem) fail(SPMV_ERR_CUDA, "a long-row chunk did not fit the launch's shared memory");
  });
  return status != SPMV_OK ? status : (timed_out ? SPMV_ERR_TIMEOUT : SPMV_OK);
}

int spmv_operator_get_arrays(const spmv_operator* op, spmv_operator_arrays* arrays) {
  return guarded([&] {
    require(op && arrays, "op and arrays are required");
    arrays->row_ptr = op->row_ptr;
    arrays->columns = op->columns;
    arrays->row_base = op->row_base;
    arrays->row_word = op->row_word;
    arrays->row_width = op->row_width;
    arrays->words = op->words;
    arrays->values = op->values;
  });
}

void spmv_operator_destroy(spmv_operator* op) { delete op; }

int spmv_launch(int layout, int dtype, int tpr, const spmv_device_matrix* matrix, void* stream) {
  return guarded([&] {
    require(matrix, "matrix is required");
    value_bytes_of(dtype);
    column_bytes_of(layout);
    require(valid_tpr(tpr), "threads per row must be 2, 4, 8, 16 or 32");
    require(matrix->rows >= 0 && matrix->row_ptr && matrix->values && matrix->x && matrix->y, "missing arrays");
    if (layout == SPMV_LAYOUT_LP) require(matrix->row_base && matrix->row_word && matrix->row_width && matrix->words, "missing lp arrays");
    else require(matrix->columns != nullptr, "missing columns");
    if (layout == SPMV_LAYOUT_R16 || layout == SPMV_LAYOUT_R8) require(matrix->row_base != nullptr, "missing row_base");
    KernelArgs a{};
    a.rows = matrix->rows;
    a.cols = matrix->cols;
    a.row_ptr = matrix->row_ptr;
    a.columns = matrix->columns;
    a.row_base = matrix->row_base;
    a.row_word = matrix->row_word;
    a.row_width = matrix->row_width;
    a.words = matrix->words;
    a.values = matrix->values;
    a.x = matrix->x;
    a.y = matrix->y;
    a.row_list = nullptr;
    a.row_count = matrix->rows;
    // one vector of T threads per row, as the reference launches (bench_csr_width.cu:525-526)
    const int64_t blocks = ((int64_t)matrix->rows * tpr + kVectorBlock - 1) / kVectorBlock;
    require(blocks <= 0x7fffffff, "too many rows for one launch");
    cuda_check(launch_vector(dtype, layout, tpr, a, blocks, static_cast<cudaStream_t>(stream)), "SpMV launch");
  });
}

}  // extern "C"

// ---- measured read bandwidth (the roof of the reference's epsilon, roofline.cuh:101) --------------------
namespace spmvb200 {
namespace {

// Every thread streams 16-byte vectors of the buffer with no reuse; the reduction result is kept only to
// stop the loads being dropped.
__global__ void __launch_bounds__(512) k_read_stream(const uint4* __restrict__ source, size_t vectors, unsigned* sink) {
  unsigned accumulator = 0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t index = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
#pragma unroll 4
  for (; index < vectors; index += stride) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(source + index));
    accumulator ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  if (accumulator == 0x9e3779b9u) *sink = accumulator;   // practically never: keeps the loads alive
}

// Random gathers: every thread reads 16 elements at hashed positions (an integer mix, in bounds by the
// power-of-two mask) and folds them into a hash only to stop the loads being dropped.
__device__ __forceinline__ uint32_t gather_position(uint32_t value) {
  value ^= value >> 16;
  value *= 0x7feb352du;
  value ^= value >> 15;
  value *= 0x846ca68bu;
  return value ^ (value >> 16);
}

template <class E>
__global__ void __launch_bounds__(256) k_gather_random(const E* __restrict__ source, uint32_t mask, uint32_t seed, unsigned* sink) {
  const uint32_t thread = blockIdx.x * blockDim.x + threadIdx.x;
  E values[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) values[k] = __ldg(source + (gather_position(thread * 16 + k + seed) & mask));
  unsigned folded = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) folded = folded * 0x01000193u ^ (unsigned)values[k];   // can take any value
  if (folded == 0x9e3779b9u) *sink = folded;   // practically never: keeps the loads alive
}

}  // namespace
}  // namespace spmvb200


extern "C" int spmv_gather_rate(int64_t elements, int value_bytes, int reps, double* elements_per_second) {
  return guarded([&] {
    require(elements_per_second && reps >= 1 && elements >= 1024 && elements <= (1LL << 31) &&
                (value_bytes == 2 || value_bytes == 4 || value_bytes == 8),
            "bad arguments");
    int64_t size = 1;
    while (size * 2 <= elements) size *= 2;   // a power of two, so that the mask keeps positions in bounds
    void* buffer = nullptr;
    unsigned* sink = nullptr;
    cuda_check(cudaMalloc(&buffer, (size_t)size * value_bytes), "cudaMalloc");
    cudaError_t status = cudaMalloc(&sink, sizeof(unsigned));
    if (status == cudaSuccess) status = cudaMemset(buffer, 1, (size_t)size * value_bytes);
    int multiprocessors = 0, device = 0;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device);
    const unsigned blocks = (unsigned)multiprocessors * 8 * 32;
    const uint32_t mask = (uint32_t)(size - 1);
    cudaEvent_t start = nullptr, end = nullptr;
    std::vector<float> times;
    if (status == cudaSuccess) status = cudaEventCreate(&start);
    if (status == cudaSuccess) status = cudaEventCreate(&end);
    for (int rep = -3; rep < reps && status == cudaSuccess; ++rep) {
      const uint32_t seed = (uint32_t)(rep + 3) * 0x9e3779b9u;
      cudaEventRecord(start);
      if (value_bytes == 2) k_gather_random<unsigned short><<<blocks, 256>>>(static_cast<unsigned short*>(buffer), mask, seed, sink);
      else if (value_bytes == 4) k_gather_random<unsigned><<<blocks, 256>>>(static_cast<unsigned*>(buffer), mask, seed, sink);
      else k_gather_random<unsigned long long><<<blocks, 256>>>(static_cast<unsigned long long*>(buffer), mask, seed, sink);
      cudaEventRecord(end);
      status = cudaGetLastError();
      if (status == cudaSuccess) status = cudaEventSynchronize(end);
      float ms = 0.0f;
      if (status == cudaSuccess) status = cudaEventElapsedTime(&ms, start, end);
      if (rep >= 0) times.push_back(ms);
    }
    if (start) cudaEventDestroy(start);
    if (end) cudaEventDestroy(end);
    cudaFree(buffer);
    if (sink) cudaFree(sink);
    cuda_check(status, "gather rate");
    std::sort(times.begin(), times.end());
    const double median = times[times.size() / 2];
    *elements_per_second = (double)blocks * 256.0 * 16.0 / (median * 1e-3);
  });
}

extern "C" int spmv_read_bandwidth(int64_t bytes, int reps, double* gigabytes_per_second) {
  return guarded([&] {
    require(gigabytes_per_second && reps >= 1 && bytes >= (1 << 20), "bad arguments");
    const size_t vectors = (size_t)bytes / sizeof(uint4);
    uint4* buffer = nullptr;
    unsigned* sink = nullptr;
    cuda_check(cudaMalloc(&buffer, vectors * sizeof(uint4)), "cudaMalloc");
    cudaError_t status = cudaMalloc(&sink, sizeof(unsigned));
    if (status == cudaSuccess) status = cudaMemset(buffer, 1, vectors * sizeof(uint4));
    int multiprocessors = 0, device = 0;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&multiprocessors, cudaDevAttrMultiProcessorCount, device);
    const unsigned blocks = (unsigned)multiprocessors * 4;
    cudaEvent_t start = nullptr, end = nullptr;
    std::vector<float> times;
    if (status == cudaSuccess) status = cudaEventCreate(&start);
    if (status == cudaSuccess) status = cudaEventCreate(&end);
    for (int rep = -3; rep < reps && status == cudaSuccess; ++rep) {
      cudaEventRecord(start);
      k_read_stream<<<blocks, 512>>>(buffer, vectors, sink);
      cudaEventRecord(end);
      status = cudaGetLastError();
      if (status == cudaSuccess) status = cudaEventSynchronize(end);
      float ms = 0.0f;
      if (status == cudaSuccess) status = cudaEventElapsedTime(&ms, start, end);
      if (rep >= 0) times.push_back(ms);
    }
    if (start) cudaEventDestroy(start);
    if (end) cudaEventDestroy(end);
    cudaFree(buffer);
    if (sink) cudaFree(sink);
    cuda_check(status, "read bandwidth");
    std::sort(times.begin(), times.end());
    const double median = times[times.size() / 2];
    *gigabytes_per_second = (double)(vectors * sizeof(uint4)) / (median * 1e-3) / 1e9;
  });
}
