// spmv_bench.cpp — the benchmark program of the study, on libspmvb200: the same command line, the same
// measurement protocol and the same CSV files as src/bench_csr_width.cu (main :1317, run_precision
// :1140), so its campaign scripts and analysis (analysis/compare_campaign.py) run on its output unchanged.
//
//   spmv_bench --matrix A.mtx [--matrix B.mtx ...] [--reps 30] [--warmup 10] [--ordering original|rcm]
//              [--min-sample-ms 0] [--tpr-csv FILE] [--csv FILE] [--precision all|fp64|fp32|fp16]
//              [--accumulate wide|half] [--r16-control lane|pair|wide|unroll16]
//
// Per matrix and precision: every layout (i32, i16, i8, r16, r8, lp) at every threads per row T; every
// result checked against CSR-i32 of the same precision at the same T (it must be bit-identical, so
// max_abs_diff = 0); cuSPARSE CSR_ALG1 and CSR_ALG2 on the same int32 arrays, checked by max |dy| against
// CSR-i32 at T = 8. Times: warm-ups, then `reps` samples of a batch of back-to-back products lasting at
// least min_sample_ms, median per product (bench_csr_width.cu:631-663). The schema of both CSV files is
// the reference's (ResultRow, :99-125, and append_thread_samples, :990-1005).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cusparse.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <functional>
#include <map>
#include <string>
#include <vector>

#include "spmvb200.h"

namespace {

struct Args {
  std::vector<std::string> matrices;
  std::string csv = "results/csr_width.csv";
  std::string tpr_csv;
  std::string ordering = "original";
  std::string precision = "all";
  // "half": FP16 values summed in FP16, FP16 only (the reference's bench_csr_width_fp16acc build)
  std::string accumulate = "wide";
  std::string r16_control;   // "", lane, pair, wide or unroll16: the reference's control builds of CSR-r16
  int reps = 30;
  int warmup = 10;
  double min_sample_ms = 0.0;
};

[[noreturn]] void die(const std::string& message) {
  std::fprintf(stderr, "spmv_bench: %s\n", message.c_str());
  std::exit(1);
}

void check(int status, const char* what) {
  if (status != SPMV_OK) die(std::string(what) + ": " + spmv_status_string(status) + ": " + spmv_last_error());
}

void cuda(cudaError_t status, const char* what) {
  if (status != cudaSuccess) die(std::string(what) + ": " + cudaGetErrorString(status));
}

struct Row {   // ResultRow (bench_csr_width.cu:99)
  std::string matrix, precision, encoding = "cumulative", column_mode, status = "ok", kernel = "custom", ordering;
  int value_bytes = 0, column_bytes = 0, length_bytes = 4, rows = 0, cols = 0, best_tpr = 0, batch = 1;
  long long nnz = 0;
  spmv_memory memory{};
  double time_ms = 0, gflops = 0, bw_gbs = 0, epsilon = 0, speedup_measured = 0, speedup_predicted = 0;
  double max_abs_diff = 0, workspace_bytes = 0, max_rel_diff = 0;

  static const char* header() {
    return "matrix,prec,row_encoding,value_bytes,column_bytes,length_bytes,status,rows,cols,nnz,"
           "bytes_values,bytes_columns,bytes_row_pointer,bytes_vectors,bytes_total,bytes_per_nnz,"
           "best_tpr,t_ms,gflops,bw_gbs,epsilon,speedup_meas,speedup_pred,max_abs_diff,column_mode,bytes_column_bases,"
           "kernel,bytes_workspace,max_rel_diff,ordering,batch";
  }
  std::string csv() const {
    char line[1024];
    std::snprintf(line, sizeof(line),
                  "%s,%s,%s,%d,%d,%d,%s,%d,%d,%lld,%.0f,%.0f,%.0f,%.0f,%.0f,%.4f,%d,%.6f,%.3f,%.2f,%.4f,%.4f,%.4f,%.3e,%s,"
                  "%.0f,%s,%.0f,%.3e,%s,%d",
                  matrix.c_str(), precision.c_str(), encoding.c_str(), value_bytes, column_bytes, length_bytes,
                  status.c_str(), rows, cols, nnz, memory.values, memory.columns, memory.row_pointer, memory.vectors,
                  memory.total, memory.total / (double)std::max(nnz, 1LL), best_tpr, time_ms, gflops, bw_gbs, epsilon,
                  speedup_measured, speedup_predicted, max_abs_diff, column_mode.c_str(), memory.column_bases,
                  kernel.c_str(), workspace_bytes, max_rel_diff, ordering.c_str(), batch);
    return line;
  }
};

void append(const std::string& path, const std::string& header, const std::string& line) {
  std::ifstream probe(path);
  const bool empty = !probe.good() || probe.peek() == std::ifstream::traits_type::eof();
  std::ofstream out(path, std::ios::app);
  if (!out) return;
  if (empty) out << header << "\n";
  out << line << "\n";
}

// CUDA-event timing on one stream (EventTimer, include/common.cuh:164).
struct Timer {
  cudaEvent_t begin{}, end{};
  cudaStream_t stream;
  explicit Timer(cudaStream_t s) : stream(s) {
    cuda(cudaEventCreate(&begin), "event");
    cuda(cudaEventCreate(&end), "event");
  }
  ~Timer() {
    cudaEventDestroy(begin);
    cudaEventDestroy(end);
  }
  double time(const std::function<void()>& run, int repeats) {
    cuda(cudaEventRecord(begin, stream), "event record");
    for (int i = 0; i < repeats; ++i) run();
    cuda(cudaEventRecord(end, stream), "event record");
    cuda(cudaEventSynchronize(end), "event sync");
    float ms = 0;
    cuda(cudaEventElapsedTime(&ms, begin, end), "elapsed");
    return ms;
  }
};

// batch_for + batched_median_ms (bench_csr_width.cu:635-663).
double median_ms(const std::function<void()>& run, const Args& args, cudaStream_t stream, int& batch) {
  Timer timer(stream);
  for (int i = 0; i < args.warmup; ++i) run();
  cuda(cudaStreamSynchronize(stream), "warm-up");
  batch = 1;
  if (args.min_sample_ms > 0) {
    double sample = 0;
    for (;;) {
      sample = timer.time(run, batch);
      if (sample >= 0.25 * args.min_sample_ms || batch >= (1 << 20)) break;
      batch *= 4;
    }
    batch = (int)std::min<double>(1 << 20, std::max(1.0, std::ceil(batch * args.min_sample_ms / std::max(sample, 1e-3))));
  }
  std::vector<double> samples;
  for (int rep = 0; rep < args.reps; ++rep) samples.push_back(timer.time(run, batch));
  std::sort(samples.begin(), samples.end());
  const size_t n = samples.size();
  const double median = (n % 2) ? samples[n / 2] : 0.5 * (samples[n / 2 - 1] + samples[n / 2]);
  return median / batch;
}

double widen(const void* data, int dtype, size_t index) {
  if (dtype == SPMV_F64) return static_cast<const double*>(data)[index];
  if (dtype == SPMV_F32) return static_cast<const float*>(data)[index];
  return (double)(float)static_cast<const _Float16*>(data)[index];
}

const char* precision_name(int dtype) { return dtype == SPMV_F64 ? "fp64" : (dtype == SPMV_F32 ? "fp32" : "fp16"); }
int value_bytes_of(int dtype) { return dtype == SPMV_F64 ? 8 : (dtype == SPMV_F32 ? 4 : 2); }

struct Layout {
  int code;
  const char* mode;
  int column_bytes;
  const char* label;
};
const Layout kLayouts[] = {{SPMV_LAYOUT_I32, "absolute", 4, "i32"}, {SPMV_LAYOUT_I16, "absolute", 2, "i16"},
                           {SPMV_LAYOUT_I8, "absolute", 1, "i8"},   {SPMV_LAYOUT_R16, "row-base", 2, "r16"},
                           {SPMV_LAYOUT_R8, "row-base", 1, "r8"},   {SPMV_LAYOUT_LP, "lane-packed", 0, "lp"}};
const int kThreadsPerRow[] = {2, 4, 8, 16, 32};

struct Vectors {
  void* x = nullptr;
  void* y = nullptr;
  size_t rows = 0;
  int dtype = 0;
  std::vector<double> read(cudaStream_t stream) const {
    std::vector<unsigned char> host(rows * value_bytes_of(dtype));
    cuda(cudaStreamSynchronize(stream), "sync");
    cuda(cudaMemcpy(host.data(), y, host.size(), cudaMemcpyDeviceToHost), "copy y");
    std::vector<double> out(rows);
    for (size_t i = 0; i < rows; ++i) out[i] = widen(host.data(), dtype, i);
    return out;
  }
};

double max_difference(const std::vector<double>& a, const std::vector<double>& b) {
  double largest = 0;
  for (size_t i = 0; i < a.size(); ++i) largest = std::max(largest, std::fabs(a[i] - b[i]));
  return largest;
}

void run_cusparse(cusparseHandle_t handle, cusparseSpMVAlg_t algorithm, const spmv_operator* i32, const Vectors& v,
                  const std::vector<double>& reference_y, double reference_scale, Row row, double baseline_ms,
                  double read_bandwidth, const Args& args, cudaStream_t stream) {
  spmv_operator_arrays arrays;
  spmv_operator_info info;
  check(spmv_operator_get_arrays(i32, &arrays), "arrays");
  check(spmv_operator_get_info(i32, &info), "info");
  const cudaDataType value_type = v.dtype == SPMV_F64 ? CUDA_R_64F : (v.dtype == SPMV_F32 ? CUDA_R_32F : CUDA_R_16F);
  const cudaDataType compute = v.dtype == SPMV_F16 ? CUDA_R_32F : value_type;   // FP16 computed in FP32 (:1066)
  const double alpha64 = 1.0, beta64 = 0.0;
  const float alpha32 = 1.0f, beta32 = 0.0f;
  const void* alpha = v.dtype == SPMV_F64 ? (const void*)&alpha64 : (const void*)&alpha32;
  const void* beta = v.dtype == SPMV_F64 ? (const void*)&beta64 : (const void*)&beta32;
  cusparseSpMatDescr_t matrix = nullptr;
  cusparseDnVecDescr_t x = nullptr, y = nullptr;
  size_t workspace = 0;
  void* buffer = nullptr;
  cusparseSetStream(handle, stream);
  cusparseCreateCsr(&matrix, info.rows, info.cols, info.nnz, (void*)arrays.row_ptr, (void*)arrays.columns,
                    (void*)arrays.values, CUSPARSE_INDEX_32I, CUSPARSE_INDEX_32I, CUSPARSE_INDEX_BASE_ZERO, value_type);
  cusparseCreateDnVec(&x, info.cols, v.x, value_type);
  cusparseCreateDnVec(&y, info.rows, v.y, value_type);
  row.kernel = algorithm == CUSPARSE_SPMV_CSR_ALG1 ? "cusparse_csr_alg1" : "cusparse_csr_alg2";
  cusparseStatus_t status = cusparseSpMV_bufferSize(handle, CUSPARSE_OPERATION_NON_TRANSPOSE, alpha, matrix, x, beta, y,
                                                    compute, algorithm, &workspace);
  cudaError_t allocated = cudaSuccess;
  if (status == CUSPARSE_STATUS_SUCCESS && workspace > 0) allocated = cudaMalloc(&buffer, workspace);
  if (status == CUSPARSE_STATUS_SUCCESS && allocated == cudaSuccess)
    status = cusparseSpMV_preprocess(handle, CUSPARSE_OPERATION_NON_TRANSPOSE, alpha, matrix, x, beta, y, compute,
                                     algorithm, buffer);
  auto multiply = [&] {
    cusparseSpMV(handle, CUSPARSE_OPERATION_NON_TRANSPOSE, alpha, matrix, x, beta, y, compute, algorithm, buffer);
  };
  if (status == CUSPARSE_STATUS_SUCCESS && allocated == cudaSuccess)
    status = cusparseSpMV(handle, CUSPARSE_OPERATION_NON_TRANSPOSE, alpha, matrix, x, beta, y, compute, algorithm, buffer);
  row.workspace_bytes = (double)workspace;
  if (status != CUSPARSE_STATUS_SUCCESS || allocated != cudaSuccess) {
    row.status = allocated != cudaSuccess ? "workspace allocation failed" : cusparseGetErrorString(status);
  } else {
    row.max_abs_diff = max_difference(v.read(stream), reference_y);
    row.max_rel_diff = reference_scale > 0 ? row.max_abs_diff / reference_scale : row.max_abs_diff;
    row.time_ms = median_ms(multiply, args, stream, row.batch);
    row.gflops = 2.0 * row.nnz / (row.time_ms * 1e-3) / 1e9;
    row.bw_gbs = row.memory.total / (row.time_ms * 1e-3) / 1e9;
    row.epsilon = row.bw_gbs / read_bandwidth;
    row.speedup_measured = baseline_ms / row.time_ms;
    row.speedup_predicted = 1.0;
  }
  std::printf("  %-4s %-21s %8.3f ms %8.2f GFLOP/s max rel |dy| %.1e  %s\n", row.precision.c_str(), row.kernel.c_str(),
              row.time_ms, row.gflops, row.max_rel_diff, row.status.c_str());
  append(args.csv, Row::header(), row.csv());
  if (buffer) cudaFree(buffer);
  cusparseDestroyDnVec(x);
  cusparseDestroyDnVec(y);
  cusparseDestroySpMat(matrix);
}

// The control build of CSR-r16 named by --r16-control (0: none).
int r16_control_code(const std::string& name) {
  if (name == "lane") return SPMV_R16_CONTROL_LANE;
  if (name == "pair") return SPMV_R16_CONTROL_PAIR;
  if (name == "wide") return SPMV_R16_CONTROL_WIDE;
  if (name == "unroll16") return SPMV_R16_CONTROL_UNROLL16;
  return 0;
}

void run_precision(spmv_csr* matrix, const std::string& name, int dtype, const Args& args, double read_bandwidth,
                   cusparseHandle_t sparse, cudaStream_t stream) {
  spmv_csr_info info;
  check(spmv_csr_get_info(matrix, &info), "info");
  spmv_facts facts;
  check(spmv_matrix_facts(matrix, &facts), "facts");
  const int value_bytes = value_bytes_of(dtype);
  Vectors v;
  v.rows = (size_t)info.rows;
  v.dtype = dtype;
  std::vector<unsigned char> x_host((size_t)info.cols * value_bytes);
  check(spmv_fill_reference_x(dtype, info.cols, x_host.data()), "x");
  cuda(cudaMalloc(&v.x, std::max<size_t>(x_host.size(), 16)), "cudaMalloc x");
  cuda(cudaMalloc(&v.y, std::max<size_t>((size_t)info.rows * value_bytes, 16)), "cudaMalloc y");
  cuda(cudaMemcpy(v.x, x_host.data(), x_host.size(), cudaMemcpyHostToDevice), "copy x");

  // CSR-i32 at every T: the reference results every layout must equal (max_difference_at, :709)
  std::map<int, std::vector<double>> i32_at;
  spmv_operator* i32_t8 = nullptr;
  for (int tpr : kThreadsPerRow) {
    spmv_operator_config config;
    spmv_operator_config_init(&config, SPMV_LAYOUT_I32, dtype, tpr);
    if (args.accumulate == "half") config.accumulate = SPMV_ACCUMULATE_HALF;
    spmv_operator* op = nullptr;
    check(spmv_operator_create(matrix, &config, &op), "operator");
    check(spmv_operator_run(op, v.x, v.y, stream), "run");
    i32_at[tpr] = v.read(stream);
    if (tpr == 8) i32_t8 = op;
    else spmv_operator_destroy(op);
  }
  const std::vector<double>& reference_y = i32_at[8];
  double reference_scale = 0;
  for (double value : reference_y) reference_scale = std::max(reference_scale, std::fabs(value));
  spmv_memory baseline_memory;
  check(spmv_memory_of(matrix, &facts, SPMV_LAYOUT_I32, dtype, 8, &baseline_memory), "memory_of");
  double baseline_ms = 0;
  Row baseline_row;

  for (const Layout& layout : kLayouts) {
    Row row;
    row.matrix = name;
    row.ordering = args.ordering;
    row.precision = precision_name(dtype);
    row.column_mode = layout.mode;
    row.value_bytes = value_bytes;
    row.column_bytes = layout.column_bytes;
    row.rows = info.rows;
    row.cols = info.cols;
    row.nnz = (long long)info.nnz;
    struct Sample {
      int tpr, batch;
      double ms, bytes, diff;
    };
    std::vector<Sample> samples;
    double best_ms = 1e30;
    int best_tpr = 0, best_batch = 1;
    for (int tpr : kThreadsPerRow) {
      int admissible = 0;
      check(spmv_admissible(matrix, &facts, layout.code, tpr, &admissible), "admissible");
      if (!admissible) continue;
      spmv_operator_config config;
      spmv_operator_config_init(&config, layout.code, dtype, tpr);
      if (args.accumulate == "half") config.accumulate = SPMV_ACCUMULATE_HALF;
      spmv_operator* op = nullptr;
      check(spmv_operator_create(matrix, &config, &op), "operator");
      spmv_memory memory;
      check(spmv_memory_of(matrix, &facts, layout.code, dtype, tpr, &memory), "memory_of");
      // a control build of CSR-r16: the control's kernel on the operator's row_ptr, row_base and values and the
      // control's offsets (bench_csr_width.cu:615-620); WIDE counts 4 bytes an offset (memory_of, :270)
      const int control = layout.code == SPMV_LAYOUT_R16 ? r16_control_code(args.r16_control) : 0;
      void* control_offsets = nullptr;
      spmv_device_matrix device{};
      if (control) {
        spmv_operator_arrays arrays;
        check(spmv_operator_get_arrays(op, &arrays), "arrays");
        device.rows = info.rows;
        device.cols = info.cols;
        device.nnz = info.nnz;
        device.row_ptr = arrays.row_ptr;
        device.row_base = arrays.row_base;
        device.values = arrays.values;
        device.x = v.x;
        device.y = v.y;
        device.columns = arrays.columns;
        if (control != SPMV_R16_CONTROL_UNROLL16) {
          const bool wide = control == SPMV_R16_CONTROL_WIDE;
          const size_t count = wide ? (size_t)info.nnz : (size_t)((info.nnz + 1) / 2 * 2);
          std::vector<unsigned char> host(std::max<size_t>(count * (wide ? 4 : 2), 4));
          if (wide) check(spmv_encode_relative(matrix, 4, host.data()), "wide offsets");
          else check(spmv_encode_relative_lane(matrix, tpr, reinterpret_cast<uint16_t*>(host.data())), "lane offsets");
          cuda(cudaMalloc(&control_offsets, host.size()), "cudaMalloc offsets");
          cuda(cudaMemcpy(control_offsets, host.data(), host.size(), cudaMemcpyHostToDevice), "copy offsets");
          device.columns = control_offsets;
          if (wide) {
            memory.total += (double)info.nnz * 2;
            memory.columns = (double)info.nnz * 4;
          }
        }
      }
      auto product = [&] {
        return control ? spmv_launch_r16_control(control, dtype, tpr, &device, stream) : spmv_operator_run(op, v.x, v.y, stream);
      };
      check(product(), "run");
      const double diff = max_difference(v.read(stream), i32_at[tpr]);
      int batch = 1;
      const double ms = median_ms(product, args, stream, batch);
      check(spmv_operator_check(op), "device status");
      if (control_offsets) cudaFree(control_offsets);
      spmv_operator_destroy(op);
      samples.push_back({tpr, batch, ms, memory.total, diff});
      if (ms < best_ms) { best_ms = ms; best_tpr = tpr; best_batch = batch; }
    }
    check(spmv_memory_of(matrix, &facts, layout.code, dtype, best_tpr > 0 ? best_tpr : 8, &row.memory), "memory_of");
    if (layout.code == SPMV_LAYOUT_R16 && r16_control_code(args.r16_control) == SPMV_R16_CONTROL_WIDE) {
      row.memory.total += (double)info.nnz * 2;
      row.memory.columns = (double)info.nnz * 4;
    }
    if (samples.empty()) {
      row.status = "not admissible";
      append(args.csv, Row::header(), row.csv());
      continue;
    }
    // the check of the row: CSR-lp at the T it was built for, the others at T = 8 (:1205)
    for (const Sample& sample : samples)
      if (sample.tpr == (layout.code == SPMV_LAYOUT_LP ? best_tpr : 8)) row.max_abs_diff = sample.diff;
    row.max_rel_diff = reference_scale > 0 ? row.max_abs_diff / reference_scale : row.max_abs_diff;
    row.time_ms = best_ms;
    row.best_tpr = best_tpr;
    row.batch = best_batch;
    if (layout.code == SPMV_LAYOUT_I32) { baseline_ms = best_ms; baseline_row = row; }
    row.gflops = 2.0 * info.nnz / (row.time_ms * 1e-3) / 1e9;
    row.bw_gbs = row.memory.total / (row.time_ms * 1e-3) / 1e9;
    row.epsilon = row.bw_gbs / read_bandwidth;
    row.speedup_measured = baseline_ms / row.time_ms;
    row.speedup_predicted = baseline_memory.total / row.memory.total;
    std::printf("  %-4s %-10s %-3s T=%2d %8.4f ms %8.2f GFLOP/s %8.1f GB/s eps %.3f pred %.3f meas %.3f max|dy| %.1e\n",
                row.precision.c_str(), row.encoding.c_str(), layout.label, row.best_tpr, row.time_ms, row.gflops,
                row.bw_gbs, row.epsilon, row.speedup_predicted, row.speedup_measured, row.max_abs_diff);
    append(args.csv, Row::header(), row.csv());
    if (!args.tpr_csv.empty())
      for (const Sample& sample : samples) {
        char line[512];
        std::snprintf(line, sizeof(line), "%s,%s,%s,%s,%d,%.6f,%d,%.0f,%lld,%.3e", row.matrix.c_str(), row.ordering.c_str(),
                      row.precision.c_str(), layout.label, sample.tpr, sample.ms, sample.batch, sample.bytes, row.nnz, sample.diff);
        append(args.tpr_csv, "matrix,ordering,prec,layout,tpr,t_ms,batch,bytes_total,nnz,max_abs_diff", line);
      }
  }
  baseline_row.best_tpr = 0;
  baseline_row.time_ms = 0;
  run_cusparse(sparse, CUSPARSE_SPMV_CSR_ALG1, i32_t8, v, reference_y, reference_scale, baseline_row, baseline_ms,
               read_bandwidth, args, stream);
  run_cusparse(sparse, CUSPARSE_SPMV_CSR_ALG2, i32_t8, v, reference_y, reference_scale, baseline_row, baseline_ms,
               read_bandwidth, args, stream);
  spmv_operator_destroy(i32_t8);
  cudaFree(v.x);
  cudaFree(v.y);
}

// print_memory_table (bench_csr_width.cu:1033): the byte model of every layout but lp, in MiB.
void print_memory_table(const spmv_csr* matrix, const spmv_facts& facts, int64_t nnz) {
  const double mebibyte = 1048576.0;
  std::printf("  memory occupancy (MiB)  %-4s %-3s %9s %9s %9s %9s %9s %9s %7s\n", "prec", "col", "values", "columns",
              "bases", "row ptr", "vectors", "total", "B/nnz");
  for (int dtype : {SPMV_F64, SPMV_F32, SPMV_F16})
    for (const Layout& layout : kLayouts) {
      if (layout.code == SPMV_LAYOUT_LP) continue;
      spmv_memory memory;
      int admissible = 0;
      check(spmv_memory_of(matrix, &facts, layout.code, dtype, 8, &memory), "memory_of");
      check(spmv_admissible(matrix, &facts, layout.code, 8, &admissible), "admissible");
      std::printf("                          %-4s %-3s %9.1f %9.1f %9.2f %9.2f %9.1f %9.1f %7.3f %s\n",
                  precision_name(dtype), layout.label, memory.values / mebibyte, memory.columns / mebibyte,
                  memory.column_bases / mebibyte, memory.row_pointer / mebibyte, memory.vectors / mebibyte,
                  memory.total / mebibyte, memory.total / (double)nnz,
                  admissible ? "" : (layout.column_bytes && std::string(layout.mode) == "absolute"
                                         ? "(not admissible: n too large)"
                                         : "(not admissible: a row spans too many columns)"));
    }
}

Args parse(int argc, char** argv) {
  Args args;
  for (int i = 1; i < argc; ++i) {
    const std::string option = argv[i];
    if (option == "--help" || i + 1 >= argc) {
      std::printf("usage: spmv_bench --matrix A.mtx [--matrix B.mtx ...] [--reps 30] [--warmup 10] "
                  "[--ordering original|rcm] [--min-sample-ms 0] [--tpr-csv FILE] [--csv FILE] "
                  "[--precision all|fp64|fp32|fp16] [--accumulate wide|half] [--r16-control lane|pair|wide|unroll16]\n");
      std::exit(option == "--help" ? 0 : 1);
    }
    const std::string value = argv[++i];
    if (option == "--matrix") args.matrices.push_back(value);
    else if (option == "--csv") args.csv = value;
    else if (option == "--reps") args.reps = std::stoi(value);
    else if (option == "--warmup") args.warmup = std::stoi(value);
    else if (option == "--ordering") args.ordering = value;
    else if (option == "--min-sample-ms") args.min_sample_ms = std::stod(value);
    else if (option == "--tpr-csv") args.tpr_csv = value;
    else if (option == "--precision") args.precision = value;
    else if (option == "--accumulate") args.accumulate = value;
    else if (option == "--r16-control") args.r16_control = value;
    else die("unknown option " + option);
  }
  if (args.matrices.empty()) die("at least one --matrix is required");
  if (args.ordering != "original" && args.ordering != "rcm") die("--ordering must be original or rcm");
  if (args.precision != "all" && args.precision != "fp64" && args.precision != "fp32" && args.precision != "fp16")
    die("--precision must be all, fp64, fp32 or fp16");
  if (args.accumulate != "wide" && args.accumulate != "half") die("--accumulate must be wide or half");
  if (!args.r16_control.empty() && r16_control_code(args.r16_control) == 0)
    die("--r16-control must be lane, pair, wide or unroll16");
  if (!args.r16_control.empty() && args.accumulate == "half") die("--r16-control runs with --accumulate wide");
  return args;
}

}  // namespace

int main(int argc, char** argv) {
  const Args args = parse(argc, argv);
  cudaStream_t stream;
  cuda(cudaStreamCreate(&stream), "stream");
  cusparseHandle_t sparse = nullptr;
  if (cusparseCreate(&sparse) != CUSPARSE_STATUS_SUCCESS) die("cusparseCreate failed");
  double read_bandwidth = 0;
  check(spmv_read_bandwidth(4LL << 30, 20, &read_bandwidth), "read bandwidth");
  cudaDeviceProp properties;
  cuda(cudaGetDeviceProperties(&properties, 0), "properties");
  std::printf("device %s (cc %d.%d), read bandwidth %.1f GB/s, L2 %.1f MiB\n", properties.name, properties.major,
              properties.minor, read_bandwidth, properties.l2CacheSize / 1048576.0);
  for (const std::string& path : args.matrices) {
    spmv_csr* matrix = nullptr;
    if (spmv_csr_read_matrix_market(path.c_str(), &matrix) != SPMV_OK) {
      std::fprintf(stderr, "[skip] %s\n", spmv_last_error());
      continue;
    }
    std::string name = spmv_csr_name(matrix);
    if (args.ordering == "rcm") {
      spmv_csr* reordered = nullptr;
      double seconds = 0;
      if (spmv_csr_reorder_rcm(path.c_str(), matrix, &reordered, &seconds) != SPMV_OK) {
        std::fprintf(stderr, "[skip] %s\n", spmv_last_error());
        spmv_csr_destroy(matrix);
        continue;
      }
      spmv_csr_destroy(matrix);
      matrix = reordered;
      std::printf("  ordering: rcm, symmetric permutation P A P^T (ordering computed in %.2f s)\n", seconds);
    }
    spmv_csr_info info;
    check(spmv_csr_get_info(matrix, &info), "info");
    std::printf("\n=== %s: m=%d n=%d nnz=%lld, %.1f nnz/row (max %d) ===\n", name.c_str(), info.rows, info.cols,
                (long long)info.nnz, info.nnz_per_row_mean, info.nnz_per_row_max);
    spmv_facts facts;
    check(spmv_matrix_facts(matrix, &facts), "facts");
    std::printf("  widest row span %d columns\n", facts.widest_row_span);
    print_memory_table(matrix, facts, info.nnz);
    std::printf("  %-4s %-10s %-3s %-4s %8s %8s %8s %8s %5s %6s %6s %9s\n", "prec", "row ptr", "col", "tpr", "t[ms]",
                "GFLOP/s", "GB/s", "", "eps", "pred", "meas", "max|dy|");
    for (int dtype : {SPMV_F64, SPMV_F32, SPMV_F16})
      if ((args.precision == "all" || args.precision == precision_name(dtype)) &&
          (args.accumulate == "wide" || dtype == SPMV_F16))   // FP16 sums: the FP16 products only
        run_precision(matrix, name, dtype, args, read_bandwidth, sparse, stream);
    spmv_csr_destroy(matrix);
  }
  cusparseDestroy(sparse);
  cudaStreamDestroy(stream);
  std::printf("\nresults appended to %s\n", args.csv.c_str());
  return 0;
}
