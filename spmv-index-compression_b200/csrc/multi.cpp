// multi.cpp — the multi-GPU layer: an NCCL communicator over the ranks of a job (one process per GPU)
// and chained products over nnz-balanced row shards with x replicated.
//
// A chained product y -> x: every rank multiplies its row shard into its slice of the next x, then the
// slices are all-gathered: one in-place ncclAllGather when the shards have equal rows, else (shards differ
// in size after nnz balancing) a group of in-place broadcasts, one per rank (an all-gather of unequal
// pieces). NCCL is opened at run time
// (dlopen, reusing a libnccl.so.2 the process already loaded, e.g. PyTorch's), so the library does not
// pin an NCCL version of its own.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "capi_internal.hpp"

namespace spmvb200 {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*get_error_string)(ncclResult_t) = nullptr;
  bool loaded = false;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!handle) handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!handle) handle = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!handle) return;
    bool ok = true;
    auto bind = [&](auto& pointer, const char* name) {
      pointer = reinterpret_cast<std::remove_reference_t<decltype(pointer)>>(dlsym(handle, name));
      ok = ok && pointer != nullptr;
    };
    bind(api.get_unique_id, "ncclGetUniqueId");
    bind(api.comm_init_rank, "ncclCommInitRank");
    bind(api.comm_destroy, "ncclCommDestroy");
    bind(api.comm_abort, "ncclCommAbort");
    bind(api.comm_get_async_error, "ncclCommGetAsyncError");
    bind(api.group_start, "ncclGroupStart");
    bind(api.group_end, "ncclGroupEnd");
    bind(api.broadcast, "ncclBroadcast");
    bind(api.all_gather, "ncclAllGather");
    bind(api.get_error_string, "ncclGetErrorString");
    api.loaded = ok;
  });
  if (!api.loaded) fail(SPMV_ERR_NCCL, "NCCL (libnccl.so.2) could not be loaded");
  return api;
}

void nccl_check(ncclResult_t result, const char* what) {
  if (result == ncclSuccess) return;
  fail(SPMV_ERR_NCCL, std::string(what) + ": " + nccl().get_error_string(result));
}

ncclDataType_t nccl_type(int dtype) {
  switch (dtype) {
    case SPMV_F64: return ncclFloat64;
    case SPMV_F32: return ncclFloat32;
    default: return ncclFloat16;
  }
}

}  // namespace
}  // namespace spmvb200

struct spmv_comm {
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
  int device = 0;
  bool aborted = false;
  cudaStream_t side = nullptr;   // the all-gathers of spmv_chain_run_blocks, beside the products
};


using namespace spmvb200;

extern "C" {

int spmv_comm_unique_id(void* id128) {
  return guarded([&] {
    require(id128 != nullptr, "id128 is required");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    ncclUniqueId id;
    nccl_check(nccl().get_unique_id(&id), "ncclGetUniqueId");
    std::memcpy(id128, &id, sizeof(id));
  });
}

int spmv_comm_create(int nranks, int rank, const void* id128, int device, spmv_comm** out) {
  return guarded([&] {
    require(out && id128 && nranks >= 1 && rank >= 0 && rank < nranks, "bad communicator arguments");
    *out = nullptr;
    std::unique_ptr<spmv_comm> comm(new spmv_comm);
    comm->nranks = nranks;
    comm->rank = rank;
    if (device >= 0) {
      const cudaError_t status = cudaSetDevice(device);
      if (status != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(status));
    }
    cudaGetDevice(&comm->device);
    ncclUniqueId id;
    std::memcpy(&id, id128, sizeof(id));
    nccl_check(nccl().comm_init_rank(&comm->comm, nranks, id, rank), "ncclCommInitRank");
    *out = comm.release();
  });
}

void spmv_comm_destroy(spmv_comm* comm) {
  if (!comm) return;
  if (comm->side) cudaStreamDestroy(comm->side);
  if (comm->comm) {
    if (comm->aborted) nccl().comm_abort(comm->comm);
    else nccl().comm_destroy(comm->comm);
  }
  delete comm;
}

// Waits until the stream's work is done or a collective failed, for at most timeout_ms; on an NCCL error
// or the timeout the communicator is aborted (so that no rank stays blocked) and the call fails.
int spmv_comm_check(spmv_comm* comm, void* stream, int timeout_ms) {
  return guarded([&] {
    require(comm && comm->comm, "comm is required");
    const auto start = std::chrono::steady_clock::now();
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (;;) {
      ncclResult_t async = ncclSuccess;
      nccl_check(nccl().comm_get_async_error(comm->comm, &async), "ncclCommGetAsyncError");
      if (async != ncclSuccess && async != ncclInProgress) {
        comm->aborted = true;
        fail(SPMV_ERR_NCCL, std::string("collective failed: ") + nccl().get_error_string(async));
      }
      const cudaError_t query = cudaStreamQuery(s);
      if (query == cudaSuccess) return;
      if (query != cudaErrorNotReady) fail(SPMV_ERR_CUDA, std::string("stream: ") + cudaGetErrorString(query));
      if (std::chrono::steady_clock::now() - start > std::chrono::milliseconds(timeout_ms)) {
        comm->aborted = true;
        fail(SPMV_ERR_TIMEOUT, "collectives did not complete in time; the communicator is aborted");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
  });
}

}  // extern "C"

namespace {
// Waits until the stream's work is done or a collective failed, for at most timeout_ms; on an NCCL error or
// the timeout the communicator is marked aborted. Returns SPMV_OK, SPMV_ERR_NCCL, SPMV_ERR_CUDA or
// SPMV_ERR_TIMEOUT.
int wait_for_stream(spmv_comm* comm, cudaStream_t s, int timeout_ms) {
  const auto start = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t async = ncclSuccess;
    if (nccl().comm_get_async_error(comm->comm, &async) != ncclSuccess ||
        (async != ncclSuccess && async != ncclInProgress)) {
      comm->aborted = true;
      return SPMV_ERR_NCCL;
    }
    const cudaError_t query = cudaStreamQuery(s);
    if (query == cudaSuccess) return SPMV_OK;
    if (query != cudaErrorNotReady) return SPMV_ERR_CUDA;
    if (std::chrono::steady_clock::now() - start > std::chrono::milliseconds(timeout_ms)) {
      comm->aborted = true;
      return SPMV_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}
// How long a call that drains its own streams waits for collectives before it gives up.
constexpr int kDrainTimeoutMs = 120000;
}  // namespace

extern "C" {

// End-to-end products of a row shard from host memory, x split over the ranks: every rank copies its
// 1/nranks slice of each x in from host memory and the slices are all-gathered in place (one
// ncclAllGather), then the shard's product runs and its rows of y are copied out. Vectors pipeline over two
// device buffers and three streams (copies in and the all-gathers on the caller's stream, products on a
// second, copies out on a third), as spmv_operator_run_host_batch does on one GPU.
int spmv_shard_run_host_batch(const spmv_operator* shard_op, spmv_comm* comm, const void* x_host, int64_t x_stride,
                              void* y_host, int64_t y_stride, int count, void* x_device, void* y_device, void* stream) {
  return guarded([&] {
    require(shard_op && comm && comm->comm && x_host && y_host && x_device && y_device && count >= 0, "bad arguments");
    require(!comm->aborted, "the communicator was aborted");
    spmv_operator_info info;
    if (spmv_operator_get_info(shard_op, &info) != SPMV_OK) fail(SPMV_ERR_INVALID_ARGUMENT, "bad operator");
    const int nranks = comm->nranks, rank = comm->rank;
    const size_t value_bytes = (size_t)value_bytes_of(info.dtype);
    const int64_t slice = ((int64_t)info.cols + nranks - 1) / nranks;   // x entries a rank copies in
    const int64_t mine_first = std::min<int64_t>((int64_t)rank * slice, info.cols);
    const int64_t mine_count = std::min<int64_t>(info.cols, mine_first + slice) - mine_first;
    const size_t x_pitch = (value_bytes * (size_t)(slice * nranks) + 15) / 16 * 16;
    const size_t y_bytes = value_bytes * (size_t)info.rows, y_pitch = (y_bytes + 15) / 16 * 16;
    char* xd = static_cast<char*>(x_device);
    char* yd = static_cast<char*>(y_device);
    NcclApi& api = nccl();
    DeviceScope scope(comm->device);
    const cudaStream_t copy_in = static_cast<cudaStream_t>(stream);
    cudaStream_t compute = nullptr, copy_out = nullptr;
    cudaEvent_t gathered[2] = {}, computed[2] = {}, copied_out[2] = {};
    cudaError_t status = cudaStreamCreateWithFlags(&compute, cudaStreamNonBlocking);
    if (status == cudaSuccess) status = cudaStreamCreateWithFlags(&copy_out, cudaStreamNonBlocking);
    for (int b = 0; b < 2 && status == cudaSuccess; ++b) {
      status = cudaEventCreateWithFlags(&gathered[b], cudaEventDisableTiming);
      if (status == cudaSuccess) status = cudaEventCreateWithFlags(&computed[b], cudaEventDisableTiming);
      if (status == cudaSuccess) status = cudaEventCreateWithFlags(&copied_out[b], cudaEventDisableTiming);
    }
    ncclResult_t collective = ncclSuccess;
    // vector i uses buffers i mod 2: its copy in waits until the product of vector i - 2 has read x, its
    // product until the copy out of vector i - 2 has read y
    for (int i = 0; i < count && status == cudaSuccess && collective == ncclSuccess; ++i) {
      const int b = i & 1;
      char* x_b = xd + b * x_pitch;
      const char* xh = static_cast<const char*>(x_host) + (int64_t)i * x_stride;
      char* yh = static_cast<char*>(y_host) + (int64_t)i * y_stride;
      if (i >= 2) status = cudaStreamWaitEvent(copy_in, computed[b], 0);
      if (status == cudaSuccess && mine_count > 0)
        status = cudaMemcpyAsync(x_b + value_bytes * mine_first, xh + value_bytes * mine_first,
                                 value_bytes * (size_t)mine_count, cudaMemcpyHostToDevice, copy_in);
      if (status != cudaSuccess) break;
      collective = api.all_gather(x_b + value_bytes * (size_t)(rank * slice), x_b, (size_t)slice, nccl_type(info.dtype),
                                  comm->comm, copy_in);
      if (collective != ncclSuccess) break;
      status = cudaEventRecord(gathered[b], copy_in);
      if (status == cudaSuccess) status = cudaStreamWaitEvent(compute, gathered[b], 0);
      if (status == cudaSuccess && i >= 2) status = cudaStreamWaitEvent(compute, copied_out[b], 0);
      if (status == cudaSuccess) status = run_operator_leaving_sms(shard_op, x_b, yd + b * y_pitch, compute, 0);
      if (status == cudaSuccess) status = cudaEventRecord(computed[b], compute);
      if (status == cudaSuccess) status = cudaStreamWaitEvent(copy_out, computed[b], 0);
      if (status == cudaSuccess) status = cudaMemcpyAsync(yh, yd + b * y_pitch, y_bytes, cudaMemcpyDeviceToHost, copy_out);
      if (status == cudaSuccess) status = cudaEventRecord(copied_out[b], copy_out);
    }
    if (status == cudaSuccess && collective == ncclSuccess && count > 0)
      status = cudaStreamWaitEvent(copy_in, copied_out[(count - 1) & 1], 0);
    // every stream drains before the call returns, after an error too; a collective that another rank
    // never joins ends in a timeout (the communicator is then aborted) instead of blocking forever
    for (cudaStream_t drained : {copy_in, compute, copy_out}) {
      if (!drained) continue;
      const int waited = wait_for_stream(comm, drained, kDrainTimeoutMs);
      if (waited != SPMV_OK && status == cudaSuccess && collective == ncclSuccess) status = cudaErrorLaunchTimeout;
    }
    for (int b = 0; b < 2; ++b)
      for (cudaEvent_t event : {gathered[b], computed[b], copied_out[b]})
        if (event) cudaEventDestroy(event);
    if (compute) cudaStreamDestroy(compute);
    if (copy_out) cudaStreamDestroy(copy_out);
    nccl_check(collective, "ncclAllGather");
    if (status != cudaSuccess) fail(SPMV_ERR_CUDA, std::string("sharded products through host buffers: ") + cudaGetErrorString(status));
  });
}

int spmv_chain_run(const spmv_operator* shard_op, spmv_comm* comm, const int* shard_row_begin, void* x_current,
                   void* x_next, int products, void* stream) {
  return guarded([&] {
    require(shard_op && comm && comm->comm && shard_row_begin && x_current && x_next && products >= 0, "bad arguments");
    require(!comm->aborted, "the communicator was aborted");
    spmv_operator_info info;
    if (spmv_operator_get_info(shard_op, &info) != SPMV_OK) fail(SPMV_ERR_INVALID_ARGUMENT, "bad operator");
    const int nranks = comm->nranks, rank = comm->rank;
    const int64_t total_rows = shard_row_begin[nranks];
    require(shard_row_begin[0] == 0 && shard_row_begin[rank + 1] - shard_row_begin[rank] == info.rows,
            "the operator's rows do not match its shard");
    require(info.cols == total_rows, "chained products need a square matrix (cols = total rows)");
    const size_t value_bytes = (size_t)value_bytes_of(info.dtype);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    NcclApi& api = nccl();
    char* current = static_cast<char*>(x_current);
    char* next = static_cast<char*>(x_next);
    // shards of equal rows (and so slices of equal size) are gathered by one in-place all-gather; others by
    // a group of broadcasts, one per rank (an all-gather of unequal pieces)
    bool equal = true;
    for (int root = 0; root < nranks; ++root)
      equal = equal && shard_row_begin[root + 1] - shard_row_begin[root] == shard_row_begin[1] - shard_row_begin[0];
    for (int product = 0; product < products; ++product) {
      // this rank's rows of y go straight into its slice of the next x
      const int status = spmv_operator_run(shard_op, current, next + value_bytes * shard_row_begin[rank], stream);
      if (status != SPMV_OK) fail(status, spmv_last_error());
      if (equal) {
        const size_t count = (size_t)(shard_row_begin[1] - shard_row_begin[0]);
        if (count > 0)
          nccl_check(api.all_gather(next + value_bytes * shard_row_begin[rank], next, count, nccl_type(info.dtype),
                                    comm->comm, s),
                     "ncclAllGather");
      } else {
        nccl_check(api.group_start(), "ncclGroupStart");
        for (int root = 0; root < nranks; ++root) {
          const size_t count = (size_t)(shard_row_begin[root + 1] - shard_row_begin[root]);
          if (count == 0) continue;
          char* slice = next + value_bytes * shard_row_begin[root];
          nccl_check(api.broadcast(slice, slice, count, nccl_type(info.dtype), root, comm->comm, s), "ncclBroadcast");
        }
        nccl_check(api.group_end(), "ncclGroupEnd");
      }
      std::swap(current, next);
    }
  });
}

// Multiprocessors the products leave to the all-gathers running beside them.
constexpr int kCollectiveSms = 8;

int spmv_chain_run_blocks(const spmv_operator* const* block_ops, int blocks_per_rank, int block_rows, spmv_comm* comm,
                          void* x_current, void* x_next, int products, void* stream) {
  return guarded([&] {
    require(block_ops && blocks_per_rank >= 1 && block_rows >= 1 && comm && comm->comm && x_current && x_next &&
                products >= 0,
            "bad arguments");
    require(!comm->aborted, "the communicator was aborted");
    const int nranks = comm->nranks, rank = comm->rank;
    const int64_t n = (int64_t)nranks * blocks_per_rank * block_rows;
    spmv_operator_info info;
    for (int c = 0; c < blocks_per_rank; ++c) {
      if (!block_ops[c] || spmv_operator_get_info(block_ops[c], &info) != SPMV_OK) fail(SPMV_ERR_INVALID_ARGUMENT, "bad operator");
      require(info.rows == block_rows && info.cols == n, "every block operator must have block_rows rows and n columns");
    }
    const int dtype = info.dtype;
    const size_t value_bytes = (size_t)value_bytes_of(dtype);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    NcclApi& api = nccl();
    // the side stream and the events live on the communicator's device, whichever device is current
    DeviceScope scope(comm->device);
    if (!comm->side) {
      const cudaError_t created = cudaStreamCreateWithFlags(&comm->side, cudaStreamNonBlocking);
      if (created != cudaSuccess) {
        comm->side = nullptr;
        fail(SPMV_ERR_CUDA, std::string("side stream: ") + cudaGetErrorString(created));
      }
    }
    // computed[c]: block c's product of the current x is in place; computed[blocks_per_rank]: the last round
    // of all-gathers is done
    struct Events {
      std::vector<cudaEvent_t> e;
      ~Events() {
        for (cudaEvent_t event : e)
          if (event) cudaEventDestroy(event);
      }
    } events;
    events.e.assign((size_t)blocks_per_rank + 1, nullptr);
    std::vector<cudaEvent_t>& computed = events.e;
    cudaEvent_t& gathered = events.e[(size_t)blocks_per_rank];
    cudaError_t status = cudaSuccess;
    for (cudaEvent_t& event : events.e)
      if (status == cudaSuccess) status = cudaEventCreateWithFlags(&event, cudaEventDisableTiming);
    char* current = static_cast<char*>(x_current);
    char* next = static_cast<char*>(x_next);
    for (int product = 0; product < products && status == cudaSuccess; ++product) {
      for (int c = 0; c < blocks_per_rank && status == cudaSuccess; ++c) {
        // block c * nranks + rank of y into its place in the next x; then, beside the next block's product,
        // the round of blocks c * nranks .. c * nranks + nranks - 1 all-gathered in place
        const int64_t mine = ((int64_t)c * nranks + rank) * block_rows;
        status = run_operator_leaving_sms(block_ops[c], current, next + value_bytes * mine, s, kCollectiveSms);
        if (status == cudaSuccess) status = cudaEventRecord(computed[c], s);
        if (status == cudaSuccess) status = cudaStreamWaitEvent(comm->side, computed[c], 0);
        if (status != cudaSuccess) break;
        nccl_check(api.all_gather(next + value_bytes * mine, next + value_bytes * (int64_t)c * nranks * block_rows,
                                  (size_t)block_rows, nccl_type(dtype), comm->comm, comm->side),
                   "ncclAllGather");
      }
      // the next product reads this one's x: it waits for every round of the all-gather
      if (status == cudaSuccess) status = cudaEventRecord(gathered, comm->side);
      if (status == cudaSuccess) status = cudaStreamWaitEvent(s, gathered, 0);
      std::swap(current, next);
    }
    if (status != cudaSuccess) {
      // all-gathers already queued on the side stream may still write x_next: let them finish before the
      // call returns its error (x_next is undefined after an error)
      cudaStreamSynchronize(comm->side);
      fail(SPMV_ERR_CUDA, std::string("chained products over row blocks: ") + cudaGetErrorString(status));
    }
  });
}

}  // extern "C"
