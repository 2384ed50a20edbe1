// peer.cu — chained products y -> x whose all-gather happens inside the product, over NVLink peer memory.
//
// Every rank (one process per GPU) holds one allocation of its own: two x buffers (the current x and the
// next) and a block of barrier flags, exported to the other ranks by CUDA IPC and mapped by each of them.
// A chained product on rank r runs its row shard with y = its rows of the next x, and the product kernel
// also stores those rows into every other rank's next x through the mapped peer pointers: the thread that
// stores a row's result into y stores it into each peer as well, and each CTA ends with one system-scope
// fence. So when every rank's product is done, every rank's next x is whole: the all-gather took no
// collective library, no multiprocessors of its own and no pass over x after the product. (Measured on two
// B200s, block FEM, 16 M rows a rank: 1.858 ms a step against 1.746 ms for the product alone, and 1.92 ms
// for the product followed by an NCCL all-gather; a tile's rows stored into the peers by the last warp out
// of the tile cost 0.2 ms more, the same with the peers' buffers replaced by local ones.) A barrier between the ranks' GPUs then
// closes the product: each rank stores the barrier's epoch into its slot of every rank's flags (a release
// store at system scope) and waits until its own flags all hold it (acquire loads), for a bounded time
// after which it sets the group's status word. The barrier orders both ways: no rank reads the next x
// before every rank has stored into it, and no rank stores into a buffer another rank still reads (the
// next product's stores go to the other buffer, which every rank finished reading before the barrier).
//
// Halo mode (spmv_peer_group_set_halo): a rank's rows usually read few of the other ranks' entries of x (a
// block FEM matrix, rows coupled within +-50,000: about 100,000 entries of 4 M a rank). After the set-up
// lists those entries (runs, split into chunks per owner), a chained product stores nothing into the peers;
// after the barrier one small kernel pulls the listed entries of the next x from their owners' memory
// (peer loads over NVLink) into this rank's next x. Each rank's x then holds its own rows and the entries
// its rows read; the others are not kept up to date.
//
// No counterpart in the reference (its benchmark runs on one GPU); the per-row results are the
// single-GPU operator's, so chained results are bit-identical to the oracle's chain.
#include <cuda_runtime.h>

#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "capi_internal.hpp"
#include "kernels.cuh"

namespace spmvb200 {
namespace {

constexpr int kMaxRanks = kMaxPeers + 1;
constexpr size_t kFlagBlock = 256;   // kMaxRanks 8-byte flags, then the 4-byte status word

void cuda_ok(cudaError_t status, const char* what) {
  if (status == cudaSuccess) return;
  fail(status == cudaErrorMemoryAllocation ? SPMV_ERR_OUT_OF_MEMORY : SPMV_ERR_CUDA,
       std::string(what) + ": " + cudaGetErrorString(status));
}

struct BarrierArgs {
  unsigned long long* flags[kMaxRanks];   // every rank's flag block as mapped here (null: not mapped)
  const unsigned long long* own;           // this rank's flags
  unsigned* status;                        // this rank's status word
  unsigned long long epoch;
  unsigned long long limit_ns;
  int nranks;
  int rank;
};

__device__ __forceinline__ void store_release_system(unsigned long long* address, unsigned long long value) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(address), "l"(value) : "memory");
}

__device__ __forceinline__ unsigned long long load_acquire_system(const unsigned long long* address) {
  unsigned long long value;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(value) : "l"(address) : "memory");
  return value;
}

// Thread t < nranks: stores the epoch into slot `rank` of rank t's flags, then waits until slot t of this
// rank's flags holds at least the epoch, for at most limit_ns (and a bounded number of polls); a wait that
// gives up sets kStatusTimeout and returns. Flags only grow, so a rank already at a later barrier passes.
__global__ void __launch_bounds__(32) k_peer_barrier(const BarrierArgs a) {
  const int t = threadIdx.x;
  if (t >= a.nranks) return;
  // this rank's earlier kernels' stores (its rows of the next x, into its own memory and its peers') are
  // visible at system scope before any rank can see the flag
  __threadfence_system();
  if (a.flags[t]) store_release_system(a.flags[t] + a.rank, a.epoch);
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 0; spin < (1u << 24); ++spin) {
    if (load_acquire_system(a.own + t) >= a.epoch) return;
    if (global_timer_ns() - start > a.limit_ns) break;
    __nanosleep(256);
  }
  atomicOr(a.status, kStatusTimeout);
}

// A chunk of the halo: x entries [begin, end) owned by rank `owner`, at most kHaloChunk of them.
constexpr int kHaloChunk = 2048;
struct HaloArgs {
  const int4* chunks;                  // {begin, end, owner, 0}
  int chunk_count;
  const char* sources[kMaxRanks];      // every rank's next x as mapped here
  char* target;                        // this rank's next x
  int value_bytes;
};

// Block b copies chunk b of the halo from its owner's next x into this rank's next x. The loads read another
// GPU's memory that this kernel's rank saw published by the barrier: they bypass the caches (ld.global.cv),
// so that no copy from before the barrier is read.
__global__ void __launch_bounds__(256) k_halo_pull(const HaloArgs a) {
  const int4 chunk = a.chunks[blockIdx.x];
  const char* source = a.sources[chunk.z];
  if (a.value_bytes == 8) {
    const unsigned long long* from = reinterpret_cast<const unsigned long long*>(source);
    unsigned long long* to = reinterpret_cast<unsigned long long*>(a.target);
    for (int i = chunk.x + (int)threadIdx.x; i < chunk.y; i += blockDim.x) to[i] = __ldcv(from + i);
  } else if (a.value_bytes == 4) {
    const unsigned* from = reinterpret_cast<const unsigned*>(source);
    unsigned* to = reinterpret_cast<unsigned*>(a.target);
    for (int i = chunk.x + (int)threadIdx.x; i < chunk.y; i += blockDim.x) to[i] = __ldcv(from + i);
  } else {
    const unsigned short* from = reinterpret_cast<const unsigned short*>(source);
    unsigned short* to = reinterpret_cast<unsigned short*>(a.target);
    for (int i = chunk.x + (int)threadIdx.x; i < chunk.y; i += blockDim.x) to[i] = __ldcv(from + i);
  }
}

}  // namespace
}  // namespace spmvb200

struct spmv_peer_group {
  int device = 0;
  int nranks = 0;
  int rank = 0;
  int64_t x_bytes = 0;
  size_t pitch = 0;                      // bytes of one x buffer, rounded up to 256
  char* local = nullptr;                 // [x buffer 0 | x buffer 1 | flag block]
  char* mapped[spmvb200::kMaxPeers + 1] = {};   // every rank's allocation as mapped here (own: local)
  bool opened = false;
  bool failed = false;
  int current = 0;                       // the buffer holding the current x (the next product's input)
  unsigned long long epoch = 0;
  // halo mode (spmv_peer_group_set_halo): the x entries other ranks own that this rank's rows read, as
  // chunks {begin, end, owner} on the device; pulled from their owners after each product's barrier
  int4* halo = nullptr;
  int halo_chunks = 0;
  bool halo_set = false;
  int64_t halo_entries = 0;
  int halo_rows_begin = 0, halo_rows_end = 0;   // the row shard the halo was planned for

  char* x_buffer(int rank_of, int which) const { return mapped[rank_of] + (size_t)which * pitch; }
  unsigned long long* flags(int rank_of) const {
    return mapped[rank_of] ? reinterpret_cast<unsigned long long*>(mapped[rank_of] + 2 * pitch) : nullptr;
  }
  unsigned* status() const { return reinterpret_cast<unsigned*>(local + 2 * pitch + 8 * (spmvb200::kMaxPeers + 1)); }

  ~spmv_peer_group() {   // never throws: the device is switched by hand and switched back
    int previous = -1;
    cudaGetDevice(&previous);
    if (previous != device) cudaSetDevice(device);
    for (int r = 0; r < nranks; ++r)
      if (r != rank && mapped[r]) cudaIpcCloseMemHandle(mapped[r]);
    if (local) cudaFree(local);
    if (halo) cudaFree(halo);
    if (previous >= 0 && previous != device) cudaSetDevice(previous);
  }
};

using namespace spmvb200;

namespace {

// One barrier launch on the stream (epoch advanced), waiting at most limit_ms.
void launch_barrier(spmv_peer_group* group, int limit_ms, cudaStream_t stream) {
  BarrierArgs a{};
  for (int r = 0; r < group->nranks; ++r) a.flags[r] = group->flags(r);
  a.own = group->flags(group->rank);
  a.status = group->status();
  a.epoch = ++group->epoch;
  a.limit_ns = (unsigned long long)limit_ms * 1000000ull;
  a.nranks = group->nranks;
  a.rank = group->rank;
  k_peer_barrier<<<1, 32, 0, stream>>>(a);
  cuda_ok(cudaGetLastError(), "peer barrier launch");
}

}  // namespace

extern "C" {

int spmv_peer_group_create(int nranks, int rank, int64_t x_bytes, int device, spmv_peer_group** out) {
  return guarded([&] {
    require(out && nranks >= 1 && nranks <= kMaxPeers + 1 && rank >= 0 && rank < nranks && x_bytes >= 0,
            "bad peer group arguments (at most 16 ranks)");
    *out = nullptr;
    DeviceScope scope(device);
    std::unique_ptr<spmv_peer_group> group(new spmv_peer_group);
    cuda_ok(cudaGetDevice(&group->device), "cudaGetDevice");
    group->nranks = nranks;
    group->rank = rank;
    group->x_bytes = x_bytes;
    group->pitch = ((size_t)x_bytes + 255) / 256 * 256;
    const size_t bytes = 2 * group->pitch + kFlagBlock;
    cuda_ok(cudaMalloc(reinterpret_cast<void**>(&group->local), bytes), "cudaMalloc");
    cuda_ok(cudaMemset(group->local, 0, bytes), "cudaMemset");
    cuda_ok(cudaDeviceSynchronize(), "peer group set-up");
    group->mapped[rank] = group->local;
    group->opened = nranks == 1;
    *out = group.release();
  });
}

int spmv_peer_group_handle(const spmv_peer_group* group, void* handle) {
  return guarded([&] {
    require(group && handle, "group and handle are required");
    static_assert(sizeof(cudaIpcMemHandle_t) == SPMV_PEER_HANDLE_BYTES, "an IPC handle is 64 bytes");
    DeviceScope scope(group->device);
    cudaIpcMemHandle_t exported;
    cuda_ok(cudaIpcGetMemHandle(&exported, group->local), "cudaIpcGetMemHandle");
    std::memcpy(handle, &exported, sizeof(exported));
  });
}

int spmv_peer_group_open(spmv_peer_group* group, const void* handles) {
  return guarded([&] {
    require(group && handles, "group and handles are required");
    require(!group->opened || group->nranks == 1, "the group is open already");
    DeviceScope scope(group->device);
    const char* bytes = static_cast<const char*>(handles);
    for (int r = 0; r < group->nranks; ++r) {
      if (r == group->rank) continue;
      cudaIpcMemHandle_t handle;
      std::memcpy(&handle, bytes + (size_t)r * SPMV_PEER_HANDLE_BYTES, sizeof(handle));
      void* pointer = nullptr;
      cuda_ok(cudaIpcOpenMemHandle(&pointer, handle, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
      group->mapped[r] = static_cast<char*>(pointer);
    }
    group->opened = true;
  });
}

int spmv_peer_group_x(const spmv_peer_group* group, int which, void** x) {
  return guarded([&] {
    require(group && x && (which == 0 || which == 1), "which must be 0 (current x) or 1 (next x)");
    *x = group->x_buffer(group->rank, which == 0 ? group->current : 1 - group->current);
  });
}

int spmv_peer_group_copy_x(spmv_peer_group* group, int direction, void* buffer, int64_t bytes, void* stream) {
  return guarded([&] {
    require(group && buffer && bytes >= 0 && bytes <= group->x_bytes && (direction == 0 || direction == 1),
            "bad copy arguments");
    DeviceScope scope(group->device);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    char* x = group->x_buffer(group->rank, group->current);
    cuda_ok(direction == 0 ? cudaMemcpyAsync(x, buffer, (size_t)bytes, cudaMemcpyDefault, s)
                           : cudaMemcpyAsync(buffer, x, (size_t)bytes, cudaMemcpyDefault, s),
            "copy of the current x");
    cuda_ok(cudaStreamSynchronize(s), "stream synchronize");
  });
}

int spmv_peer_group_barrier(spmv_peer_group* group, int timeout_ms, void* stream) {
  return guarded([&] {
    require(group && timeout_ms > 0, "group and a positive timeout are required");
    require(!group->failed, "a barrier of this group timed out before; its buffers are undefined");
    DeviceScope scope(group->device);
    launch_barrier(group, timeout_ms, static_cast<cudaStream_t>(stream));
  });
}

int spmv_peer_group_check(spmv_peer_group* group) {
  int timed_out = 0;
  const int status = guarded([&] {
    require(group, "group is required");
    DeviceScope scope(group->device);
    cuda_ok(cudaDeviceSynchronize(), "device synchronize");
    unsigned word = 0;
    cuda_ok(cudaMemcpy(&word, group->status(), sizeof(word), cudaMemcpyDeviceToHost), "read status");
    if (word & kStatusTimeout) {
      group->failed = true;
      timed_out = 1;
      set_last_error("a peer barrier gave up waiting for another rank");
    }
  });
  return status != SPMV_OK ? status : (timed_out ? SPMV_ERR_TIMEOUT : SPMV_OK);
}

int spmv_peer_group_set_halo(spmv_peer_group* group, const spmv_csr* shard, const int* shard_row_begin) {
  return guarded([&] {
    require(group && shard && shard_row_begin, "group, shard and shard_row_begin are required");
    const Csr& m = shard->m;
    const int nranks = group->nranks, rank = group->rank;
    const int64_t n = shard_row_begin[nranks];
    require(shard_row_begin[0] == 0 && shard_row_begin[rank + 1] - shard_row_begin[rank] == m.rows && m.cols == n,
            "the shard's rows or columns do not match shard_row_begin");
    const int own_begin = shard_row_begin[rank], own_end = shard_row_begin[rank + 1];
    // the columns outside this rank's rows that its rows read
    std::vector<unsigned char> read((size_t)n, 0);   // set by several host threads: relaxed atomic stores
    parallel_for(m.rows, [&](int64_t first, int64_t last) {
      for (int64_t row = first; row < last; ++row)
        for (int entry = m.row_ptr[row]; entry < m.row_ptr[row + 1]; ++entry) {
          const int column = m.col_ind[entry];
          if (column < own_begin || column >= own_end) __atomic_store_n(&read[(size_t)column], 1, __ATOMIC_RELAXED);
        }
    });
    // runs of them (gaps of up to 32 entries bridged), split at the owners' bounds and into chunks
    std::vector<int4> chunks;
    int64_t entries = 0;
    int owner = 0;
    for (int64_t column = 0; column < n;) {
      if (!read[(size_t)column]) { ++column; continue; }
      while (shard_row_begin[owner + 1] <= column) ++owner;
      int64_t end = column + 1, last_read = column;
      while (end < shard_row_begin[owner + 1] && end - last_read <= 32) {
        if (read[(size_t)end]) last_read = end;
        ++end;
      }
      for (int64_t begin = column; begin <= last_read; begin += kHaloChunk)
        chunks.push_back(make_int4((int)begin, (int)std::min<int64_t>(begin + kHaloChunk, last_read + 1), owner, 0));
      entries += last_read + 1 - column;
      column = last_read + 1;
    }
    require(chunks.size() < 0x7fffffff, "halo too large");
    DeviceScope scope(group->device);
    if (group->halo) cudaFree(group->halo);
    group->halo = nullptr;
    if (!chunks.empty()) {
      cuda_ok(cudaMalloc(reinterpret_cast<void**>(&group->halo), sizeof(int4) * chunks.size()), "cudaMalloc");
      cuda_ok(cudaMemcpy(group->halo, chunks.data(), sizeof(int4) * chunks.size(), cudaMemcpyHostToDevice), "halo upload");
    }
    group->halo_chunks = (int)chunks.size();
    group->halo_entries = entries;
    group->halo_rows_begin = own_begin;
    group->halo_rows_end = own_end;
    group->halo_set = true;
  });
}

int spmv_peer_group_halo_entries(const spmv_peer_group* group, int64_t* entries) {
  return guarded([&] {
    require(group && entries, "group and entries are required");
    *entries = group->halo_set ? group->halo_entries : -1;
  });
}

int spmv_chain_run_peer(const spmv_operator* shard_op, spmv_peer_group* group, const int* shard_row_begin, int products,
                        int timeout_ms, void* stream) {
  return guarded([&] {
    require(shard_op && group && shard_row_begin && products >= 0 && timeout_ms > 0, "bad arguments");
    require(group->opened, "open the group (spmv_peer_group_open) before chained products");
    require(!group->failed, "a barrier of this group timed out before; its buffers are undefined");
    spmv_operator_info info;
    if (spmv_operator_get_info(shard_op, &info) != SPMV_OK) fail(SPMV_ERR_INVALID_ARGUMENT, "bad operator");
    const int nranks = group->nranks, rank = group->rank;
    const int64_t n = shard_row_begin[nranks];
    require(shard_row_begin[0] == 0 && shard_row_begin[rank + 1] - shard_row_begin[rank] == info.rows,
            "the operator's rows do not match its shard");
    for (int r = 0; r < nranks; ++r) require(shard_row_begin[r + 1] >= shard_row_begin[r], "shard bounds must not decrease");
    require(info.cols == n, "chained products need a square matrix (cols = total rows)");
    const size_t value_bytes = (size_t)value_bytes_of(info.dtype);
    require((int64_t)(value_bytes * (size_t)n) <= group->x_bytes, "the group's x buffers hold fewer than n entries");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    DeviceScope scope(group->device);
    const size_t offset = value_bytes * (size_t)shard_row_begin[rank];
    // every rank has reached this point in its stream before any stores into its buffers
    launch_barrier(group, timeout_ms, s);
    if (group->halo_set)
      require(group->halo_rows_begin == shard_row_begin[rank] && group->halo_rows_end == shard_row_begin[rank + 1],
              "the halo was planned for another row shard");
    for (int product = 0; product < products; ++product) {
      const int next = 1 - group->current;
      void* peers[kMaxPeers];
      int count = 0;
      if (!group->halo_set)   // every row stored into every rank's next x as well
        for (int r = 0; r < nranks; ++r)
          if (r != rank) peers[count++] = group->x_buffer(r, next) + offset;
      cuda_ok(run_operator_with_peers(shard_op, group->x_buffer(rank, group->current), group->x_buffer(rank, next) + offset,
                                      peers, count, s),
              "chained product");
      launch_barrier(group, timeout_ms, s);
      if (group->halo_set && group->halo_chunks > 0) {   // the entries of the next x this rank's rows read
        HaloArgs h{};
        h.chunks = group->halo;
        h.chunk_count = group->halo_chunks;
        for (int r = 0; r < nranks; ++r) h.sources[r] = group->x_buffer(r, next);
        h.target = group->x_buffer(rank, next);
        h.value_bytes = (int)value_bytes;
        k_halo_pull<<<(unsigned)group->halo_chunks, 256, 0, s>>>(h);
        cuda_ok(cudaGetLastError(), "halo pull");
      }
      group->current = next;
    }
  });
}

void spmv_peer_group_destroy(spmv_peer_group* group) { delete group; }

}  // extern "C"
