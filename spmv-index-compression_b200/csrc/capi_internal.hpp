// capi_internal.hpp — error plumbing and internals shared by the C entry points.
#pragma once

#include <cuda_runtime.h>

#include <functional>
#include <memory>
#include <string>

#include "internal.hpp"

namespace spmvb200 {

void set_last_error(const std::string& message);
// Runs body, returning SPMV_OK or the status of the exception it threw (message kept for spmv_last_error).
int guarded(const std::function<void()>& body);
// Throws SPMV_ERR_INVALID_ARGUMENT with message unless condition holds.
void require(bool condition, const char* message);
// The caller's facts, or facts_of(matrix) when facts is null.
Facts facts_for(const spmv_csr* matrix, const spmv_facts* facts);
// Makes `device` current (when it is >= 0 and not already) and restores the caller's device when it goes
// out of scope.
struct DeviceScope {
  int previous = -1;
  explicit DeviceScope(int device);
  ~DeviceScope();
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;
};
// One product on `stream` whose tile kernel launches free_sms multiprocessors' worth of persistent CTAs
// fewer, so that kernels running beside it (collectives) find free multiprocessors (operator.cu).
cudaError_t run_operator_leaving_sms(const spmv_operator* op, const void* x, void* y, cudaStream_t stream, int free_sms);
// One product on `stream` that also stores every row of y into the peer_count copies of y at peers[] (other
// GPUs' memory, indexed by the same rows), at most kMaxPeers (operator.cu).
cudaError_t run_operator_with_peers(const spmv_operator* op, const void* x, void* y, void* const* peers, int peer_count,
                                    cudaStream_t stream);

}  // namespace spmvb200
