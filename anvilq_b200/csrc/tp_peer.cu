// tp_peer.cu -- device memory that the ranks of one node write into each other,
// for the column-split GEMV whose all-gather is fused into its epilogue
// (anvilq_w4a16_gemv_allgather).
//
// A rank exports a buffer it allocated (any pointer inside a cudaMalloc
// allocation, e.g. a torch tensor) as a CUDA IPC handle plus the pointer's
// offset from the allocation's base; the other ranks import it and write with
// plain stores over NVLink.  No multicast object is created.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <cstring>
#include <mutex>

#include "../../include/anvilq.h"

namespace {

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static std::once_flag once;
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
    cudaGetLastError();
  });
  return fn;
}

}  // namespace

extern "C" {

size_t anvilq_peer_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

int anvilq_peer_export(const void* dev_ptr, void* handle_out, size_t* offset_out) {
  if (!dev_ptr || !handle_out || !offset_out) return ANVILQ_EINVAL;
  auto range = address_range_fn();
  if (!range) return ANVILQ_ECUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return ANVILQ_ECUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uintptr_t>(dev_ptr) - static_cast<uintptr_t>(base);
  return ANVILQ_OK;
}

int anvilq_peer_import(const void* handle, size_t offset, void** base_out, void** dev_ptr_out) {
  if (!handle || !base_out || !dev_ptr_out) return ANVILQ_EINVAL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  *base_out = base;
  *dev_ptr_out = static_cast<char*>(base) + offset;
  return ANVILQ_OK;
}

int anvilq_peer_close(void* base) {
  if (!base) return ANVILQ_EINVAL;
  if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
    cudaGetLastError();
    return ANVILQ_ECUDA;
  }
  return ANVILQ_OK;
}

}  // extern "C"
