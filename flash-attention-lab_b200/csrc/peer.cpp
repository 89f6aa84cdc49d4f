// Peer memory for the cross-GPU decode exchange: device buffers that the other ranks (one
// process per GPU) map through CUDA IPC and write over NVLink / NVSwitch. No counterpart in the
// reference, which is single-GPU.
#include <cuda_runtime.h>

#include <cstring>

#include "flash_lab_b200.h"
#include "host_common.h"

using namespace flb;

extern "C" size_t flb_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int flb_peer_alloc(size_t bytes, void** ptr, void* handle) {
  clear_error();
  if (ptr == nullptr || handle == nullptr || bytes == 0)
    return fail(FLB_ERR_INVALID_ARGUMENT, "flb_peer_alloc: bad arguments");
  *ptr = nullptr;
  void* p = nullptr;
  if (int st = check_cuda(cudaMalloc(&p, bytes), "cudaMalloc(peer buffer)")) return st;
  // Arrival counters start at zero; the partial regions are always written before being read.
  if (int st = check_cuda(cudaMemset(p, 0, bytes), "cudaMemset(peer buffer)")) {
    cudaFree(p);
    return st;
  }
  cudaIpcMemHandle_t h;
  if (int st = check_cuda(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle")) {
    cudaFree(p);
    return st;
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return FLB_OK;
}

extern "C" int flb_peer_open(const void* handle, void** ptr) {
  clear_error();
  if (ptr == nullptr || handle == nullptr)
    return fail(FLB_ERR_INVALID_ARGUMENT, "flb_peer_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess),
                    "cudaIpcOpenMemHandle");
}

extern "C" int flb_peer_close(void* ptr) {
  clear_error();
  if (ptr == nullptr) return FLB_OK;
  return check_cuda(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

extern "C" int flb_peer_free(void* ptr) {
  clear_error();
  if (ptr == nullptr) return FLB_OK;
  return check_cuda(cudaFree(ptr), "cudaFree(peer buffer)");
}
