// Peer memory of the sequence-split exchange: device allocations that the other processes of
// the node map through CUDA IPC (one process per GPU), so a kernel can store into another GPU's
// memory over NVLink.
#include <cuda_runtime.h>

#include <cstring>

#include "hla_s6.h"
#include "hla_s6_internal.h"

using namespace hla;

static_assert(sizeof(cudaIpcMemHandle_t) <= HLA_S6_PEER_HANDLE_BYTES, "IPC handle does not fit");

extern "C" {

int hla_s6_peer_alloc(int64_t bytes, void** ptr, void* handle) {
  if (bytes <= 0 || !ptr || !handle) {
    set_error("peer alloc needs a positive size and output pointers");
    return kStatusInvalid;
  }
  void* p = nullptr;
  int rc = cuda_status(cudaMalloc(&p, static_cast<size_t>(bytes)), "peer alloc");
  if (rc) return rc;
  if ((rc = cuda_status(cudaMemset(p, 0, static_cast<size_t>(bytes)), "peer alloc zero-fill"))) {
    cudaFree(p);
    return rc;
  }
  cudaIpcMemHandle_t h;
  if ((rc = cuda_status(cudaIpcGetMemHandle(&h, p), "peer alloc IPC handle"))) {
    cudaFree(p);
    return rc;
  }
  std::memset(handle, 0, HLA_S6_PEER_HANDLE_BYTES);
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return kStatusOk;
}

int hla_s6_peer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) {
    set_error("peer open needs a handle and an output pointer");
    return kStatusInvalid;
  }
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const int rc = cuda_status(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "peer open");
  if (rc) return rc;
  *ptr = p;
  return kStatusOk;
}

int hla_s6_peer_close(void* ptr) {
  if (!ptr) return kStatusOk;
  return cuda_status(cudaIpcCloseMemHandle(ptr), "peer close");
}

int hla_s6_peer_free(void* ptr) {
  if (!ptr) return kStatusOk;
  return cuda_status(cudaFree(ptr), "peer free");
}

}  // extern "C"
