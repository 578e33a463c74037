// Device buffers shared between the processes of one node (one process per
// GPU), for the data-parallel optimizer: each process allocates its parameter
// buckets here, exports a CUDA IPC handle per buffer, and maps the other
// processes' buffers into its own address space (peer access over NVLink), so
// that packr_adam8_multi_push can store the updated parameters straight into
// every other GPU's copy.  The reference has no distributed code.
//
// Plain cudaMalloc allocations: an IPC handle names a whole allocation, so a
// buffer from a caching allocator (a sub-range of a larger block) would not
// map back to the same address range.
#include <cstring>

#include "common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == PACKR_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int packr_device_alloc(size_t bytes, void** ptr) {
  using namespace packr;
  if (ptr == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  if (bytes == 0) return PACKR_ERR_SHAPE;
  const int st = check_device();
  if (st != PACKR_OK) return st;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return PACKR_ERR_CUDA;
  }
  *ptr = p;
  return PACKR_OK;
}

extern "C" int packr_device_free(void* ptr) {
  if (ptr == nullptr) return PACKR_OK;
  return cudaFree(ptr) == cudaSuccess ? PACKR_OK : PACKR_ERR_CUDA;
}

extern "C" int packr_ipc_export(const void* ptr, void* handle) {
  using namespace packr;
  if (ptr == nullptr || handle == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) {
    cudaGetLastError();
    return PACKR_ERR_CUDA;
  }
  std::memcpy(handle, &h, sizeof(h));
  return PACKR_OK;
}

extern "C" int packr_ipc_open(const void* handle, void** ptr) {
  using namespace packr;
  if (handle == nullptr || ptr == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  const int st = check_device();
  if (st != PACKR_OK) return st;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return PACKR_ERR_CUDA;
  }
  *ptr = p;
  return PACKR_OK;
}

extern "C" int packr_ipc_close(void* ptr) {
  if (ptr == nullptr) return PACKR_OK;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? PACKR_OK : PACKR_ERR_CUDA;
}
