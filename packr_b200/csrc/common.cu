// Status plumbing and the per-device attribute cache.
#include <atomic>

#include "common.cuh"

namespace packr {

namespace {
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<int> g_cc_major[kMaxDevices];

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}
}  // namespace

int sm_count() {
  int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  int c = g_sm_count[dev].load(std::memory_order_relaxed);
  if (c > 0) return c;
  if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
  g_sm_count[dev].store(c, std::memory_order_relaxed);
  return c;
}

int check_device() {
  int dev = current_device();
  if (dev < 0) return PACKR_ERR_CUDA;
  if (dev >= kMaxDevices) return PACKR_ERR_DEVICE;
  int major = g_cc_major[dev].load(std::memory_order_relaxed);
  if (major == 0) {
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return PACKR_ERR_CUDA;
    g_cc_major[dev].store(major, std::memory_order_relaxed);
  }
  return major == 10 ? PACKR_OK : PACKR_ERR_DEVICE;
}

int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return PACKR_OK;
  return PACKR_ERR_LAUNCH;
}

}  // namespace packr

extern "C" const char* packr_error_string(int code) {
  switch (code) {
    case PACKR_OK: return "ok";
    case PACKR_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PACKR_ERR_SHAPE: return "bad shape";
    case PACKR_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case PACKR_ERR_WORKSPACE: return "workspace missing or too small";
    case PACKR_ERR_LAUNCH: return "kernel launch failed";
    case PACKR_ERR_DEVICE: return "current device is not sm_100";
    case PACKR_ERR_TIMEOUT: return "device-side wait timed out";
    case PACKR_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

extern "C" int packr_abi_version(void) { return 1; }

extern "C" int packr_device_status(void* stream) {
  if (cudaStreamSynchronize(packr::as_stream(stream)) != cudaSuccess) return PACKR_ERR_CUDA;
  unsigned int word = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&word, packr::g_wait_timeout, sizeof(word)) != cudaSuccess) return PACKR_ERR_CUDA;
  if (word != 0 && cudaMemcpyToSymbol(packr::g_wait_timeout, &zero, sizeof(zero)) != cudaSuccess)
    return PACKR_ERR_CUDA;
  return word ? PACKR_ERR_TIMEOUT : PACKR_OK;
}
