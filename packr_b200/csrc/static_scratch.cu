// packr_backward_static_scratch: the PackRLinear backward for callers that
// cannot allocate device memory themselves — for example a host runtime with
// a fixed device-memory budget and no allocator of its own, or a language
// binding that can hand over tensors it was given but has no way to obtain a
// temporary device buffer.  Its scratch (bf16 dY, split parts, bias and lut
// partial sums) lives in one file-scope device array of
// PACKR_STATIC_SCRATCH_BYTES that every GPU loading this library holds until
// the process exits.
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace packr {
namespace static_scratch {

static __device__ __align__(256) unsigned char g_scratch[PACKR_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu[kMaxDevices];
std::atomic<void*> g_ptr[kMaxDevices];

// Device address of g_scratch on the current device.  The host-side name
// g_scratch is only a stand-in for the symbol and must never be passed to a
// kernel; cudaGetSymbolAddress is asked with that device current, and only a
// successful answer is kept (the first successful call on each device
// performs this set-up; a failed lookup, e.g. one made during a stream
// capture, is retried by the next call).
int device_ptr(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return PACKR_ERR_CUDA;
  void* p = g_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_mu[dev]);
    p = g_ptr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        return PACKR_ERR_CUDA;
      }
      g_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return PACKR_OK;
}

}  // namespace static_scratch
}  // namespace packr

extern "C" int packr_backward_static_scratch(const float* dY, const void* x, int x_dtype, const uint8_t* W_p,
                                             const uint16_t* W_f, const float* lut, const int32_t* lut_counts,
                                             void* dX, uint16_t* dW_f, float* dlut, uint16_t* dbias, int64_t M,
                                             int64_t K, int64_t N, int flags, void* stream) {
  using namespace packr;
  if (M > 0 && K > 0 && N > 0) {
    linear::Carve c{nullptr};
    linear::BwdPlan p;
    const size_t need = linear::plan_backward(c, p, M, K, N, x_dtype, flags, dX != nullptr, dW_f != nullptr,
                                              dlut != nullptr, dbias != nullptr, lut_counts != nullptr, false);
    if (need > (size_t)PACKR_STATIC_SCRATCH_BYTES) return PACKR_ERR_WORKSPACE;  // beyond the static maximum
  }
  void* scratch = nullptr;
  int st = static_scratch::device_ptr(&scratch);
  if (st != PACKR_OK) return st;
  return packr_backward(dY, x, x_dtype, W_p, W_f, lut, lut_counts, dX, dW_f, dlut, dbias, M, K, N, flags, scratch,
                        (size_t)PACKR_STATIC_SCRATCH_BYTES, stream);
}
