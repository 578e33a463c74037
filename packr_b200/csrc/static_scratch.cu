// packr_backward_static_scratch: the PackRLinear backward for callers that
// cannot allocate device memory themselves — for example a host runtime with
// a fixed device-memory budget and no allocator of its own, or a language
// binding that can hand over tensors it was given but has no way to obtain a
// temporary device buffer.  Its scratch (bf16 dY, split parts, bias and lut
// partial sums) lives in one file-scope device array of
// PACKR_STATIC_SCRATCH_BYTES that every GPU loading this library holds until
// the process exits.
#include <mutex>

#include "common.cuh"

namespace packr {
namespace static_scratch {

static __device__ __align__(256) unsigned char g_scratch[PACKR_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::once_flag g_once[kMaxDevices];
void* g_ptr[kMaxDevices];
cudaError_t g_err[kMaxDevices];

// Device address of g_scratch on the current device.  The host-side name
// g_scratch is only a stand-in for the symbol and must never be passed to a
// kernel; cudaGetSymbolAddress is asked once per device, with that device
// current (the first call on each device performs this set-up).
int device_ptr(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return PACKR_ERR_CUDA;
  std::call_once(g_once[dev], [dev] { g_err[dev] = cudaGetSymbolAddress(&g_ptr[dev], g_scratch); });
  if (g_err[dev] != cudaSuccess || g_ptr[dev] == nullptr) return PACKR_ERR_CUDA;
  *out = g_ptr[dev];
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
