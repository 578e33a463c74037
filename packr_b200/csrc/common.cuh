// Shared helpers for the libpackr_b200 kernels: status plumbing, the
// per-device attribute cache and small bit-exact conversions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/packr_b200.h"

namespace packr {

// Device-side word set by any kernel whose bounded wait gave up.  It is the
// only device global the library writes; packr_device_status() reads and
// clears it.  (The library is one translation unit, so a plain definition in
// this header is shared by every kernel.)
__device__ unsigned int g_wait_timeout = 0;

// Number of SMs of the current device (cached per device ordinal).
int sm_count();
// PACKR_OK if the current device is compute capability 10.x, else PACKR_ERR_DEVICE.
int check_device();
// Maps the last CUDA launch error to a status code (and clears it).
int launch_status();

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

__host__ __device__ inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// float -> bf16 bit pattern, round to nearest even, by the integer method the
// reference uses for its bf16 parameter store (packr/cuda_adam_kernel.cu:62-64)
// and that torch's float->bfloat16 conversion uses for finite values.
__device__ __forceinline__ uint32_t f32_to_bf16_rne(float f) {
  uint32_t u = __float_as_uint(f);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return u >> 16;
}

__device__ __forceinline__ float bf16_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// Two floats -> packed bf16x2 (lo in bits 0-15), round to nearest even: the
// hardware conversion, identical to f32_to_bf16_rne for every non-NaN input.
__device__ __forceinline__ uint32_t pack_bf16x2_rne(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

}  // namespace packr
