/*
 * packr_b200.h — C ABI of libpackr_b200.so, the sm_100a (B200) kernels behind
 * PackR's training hot path.
 *
 * Conventions (every entry point):
 *   - The caller owns every buffer.  No entry point allocates device memory;
 *     temporaries live in a caller-provided workspace whose size is returned
 *     by the matching *_workspace_bytes() query.
 *   - All pointers are device pointers of the current CUDA device.
 *   - Work is enqueued asynchronously on `stream` (a cudaStream_t passed as
 *     void*; NULL is the legacy default stream).  Nothing synchronises.
 *   - Return 0 (PACKR_OK) or a PACKR_ERR_* code; nothing aborts the process.
 *     packr_error_string() names the code.
 *   - Sizes are 64-bit.  bf16 tensors are passed as uint16_t bit patterns.
 *   - W_p and W_f are [K, N] row-major (in_features x out_features), exactly
 *     as PackRLinear stores them (reference packr/layer.py:53-59).
 *   - No entry point keeps mutable global state except the per-device
 *     attribute cache and the device-side wait-timeout word read by
 *     packr_device_status().
 */
#ifndef PACKR_B200_H
#define PACKR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define PACKR_OK 0
#define PACKR_ERR_INVALID_ARGUMENT 1 /* null pointer, bad dtype, bad hyper-parameter */
#define PACKR_ERR_SHAPE 2            /* a size is negative or exceeds a kernel limit */
#define PACKR_ERR_ALIGNMENT 3        /* a pointer or row stride breaks a 16-byte TMA rule */
#define PACKR_ERR_WORKSPACE 4        /* workspace missing or smaller than required */
#define PACKR_ERR_LAUNCH 5           /* the CUDA launch itself failed */
#define PACKR_ERR_DEVICE 6           /* current device is not sm_100 */
#define PACKR_ERR_TIMEOUT 7          /* a bounded device-side wait gave up */
#define PACKR_ERR_CUDA 8             /* another CUDA runtime/driver error */

/* ---- dtypes ------------------------------------------------------------ */
#define PACKR_DTYPE_F32 0
#define PACKR_DTYPE_BF16 1

const char* packr_error_string(int code);
int packr_abi_version(void);

/* Reads (and clears) the device-side wait-timeout word on the current
 * device.  Synchronises `stream`.  Returns PACKR_OK or PACKR_ERR_TIMEOUT. */
int packr_device_status(void* stream);

/* ---- 8-bit block-absmax AdamW -------------------------------------------
 * One parameter tensor: p/g are bf16 or f32 (dtype), m/v are int8 with one
 * f32 scale per 256-element block of the flat view (ceil(numel/256) scales).
 * Replaces the pybind binding launch_adam_8bit(p, g, m, v, ms, vs, is_bf16,
 * lr, b1, b2, eps, bc1, bc2, wd) of reference packr/cuda_adam_kernel.cu:72-88
 * (called once per parameter by packr/cuda_adam.py:178-192); here one call
 * updates every tensor of a parameter group.
 */
typedef struct packr_adam_tensor {
  void* p;            /* [numel] bf16 or f32, updated in place           */
  const void* g;      /* [numel] same dtype as p                          */
  int8_t* m;          /* [numel] int8 first moment codes                  */
  int8_t* v;          /* [numel] int8 second moment codes, in [1,127]     */
  float* m_scale;     /* [ceil(numel/256)] block scales of m              */
  float* v_scale;     /* [ceil(numel/256)] block scales of v              */
  int64_t numel;
  int32_t dtype;      /* PACKR_DTYPE_BF16 or PACKR_DTYPE_F32              */
  int32_t reserved;   /* must be 0                                        */
} packr_adam_tensor;

/* bc1 = 1 - beta1^t and bc2 = 1 - beta2^t, as the caller computes them
 * (reference packr/cuda_adam.py:175-176). */
int packr_adam8_multi(const packr_adam_tensor* tensors, int n_tensors, float lr,
                      float beta1, float beta2, float eps, float bc1, float bc2,
                      float weight_decay, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PACKR_B200_H */
