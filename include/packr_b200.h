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
 *     attribute cache, the device-side wait-timeout word read by
 *     packr_device_status(), and the static scratch array (with its cached
 *     per-device address) of packr_backward_static_scratch, the one entry
 *     point that brings its own workspace.
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
#define PACKR_DTYPE_F16 2 /* weights of packr_from_linear_encode only */

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

/* packr_adam8_multi that also stores every updated parameter value into
 * n_peers (0..7) other copies of the same tensor: peer_p[i * n_peers + q] is
 * tensor i's p in the memory of another GPU of this node (a pointer from
 * packr_ipc_open, plus the tensor's offset in that buffer).  The data-parallel
 * optimizer uses it to replace the parameter all-gather: each process updates
 * its 1/N shard and writes it into every other process's parameter buffer in
 * the same kernel.  The kernel ends with a system-scope fence; the caller
 * still needs a barrier (e.g. a one-element all-reduce on `stream`) before
 * other GPUs read the values.  The reference has no counterpart (it has no
 * distributed code; it replaces no reference interface). */
int packr_adam8_multi_push(const packr_adam_tensor* tensors, int n_tensors, void* const* peer_p,
                           int n_peers, float lr, float beta1, float beta2, float eps, float bc1,
                           float bc2, float weight_decay, void* stream);

/* Buffers shared between the processes of one node (CUDA IPC).  An IPC
 * handle names a whole cudaMalloc allocation, hence packr_device_alloc.
 * packr_ipc_open maps another process's buffer into this process on the
 * current device (peer access enabled on first use); packr_ipc_close unmaps
 * it.  Host-side calls, synchronous.  No counterpart in the reference. */
#define PACKR_IPC_HANDLE_BYTES 64
int packr_device_alloc(size_t bytes, void** ptr);
int packr_device_free(void* ptr);
int packr_ipc_export(const void* ptr, void* handle /* PACKR_IPC_HANDLE_BYTES */);
int packr_ipc_open(const void* handle, void** ptr);
int packr_ipc_close(void* ptr);

/* Self-check of the short correctly rounded sequences packr_adam8_multi uses
 * on most blocks, against CUDA's IEEE operations, on the current device:
 * mismatches (device, 4 x u64) = [0] reciprocals over every positive normal
 * argument with a normal result, [1] square roots over every argument in
 * [2^-100, 2^128), [2] quotients on 2^30 pseudo-random pairs, [3] the whole
 * parameter update on 2^30 pseudo-random moments.  All four are 0 on a
 * correct device.  No counterpart in the reference.  A few milliseconds. */
int packr_selfcheck_rounding(unsigned long long* mismatches, void* stream);

/* ---- PackRLinear ---------------------------------------------------------
 * out[M,N] (f32) = x[M,K] @ W + bias,  W = bf16(W_f + bf16(lut[W_p])),
 * computed on the tensor cores with x and W as bf16 operands and an f32
 * accumulator.  Below 129 rows W is decoded tile by tile in shared memory
 * and never written to HBM; from 129 rows on (N % 16 == 0, 16-byte aligned
 * W_p / W_f) W is decoded once into the workspace and read back by TMA,
 * provided the workspace holds it (packr_forward_workspace_bytes counts it;
 * a smaller workspace that fits the fused route selects that route).  For
 * 5..128 rows (N % 16 == 0) W is streamed once through a tcgen05 GEMM that
 * takes 128 weight columns as the MMA's rows and the tokens as its N, split
 * over K; up to 4 rows (N % 4 == 0, 8-byte aligned W_p) through the CUDA
 * cores, decoding as the reference's forward does (f32(W_f) +
 * f32(fp16(lut[W_p]))) with f32 accumulation.
 * x is bf16 or f32 (f32 x is rounded to bf16 in the workspace first).
 * bias: [N] of bias_dtype (bf16 or f32, added in f32 in the epilogue) or
 * NULL.  M = 0 is a no-op; K, N >= 1.
 * Replaces packr_matmul(x, W_p, W_f, lut, bias) of reference
 * packr/kernel.py:98-141 plus the bias add of packr/layer.py:96-97.
 */
size_t packr_forward_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype);
int packr_forward(const void* x, int x_dtype, const uint8_t* W_p, const uint16_t* W_f, const float* lut,
                  const void* bias, int bias_dtype, float* out, int64_t M, int64_t K, int64_t N, void* workspace,
                  size_t workspace_bytes, void* stream);

/* The forward GEMM over a W already decoded to bf16 [K, N] (for example by
 * packr_predecode_bf16, cached by a caller that runs many forwards with the
 * same weights): out = x @ Wd + bias, same x / bias / out conventions as
 * packr_forward.  N % 8 == 0 and Wd 16-byte aligned.  No counterpart in the
 * reference (it decodes inside every packr_matmul call). */
size_t packr_forward_decoded_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype);
int packr_forward_decoded(const void* x, int x_dtype, const uint16_t* Wd, const void* bias, int bias_dtype,
                          float* out, int64_t M, int64_t K, int64_t N, void* workspace, size_t workspace_bytes,
                          void* stream);

/* Backward of the forward above; replaces PackRMatmulFunction.backward of
 * reference packr/autograd.py:56-88 and the bias gradient of layer.py:97:
 *   dX[M,K]   = bf16(bf16(dY) @ W^T)      stored as x's dtype (NULL: skipped)
 *   dW_f[K,N] = bf16(x^T @ dY)             fp32 accumulate     (NULL: skipped)
 *   dlut[256] = sum_{W_p==b} (x^T @ dY) / (count[b] + 1e-8)     (NULL: skipped)
 *   dbias[N]  = bf16(sum_m dY)                                  (NULL: skipped)
 * dY is the f32 upstream gradient [M,N].  lut_counts = bincount(W_p, 256)
 * (packr_bincount256; W_p is frozen, so callers cache it) or NULL to count
 * here.  flags: PACKR_BWD_DW_SPLIT makes the dW product fp32-faithful by
 * splitting dY (and an f32 x) into bf16 hi + lo parts (x.dY_hi + x.dY_lo
 * [+ x_lo.dY_hi]); without it dY is rounded to bf16 as the reference does for
 * dX.  A workspace of packr_backward_workspace_bytes(M, K, N, x_dtype, flags)
 * bytes (256-byte aligned) holds bf16(dY), its split parts, a bf16 copy of an
 * f32 x, the partial sums and, for dX from 129 rows on, the decoded W (the
 * same route choice as packr_forward). */
#define PACKR_BWD_DW_SPLIT 1
size_t packr_backward_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype, int flags);
int packr_backward(const float* dY, const void* x, int x_dtype, const uint8_t* W_p, const uint16_t* W_f,
                   const float* lut, const int32_t* lut_counts, void* dX, uint16_t* dW_f, float* dlut,
                   uint16_t* dbias, int64_t M, int64_t K, int64_t N, int flags, void* workspace,
                   size_t workspace_bytes, void* stream);

/* counts[b] = number of bytes equal to b in W_p[0..n) (the
 * torch.bincount(W_p, minlength=256) of reference packr/autograd.py:80). */
int packr_bincount256(const uint8_t* W_p, int64_t n, int32_t* counts, void* stream);

/* dlut[b] = dlut_sum[b] / (counts[b] + 1e-8)  (reference autograd.py:83). */
int packr_lut_finalize(float* dlut, const float* dlut_sum, const int32_t* counts, void* stream);

/* out[K,N] = bf16(W_f + bf16(lut[W_p])) through the GEMM's own decode path
 * (reference packr/autograd.py:66-67); for bit-exactness checks. */
int packr_decode_bf16(const uint8_t* W_p, const uint16_t* W_f, const float* lut, uint16_t* out, int64_t K,
                      int64_t N, void* stream);

/* out[K,N] = bf16(W_f + bf16(lut[W_p])) by the streaming decode kernel that
 * feeds the plain GEMMs (same bits as packr_decode_bf16).  N % 16 == 0;
 * W_p, W_f and out 16-byte aligned. */
int packr_predecode_bf16(const uint8_t* W_p, const uint16_t* W_f, const float* lut, uint16_t* out, int64_t K,
                         int64_t N, void* stream);

/* Backward with the caller's decoded W (Wd [K, N] bf16, 16-byte aligned,
 * equal to packr_predecode_bf16(W_p, W_f, lut)): where packr_backward would
 * predecode W for the plain dX GEMM (M >= 129, N % 16 == 0, 16-byte aligned
 * W_p / W_f) it uses Wd instead; otherwise Wd is ignored.  A forward that
 * predecodes (packr_predecode_bf16 + packr_forward_decoded, which is what
 * packr_forward runs on the same route) can keep its W for the backward and
 * save one decode pass.  Same results as packr_backward; workspace from
 * packr_backward_decoded_workspace_bytes (no decoded-W buffer in it).  No
 * counterpart in the reference (it decodes in both passes,
 * packr/kernel.py:127-130 and packr/autograd.py:66-67). */
size_t packr_backward_decoded_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype, int flags);
int packr_backward_decoded(const float* dY, const void* x, int x_dtype, const uint8_t* W_p, const uint16_t* W_f,
                           const float* lut, const uint16_t* Wd, const int32_t* lut_counts, void* dX,
                           uint16_t* dW_f, float* dlut, uint16_t* dbias, int64_t M, int64_t K, int64_t N,
                           int flags, void* workspace, size_t workspace_bytes, void* stream);
/* 1 when packr_forward takes its predecode route for this problem (given a
 * workspace of packr_forward_workspace_bytes), else 0. */
int packr_predecode_route(int64_t M, int64_t K, int64_t N, const uint8_t* W_p, const uint16_t* W_f);

/* ---- PackRLinear.from_linear (reference packr/layer.py:106-159) ----------
 * Step 1: the rank_lo-th and rank_hi-th smallest |w| (0-based; rank_hi is
 * rank_lo or rank_lo + 1) of n weights (f32 or bf16), as f32, written to
 * out2[0..1] on the device: the two order statistics torch.quantile
 * interpolates (layer.py:127), found by an exact radix select without
 * sorting and without torch.quantile's 2^24-element limit.  Workspace of
 * packr_abs_order_stats_workspace_bytes(), 16-byte aligned. */
size_t packr_abs_order_stats_workspace_bytes(void);
int packr_abs_order_stats(const void* w, int dtype, int64_t n, int64_t rank_lo, int64_t rank_hi,
                          float* out2, void* workspace, size_t workspace_bytes, void* stream);
/* Step 2: weight [out_features, in_features] (nn.Linear layout, f32, bf16 or
 * f16) -> W_p u8 and W_f bf16 [in_features, out_features], lut f32 [256]:
 * t = clamp(w * target_scale, -1.6, 1.6) (rounded to the weight's type for
 * bf16 / f16, the clamp bounds too),
 * W_p = the nearest codebook entry (lowest index on ties; layer.py:137-141),
 * lut = codebook / scale (layer.py:144), W_f = bf16(w - lut[W_p])
 * (layer.py:148).  codebook (256 f32), scale and target_scale (1 f32 each;
 * target_scale may be NULL = scale) on the device. */
int packr_from_linear_encode(const void* weight, int dtype, int64_t out_features, int64_t in_features,
                             const float* codebook, const float* scale, const float* target_scale,
                             uint8_t* W_p, uint16_t* W_f, float* lut, void* stream);

/* ---- VelvetController support ---------------------------------------------
 * sums[i] (double, device) = sum of parameter i's int8 second-moment codes,
 * each times its block's v_scale when block_size > 0, unweighted when
 * block_size == 0 (reference packr/velvet.py:270-300
 * takes the mean of the [blocks, block_size] view, or of the raw codes when
 * that view would need padding; the caller divides by numel).  One launch for
 * all parameters (the reference reads one `.item()` per parameter). */
typedef struct packr_vsum_desc {
  const int8_t* v;
  const float* v_scale;  /* used when block_size > 0 */
  int64_t numel;
  int64_t block_size;    /* 0: sum of the raw codes */
  int64_t block_origin;  /* element i is scaled by v_scale[(block_origin + i) / block_size] */
} packr_vsum_desc;
int packr_state_v_sums(const packr_vsum_desc* descs, int n, double* sums, void* stream);

/* packr_backward without a caller-provided workspace, for callers that cannot
 * allocate device memory (a host runtime with a fixed device-memory budget
 * and no allocator of its own, a binding that can pass tensors it was given
 * but cannot obtain a temporary buffer).  No counterpart in the reference.
 * Same arguments and results as packr_backward minus the workspace: the
 * scratch is one static device array of PACKR_STATIC_SCRATCH_BYTES per GPU,
 * held from the library's load until process exit.  Problems whose scratch
 * need exceeds that size return PACKR_ERR_WORKSPACE before any launch (the
 * need for bf16 x without PACKR_BWD_DW_SPLIT is about M*round8(N)*2 bytes).
 * Within the array the backward takes the fastest route whose scratch fits,
 * exactly as packr_backward does with a workspace of that size: for dX the
 * decode-first route (W decoded into the array, K*N*2 more bytes, plus the
 * stream-K partial tiles when those fit too) from 129 rows on, otherwise
 * the GEMM that decodes W in shared memory.
 * The first successful call on each device looks up the array's device
 * address (make it before any stream capture; a failed lookup is retried by
 * the next call).  Every call shares the array and finds the previous call's
 * contents there; calls that overlap on the GPU (different streams,
 * different threads) race on it. */
#define PACKR_STATIC_SCRATCH_BYTES (32u << 20)
int packr_backward_static_scratch(const float* dY, const void* x, int x_dtype, const uint8_t* W_p,
                                  const uint16_t* W_f, const float* lut, const int32_t* lut_counts, void* dX,
                                  uint16_t* dW_f, float* dlut, uint16_t* dbias, int64_t M, int64_t K, int64_t N,
                                  int flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PACKR_B200_H */
