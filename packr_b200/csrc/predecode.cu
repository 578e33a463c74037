// Streaming decode of the packed weight, W = bf16(W_f + bf16(lut[W_p]))
// (packr/autograd.py:66-67), into a row-major bf16 [K, N] array.  For large
// token counts the FWD and DX GEMMs read this array by TMA instead of
// decoding each weight tile once per 512-row output tile: the decode then
// costs one HBM pass (3 bytes in, 2 bytes out per weight) and the GEMM's
// shared memory serves only the tensor cores.
//
// HBM-bound: each thread decodes 8 consecutive weights per chunk (one 16-byte
// W_f load, one 8-byte W_p load, one 16-byte store), kUnroll chunks in flight;
// the lut sits in a lane-replicated shared-memory copy as in the GEMM's decode
// warps, and the add is the same add.rn.bf16x2, so both decodes give the same
// bits.  W_f and W_p are read with the evict-first hint so that the decoded
// array stays in L2 for the GEMM that follows.
#include <atomic>

#include "common.cuh"

namespace packr {
namespace gemm {

constexpr int kPredecodeThreads = 256;
constexpr int kPredecodeUnroll = 8;

__device__ __forceinline__ uint4 decode8(const uint4 f, const uint2 w, const uint32_t* lut_lane) {
  const uint32_t ww[2] = {w.x, w.y};
  const uint32_t ff[4] = {f.x, f.y, f.z, f.w};
  uint32_t r[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t word = ww[p >> 1];
    const int sh = 16 * (p & 1);
    const uint32_t l0 = lut_lane[((word >> sh) & 0xFFu) * 32];
    const uint32_t l1 = lut_lane[((word >> (sh + 8)) & 0xFFu) * 32];
    r[p] = bf16x2_add(ff[p], prmt(l0, l1, 0x5410u));
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// chunks = K * N / 8; chunk c covers weights 8c .. 8c + 7 of the row-major W.
__global__ void __launch_bounds__(kPredecodeThreads) predecode_kernel(const uint2* __restrict__ W_p,
                                                                      const uint4* __restrict__ W_f,
                                                                      const float* __restrict__ lut,
                                                                      uint4* __restrict__ out, long long chunks) {
  __shared__ uint32_t lut_s[256 * 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = warp; e < 256; e += kPredecodeThreads / 32) lut_s[e * 32 + lane] = f32_to_bf16_rne(__ldg(lut + e));
  __syncthreads();
  const uint32_t* lut_lane = lut_s + lane;
  const long long stride = (long long)gridDim.x * kPredecodeThreads;
  long long c = (long long)blockIdx.x * kPredecodeThreads + threadIdx.x;
  for (; c + (kPredecodeUnroll - 1) * stride < chunks; c += kPredecodeUnroll * stride) {
    uint4 f[kPredecodeUnroll];
    uint2 w[kPredecodeUnroll];
#pragma unroll
    for (int u = 0; u < kPredecodeUnroll; ++u) {
      f[u] = __ldcs(W_f + c + u * stride);
      w[u] = __ldcs(W_p + c + u * stride);
    }
#pragma unroll
    for (int u = 0; u < kPredecodeUnroll; ++u) out[c + u * stride] = decode8(f[u], w[u], lut_lane);
  }
  for (; c < chunks; c += stride) out[c] = decode8(__ldcs(W_f + c), __ldcs(W_p + c), lut_lane);
}

// out: [K, N] bf16, row-major, 16-byte aligned.  Requires N % 16 == 0 and
// 16-byte aligned W_p / W_f (the layout the TMA-fed GEMMs require as well).
int predecode(const uint8_t* W_p, const uint16_t* W_f, const float* lut, uint16_t* out, long long K, long long N,
              cudaStream_t st) {
  if (!wtma_ok(W_p, W_f, N) || !aligned(out, 16)) return PACKR_ERR_ALIGNMENT;
  const long long chunks = K * N / 8;
  if (chunks == 0) return PACKR_OK;
  // as many resident blocks as fit (smem, registers), one wave: the loop
  // strides over the chunks.  Blocks per SM are cached per device (relaxed
  // atomics: concurrent first calls store the same value).
  static std::atomic<int> per_sm[64];
  int dev = 0;
  cudaGetDevice(&dev);
  int n = per_sm[dev & 63].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, predecode_kernel, kPredecodeThreads, 0) != cudaSuccess || n < 1)
      n = 4;
    per_sm[dev & 63].store(n, std::memory_order_relaxed);
  }
  const long long want = (chunks + kPredecodeThreads - 1) / kPredecodeThreads;
  const long long cap = (long long)n * sm_count();
  predecode_kernel<<<(int)(want < cap ? want : cap), kPredecodeThreads, 0, st>>>(
      reinterpret_cast<const uint2*>(W_p), reinterpret_cast<const uint4*>(W_f), lut, reinterpret_cast<uint4*>(out),
      chunks);
  return launch_status();
}

}  // namespace gemm
}  // namespace packr
