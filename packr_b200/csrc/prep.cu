// Memory-bound helpers around the GEMMs: activation / upstream-gradient
// conversion to bf16 (with optional hi/lo split and column sums), the lut
// gradient and bias gradient finalisation, the 256-bin W_p histogram and the
// stand-alone decode check.
#include "common.cuh"

namespace packr {
namespace prep {

constexpr int kThreads = 256;
constexpr int kRowsPerCta = 32;

// src [R, C] (f32 or bf16, row stride ld_src elements) ->
//   hi[r, c] = bf16(v)           (row stride ld_dst)
//   lo[r, c] = bf16(v - f32(hi))  (optional; v - f32(hi) is exact in f32)
//   colsum[c] += sum over rows of v, in f32 (optional)
// Each thread owns 8 consecutive columns of kRowsPerCta rows.
// Loads one row segment of 8 values (vector path).
template <bool SRC_F32>
__device__ __forceinline__ void load8(const void* src, long long off, float* v) {
  if (SRC_F32) {
    const float4* s = reinterpret_cast<const float4*>(static_cast<const float*>(src) + off);
    const float4 a = __ldcs(s);
    const float4 b = __ldcs(s + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 a = __ldcs(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(src) + off));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
}

// src [R, C] (f32 or bf16, row stride ld_src elements) ->
//   hi[r, c] = bf16(v)           (row stride ld_dst)
//   lo[r, c] = bf16(v - f32(hi))  (optional; v - f32(hi) is exact in f32)
//   colsum[c] += sum over rows of v, in f32 (optional)
// Each thread owns 8 consecutive columns of kRowsPerCta rows; rows go in
// groups of kRowUnroll whose loads are all issued before any is used, so
// every thread keeps several 16-byte loads in flight.
constexpr int kRowUnroll = 4;
template <bool SRC_F32>
__global__ void __launch_bounds__(kThreads) split_rows_kernel(const void* __restrict__ src, long long ld_src, int R,
                                                             int C, uint16_t* __restrict__ hi,
                                                             uint16_t* __restrict__ lo, long long ld_dst,
                                                             float* __restrict__ colsum) {
  const long long c0 = ((long long)blockIdx.x * kThreads + threadIdx.x) * 8;
  if (c0 >= C) return;
  const int r0 = blockIdx.y * kRowsPerCta;
  const int r1 = min(R, r0 + kRowsPerCta);
  const int nc = (int)min(8ll, (long long)C - c0);
  const bool vec = nc == 8 && (ld_src & 7) == 0 && (ld_dst & 7) == 0;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  auto emit = [&](int r, const float* v) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = pack_bf16x2_rne(v[2 * j], v[2 * j + 1]);
      if (lo != nullptr) {
        const float d0 = __fsub_rn(v[2 * j], __uint_as_float(h[j] << 16));
        const float d1 = __fsub_rn(v[2 * j + 1], __uint_as_float(h[j] & 0xFFFF0000u));
        l[j] = pack_bf16x2_rne(d0, d1);
      }
    }
    if (colsum != nullptr) {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], v[j]);
    }
    uint16_t* dh = hi + (long long)r * ld_dst + c0;
    uint16_t* dl = lo != nullptr ? lo + (long long)r * ld_dst + c0 : nullptr;
    if (vec) {
      *reinterpret_cast<uint4*>(dh) = make_uint4(h[0], h[1], h[2], h[3]);
      if (dl) *reinterpret_cast<uint4*>(dl) = make_uint4(l[0], l[1], l[2], l[3]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < nc) {
          dh[j] = (uint16_t)(h[j >> 1] >> (16 * (j & 1)));
          if (dl) dl[j] = (uint16_t)(l[j >> 1] >> (16 * (j & 1)));
        }
      }
    }
  };
  int r = r0;
  if (vec) {
    for (; r + kRowUnroll <= r1; r += kRowUnroll) {
      float v[kRowUnroll][8];
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u) load8<SRC_F32>(src, (long long)(r + u) * ld_src + c0, v[u]);
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u) emit(r + u, v[u]);
    }
  }
  for (; r < r1; ++r) {
    float v[8];
    if (vec) {
      load8<SRC_F32>(src, (long long)r * ld_src + c0, v);
    } else if (SRC_F32) {
      const float* s = static_cast<const float*>(src) + (long long)r * ld_src + c0;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = j < nc ? s[j] : 0.0f;
    } else {
      const uint16_t* s = static_cast<const uint16_t*>(src) + (long long)r * ld_src + c0;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = j < nc ? bf16_to_f32(s[j]) : 0.0f;
    }
    emit(r, v);
  }
  if (colsum != nullptr) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < nc) atomicAdd(colsum + c0 + j, acc[j]);
  }
}

int split_rows(const void* src, int src_f32, long long ld_src, long long R, long long C, uint16_t* hi, uint16_t* lo,
               long long ld_dst, float* colsum, cudaStream_t st) {
  if (R <= 0 || C <= 0) return PACKR_OK;
  if (R > 0x7FFFFFFFll || C > 0x7FFFFFFFll) return PACKR_ERR_SHAPE;
  const long long col_threads = (C + 7) / 8;
  dim3 grid((unsigned)((col_threads + kThreads - 1) / kThreads), (unsigned)((R + kRowsPerCta - 1) / kRowsPerCta));
  if (grid.y > 65535u) return PACKR_ERR_SHAPE;
  if (src_f32)
    split_rows_kernel<true><<<grid, kThreads, 0, st>>>(src, ld_src, (int)R, (int)C, hi, lo, ld_dst, colsum);
  else
    split_rows_kernel<false><<<grid, kThreads, 0, st>>>(src, ld_src, (int)R, (int)C, hi, lo, ld_dst, colsum);
  return launch_status();
}

// dlut[b] = sum[b] / (count[b] + 1e-8)   (reference packr/autograd.py:80-83)
// dbias[n] = bf16(colsum[n])              (autograd of packr/layer.py:97)
__global__ void finalize_kernel(float* __restrict__ dlut, const float* __restrict__ dlut_sum,
                                const int32_t* __restrict__ counts, uint16_t* __restrict__ dbias,
                                const float* __restrict__ colsum, int N) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (dlut != nullptr && i < 256) dlut[i] = __fdiv_rn(dlut_sum[i], __fadd_rn((float)counts[i], 1e-8f));
  if (dbias != nullptr) {
    for (int n = i; n < N; n += gridDim.x * blockDim.x) dbias[n] = (uint16_t)f32_to_bf16_rne(colsum[n]);
  }
}

int finalize(float* dlut, const float* dlut_sum, const int32_t* counts, uint16_t* dbias, const float* colsum,
             long long N, cudaStream_t st) {
  if (dlut == nullptr && dbias == nullptr) return PACKR_OK;
  long long work = dbias != nullptr ? (N > 256 ? N : 256) : 256;
  int blocks = (int)((work + 255) / 256);
  if (blocks > 4 * sm_count()) blocks = 4 * sm_count();
  finalize_kernel<<<blocks, 256, 0, st>>>(dlut, dlut_sum, counts, dbias, colsum, (int)N);
  return launch_status();
}

// 256-bin histogram of bytes: per-warp shared-memory sub-histograms, one
// global atomic per bin per CTA.
__global__ void __launch_bounds__(kThreads) bincount256_kernel(const uint8_t* __restrict__ p, long long n,
                                                              int32_t* __restrict__ counts) {
  __shared__ int h[kThreads / 32][256];
  const int w = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (kThreads / 32) * 256; i += kThreads) (&h[0][0])[i] = 0;
  __syncthreads();
  const bool vec = aligned(p, 16);
  const long long stride = (long long)gridDim.x * kThreads;
  if (vec) {
    const long long nv = n / 16;
    for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < nv; i += stride) {
      const uint4 q = __ldcs(reinterpret_cast<const uint4*>(p) + i);
      const uint32_t ws[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int b = 0; b < 4; ++b) atomicAdd(&h[w][(ws[k] >> (8 * b)) & 0xFF], 1);
    }
    for (long long i = nv * 16 + (long long)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride)
      atomicAdd(&h[w][p[i]], 1);
  } else {
    for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) atomicAdd(&h[w][p[i]], 1);
  }
  __syncthreads();
  for (int b = threadIdx.x; b < 256; b += kThreads) {
    int s = 0;
#pragma unroll
    for (int k = 0; k < kThreads / 32; ++k) s += h[k][b];
    if (s) atomicAdd(counts + b, s);
  }
}

int bincount256(const uint8_t* p, long long n, int32_t* counts, cudaStream_t st) {
  if (cudaMemsetAsync(counts, 0, 256 * sizeof(int32_t), st) != cudaSuccess) return PACKR_ERR_CUDA;
  if (n == 0) return PACKR_OK;
  long long want = (n / 16 + kThreads - 1) / kThreads;
  int blocks = (int)(want < 2 * sm_count() ? (want > 0 ? want : 1) : 2 * sm_count());
  bincount256_kernel<<<blocks, kThreads, 0, st>>>(p, n, counts);
  return launch_status();
}

}  // namespace prep
}  // namespace packr
