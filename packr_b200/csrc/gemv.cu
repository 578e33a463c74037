// Forward for very few rows (decode-bound; used up to 4 tokens, built for up
// to 16): out = x @ W + bias
// with W decoded exactly as the reference's forward decodes it,
// W = f32(W_f) + f32(fp16(lut[W_p])) (packr/kernel.py:127-130), and an f32
// accumulation on the CUDA cores.  At these sizes the work is streaming W
// once from HBM (3 bytes per weight); a 256-row tensor-core tile would waste
// almost all of its rows, and the fused decode GEMM can only spread N/256
// tiles over the SMs.
//
// Pass 1 (gemv_partial_kernel): CTA (column block, K split); each of its 8
// warps owns 32 * CPT columns and walks every row of the split for them.  Per
// row a lane loads CPT W_f values and CPT W_p bytes with one vector load each
// (the next group of rows in flight while one is used), looks the bytes up in
// a lane-replicated shared copy of the fp16-rounded lut (bank-conflict free),
// and accumulates x[m, k] * W[k, n] for every m in packed f32 pairs, x[:,
// split] staged in shared memory as f32.  The sums of each split go to
// partial[split][m][n].  Pass 2 (gemv_reduce_kernel) adds the splits in a
// fixed order and the bias: the result does not depend on timing.
#include "common.cuh"

#include <cuda_fp16.h>

namespace packr {
namespace gemv {

// Packed pairs of f32 (first element in the low half) with the sm_100 f32x2
// fma; each half is rounded exactly as the scalar fma.rn.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pk2(float a, float b) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(f32x2 v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRowUnroll = 4;
constexpr int kMaxM = 16;

// Vector loads of CPT consecutive W_f (bf16) and W_p (u8) values.
template <int CPT>
struct WVec;
template <>
struct WVec<8> {
  uint4 f;
  uint2 p;
  __device__ __forceinline__ void load(const uint16_t* wf, const uint8_t* wp) {
    f = __ldcs(reinterpret_cast<const uint4*>(wf));
    p = __ldcs(reinterpret_cast<const uint2*>(wp));
  }
  __device__ __forceinline__ uint32_t fword(int i) const { return i == 0 ? f.x : i == 1 ? f.y : i == 2 ? f.z : f.w; }
  __device__ __forceinline__ uint32_t pword(int i) const { return i == 0 ? p.x : p.y; }
};
template <>
struct WVec<4> {
  uint2 f;
  uint32_t p;
  __device__ __forceinline__ void load(const uint16_t* wf, const uint8_t* wp) {
    f = __ldcs(reinterpret_cast<const uint2*>(wf));
    p = __ldcs(reinterpret_cast<const unsigned int*>(wp));
  }
  __device__ __forceinline__ uint32_t fword(int i) const { return i == 0 ? f.x : f.y; }
  __device__ __forceinline__ uint32_t pword(int) const { return p; }
};

template <>
struct WVec<2> {
  uint32_t f;
  uint32_t p;
  __device__ __forceinline__ void load(const uint16_t* wf, const uint8_t* wp) {
    f = __ldcs(reinterpret_cast<const unsigned int*>(wf));
    p = __ldcs(reinterpret_cast<const unsigned short*>(wp));
  }
  __device__ __forceinline__ uint32_t fword(int) const { return f; }
  __device__ __forceinline__ uint32_t pword(int) const { return p; }
};

// Dynamic shared memory: lut copy [256][32] u32 | x [rows][M] as (x, x) f32
// pairs, ready to be the packed multiplier of fma.rn.f32x2.
// M is a compile-time bound on the rows; Mr <= M rows are real (x rows past
// Mr read as zero and their sums are not written).  Warp w of the CTA owns
// the 32 * CPT columns starting at (blockIdx.x * 8 + w) * 32 * CPT and walks
// every row of the CTA's K range for them, kRowUnroll rows per load group
// with the next group in flight; its sums go straight to the partial array.
template <int M, int CPT, int U>
__global__ void __launch_bounds__(kThreads, (M <= 2 ? 4 : 3))
    gemv_partial_kernel(const void* __restrict__ x, int x_f32, int Mr, const uint8_t* __restrict__ W_p,
                        const uint16_t* __restrict__ W_f, const float* __restrict__ lut,
                        float* __restrict__ partial, int K, int N, int rows_per_split) {
  extern __shared__ __align__(16) uint32_t gsm[];
  uint32_t* lut_s = gsm;                                 // 256 * 32
  f32x2* xs = reinterpret_cast<f32x2*>(gsm + 256 * 32);  // rows_per_split * M
  constexpr int kStrip = 32 * CPT;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k0 = blockIdx.y * rows_per_split;
  const int k1 = min(K, k0 + rows_per_split);
  const int nrows = k1 - k0;
  for (int e = warp; e < 256; e += kWarps)
    lut_s[e * 32 + lane] = __float_as_uint(__half2float(__float2half_rn(__ldg(lut + e))));
  for (int i = threadIdx.x; i < nrows * M; i += kThreads) {
    const int r = i / M, m = i - r * M;
    const long long src = (long long)m * K + k0 + r;
    const float v = m >= Mr ? 0.0f
                            : x_f32 ? __ldg(static_cast<const float*>(x) + src)
                                    : bf16_to_f32(__ldg(static_cast<const uint16_t*>(x) + src));
    xs[i] = pk2(v, v);
  }
  __syncthreads();

  const long long n0 = ((long long)blockIdx.x * kWarps + warp) * kStrip + lane * CPT;
  if (n0 >= N) return;  // N % CPT == 0: a chunk is whole or absent
  const uint32_t* lut_lane = lut_s + lane;
  // accumulators as packed pairs of adjacent columns (fma.rn.f32x2 rounds
  // each half exactly as the scalar fma would)
  f32x2 acc[M][CPT / 2];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int j = 0; j < CPT / 2; ++j) acc[m][j] = 0ull;

  auto consume = [&](const WVec<CPT>& w, int r) {
    f32x2 wv[CPT / 2];
#pragma unroll
    for (int j = 0; j < CPT / 2; ++j) {
      const uint32_t fw = w.fword(j);
      const uint32_t pw = w.pword(j >> 1) >> (16 * (j & 1));
      const float f0 = __fadd_rn(__uint_as_float(fw << 16), __uint_as_float(lut_lane[(pw & 0xFFu) * 32]));
      const float f1 = __fadd_rn(__uint_as_float(fw & 0xFFFF0000u), __uint_as_float(lut_lane[((pw >> 8) & 0xFFu) * 32]));
      wv[j] = pk2(f0, f1);
    }
    const f32x2* xr = xs + r * M;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const f32x2 x2 = xr[m];
#pragma unroll
      for (int j = 0; j < CPT / 2; ++j) acc[m][j] = fma2(x2, wv[j], acc[m][j]);
    }
  };
  auto load_group = [&](WVec<CPT>* w, int r) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (r + u < nrows) {
        const long long off = (long long)(k0 + r + u) * N + n0;
        w[u].load(W_f + off, W_p + off);
      }
    }
  };
  WVec<CPT> cur[U], nxt[U];
  load_group(cur, 0);
  for (int r = 0; r < nrows; r += U) {
    load_group(nxt, r + U);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (r + u < nrows) consume(cur[u], r + u);
#pragma unroll
    for (int u = 0; u < U; ++u) cur[u] = nxt[u];
  }
  float* dst = partial + (long long)blockIdx.y * Mr * N + n0;
#pragma unroll
  for (int m = 0; m < M; ++m) {
    if (m < Mr) {
#pragma unroll
      for (int j = 0; j < CPT / 2; ++j) {
        float a0, a1;
        upk2(acc[m][j], a0, a1);
        *reinterpret_cast<float2*>(dst + (long long)m * N + 2 * j) = make_float2(a0, a1);
      }
    }
  }
}

// out[m, n] = sum over splits of partial[s][m][n] + bias[n], in a fixed
// order: warp w of the CTA sums splits w, w+8, ... (four loads in flight),
// then the 8 warp sums are added in warp order.  One CTA per 32 columns of
// one row m.
__global__ void __launch_bounds__(256) gemv_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N,
                                                         const void* __restrict__ bias, int bias_f32,
                                                         float* __restrict__ out, long long ld_out) {
  __shared__ float red[kWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m = blockIdx.y;
  const long long n = (long long)blockIdx.x * 32 + lane;
  float s = 0.0f;
  if (n < N) {
    const float* p = partial + (long long)m * N + n;
    const long long step = (long long)M * N;
    int sp = warp;
    for (; sp + 3 * kWarps < splits; sp += 4 * kWarps) {
      const float a = __ldcs(p + sp * step), b = __ldcs(p + (sp + kWarps) * step);
      const float c = __ldcs(p + (sp + 2 * kWarps) * step), d = __ldcs(p + (sp + 3 * kWarps) * step);
      s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, a), b), c), d);
    }
    for (; sp < splits; sp += kWarps) s = __fadd_rn(s, __ldcs(p + sp * step));
  }
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && n < N) {
    float t = red[0][lane];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) t = __fadd_rn(t, red[w][lane]);
    if (bias != nullptr)
      t = __fadd_rn(t, bias_f32 ? __ldg(static_cast<const float*>(bias) + n)
                                : bf16_to_f32(__ldg(static_cast<const uint16_t*>(bias) + n)));
    out[(long long)m * ld_out + n] = t;
  }
}

struct Plan {
  int mb;  // compile-time row bound used for M
  int cpt, splits, rows_per_split;
  size_t smem;
};

inline int row_bound(long long M) { return M <= 2 ? (int)M : M <= 4 ? 4 : M <= 8 ? 8 : M <= 12 ? 12 : 16; }

// Columns per thread: 8 for one row (one 16-byte W_f load), 4 up to 8 rows,
// 2 beyond (the accumulators of 12-16 rows would cost occupancy).  K is split so that the grid is about one wave of
// `resident` CTAs per SM, with the partial sums (splits x M x N f32) at most
// about a tenth of W's bytes and the x slice of a split (8 bytes per value)
// at most 32 KB.
inline Plan plan(long long M, long long K, long long N, int resident = 8) {
  Plan p{};
  p.mb = row_bound(M);
  p.cpt = (N % 8 == 0 && p.mb <= 1) ? 8 : p.mb >= 12 ? 2 : 4;
  const long long col_blocks = (N + (long long)kWarps * 32 * p.cpt - 1) / ((long long)kWarps * 32 * p.cpt);
  long long splits = ((long long)resident * sm_count() + col_blocks - 1) / col_blocks;
  long long cap = (3 * K) / (40 * M);  // partial bytes <= ~W bytes / 10
  if (cap < 1) cap = 1;
  if (splits > cap) splits = cap;
  const long long min_splits = (K * p.mb * 8 + 32767) / 32768;  // x slice <= 32 KB
  if (splits < min_splits) splits = min_splits;
  if (splits > K) splits = K;
  if (splits < 1) splits = 1;
  const long long rows = (K + splits - 1) / splits;
  p.rows_per_split = (int)rows;
  p.splits = (int)((K + rows - 1) / rows);
  p.smem = 256 * 32 * 4 + (size_t)rows * p.mb * 8;
  return p;
}

// Usable for this problem: few rows, W rows whole vector chunks, aligned bases.
inline bool eligible(long long M, long long K, long long N, const uint8_t* W_p, const uint16_t* W_f) {
  if (M < 1 || M > kMaxM || (N % 4) != 0 || K < 1) return false;
  const Plan p = plan(M, K, N);
  const uintptr_t va = 2 * p.cpt;  // bytes of one W_f chunk
  return aligned(W_f, va) && aligned(W_p, va / 2);
}

// Upper bound over the resident count (at most 8 CTAs of 256 threads per SM).
inline size_t workspace_bytes(long long M, long long K, long long N) {
  const Plan p = plan(M, K, N, 8);
  return (size_t)p.splits * M * N * sizeof(float);
}

template <int M, int CPT, int U = 4>
int launch_m(Plan p, const void* x, int x_f32, int Mr, const uint8_t* W_p, const uint16_t* W_f,
             const float* lut, float* partial, long long K, long long N, cudaStream_t st, int* splits_out) {
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    if (cudaFuncSetAttribute(gemv_partial_kernel<M, CPT, U>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
        cudaSuccess)
      return PACKR_ERR_CUDA;
    attr_done[dev & 63] = 1;
  }
  // one wave: the most CTAs per SM whose own plan (its x slice in shared
  // memory) still lets that many be resident
  for (int c = 8; c >= 1; --c) {
    const Plan q = plan((long long)Mr, K, N, c);
    int fit = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&fit, gemv_partial_kernel<M, CPT, U>, kThreads, q.smem) !=
        cudaSuccess) {
      cudaGetLastError();
      fit = 0;
    }
    p = q;
    if (fit >= c) break;
  }
  *splits_out = p.splits;
  dim3 grid((unsigned)((N + kWarps * 32 * CPT - 1) / (kWarps * 32 * CPT)), (unsigned)p.splits);
  gemv_partial_kernel<M, CPT, U><<<grid, kThreads, p.smem, st>>>(x, x_f32, Mr, W_p, W_f, lut, partial, (int)K,
                                                                 (int)N, p.rows_per_split);
  return launch_status();
}

template <int M>
int launch_cpt(const Plan& p, const void* x, int x_f32, int Mr, const uint8_t* W_p, const uint16_t* W_f,
               const float* lut, float* partial, long long K, long long N, cudaStream_t st) {
  int splits = 0;
  int rc;
  if constexpr (M == 1) {
    if (p.cpt == 8) {
      rc = launch_m<M, 8>(p, x, x_f32, Mr, W_p, W_f, lut, partial, K, N, st, &splits);
      return rc == PACKR_OK ? splits : -rc;
    }
  }
  if constexpr (M >= 12) {
    rc = launch_m<M, 2>(p, x, x_f32, Mr, W_p, W_f, lut, partial, K, N, st, &splits);
  } else {
    rc = launch_m<M, 4>(p, x, x_f32, Mr, W_p, W_f, lut, partial, K, N, st, &splits);
  }
  return rc == PACKR_OK ? splits : -rc;
}

int forward(const void* x, int x_f32, const uint8_t* W_p, const uint16_t* W_f, const float* lut, const void* bias,
            int bias_f32, float* out, long long M, long long K, long long N, float* partial, cudaStream_t st) {
  const Plan p = plan(M, K, N);
  const int Mr = (int)M;
  int rc;
  switch (p.mb) {
    case 1: rc = launch_cpt<1>(p, x, x_f32, Mr, W_p, W_f, lut, partial, K, N, st); break;
    case 2: rc = launch_cpt<2>(p, x, x_f32, Mr, W_p, W_f, lut, partial, K, N, st); break;
    case 4: rc = launch_cpt<4>(p, x, x_f32, Mr, W_p, W_f, lut, partial, K, N, st); break;
    case 8: rc = launch_cpt<8>(p, x, x_f32, Mr, W_p, W_f, lut, partial, K, N, st); break;
    case 12: rc = launch_cpt<12>(p, x, x_f32, Mr, W_p, W_f, lut, partial, K, N, st); break;
    default: rc = launch_cpt<16>(p, x, x_f32, Mr, W_p, W_f, lut, partial, K, N, st); break;
  }
  if (rc <= 0) return -rc;  // launch_cpt returns the split count, or -status
  gemv_reduce_kernel<<<dim3((unsigned)((N + 31) / 32), (unsigned)M), 256, 0, st>>>(partial, rc, (int)M, (int)N, bias,
                                                                                   bias_f32, out, N);
  return launch_status();
}

}  // namespace gemv
}  // namespace packr
