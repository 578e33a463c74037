// Forward for very few rows (decode-bound; used up to 4 tokens, built for up
// to 16): out = x @ W + bias
// with W decoded exactly as the reference's forward decodes it,
// W = f32(W_f) + f32(fp16(lut[W_p])) (packr/kernel.py:127-130), and an f32
// accumulation on the CUDA cores.  At these sizes the work is streaming W
// once from HBM (3 bytes per weight); a 128-row tensor-core tile would waste
// almost all of its rows.
//
// One launch (gemv_cluster_kernel): a CTA owns 32 * CPT columns (each lane
// CPT adjacent columns, loaded with one vector load of W_f and one of W_p per
// row) and a K range; its 8 warps split that range, each streaming its rows
// with the next group of rows in flight, looking the bytes up in a
// lane-replicated shared copy of the fp16-rounded lut (bank-conflict free)
// and accumulating x[m, k] * W[k, n] for every m in packed f32 pairs (x of
// the CTA's range staged in shared memory).  The C CTAs of a thread-block
// cluster (C = 8 or 16) split K for the same columns.  The sums are combined
// in a fixed order (the 8 warps in order inside a CTA, then the C CTAs in
// rank order through distributed shared memory, each CTA finishing a 1/C
// slice of the columns and adding the bias), so the result does not depend
// on timing and no partial sums go through global memory.
//
// gemv_reduce_kernel (a fixed-order sum of split partials plus the bias) is
// the final pass of the skinny tensor-core forward.
#include <atomic>

#include "common.cuh"
#include "sm100.cuh"

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

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Dynamic shared memory: lut copy [256][32] u32 (reused for the 8 warps'
// sums [8][MB][32 * CPT] f32 after the stream) | x [rows][MB] as (x, x) f32
// pairs | this CTA's sums [MB][32 * CPT] f32.  MB is a compile-time bound
// on the rows; Mr <= MB rows are real (rows past Mr read x as zero and are
// not written).
template <int MB, int CPT>
__host__ __device__ constexpr size_t cluster_smem(int rows_per_cta) {
  return 256 * 32 * 4 + (size_t)rows_per_cta * MB * 8 + (size_t)MB * 32 * CPT * 4;
}

#ifndef PACKR_GEMV_ROWS_IN_FLIGHT
#define PACKR_GEMV_ROWS_IN_FLIGHT 4
#endif
#ifndef PACKR_GEMV_MIN_CTAS
#define PACKR_GEMV_MIN_CTAS 3
#endif
template <int MB, int CPT, int U>
__global__ void __launch_bounds__(kThreads, (MB <= 2 ? PACKR_GEMV_MIN_CTAS : 2))
    gemv_cluster_kernel(const void* __restrict__ x, int x_f32, int Mr, const uint8_t* __restrict__ W_p,
                        const uint16_t* __restrict__ W_f, const float* __restrict__ lut,
                        const void* __restrict__ bias, int bias_f32, float* __restrict__ out, int K, int N,
                        int rows_per_cta, int rows_per_warp) {
  static_assert(8 * MB * 32 * CPT <= 256 * 32, "warp sums must fit in the lut region");
  static_assert(kThreads == 256, "one lut entry per thread");
  constexpr int kCols = 32 * CPT;
  extern __shared__ __align__(16) uint32_t gsm[];
  uint32_t* lut_s = gsm;                                   // 256 * 32
  float* red = reinterpret_cast<float*>(gsm);              // [8][MB][kCols], after the stream
  f32x2* xs = reinterpret_cast<f32x2*>(gsm + 256 * 32);    // rows_per_cta * MB
  float* part = reinterpret_cast<float*>(gsm + 256 * 32 + 2 * rows_per_cta * MB);  // [MB][kCols]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int C = (int)gridDim.y;  // one cluster spans the K splits of a column block
  const int rank = (int)sm100::cluster_ctarank();
  const int k0 = rank * rows_per_cta;
  const int k1 = min(K, k0 + rows_per_cta);
  const int nrows_cta = max(0, k1 - k0);
  {
    // thread t loads lut[t] once and writes its 32 lane copies, rotated so
    // that the warp's stores fall in 32 different banks
    const uint32_t v = __float_as_uint(__half2float(__float2half_rn(__ldg(lut + threadIdx.x))));
#pragma unroll 8
    for (int l = 0; l < 32; ++l) lut_s[threadIdx.x * 32 + ((l + lane) & 31)] = v;
  }
  for (int i = threadIdx.x; i < nrows_cta * MB; i += kThreads) {
    const int r = i / MB, m = i - r * MB;
    const long long src = (long long)m * K + k0 + r;
    const float v = m >= Mr ? 0.0f
                            : x_f32 ? __ldg(static_cast<const float*>(x) + src)
                                    : bf16_to_f32(__ldg(static_cast<const uint16_t*>(x) + src));
    xs[i] = pk2(v, v);
  }
  __syncthreads();

  const long long n0 = (long long)blockIdx.x * kCols + lane * CPT;
  const bool live = n0 < N;  // N % CPT == 0: a lane's columns are whole or absent
  const int r0 = warp * rows_per_warp;  // rows of this warp, relative to k0
  const int r1 = min(nrows_cta, r0 + rows_per_warp);
  const uint32_t* lut_lane = lut_s + lane;
  f32x2 acc[MB][CPT / 2];
#pragma unroll
  for (int m = 0; m < MB; ++m)
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
    const f32x2* xr = xs + r * MB;
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      const f32x2 x2 = xr[m];
#pragma unroll
      for (int j = 0; j < CPT / 2; ++j) acc[m][j] = fma2(x2, wv[j], acc[m][j]);
    }
  };
  // Rows of this warp in groups of U, loads of the next group in flight
  // while one is consumed (ping-pong buffers, row pointers advanced by N).
  if (live && r1 > r0) {
    const long long base = (long long)(k0 + r0) * N + n0;
    const uint16_t* pf = W_f + base;
    const uint8_t* pp = W_p + base;
    const int full = (r1 - r0) / U;  // whole groups
    auto load = [&](WVec<CPT>* w) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        w[u].load(pf, pp);
        pf += N;
        pp += N;
      }
    };
    auto eat = [&](const WVec<CPT>* w, int r) {
#pragma unroll
      for (int u = 0; u < U; ++u) consume(w[u], r + u);
    };
    int r = r0;
    WVec<CPT> a[U], b[U];
    if (full > 0) {
      load(a);
      int g = 1;
      for (; g + 1 < full; g += 2) {
        load(b);
        eat(a, r);
        r += U;
        load(a);
        eat(b, r);
        r += U;
      }
      if (g < full) {
        load(b);
        eat(a, r);
        r += U;
        eat(b, r);
        r += U;
      } else {
        eat(a, r);
        r += U;
      }
    }
    for (; r < r1; ++r) {  // the last rows, one at a time
      WVec<CPT> t;
      t.load(pf, pp);
      pf += N;
      pp += N;
      consume(t, r);
    }
  }
  __syncthreads();  // every warp is done with the lut and x copies
#pragma unroll
  for (int m = 0; m < MB; ++m)
#pragma unroll
    for (int j = 0; j < CPT / 2; ++j) {
      float a0, a1;
      upk2(acc[m][j], a0, a1);
      *reinterpret_cast<float2*>(&red[(warp * MB + m) * kCols + lane * CPT + 2 * j]) = make_float2(a0, a1);
    }
  __syncthreads();
  for (int i = threadIdx.x; i < MB * kCols; i += kThreads) {
    float t = red[i];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) t = __fadd_rn(t, red[w * MB * kCols + i]);
    part[i] = t;
  }
  cluster_sync_all();  // every CTA's sums are visible to the cluster
  // CTA `rank` finishes columns [rank * kCols / C, (rank + 1) * kCols / C)
  const int c_lo = rank * kCols / C;
  const int per = (rank + 1) * kCols / C - c_lo;
  const uint32_t part_s = sm100::smem_u32(part);
  for (int i = threadIdx.x; i < MB * per; i += kThreads) {
    const int m = i / per, c = c_lo + (i - m * per);
    const long long n = (long long)blockIdx.x * kCols + c;
    float t = 0.0f;
    for (int q = 0; q < C; ++q) t = __fadd_rn(t, ld_cluster_f32(sm100::mapa(part_s + 4u * (uint32_t)(m * kCols + c), q)));
    if (m < Mr && n < N) {
      if (bias != nullptr)
        t = __fadd_rn(t, bias_f32 ? __ldg(static_cast<const float*>(bias) + n)
                                  : bf16_to_f32(__ldg(static_cast<const uint16_t*>(bias) + n)));
      out[(long long)m * N + n] = t;
    }
  }
  cluster_sync_all();  // no CTA leaves while a peer may still read its sums
}

// out[m, n] = sum over splits of partial[s][m][n] (added in split order
// 0, 1, ...) + bias[n].  One thread per 4 consecutive columns of one row:
// 16-byte loads of the splits, four in flight, and one 16-byte store where
// N and the output allow it.
__global__ void __launch_bounds__(256) gemv_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N,
                                                         const void* __restrict__ bias, int bias_f32,
                                                         float* __restrict__ out, long long ld_out) {
  const long long qpr = (N + 3) / 4;  // column quads per row
  const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= (long long)M * qpr) return;
  const int m = (int)(q / qpr);
  const int n = (int)(q - (long long)m * qpr) * 4;
  const int nv = min(4, N - n);
  const long long step = (long long)M * N;
  const float* p = partial + (long long)m * N + n;
  float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (nv == 4 && (N & 3) == 0) {  // partial rows are 16-byte aligned
    auto add4 = [&](const float4 v) {
      s[0] = __fadd_rn(s[0], v.x);
      s[1] = __fadd_rn(s[1], v.y);
      s[2] = __fadd_rn(s[2], v.z);
      s[3] = __fadd_rn(s[3], v.w);
    };
    int sp = 0;
    for (; sp + 4 <= splits; sp += 4) {
      const float4 a = __ldcs(reinterpret_cast<const float4*>(p + sp * step));
      const float4 b = __ldcs(reinterpret_cast<const float4*>(p + (sp + 1) * step));
      const float4 c = __ldcs(reinterpret_cast<const float4*>(p + (sp + 2) * step));
      const float4 d = __ldcs(reinterpret_cast<const float4*>(p + (sp + 3) * step));
      add4(a);
      add4(b);
      add4(c);
      add4(d);
    }
    for (; sp < splits; ++sp) add4(__ldcs(reinterpret_cast<const float4*>(p + sp * step)));
  } else {
    for (int sp = 0; sp < splits; ++sp)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j < nv) s[j] = __fadd_rn(s[j], __ldcs(p + sp * step + j));
  }
  if (bias != nullptr) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < nv)
        s[j] = __fadd_rn(s[j], bias_f32 ? __ldg(static_cast<const float*>(bias) + n + j)
                                        : bf16_to_f32(__ldg(static_cast<const uint16_t*>(bias) + n + j)));
  }
  float* o = out + (long long)m * ld_out + n;
  if (nv == 4 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
    *reinterpret_cast<float4*>(o) = make_float4(s[0], s[1], s[2], s[3]);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < nv) o[j] = s[j];
  }
}

// Grid of gemv_reduce_kernel for M rows of N columns.
inline unsigned reduce_blocks(long long M, long long N) { return (unsigned)((M * ((N + 3) / 4) + 255) / 256); }

inline int row_bound(long long M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16; }

struct Plan {
  int mb, cpt, cluster, rows_per_cta, rows_per_warp;
  long long col_blocks;
  size_t smem;
};

// Columns per lane: 8 up to 4 rows (16-byte W_f loads), 4 for 8 rows, 2 for
// 16 (more accumulators would cost occupancy); 4 or 2 when N needs it.
// Cluster size C (CTAs along K, at most 16, at least 64 rows each): measured
// on B200 over the Llama FFN shapes, the stream runs fastest with about 2.35
// CTAs per SM for one or two rows (e.g. 43 column blocks x 8 for 4096 ->
// 11008, 16 x 16 for 11008 -> 4096) and about 1.75 for four (at most 12
// along K): more CTAs per SM lengthen the start and the reduction more than
// they add to the stream.
inline Plan plan(long long M, long long K, long long N) {
  Plan p{};
  p.mb = row_bound(M);
  const int pref = p.mb <= 4 ? 8 : p.mb <= 8 ? 4 : 2;
  p.cpt = N % pref == 0 ? pref : (N % 4 == 0 && pref > 4 ? 4 : (N % 2 == 0 ? 2 : 0));
  if (p.cpt == 0) return p;
  p.col_blocks = (N + 32LL * p.cpt - 1) / (32LL * p.cpt);
  const double per_sm = p.mb <= 2 ? 2.35 : 1.75;
  const int cmax = p.mb <= 2 ? 16 : 12;
  long long c = (long long)(per_sm * sm_count() / (double)p.col_blocks);
  c = c < 1 ? 1 : (c > cmax ? cmax : c);
  while (c > 1 && K < 64LL * c) --c;
  p.cluster = (int)c;
  if (p.cpt == 0) return p;
  p.rows_per_cta = (int)((K + p.cluster - 1) / p.cluster);
  p.rows_per_warp = (p.rows_per_cta + kWarps - 1) / kWarps;
  return p;
}

// Usable for this problem: few rows, whole vector chunks, aligned bases, and
// the x slice of a CTA in shared memory.
inline bool eligible(long long M, long long K, long long N, const uint8_t* W_p, const uint16_t* W_f) {
  if (M < 1 || M > kMaxM || K < 1 || N < 2 || K > 0x7FFFFFFFLL || N > 0x7FFFFFFFLL) return false;
  const Plan p = plan(M, K, N);
  if (p.cpt == 0 || (long long)p.rows_per_cta * p.mb * 8 > 96 * 1024) return false;
  const uintptr_t va = 2 * p.cpt;  // bytes of one W_f chunk
  return aligned(W_f, va) && aligned(W_p, va / 2);
}

inline size_t workspace_bytes(long long, long long, long long) { return 0; }

template <int MB, int CPT, int U = PACKR_GEMV_ROWS_IN_FLIGHT>
int launch(const Plan& p, const void* x, int x_f32, int Mr, const uint8_t* W_p, const uint16_t* W_f, const float* lut,
           const void* bias, int bias_f32, float* out, long long K, long long N, cudaStream_t st) {
  auto kern = gemv_cluster_kernel<MB, CPT, U>;
  // per-device flag; relaxed atomics: concurrent first calls set the same attributes
  static std::atomic<int> attr_done[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
      return PACKR_ERR_CUDA;
    attr_done[dev & 63].store(1, std::memory_order_relaxed);
  }
  Plan q = p;
  for (;;) {
    q.rows_per_cta = (int)((K + q.cluster - 1) / q.cluster);
    q.rows_per_warp = (q.rows_per_cta + kWarps - 1) / kWarps;
    q.smem = cluster_smem<MB, CPT>(q.rows_per_cta);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)q.col_blocks, (unsigned)q.cluster, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = q.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)q.cluster;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      clusters = 0;
    }
    if (clusters < 1 && q.cluster > 1) {  // a cluster this large does not fit: shrink it
      q.cluster -= 1;
      continue;
    }
    if (cudaLaunchKernelEx(&cfg, kern, x, x_f32, Mr, W_p, W_f, lut, bias, bias_f32, out, (int)K, (int)N,
                           q.rows_per_cta, q.rows_per_warp) != cudaSuccess)
      return launch_status();
    return launch_status();
  }
}

template <int MB>
int launch_cpt(const Plan& p, const void* x, int x_f32, int Mr, const uint8_t* W_p, const uint16_t* W_f,
               const float* lut, const void* bias, int bias_f32, float* out, long long K, long long N,
               cudaStream_t st) {
  if constexpr (MB <= 4) {
    if (p.cpt == 8) return launch<MB, 8>(p, x, x_f32, Mr, W_p, W_f, lut, bias, bias_f32, out, K, N, st);
  }
  if constexpr (MB <= 8) {
    if (p.cpt == 4) return launch<MB, 4>(p, x, x_f32, Mr, W_p, W_f, lut, bias, bias_f32, out, K, N, st);
  }
  return launch<MB, 2>(p, x, x_f32, Mr, W_p, W_f, lut, bias, bias_f32, out, K, N, st);
}

int forward(const void* x, int x_f32, const uint8_t* W_p, const uint16_t* W_f, const float* lut, const void* bias,
            int bias_f32, float* out, long long M, long long K, long long N, float* /*unused*/, cudaStream_t st) {
  const Plan p = plan(M, K, N);
  const int Mr = (int)M;
  switch (p.mb) {
    case 1: return launch_cpt<1>(p, x, x_f32, Mr, W_p, W_f, lut, bias, bias_f32, out, K, N, st);
    case 2: return launch_cpt<2>(p, x, x_f32, Mr, W_p, W_f, lut, bias, bias_f32, out, K, N, st);
    case 4: return launch_cpt<4>(p, x, x_f32, Mr, W_p, W_f, lut, bias, bias_f32, out, K, N, st);
    case 8: return launch_cpt<8>(p, x, x_f32, Mr, W_p, W_f, lut, bias, bias_f32, out, K, N, st);
    default: return launch_cpt<16>(p, x, x_f32, Mr, W_p, W_f, lut, bias, bias_f32, out, K, N, st);
  }
}

}  // namespace gemv
}  // namespace packr
