// PackRLinear.from_linear on the GPU (reference packr/layer.py:106-159).
//
//   q99   = torch.quantile(|W|, 0.99) + 1e-6          (layer.py:127)
//   scale = 1.6 / q99                                  (:128)
//   t     = clamp(W * scale, -1.6, 1.6)                (:129; for a bf16 or f16
//           W the product is rounded to the weight's type and the
//           multiplier is the one torch uses, passed as target_scale)
//   W_p   = argmin_i |t - codebook[i]| (first index)   (:137-141)
//   lut   = codebook / scale                           (:144)
//   W_f   = bf16(W - lut[W_p])                         (:148)
// with W = weight^T ([in, out]; weight is nn.Linear's [out, in]).
//
// The quantile needs two order statistics of |W| (ranks floor and ceil of
// 0.99 (n - 1)); torch.quantile sorts the whole tensor and refuses more than
// 2^24 elements.  packr_abs_order_stats finds them by an exact radix select
// on the f32 bit patterns of |w| (for non-negative floats the bit patterns
// order like the values): histogram passes over the weight (the exponent,
// then 12 and 11 mantissa bits; two passes suffice for bf16), each followed
// by a one-CTA scan that picks the bin holding the rank, and at most one more
// pass for the smallest key above the first statistic.  The caller interpolates exactly as torch.quantile does.
//
// packr_from_linear_encode makes the one pass that writes W_p, W_f and lut:
// 64 x 64 tiles of the weight are transposed through shared memory, and the
// nearest codebook entry is found without the reference's 256 distance
// computations per weight.  Once per CTA, the distinct codebook values (170
// of 256) are sorted with the lowest index of each; only the two values
// around t can be nearest (|RN(t - v)| is monotone in the distance, so no
// farther entry can tie with them), and between two neighbours the choice,
// including torch.argmin's lowest-index rule on a tie, switches at one float
// found by bisection.  Per weight this leaves one 8-byte bucket record (a
// bucket is 2^-9 wide, two boundaries are at least 0.0066 apart, so a bucket
// holds at most one) and one comparison against its threshold.
#include <cuda_fp16.h>

#include "common.cuh"

namespace packr {
namespace compress {

constexpr int kBins = 4096;
constexpr int kHistThreads = 256;

struct SelectState {
  unsigned int prefix;       // key bits fixed so far
  unsigned int mask;         // which bits of prefix are fixed
  long long rank;            // rank of the first statistic within the keys matching prefix
  long long rank_hi_delta;   // 1 if the second statistic is the next rank, else 0
  unsigned int key_lo;
  unsigned int key_hi;
  unsigned int need_min;     // 1: key_hi is the smallest key > key_lo, found by min_greater_kernel
  unsigned int min_greater;  // atomicMin target
  unsigned int hist[kBins];
};

__device__ __forceinline__ unsigned int abs_key_f32(float x) { return __float_as_uint(x) & 0x7FFFFFFFu; }
__device__ __forceinline__ unsigned int abs_key_bf16(unsigned short h) { return ((unsigned int)h & 0x7FFFu) << 16; }

// Digits of a key (bit 31 is 0): D=0 the exponent, bits 30..23; D=1 bits
// 22..11; D=2 bits 10..0.  A bf16 key has bits 15..0 zero, so it is fixed
// after D=1.
template <int D>
struct Digit {
  static constexpr int kShift = D == 0 ? 23 : (D == 1 ? 11 : 0);
  static constexpr unsigned int kMask = D == 0 ? 0xFFu : (D == 1 ? 0xFFFu : 0x7FFu);
  static constexpr int kBins = (int)kMask + 1;
};

// Streams the keys of w through fn(key, valid) with every lane of every warp
// taking part in each call (16-byte loads where the base allows).
template <bool BF16, class F>
__device__ __forceinline__ void for_each_key(const void* w, long long n, F&& fn) {
  const long long stride = (long long)gridDim.x * kHistThreads;
  const long long me = (long long)blockIdx.x * kHistThreads + threadIdx.x;
  if constexpr (BF16) {
    const unsigned short* p = static_cast<const unsigned short*>(w);
    const long long n8 = (reinterpret_cast<uintptr_t>(p) & 15) == 0 ? n / 8 : 0;
    const long long iters = (n8 + stride - 1) / stride;
    for (long long it = 0; it < iters; ++it) {
      const long long i = it * stride + me;
      uint4 q = make_uint4(0, 0, 0, 0);
      const bool ok = i < n8;
      if (ok) q = __ldcs(reinterpret_cast<const uint4*>(p) + i);
      const unsigned int ws[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        fn(abs_key_bf16((unsigned short)(ws[k] & 0xFFFFu)), ok);
        fn(abs_key_bf16((unsigned short)(ws[k] >> 16)), ok);
      }
    }
    const long long tail0 = n8 * 8;
    const long long titers = (n - tail0 + stride - 1) / stride;
    for (long long it = 0; it < titers; ++it) {
      const long long i = tail0 + it * stride + me;
      fn(i < n ? abs_key_bf16(p[i]) : 0u, i < n);
    }
  } else {
    const float* p = static_cast<const float*>(w);
    const long long n4 = (reinterpret_cast<uintptr_t>(p) & 15) == 0 ? n / 4 : 0;
    const long long iters = (n4 + stride - 1) / stride;
    for (long long it = 0; it < iters; ++it) {
      const long long i = it * stride + me;
      float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
      const bool ok = i < n4;
      if (ok) q = __ldcs(reinterpret_cast<const float4*>(p) + i);
      fn(abs_key_f32(q.x), ok);
      fn(abs_key_f32(q.y), ok);
      fn(abs_key_f32(q.z), ok);
      fn(abs_key_f32(q.w), ok);
    }
    const long long tail0 = n4 * 4;
    const long long titers = (n - tail0 + stride - 1) / stride;
    for (long long it = 0; it < titers; ++it) {
      const long long i = tail0 + it * stride + me;
      fn(i < n ? abs_key_f32(p[i]) : 0u, i < n);
    }
  }
}

// D=0: the exponent histogram.  Most weights share a few exponents, so each
// lane counts into its own column (bin * 32 + lane): no two lanes of a warp
// ever hit the same shared-memory word.
template <bool BF16>
__global__ void __launch_bounds__(kHistThreads) hist_exp_kernel(const void* __restrict__ w, long long n,
                                                                SelectState* __restrict__ st) {
  __shared__ unsigned int sh[256 * 32];
  for (int i = threadIdx.x; i < 256 * 32; i += kHistThreads) sh[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for_each_key<BF16>(w, n, [&](unsigned int key, bool ok) {
    if (ok) atomicAdd(&sh[(key >> 23) * 32 + lane], 1u);
  });
  __syncthreads();
  for (int b = threadIdx.x; b < 256; b += kHistThreads) {
    unsigned int c = 0;
#pragma unroll 8
    for (int l = 0; l < 32; ++l) c += sh[b * 32 + ((l + b) & 31)];
    if (c) atomicAdd(&st->hist[b], c);
  }
}

// D=1, 2: keys matching the prefix; these are spread over many bins.
template <int D, bool BF16>
__global__ void __launch_bounds__(kHistThreads) hist_kernel(const void* __restrict__ w, long long n,
                                                            SelectState* __restrict__ st) {
  __shared__ unsigned int sh[Digit<D>::kBins];
  for (int i = threadIdx.x; i < Digit<D>::kBins; i += kHistThreads) sh[i] = 0;
  __syncthreads();
  const unsigned int prefix = st->prefix, mask = st->mask;
  for_each_key<BF16>(w, n, [&](unsigned int key, bool ok) {
    if (ok && (key & mask) == prefix) atomicAdd(&sh[(key >> Digit<D>::kShift) & Digit<D>::kMask], 1u);
  });
  __syncthreads();
  for (int i = threadIdx.x; i < Digit<D>::kBins; i += kHistThreads)
    if (sh[i]) atomicAdd(&st->hist[i], sh[i]);
}

// One CTA of 1024 threads: the bin holding `rank`, then the prefix and the
// rank inside it for the next digit.  After the last digit (LAST): key_lo,
// and key_hi when it lies in the same histogram.
template <int D, bool LAST>
__global__ void __launch_bounds__(1024) select_kernel(SelectState* __restrict__ st) {
  constexpr int kPer = (Digit<D>::kBins + 1023) / 1024;  // bins per thread
  __shared__ long long part[1024];
  const int t = threadIdx.x;
  unsigned long long h[kPer];
  unsigned long long sum = 0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int b = t * kPer + k;
    h[k] = b < Digit<D>::kBins ? st->hist[b] : 0;
    sum += h[k];
  }
  part[t] = (long long)sum;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const long long v = t >= o ? part[t - o] : 0;
    __syncthreads();
    part[t] += v;
    __syncthreads();
  }
  const long long r = st->rank;
  long long before = part[t] - (long long)sum;
  int bin = -1;
  long long below = 0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    if (bin < 0 && r >= before && r < before + (long long)h[k]) {
      bin = t * kPer + k;
      below = before;
    }
    before += (long long)h[k];
  }
  __syncthreads();  // every thread has read st->hist and st->rank
  if (bin >= 0) {
    const unsigned int prefix = st->prefix | ((unsigned int)bin << Digit<D>::kShift);
    st->prefix = prefix;
    st->mask |= Digit<D>::kMask << Digit<D>::kShift;
    st->rank = r - below;
    if constexpr (LAST) {
      st->key_lo = prefix;
      const long long cnt = (long long)st->hist[bin];
      if (st->rank_hi_delta == 0 || r + 1 < below + cnt) {
        st->key_hi = prefix;
        st->need_min = 0;
      } else {
        unsigned int nxt = 0xFFFFFFFFu;
        for (int b = bin + 1; b < Digit<D>::kBins; ++b)
          if (st->hist[b]) {
            nxt = (prefix & ~(Digit<D>::kMask << Digit<D>::kShift)) | ((unsigned int)b << Digit<D>::kShift);
            break;
          }
        st->key_hi = nxt;
        st->need_min = nxt == 0xFFFFFFFFu ? 1u : 0u;
      }
    }
  }
  __syncthreads();
  for (int i = t; i < kBins; i += 1024) st->hist[i] = 0;
}

template <bool BF16>
__global__ void __launch_bounds__(kHistThreads) min_greater_kernel(const void* __restrict__ w, long long n,
                                                                   SelectState* __restrict__ st) {
  if (!st->need_min) return;
  const unsigned int lo = st->key_lo;
  unsigned int best = 0xFFFFFFFFu;
  for_each_key<BF16>(w, n, [&](unsigned int key, bool ok) {
    if (ok && key > lo && key < best) best = key;
  });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xFFFFFFFFu, best, o));
  if ((threadIdx.x & 31) == 0 && best != 0xFFFFFFFFu) atomicMin(&st->min_greater, best);
}

__global__ void finish_kernel(SelectState* __restrict__ st, float* __restrict__ out2) {
  const unsigned int hi = st->need_min ? st->min_greater : st->key_hi;
  out2[0] = __uint_as_float(st->key_lo);
  out2[1] = __uint_as_float(hi);
}

// ---------------------------------------------------------------- encode

constexpr int kTile = 64;
constexpr int kEncThreads = 256;
constexpr int kBuckets = 2048;      // width 2^-9 over [-2, 2): bucket of t = floor(t * 512) + 1024, exact
// Tile element (row ro of the weight, column ci) sits at ro * 64 + (ci ^ swz(ro)),
// swz(ro) = 8 * ((ro >> 4) & 3): the transposed reads (lane (r, q): row
// 16q + c, column r) are free of bank conflicts; 16-byte groups stay whole.
__device__ __forceinline__ int tile_at(int ro, int ci) { return ro * 64 + (ci ^ (((ro >> 4) & 3) << 3)); }

// Nearest-codebook choice as cells of t.  With v_0 < ... < v_{U-1} the
// distinct codebook values (each with its lowest index), the entry chosen for
// t in [v_p, v_{p+1}] is p+1 exactly when |RN(t - v_{p+1})| < |RN(t - v_p)|,
// or they are equal and p+1 has the lower index; both distances are monotone
// in t, so the choice switches once, at a boundary B_p found by bisection
// over the floats between v_p and v_{p+1}.  Cell j = [B_{j-1}, B_j).  Each
// bucket records the cell of its lower edge, the boundary inside it (if any)
// and the cell above that boundary; a bucket with two boundaries (not the
// case for the reference codebook, whose boundaries are >= 0.0066 apart)
// is marked and its weights search the boundaries.
struct EncodeSm {
  float cb[256];
  float dq[256];              // lut = codebook / scale, by codebook index
  float val[256];             // distinct values, ascending
  int vidx[256];              // lowest codebook index of each
  unsigned char first[256];
  float bnd[258];             // bnd[j + 1] = B_j; bnd[0] = -inf, bnd[U] = +inf
  float2 bucket[kBuckets];    // (threshold, idx_lo | idx_hi << 8 | multi << 16)
  int u;
};

__device__ __forceinline__ int ord_of(float x) {
  const int b = __float_as_int(x);
  return b >= 0 ? b : -(b & 0x7FFFFFFF);
}
__device__ __forceinline__ float float_of_ord(int o) {
  return o >= 0 ? __int_as_float(o) : __int_as_float((-o) | (int)0x80000000);
}

// cell of t: the largest j with bnd[j] <= t
__device__ __forceinline__ int cell_of(const EncodeSm& S, float t, int U) {
  int lo = 0, hi = U - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (S.bnd[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void encode_setup(EncodeSm& S, const float* __restrict__ codebook, float scale,
                                             float* __restrict__ lut) {
  const int tid = threadIdx.x;
  {
    const float v = codebook[tid];
    S.cb[tid] = v;
    S.dq[tid] = __fdiv_rn(v, scale);
    if (blockIdx.x == 0) lut[tid] = S.dq[tid];
  }
  __syncthreads();
  {
    const float v = S.cb[tid];
    bool first = true;
    for (int j = 0; j < tid; ++j) first &= S.cb[j] != v;
    S.first[tid] = first;
  }
  __syncthreads();
  {
    const float v = S.cb[tid];
    int rank = 0;
    for (int j = 0; j < 256; ++j) rank += (S.first[j] && S.cb[j] < v) ? 1 : 0;
    if (S.first[tid]) {
      S.val[rank] = v;
      S.vidx[rank] = tid;
    }
    const int u = __syncthreads_count(S.first[tid]);
    if (tid == 0) S.u = u;
  }
  __syncthreads();
  const int U = S.u;
  if (tid == 0) {
    S.bnd[0] = -INFINITY;
    S.bnd[U] = INFINITY;
  }
  if (tid + 1 < U) {
    const float a = S.val[tid], b = S.val[tid + 1];
    const int ia = S.vidx[tid], ib = S.vidx[tid + 1];
    auto takes_b = [&](float t) {
      const float d0 = fabsf(__fsub_rn(t, a)), d1 = fabsf(__fsub_rn(t, b));
      return d1 < d0 || (d1 == d0 && ib < ia);
    };
    int lo = ord_of(a), hi = ord_of(b);  // takes_b(lo) false, takes_b(hi) true
    for (int guard = 0; guard < 40 && hi - lo > 1; ++guard) {
      const int mid = lo + (hi - lo) / 2;
      if (takes_b(float_of_ord(mid))) hi = mid; else lo = mid;
    }
    S.bnd[tid + 1] = float_of_ord(hi);
  }
  __syncthreads();
  for (int b = tid; b < kBuckets; b += kEncThreads) {
    const float e_lo = (float)(b - kBuckets / 2) * 0x1p-9f, e_hi = (float)(b + 1 - kBuckets / 2) * 0x1p-9f;
    const int j = cell_of(S, e_lo, U);
    float thr = INFINITY;
    int jh = j, multi = 0;
    if (j + 1 < U && S.bnd[j + 1] < e_hi) {
      thr = S.bnd[j + 1];
      jh = j + 1;
      multi = (j + 2 < U && S.bnd[j + 2] < e_hi) ? 1 : 0;
    }
    S.bucket[b] = make_float2(thr, __int_as_float(S.vidx[j] | (S.vidx[jh] << 8) | (multi << 16)));
  }
  __syncthreads();
}

// Weight element types of the encode pass.
enum WType { W_F32 = 0, W_BF16 = 1, W_F16 = 2 };

// A 16-bit weight (bits in the low half) as the f32 it equals exactly.
template <int WT>
__device__ __forceinline__ float half_to_f32(unsigned int h) {
  if constexpr (WT == W_BF16) return __uint_as_float(h << 16);
  return __half2float(__ushort_as_half((unsigned short)h));
}

template <int WT>
__global__ void __launch_bounds__(kEncThreads) encode_kernel(const void* __restrict__ weight, long long out_f,
                                                             long long in_f, const float* __restrict__ codebook,
                                                             const float* __restrict__ scale_p,
                                                             const float* __restrict__ target_scale_p,
                                                             uint8_t* __restrict__ W_p, uint16_t* __restrict__ W_f,
                                                             float* __restrict__ lut) {
  constexpr bool BF16 = WT == W_BF16;
  constexpr bool HALF = WT != W_F32;  // 16-bit weights
  __shared__ EncodeSm S;
  __shared__ __align__(16) float tile[kTile * kTile];
  const int tid = threadIdx.x;
  const float tscale = *target_scale_p;
  encode_setup(S, codebook, *scale_p, lut);
  const int U = S.u;

  const long long tiles_i = (in_f + kTile - 1) / kTile, tiles_o = (out_f + kTile - 1) / kTile;
  const long long ntiles = tiles_i * tiles_o;
  constexpr int kVec = HALF ? 8 : 4;  // elements per 16-byte load
  const bool vec_rows = (in_f % kVec) == 0 && (reinterpret_cast<uintptr_t>(weight) & 15) == 0;
  for (long long tl = blockIdx.x; tl < ntiles; tl += gridDim.x) {
    const long long i0 = (tl % tiles_i) * kTile;  // in (columns of weight)
    const long long o0 = (tl / tiles_i) * kTile;  // out (rows of weight)
    // load: thread -> row r = tid / 4 of the weight, columns c0 .. c0 + 15,
    // c0 = 16 (tid % 4): 16-byte loads, 16-byte shared stores
    {
      const int r = tid >> 2, c0 = 16 * (tid & 3);
      const long long o = o0 + r, i = i0 + c0;
      float v[16];
      if (o < out_f && vec_rows && i + 16 <= in_f) {
        if constexpr (HALF) {
          const uint4* src = reinterpret_cast<const uint4*>(static_cast<const unsigned short*>(weight) + o * in_f + i);
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const uint4 q = __ldcs(src + k);
            const unsigned int ws[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              v[8 * k + 2 * e] = half_to_f32<WT>(ws[e] & 0xFFFFu);
              v[8 * k + 2 * e + 1] = half_to_f32<WT>(ws[e] >> 16);
            }
          }
        } else {
          const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(weight) + o * in_f + i);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 q = __ldcs(src + k);
            v[4 * k] = q.x;
            v[4 * k + 1] = q.y;
            v[4 * k + 2] = q.z;
            v[4 * k + 3] = q.w;
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          v[c] = 0.0f;
          if (o < out_f && i + c < in_f)
            v[c] = HALF ? half_to_f32<WT>(static_cast<const unsigned short*>(weight)[o * in_f + i + c])
                        : static_cast<const float*>(weight)[o * in_f + i + c];
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k)
        *reinterpret_cast<float4*>(&tile[tile_at(r, c0 + 4 * k)]) = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
    }
    __syncthreads();
    // encode: thread -> in row r = tid / 4, out columns c0 = 16 (tid % 4)
    // .. c0 + 15 (four lanes write 64 contiguous W_p bytes of a row)
    {
      const int r = tid >> 2, c0 = 16 * (tid & 3);
      const long long i = i0 + r;
      uint32_t pb[4], pf[8];
#pragma unroll
      for (int c = 0; c < 16; c += 2) {
        float res[2];
        int idx[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float w = tile[tile_at(c0 + c + h, r)];
          float t;
          if constexpr (BF16) {
            // bf16 * f32 scalar: the product in f32, rounded to bf16; the
            // clamp bound rounds to bf16(1.6) = 1.6015625
            t = bf16_to_f32(f32_to_bf16_rne(__fmul_rn(w, tscale)));
            t = fminf(fmaxf(t, -1.6015625f), 1.6015625f);
          } else if constexpr (WT == W_F16) {
            // f16 * f32 scalar: the product in f32, rounded to f16 (RN, with
            // f16's own overflow to inf); the clamp bound rounds to
            // f16(1.6) = 1.599609375
            t = __half2float(__float2half_rn(__fmul_rn(w, tscale)));
            t = fminf(fmaxf(t, -1.599609375f), 1.599609375f);
          } else {
            t = fminf(fmaxf(__fmul_rn(w, tscale), -1.6f), 1.6f);
          }
          int b = __float2int_rd(t * 512.0f) + kBuckets / 2;  // t * 512 is exact
          b = b < 0 ? 0 : (b >= kBuckets ? kBuckets - 1 : b);
          const float2 rec = S.bucket[b];
          const unsigned int packed = __float_as_uint(rec.y);
          int id = t >= rec.x ? (int)((packed >> 8) & 0xFFu) : (int)(packed & 0xFFu);
          if (packed >> 16) id = S.vidx[cell_of(S, t, U)];
          idx[h] = id;
          res[h] = __fsub_rn(w, S.dq[id]);
        }
        const uint32_t two = (uint32_t)idx[0] | ((uint32_t)idx[1] << 8);
        if ((c & 3) == 0) pb[c >> 2] = two; else pb[c >> 2] |= two << 16;
        pf[c >> 1] = pack_bf16x2_rne(res[0], res[1]);
      }
      if (i < in_f) {
        const long long o = o0 + c0;
        uint8_t* wp = W_p + i * out_f + o;
        uint16_t* wf = W_f + i * out_f + o;
        const bool vec = o + 16 <= out_f && (reinterpret_cast<uintptr_t>(wp) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(wf) & 15) == 0;
        if (vec) {
          __stcs(reinterpret_cast<uint4*>(wp), make_uint4(pb[0], pb[1], pb[2], pb[3]));
          __stcs(reinterpret_cast<uint4*>(wf), make_uint4(pf[0], pf[1], pf[2], pf[3]));
          __stcs(reinterpret_cast<uint4*>(wf) + 1, make_uint4(pf[4], pf[5], pf[6], pf[7]));
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            if (o + c < out_f) {
              wp[c] = (uint8_t)(pb[c >> 2] >> (8 * (c & 3)));
              wf[c] = (uint16_t)(pf[c >> 1] >> (16 * (c & 1)));
            }
          }
        }
      }
    }
    __syncthreads();
  }
}

}  // namespace compress
}  // namespace packr

extern "C" size_t packr_abs_order_stats_workspace_bytes(void) { return sizeof(packr::compress::SelectState); }

extern "C" int packr_abs_order_stats(const void* w, int dtype, int64_t n, int64_t rank_lo, int64_t rank_hi,
                                     float* out2, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace packr;
  using namespace packr::compress;
  if (w == nullptr || out2 == nullptr || workspace == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
  if (dtype != PACKR_DTYPE_F32 && dtype != PACKR_DTYPE_BF16) return PACKR_ERR_INVALID_ARGUMENT;
  if (n < 1 || rank_lo < 0 || rank_lo >= n || (rank_hi != rank_lo && rank_hi != rank_lo + 1) || rank_hi >= n)
    return PACKR_ERR_SHAPE;
  if (workspace_bytes < sizeof(SelectState)) return PACKR_ERR_WORKSPACE;
  if (!aligned(workspace, 16) || !aligned(out2, 4) || !aligned(w, dtype == PACKR_DTYPE_F32 ? 4 : 2))
    return PACKR_ERR_ALIGNMENT;
  int st = check_device();
  if (st != PACKR_OK) return st;
  cudaStream_t s = as_stream(stream);
  SelectState init{};
  init.rank = rank_lo;
  init.rank_hi_delta = rank_hi - rank_lo;
  init.min_greater = 0xFFFFFFFFu;
  if (cudaMemcpyAsync(workspace, &init, sizeof(SelectState), cudaMemcpyHostToDevice, s) != cudaSuccess)
    return PACKR_ERR_CUDA;
  SelectState* ws = static_cast<SelectState*>(workspace);
  const long long per = dtype == PACKR_DTYPE_BF16 ? 8 : 4;
  long long want = (n / per + kHistThreads - 1) / kHistThreads;
  const int grid = (int)(want < 1 ? 1 : (want > sm_count() * 8 ? sm_count() * 8 : want));
  if (dtype == PACKR_DTYPE_BF16) {
    hist_exp_kernel<true><<<grid, kHistThreads, 0, s>>>(w, n, ws);
    select_kernel<0, false><<<1, 1024, 0, s>>>(ws);
    hist_kernel<1, true><<<grid, kHistThreads, 0, s>>>(w, n, ws);
    select_kernel<1, true><<<1, 1024, 0, s>>>(ws);  // bf16 keys have bits 15..0 zero
    min_greater_kernel<true><<<grid, kHistThreads, 0, s>>>(w, n, ws);
  } else {
    hist_exp_kernel<false><<<grid, kHistThreads, 0, s>>>(w, n, ws);
    select_kernel<0, false><<<1, 1024, 0, s>>>(ws);
    hist_kernel<1, false><<<grid, kHistThreads, 0, s>>>(w, n, ws);
    select_kernel<1, false><<<1, 1024, 0, s>>>(ws);
    hist_kernel<2, false><<<grid, kHistThreads, 0, s>>>(w, n, ws);
    select_kernel<2, true><<<1, 1024, 0, s>>>(ws);
    min_greater_kernel<false><<<grid, kHistThreads, 0, s>>>(w, n, ws);
  }
  finish_kernel<<<1, 1, 0, s>>>(ws, out2);
  return launch_status();
}

extern "C" int packr_from_linear_encode(const void* weight, int dtype, int64_t out_features, int64_t in_features,
                                        const float* codebook, const float* scale, const float* target_scale,
                                        uint8_t* W_p, uint16_t* W_f, float* lut, void* stream) {
  using namespace packr;
  using namespace packr::compress;
  if (!weight || !codebook || !scale || !W_p || !W_f || !lut) return PACKR_ERR_INVALID_ARGUMENT;
  if (target_scale == nullptr) target_scale = scale;
  if (dtype != PACKR_DTYPE_F32 && dtype != PACKR_DTYPE_BF16 && dtype != PACKR_DTYPE_F16)
    return PACKR_ERR_INVALID_ARGUMENT;
  if (out_features < 1 || in_features < 1) return PACKR_ERR_SHAPE;
  if (!aligned(weight, dtype == PACKR_DTYPE_F32 ? 4 : 2) || !aligned(W_f, 2) || !aligned(codebook, 4) ||
      !aligned(scale, 4) || !aligned(target_scale, 4) || !aligned(lut, 4))
    return PACKR_ERR_ALIGNMENT;
  int st = check_device();
  if (st != PACKR_OK) return st;
  const long long tiles = ((in_features + kTile - 1) / kTile) * ((out_features + kTile - 1) / kTile);
  const int grid = (int)(tiles < sm_count() * 8 ? tiles : sm_count() * 8);
  cudaStream_t s = as_stream(stream);
  if (dtype == PACKR_DTYPE_BF16)
    encode_kernel<W_BF16><<<grid, kEncThreads, 0, s>>>(weight, out_features, in_features, codebook, scale,
                                                       target_scale, W_p, W_f, lut);
  else if (dtype == PACKR_DTYPE_F16)
    encode_kernel<W_F16><<<grid, kEncThreads, 0, s>>>(weight, out_features, in_features, codebook, scale,
                                                      target_scale, W_p, W_f, lut);
  else
    encode_kernel<W_F32><<<grid, kEncThreads, 0, s>>>(weight, out_features, in_features, codebook, scale,
                                                      target_scale, W_p, W_f, lut);
  return launch_status();
}
