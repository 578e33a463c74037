// Multi-tensor 8-bit block-absmax AdamW for sm_100a.
//
// Algorithm: reference packr/cuda_adam_kernel.cu:19-69 (one 256-thread CTA per
// 256-element quantisation block, one element per thread, scalar loads).
// Here HALF a warp owns one quantisation block: each lane moves 16 contiguous
// elements with 128-bit loads (bf16 p/g: 32 B each, int8 m/v: 16 B each), the
// block absmax is a 4-step xor-shuffle inside the half-warp (no shared
// memory, no __syncthreads), the loads of the lane's next block are in
// flight while the current one is computed, and one launch per parameter
// dtype walks every tensor of a group through a block-offset table passed as
// a __grid_constant__ parameter.  The push variant (packr_adam8_multi_push)
// repeats each lane's 256-bit parameter store into up to 7 copies of the
// tensor in other GPUs' memory (a data-parallel rank's shard going to every
// other rank over NVLink) and ends with a system-scope fence.
//
// Arithmetic (every operation rounds to nearest, as the reference's does):
//   wd decay  p  = fma(-(lr*wd), p, p)                     (cuda_adam_kernel.cu:34)
//   m_new     = fma(1-b1, g, b1*(m*ms))                    (:36)
//   v_new     = fma((1-b2)*g, g, b2*(v*vs))                (:37)
//   scales    = max(absmax/127, 1e-14)                     (:48)
//   m code    = trunc(clamp(m_new/ms' +- 0.5, -127, 127))  (:53)
//   v code    = trunc(clamp(v_new/vs' + 0.5, 1, 127))      (:54)
//   p_new     = p - (lr*(m_new/bc1)) / (sqrt(v_new/bc2) + eps)   (:55)
//   bf16 store: round to nearest even                      (:62-64)
// The fused multiply-adds are where nvcc's default -fmad=true contracts the
// reference's source expressions (checked bit for bit against the reference
// kernel's outputs).
//
// Every division and square root must be correctly rounded (the results are
// compared bit for bit).  A block whose values all lie in ranges where the
// short sequences below are exact (checked once per block, see `fast`) takes
// them, on packed f32x2 pairs:
//   * x / b  by Markstein's correction with y = RN(1/b) (P. Markstein,
//     "Computation of elementary functions on the IBM RISC System/6000
//     processor", IBM J. Res. Dev. 34(1), 1990; Muller et al., Handbook of
//     Floating-Point Arithmetic, ch. 4): q = RN(x*y); r = x - b*q, exact by
//     FMA; RN(q + r*y) = RN(x/b) when x, b, x/b are normal and the exponent
//     of x is at least -102 (so that r is representable);
//   * RN(1/b) by one FMA Newton step from the hardware approximation:
//     e = RN(1 - b*y0), RN(y0 + y0*e);
//   * RN(sqrt(x)) by one residual correction of the hardware reciprocal
//     square root r0: g = RN(x*r0), h = RN(r0/2), d = RN(x - g*g),
//     RN(g + d*h).
// The last two are checked exhaustively against the IEEE operations by
// packr_selfcheck_rounding (every positive normal reciprocal argument, every
// square-root argument in [2^-100, 2^128)).  Other blocks take the IEEE
// operations.
#include <atomic>
#include <cstring>
#include <type_traits>

#include "common.cuh"

namespace packr {
namespace adam {

constexpr int kQuantBlock = 256;
constexpr int kMaxTensorsPerLaunch = 96;
constexpr int kThreads = 256;
constexpr int kMaxPeers = 7;  // packr_adam8_multi_push: other GPUs of one node
#ifndef PACKR_ADAM_WAVES
#define PACKR_ADAM_WAVES 1
#endif
// Grid = min(work, resident CTAs x kWaves): more than one wave lets CTAs start
// on the SMs that another kernel running at the same time (a collective on
// another stream) leaves free, instead of waiting for that kernel to end.
constexpr int kWaves = PACKR_ADAM_WAVES;

// Elements per lane: 16 for bf16 parameters (half a warp per block), 8 for
// f32 (a whole warp per block, to stay within 128 registers).
template <bool BF16>
struct Geo {
  static constexpr int kEpl = BF16 ? 16 : 8;
  static constexpr int kLpb = kQuantBlock / kEpl;  // lanes per quantisation block
  static constexpr int kBpw = 32 / kLpb;           // blocks per warp
  static constexpr int kPairs = kEpl / 2;
  static constexpr int kPw = kEpl * (BF16 ? 2 : 4) / 16;  // uint4 per lane for p and for g
  static constexpr int kMw = kEpl / 4;                    // 32-bit words per lane for m and for v
};

struct Slot {
  void* p;
  const void* g;
  int8_t* m;
  int8_t* v;
  float* ms;
  float* vs;
  long long numel;
  int vec_ok;  // every base pointer allows the 128-bit lane accesses
  int v8_ok;   // p and every peer copy are 32-byte aligned: one 256-bit store per lane
  char* peer[kMaxPeers];  // the same parameter in other GPUs' memory (push launches)
};

struct Launch {
  int n;
  int n_peers;  // p_new is also stored to Slot::peer[0, n_peers)
  long long block_begin[kMaxTensorsPerLaunch + 1];
  Slot t[kMaxTensorsPerLaunch];
};

typedef unsigned long long f32x2;

// Loop-invariant operands of the packed arithmetic, each float twice (both
// halves of an f32x2), computed on the host: kernel-parameter operands need
// no registers.  y_* = RN(1/x), computed as (float)(1.0 / (double)x), which
// equals RN(1/x) because 1/x is never within 2^-53 (relative) of a float
// midpoint it is not equal to.
struct Pairs {
  f32x2 b1, c1, b2, c2;  // beta1, RN(1-beta1), beta2, RN(1-beta2)
  f32x2 nlrwd;           // -RN(lr*wd)
  f32x2 yb1, nb1, nyb2, pb2;  // RN(1/bc1), -bc1, -RN(1/bc2), bc2
  f32x2 lr, eps, one, half, bias8;
};

struct Hyper {
  float lr, b1, b2, eps, bc1, bc2, wd;
  float lr_bc1;   // ~ lr / bc1 (only bounds the fast-path check)
  float inv_bc2;  // ~ 1 / bc2 (same)
  int fast_ok;    // hyper-parameters inside the fast path's ranges
  Pairs pr;
};
__device__ __forceinline__ f32x2 pk2(float a, float b) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(f32x2 v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f32x2 splat(float a) { return pk2(a, a); }

__device__ __forceinline__ float rcp_approx(float b) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
  return y;
}
__device__ __forceinline__ float rsqrt_approx(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max that returns NaN when either input is NaN (fmaxf ignores a NaN).
__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// RN(1/b) for positive normal b with 1/b normal (see the header).
__device__ __forceinline__ float rcp_rn_newton(float b) {
  const float y0 = rcp_approx(b);
  return __fmaf_rn(y0, __fmaf_rn(-b, y0, 1.0f), y0);
}
// RN(sqrt(x)) for x in [2^-100, 2^128) (see the header).
__device__ __forceinline__ float sqrt_rn_residual(float x) {
  const float r0 = rsqrt_approx(x);
  const float g = __fmul_rn(x, r0);
  const float h = __fmul_rn(0.5f, r0);
  return __fmaf_rn(__fmaf_rn(-g, g, x), h, g);
}

// Markstein's correction on pairs: q = RN(a*y), r = a - b*q (exact: fma with
// -b), RN(q + r*y).  For a = +0 it returns +0 like the IEEE quotient.
__device__ __forceinline__ f32x2 div_recip2(f32x2 a, f32x2 neg_b, f32x2 y) {
  const f32x2 q = mul2(a, y);
  const f32x2 r = fma2(q, neg_b, a);
  return fma2(r, y, q);
}

// -RN(v/bc2) by Markstein with the negated reciprocal -RN(1/bc2): RN is
// symmetric, so every step is the exact negation of the one for RN(v/bc2).
__device__ __forceinline__ f32x2 neg_div_bc2(f32x2 v, const Pairs& C) {
  const f32x2 nq = mul2(v, C.nyb2);
  return fma2(fma2(nq, C.pb2, v), C.nyb2, nq);
}

// RN(RN(lr*T1) / RN(RN(sqrt(T2)) + eps)) on a pair, given T1 = RN(m/bc1) and
// nT2 = -RN(v/bc2): the square root by the residual correction carried
// negated (ng = -g, e = g*g - x, ns = -(g + (x - g*g)*h)), d = s + eps carried
// as nd = -d, its reciprocal by one Newton step, the quotient by Markstein.
// Each step is the exact negation of the sequence in the header.
__device__ __forceinline__ f32x2 fast_update2(f32x2 T1, f32x2 nT2, const Pairs& C) {
  float x0, x1;
  upk2(nT2, x0, x1);
  const f32x2 r0 = pk2(rsqrt_approx(-x0), rsqrt_approx(-x1));
  const f32x2 ng = mul2(nT2, r0);
  const f32x2 ns = fma2(fma2(ng, ng, nT2), mul2(C.half, r0), ng);
  const f32x2 nd = sub2(ns, C.eps);
  float d0, d1;
  upk2(nd, d0, d1);
  const f32x2 y0 = pk2(rcp_approx(-d0), rcp_approx(-d1));
  const f32x2 y = fma2(y0, fma2(nd, y0, C.one), y0);
  return div_recip2(mul2(C.lr, T1), nd, y);
}

// int8 -> float without the conversion unit: (x ^ 0x80) is x + 128 in
// [0, 255]; placed in the low byte of 2^23 (0x4B000000) it forms the float
// 2^23 + 128 + x exactly, and subtracting 2^23 + 128 leaves x exactly.
__device__ __forceinline__ f32x2 i8pair(uint32_t w, int j, f32x2 bias8) {
  const uint32_t wb = w ^ 0x80808080u;
  const uint32_t lo = __byte_perm(wb, 0x4B000000u, 0x7440u + 2 * j);
  const uint32_t hi = __byte_perm(wb, 0x4B000000u, 0x7441u + 2 * j);
  return sub2(pk2(__uint_as_float(lo), __uint_as_float(hi)), bias8);
}

// The next blocks' p, g, m, v and scales are staged in shared memory by
// cp.async (kStages - 1 blocks ahead of the one being computed), so that the
// registers hold only the block in flight through the arithmetic.  Per warp
// and stage, chunk-major: 16-byte chunk k of lane l sits at k*512 + l*16, so
// each lane's 128-bit shared accesses are conflict-free.
constexpr int kStages = 2;
template <bool BF16>
struct Stage {
  static constexpr int kP = 0;                                  // p chunks
  static constexpr int kG = Geo<BF16>::kPw * 512;               // g chunks
  static constexpr int kM = 2 * Geo<BF16>::kPw * 512;           // m (one chunk, 4 * kMw bytes used)
  static constexpr int kV = kM + 512;                           // v
  static constexpr int kS = kV + 512;                           // scales: ms at l*8, vs at l*8 + 4
  static constexpr int kBytes = kS + 256;
  static constexpr int kCtaBytes = kBytes * kStages * (kThreads / 32);
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// cp.async of one lane's elements [e0, e0 + kEpl) of block blk into a stage.
template <bool BF16>
__device__ __forceinline__ void stage_issue(const Slot& s, long long blk, long long e0, uint32_t st, int lane) {
  using G = Geo<BF16>;
  using S = Stage<BF16>;
  const char* pp = static_cast<const char*>(s.p) + e0 * (BF16 ? 2 : 4);
  const char* gp = static_cast<const char*>(s.g) + e0 * (BF16 ? 2 : 4);
#pragma unroll
  for (int k = 0; k < G::kPw; ++k) {
    cp_async16(st + S::kP + k * 512 + lane * 16, pp + 16 * k);
    cp_async16(st + S::kG + k * 512 + lane * 16, gp + 16 * k);
  }
  if constexpr (G::kMw == 4) {
    cp_async16(st + S::kM + lane * 16, s.m + e0);
    cp_async16(st + S::kV + lane * 16, s.v + e0);
  } else {
    cp_async8(st + S::kM + lane * 16, s.m + e0);
    cp_async8(st + S::kV + lane * 16, s.v + e0);
  }
  cp_async4(st + S::kS + lane * 8, s.ms + blk);
  cp_async4(st + S::kS + lane * 8 + 4, s.vs + blk);
}

template <bool BF16>
__device__ __forceinline__ uint4 lds_chunk(const unsigned char* st, int off, int k, int lane) {
  return *reinterpret_cast<const uint4*>(st + off + k * 512 + lane * 16);
}

__device__ __forceinline__ uint32_t word_of(const uint4& q, int i) {
  return i == 0 ? q.x : i == 1 ? q.y : i == 2 ? q.z : q.w;
}

template <bool BF16>
__device__ __forceinline__ f32x2 raw_pair(const uint4* q, int j) {
  if constexpr (BF16) {
    const uint32_t w = word_of(q[j >> 2], j & 3);
    return pk2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  } else {
    const uint4& w4 = q[j >> 1];
    return (j & 1) == 0 ? pk2(__uint_as_float(w4.x), __uint_as_float(w4.y))
                        : pk2(__uint_as_float(w4.z), __uint_as_float(w4.w));
  }
}

// A lane's 32 bytes of parameters in one 256-bit store: a warp's store then
// covers whole 32-byte sectors (two 128-bit stores leave every sector half
// written per instruction, which costs twice the NVLink packets when the
// destination is another GPU's memory).
__device__ __forceinline__ void st_v8_cs(void* p, const uint32_t* w) {
  asm volatile("st.global.cs.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}
__device__ __forceinline__ void st_v8_cg(void* p, const uint32_t* w) {
  asm volatile("st.global.cg.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// Largest tensor index t with block_begin[t] <= b.
__device__ __forceinline__ int find_tensor(const Launch& L, long long b) {
  int lo = 0, hi = L.n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (L.block_begin[mid] <= b) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return __byte_perm(__byte_perm(a, b, 0x0040u), __byte_perm(c, d, 0x0040u), 0x5410u);
}

// PUSH: also store the new parameters into L.n_peers other GPUs' copies.
template <bool BF16, bool PUSH>
__global__ void __launch_bounds__(kThreads, 2) adam8_kernel(const __grid_constant__ Launch L, const Hyper h) {
  using Gm = Geo<BF16>;
  constexpr int kEpl = Gm::kEpl, kLpb = Gm::kLpb, kBpw = Gm::kBpw, kPairs = Gm::kPairs;
  const int lane = threadIdx.x & 31;
  const int li = lane % kLpb;  // lane within its block
  const unsigned blk_mask = kLpb == 32 ? 0xFFFFFFFFu : (((1u << kLpb) - 1u) << (lane & ~(kLpb - 1)));
  const long long warp0 = ((long long)blockIdx.x * kThreads + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * kThreads) >> 5;
  const long long total = L.block_begin[L.n];
  const long long stride = nwarps * kBpw;

  const float y_127 = __frcp_rn(127.0f);
  const Pairs& C = h.pr;

  extern __shared__ __align__(16) unsigned char adam_smem[];
  using Sg = Stage<BF16>;
  unsigned char* wbuf = adam_smem + (threadIdx.x >> 5) * (kStages * Sg::kBytes);
  const uint32_t wbuf_s = (uint32_t)__cvta_generic_to_shared(wbuf);

  long long b = warp0 * kBpw + lane / kLpb;
  int t = b < total ? find_tensor(L, b) : 0;
  auto vec_of = [&](int tt, long long bb) {
    const Slot& s = L.t[tt];
    return s.vec_ok && (bb - L.block_begin[tt] + 1) * kQuantBlock <= s.numel;
  };
  // issue cursor: block bi of tensor ti goes into stage (iteration % kStages)
  long long bi = b;
  int ti = t;
  uint32_t vec_stages = 0;  // bit k: stage k was filled by cp.async
  auto issue = [&](int stage) {
    bool vec = false;
    if (bi < total) {
      while (L.block_begin[ti + 1] <= bi) ++ti;
      vec = vec_of(ti, bi);
      if (vec) {
        const long long blk = bi - L.block_begin[ti];
        stage_issue<BF16>(L.t[ti], blk, blk * kQuantBlock + li * kEpl, wbuf_s + stage * Sg::kBytes, lane);
      }
    }
    vec_stages = vec ? (vec_stages | (1u << stage)) : (vec_stages & ~(1u << stage));
    cp_async_commit();
    bi += stride;
  };
#pragma unroll
  for (int k = 0; k < kStages - 1; ++k) issue(k);

  // Every lane of a warp runs the loop the same number of times (the
  // shuffles need them all): a lane whose block is past the end computes on
  // zeros and stores nothing.
  int stage = 0;
  for (long long bw = warp0 * kBpw; bw < total; bw += stride, b += stride) {
    issue(stage == 0 ? kStages - 1 : stage - 1);
    cp_async_wait<kStages - 1>();
    const bool live = b < total;
    if (live) {
      while (L.block_begin[t + 1] <= b) ++t;
    }
    unsigned char* st = wbuf + stage * Sg::kBytes;
    const bool cur_vec = (vec_stages >> stage) & 1u;

    const Slot& s = L.t[t];
    const long long blk = live ? b - L.block_begin[t] : 0;
    const long long e0 = blk * kQuantBlock + li * kEpl;
    const long long rem = live ? s.numel - e0 : 0;
    const int my_n = rem >= kEpl ? kEpl : (rem > 0 ? (int)rem : 0);

    if (!cur_vec) {
      // tail of a tensor, unaligned base or past the end: element loads
      // (zeros past the end) written into the stage in the staged layout
      // (unrolled and predicated, so that the words stay in registers)
      constexpr int kWords = kEpl * (BF16 ? 2 : 4) / 4;
      uint32_t pw[kWords], gw[kWords], mw0[Gm::kMw], vw0[Gm::kMw];
#pragma unroll
      for (int i = 0; i < kWords; ++i) pw[i] = gw[i] = 0u;
#pragma unroll
      for (int i = 0; i < Gm::kMw; ++i) mw0[i] = vw0[i] = 0u;
#pragma unroll
      for (int i = 0; i < kEpl; ++i) {
        if (i < my_n) {
          if constexpr (BF16) {
            pw[i >> 1] |= (uint32_t)static_cast<const uint16_t*>(s.p)[e0 + i] << (16 * (i & 1));
            gw[i >> 1] |= (uint32_t)static_cast<const uint16_t*>(s.g)[e0 + i] << (16 * (i & 1));
          } else {
            pw[i] = __float_as_uint(static_cast<const float*>(s.p)[e0 + i]);
            gw[i] = __float_as_uint(static_cast<const float*>(s.g)[e0 + i]);
          }
          mw0[i >> 2] |= (uint32_t)(uint8_t)s.m[e0 + i] << (8 * (i & 3));
          vw0[i >> 2] |= (uint32_t)(uint8_t)s.v[e0 + i] << (8 * (i & 3));
        }
      }
#pragma unroll
      for (int k = 0; k < Gm::kPw; ++k) {
        *reinterpret_cast<uint4*>(st + Sg::kP + k * 512 + lane * 16) = make_uint4(pw[4 * k], pw[4 * k + 1], pw[4 * k + 2], pw[4 * k + 3]);
        *reinterpret_cast<uint4*>(st + Sg::kG + k * 512 + lane * 16) = make_uint4(gw[4 * k], gw[4 * k + 1], gw[4 * k + 2], gw[4 * k + 3]);
      }
#pragma unroll
      for (int i = 0; i < Gm::kMw; ++i) {
        reinterpret_cast<uint32_t*>(st + Sg::kM + lane * 16)[i] = mw0[i];
        reinterpret_cast<uint32_t*>(st + Sg::kV + lane * 16)[i] = vw0[i];
      }
      reinterpret_cast<float*>(st + Sg::kS + lane * 8)[0] = live ? s.ms[blk] : 1.0f;
      reinterpret_cast<float*>(st + Sg::kS + lane * 8)[1] = live ? s.vs[blk] : 1.0f;
    }
    const float cur_ms = reinterpret_cast<const float*>(st + Sg::kS + lane * 8)[0];
    const float cur_vs = reinterpret_cast<const float*>(st + Sg::kS + lane * 8)[1];
    uint32_t cm_raw[Gm::kMw], cv_raw[Gm::kMw];
#pragma unroll
    for (int i = 0; i < Gm::kMw; ++i) {
      cm_raw[i] = reinterpret_cast<const uint32_t*>(st + Sg::kM + lane * 16)[i];
      cv_raw[i] = reinterpret_cast<const uint32_t*>(st + Sg::kV + lane * 16)[i];
    }
    uint4 graw[Gm::kPw];
#pragma unroll
    for (int k = 0; k < Gm::kPw; ++k) graw[k] = lds_chunk<BF16>(st, Sg::kG, k, lane);

    // Pass 1: moments.  Lanes past the end of the tensor hold g = m = v = 0,
    // so their moments come out as +0 and do not change the block absmax;
    // they are left out of the minima.
    f32x2 MN[kPairs], VN[kPairs];
    float amax_m = 0.0f, amax_v = 0.0f, amin_m = 0x1p+127f, amin_v = 0x1p+127f;
    // The maxima propagate NaN (so that a NaN moment fails the fast-path
    // check); the IEEE path recomputes them as the reference does.
    auto moments = [&](auto full) {
      const f32x2 ms2 = splat(cur_ms), vs2 = splat(cur_vs);
#pragma unroll
      for (int j = 0; j < kPairs; ++j) {
        const f32x2 G = raw_pair<BF16>(graw, j);
        MN[j] = fma2(C.c1, G, mul2(C.b1, mul2(i8pair(cm_raw[j >> 1], j & 1, C.bias8), ms2)));
        VN[j] = fma2(mul2(C.c2, G), G, mul2(C.b2, mul2(i8pair(cv_raw[j >> 1], j & 1, C.bias8), vs2)));
        float a0, a1, c0, c1;
        upk2(MN[j], a0, a1);
        upk2(VN[j], c0, c1);
        amax_m = max_nan(amax_m, max_nan(fabsf(a0), fabsf(a1)));
        amax_v = max_nan(amax_v, max_nan(c0, c1));
        if (decltype(full)::value || 2 * j < my_n) {
          amin_m = fminf(amin_m, fabsf(a0));
          amin_v = fminf(amin_v, c0);
        }
        if (decltype(full)::value || 2 * j + 1 < my_n) {
          amin_m = fminf(amin_m, fabsf(a1));
          amin_v = fminf(amin_v, c1);
        }
      }
    };
    if (cur_vec)
      moments(std::true_type{});
    else
      moments(std::false_type{});
#pragma unroll
    for (int o = kLpb / 2; o > 0; o >>= 1) {
      amax_m = max_nan(amax_m, __shfl_xor_sync(0xFFFFFFFFu, amax_m, o));
      amax_v = max_nan(amax_v, __shfl_xor_sync(0xFFFFFFFFu, amax_v, o));
    }

    // Fast-path check (a sufficient condition, evaluated with factor-2
    // margins for its own rounding):
    //  * every moment of the block in [2^-96, 2^100): the quotients by the
    //    scales and by bc1/bc2 meet Markstein's conditions (a quotient that
    //    underflows is far below the 0.5 that decides a code), v_new/bc2 is
    //    in the square root's range, and NaN, Inf and zero take the IEEE path;
    //  * st = lr*(m_new/bc1) has exponent >= -99 and below 2^70, and its
    //    quotient by sqrt(v_new/bc2) + eps (>= 2^-48) is normal.
    bool ok = h.fast_ok && amin_m >= 0x1p-96f && amin_v >= 0x1p-96f && amax_m < 0x1p+100f && amax_v < 0x1p+100f;
    if (ok && h.lr != 0.0f) {
      const float st_lo = amin_m * h.lr_bc1 * 0.5f;
      const float st_hi = amax_m * h.lr_bc1 * 2.0f;
      const float d_hi = (sqrt_rn_residual(amax_v * h.inv_bc2) + h.eps) * 2.0f;
      ok = st_lo >= 0x1p-99f && st_lo >= 0x1p-120f * d_hi && st_hi < 0x1p+70f;
    }
    bool fast = (__ballot_sync(0xFFFFFFFFu, ok || !live) & blk_mask) == blk_mask;
    // A block whose only obstacle is a first moment of exactly +-0 (a zero
    // gradient on a zero m code: frequent where rank-averaged gradients
    // cancel exactly) also takes the fast sequences: the same check over the
    // nonzero |m_new|, and such an element's update is m_new itself, the
    // IEEE value RN(lr * (+-0 / bc1)) / d = +-0 (Markstein's correction
    // returns +0 for -0); its code is 0 either way.
    bool zfix = false;
    if (__any_sync(0xFFFFFFFFu, !fast)) {
      float amin_nz = 0x1p+127f;
#pragma unroll
      for (int j = 0; j < kPairs; ++j) {
        float a0, a1;
        upk2(MN[j], a0, a1);
        if (2 * j < my_n && a0 != 0.0f) amin_nz = fminf(amin_nz, fabsf(a0));
        if (2 * j + 1 < my_n && a1 != 0.0f) amin_nz = fminf(amin_nz, fabsf(a1));
      }
      bool ok2 = h.fast_ok && amin_nz >= 0x1p-96f && amin_v >= 0x1p-96f && amax_m < 0x1p+100f && amax_v < 0x1p+100f;
      if (ok2 && h.lr != 0.0f) {
        const float st_lo = amin_nz * h.lr_bc1 * 0.5f;
        const float st_hi = amax_m * h.lr_bc1 * 2.0f;
        const float d_hi = (sqrt_rn_residual(amax_v * h.inv_bc2) + h.eps) * 2.0f;
        ok2 = st_lo >= 0x1p-99f && st_lo >= 0x1p-120f * d_hi && st_hi < 0x1p+70f;
      }
      const bool fz = (__ballot_sync(0xFFFFFFFFu, ok2 || !live) & blk_mask) == blk_mask;
      zfix = fz && !fast;
      fast = fast || fz;
    }

    float nms, nvs;
    if (fast) {
      // amax/127: Markstein with RN(1/127); a quotient below 2^-100 is far
      // under the 1e-14 floor, so its last bit does not matter.
      const float qm = __fmul_rn(amax_m, y_127), qv = __fmul_rn(amax_v, y_127);
      nms = fmaxf(__fmaf_rn(__fmaf_rn(-127.0f, qm, amax_m), y_127, qm), 1e-14f);
      nvs = fmaxf(__fmaf_rn(__fmaf_rn(-127.0f, qv, amax_v), y_127, qv), 1e-14f);
    } else {
      // the reference's absmax (fmaxf: a NaN moment is skipped)
      float xm = 0.0f, xv = 0.0f;
#pragma unroll
      for (int j = 0; j < kPairs; ++j) {
        float a0, a1, c0, c1;
        upk2(MN[j], a0, a1);
        upk2(VN[j], c0, c1);
        xm = fmaxf(xm, fmaxf(fabsf(a0), fabsf(a1)));
        xv = fmaxf(xv, fmaxf(c0, c1));
      }
#pragma unroll
      for (int o = kLpb / 2; o > 0; o >>= 1) {
        xm = fmaxf(xm, __shfl_sync(blk_mask, xm, li ^ o, kLpb));
        xv = fmaxf(xv, __shfl_sync(blk_mask, xv, li ^ o, kLpb));
      }
      nms = fmaxf(__fdiv_rn(xm, 127.0f), 1e-14f);
      nvs = fmaxf(__fdiv_rn(xv, 127.0f), 1e-14f);
    }
    if (live && li == 0) {
      s.ms[blk] = nms;
      s.vs[blk] = nvs;
    }

    // Pass 2: codes and parameters, pair by pair.
    //   m code: trunc(clamp(q +- 0.5, -127, 127)) with +0.5 when m_new >= 0;
    //   v code: trunc(clamp(q + 0.5, 1, 127)).
    // On the fast path |q| <= 127 (1 + 2^-23) (the scale is RN(absmax/127) or
    // larger), so q +- 0.5 truncates into [-127, 127] without the clamps.
    uint32_t mw[Gm::kMw], vw[Gm::kMw];
    uint32_t po[kEpl * (BF16 ? 2 : 4) / 4];
    uint4 praw[Gm::kPw];
#pragma unroll
    for (int k = 0; k < Gm::kPw; ++k) praw[k] = lds_chunk<BF16>(st, Sg::kP, k, lane);
    // the fast sequences, compiled twice: with the zero-moment select only
    // for the blocks that need it
    auto fast_pass = [&](auto zero_moments) {
      const f32x2 yms = splat(rcp_rn_newton(nms)), yvs = splat(rcp_rn_newton(nvs));
      const f32x2 nms2 = splat(-nms), nvs2 = splat(-nvs);
      int cm[4], cv[4];
#pragma unroll
      for (int j = 0; j < kPairs; ++j) {
        const f32x2 QM = div_recip2(MN[j], nms2, yms);
        const f32x2 QV = div_recip2(VN[j], nvs2, yvs);
        const f32x2 T1 = div_recip2(MN[j], C.nb1, C.yb1);
        const f32x2 nT2 = neg_div_bc2(VN[j], C);
        {
          float q0, q1, u0, u1;
          upk2(add2(QM, f32x2((MN[j] & 0x8000000080000000ull) | 0x3F0000003F000000ull)), q0, q1);
          upk2(add2(QV, C.half), u0, u1);
          cm[(2 * j) & 3] = __float2int_rz(q0);
          cm[(2 * j + 1) & 3] = __float2int_rz(q1);
          cv[(2 * j) & 3] = __float2int_rz(fmaxf(u0, 1.0f));
          cv[(2 * j + 1) & 3] = __float2int_rz(fmaxf(u1, 1.0f));
        }
        if (j & 1) {
          mw[j >> 1] = pack4(cm[0], cm[1], cm[2], cm[3]);
          vw[j >> 1] = pack4(cv[0], cv[1], cv[2], cv[3]);
        }
        f32x2 upd = fast_update2(T1, nT2, C);
        if constexpr (decltype(zero_moments)::value) {
          float m0, m1, u0, u1;
          upk2(MN[j], m0, m1);
          upk2(upd, u0, u1);
          upd = pk2(m0 == 0.0f ? m0 : u0, m1 == 0.0f ? m1 : u1);
        }
        f32x2 P = raw_pair<BF16>(praw, j);
        if (h.wd > 0.0f) P = fma2(C.nlrwd, P, P);
        float p0, p1;
        upk2(sub2(P, upd), p0, p1);
        if constexpr (BF16) {
          po[j] = pack_bf16x2_rne(p0, p1);
        } else {
          po[2 * j] = __float_as_uint(p0);
          po[2 * j + 1] = __float_as_uint(p1);
        }
      }
    };
    if (fast && !zfix) {
      fast_pass(std::false_type{});
    } else if (fast) {
      fast_pass(std::true_type{});
    } else {
      int cm[4], cv[4];
#pragma unroll
      for (int j = 0; j < kPairs; ++j) {
        float a[2], c[2], pn[2];
        upk2(MN[j], a[0], a[1]);
        upk2(VN[j], c[0], c[1]);
        f32x2 P = raw_pair<BF16>(praw, j);
        if (h.wd > 0.0f) P = fma2(C.nlrwd, P, P);
        float pp[2];
        upk2(P, pp[0], pp[1]);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float qm = __fdiv_rn(a[k], nms), qv = __fdiv_rn(c[k], nvs);
          const float xm = a[k] >= 0.0f ? __fadd_rn(qm, 0.5f) : __fsub_rn(qm, 0.5f);
          cm[(2 * j + k) & 3] = __float2int_rz(fminf(fmaxf(xm, -127.0f), 127.0f));
          cv[(2 * j + k) & 3] = __float2int_rz(fminf(fmaxf(__fadd_rn(qv, 0.5f), 1.0f), 127.0f));
          const float t1 = __fdiv_rn(a[k], h.bc1), t2 = __fdiv_rn(c[k], h.bc2);
          const float d = __fadd_rn(__fsqrt_rn(t2), h.eps);
          pn[k] = __fsub_rn(pp[k], __fdiv_rn(__fmul_rn(h.lr, t1), d));
        }
        if (j & 1) {
          mw[j >> 1] = pack4(cm[0], cm[1], cm[2], cm[3]);
          vw[j >> 1] = pack4(cv[0], cv[1], cv[2], cv[3]);
        }
        if constexpr (BF16) {
          // the reference's integer rounding (also for a NaN it produces)
          po[j] = f32_to_bf16_rne(pn[0]) | (f32_to_bf16_rne(pn[1]) << 16);
        } else {
          po[2 * j] = __float_as_uint(pn[0]);
          po[2 * j + 1] = __float_as_uint(pn[1]);
        }
      }
    }

    if (cur_vec) {
      static_assert(Gm::kPw == 2, "32 bytes of parameters per lane");
      if (s.v8_ok) {
        st_v8_cs(static_cast<char*>(s.p) + e0 * (BF16 ? 2 : 4), po);
        // the same store into each peer's copy (NVLink)
        if constexpr (PUSH)
          for (int q = 0; q < L.n_peers; ++q) st_v8_cg(s.peer[q] + e0 * (BF16 ? 2 : 4), po);
      } else {
        uint4* pp = reinterpret_cast<uint4*>(static_cast<char*>(s.p) + e0 * (BF16 ? 2 : 4));
#pragma unroll
        for (int k = 0; k < Gm::kPw; ++k) __stcs(pp + k, make_uint4(po[4 * k], po[4 * k + 1], po[4 * k + 2], po[4 * k + 3]));
        for (int q = 0; PUSH && q < L.n_peers; ++q) {
          uint4* qp = reinterpret_cast<uint4*>(s.peer[q] + e0 * (BF16 ? 2 : 4));
#pragma unroll
          for (int k = 0; k < Gm::kPw; ++k) __stcg(qp + k, make_uint4(po[4 * k], po[4 * k + 1], po[4 * k + 2], po[4 * k + 3]));
        }
      }
      if constexpr (Gm::kMw == 4) {
        __stcs(reinterpret_cast<uint4*>(s.m + e0), make_uint4(mw[0], mw[1], mw[2], mw[3]));
        __stcs(reinterpret_cast<uint4*>(s.v + e0), make_uint4(vw[0], vw[1], vw[2], vw[3]));
      } else {
        __stcs(reinterpret_cast<uint2*>(s.m + e0), make_uint2(mw[0], mw[1]));
        __stcs(reinterpret_cast<uint2*>(s.v + e0), make_uint2(vw[0], vw[1]));
      }
    } else {
#pragma unroll
      for (int i = 0; i < kEpl; ++i) {
        if (i < my_n) {
          if constexpr (BF16) {
            static_cast<uint16_t*>(s.p)[e0 + i] = (uint16_t)(po[i >> 1] >> (16 * (i & 1)));
            for (int q = 0; PUSH && q < L.n_peers; ++q)
              reinterpret_cast<uint16_t*>(s.peer[q])[e0 + i] = (uint16_t)(po[i >> 1] >> (16 * (i & 1)));
          } else {
            static_cast<uint32_t*>(s.p)[e0 + i] = po[i];
            for (int q = 0; PUSH && q < L.n_peers; ++q) reinterpret_cast<uint32_t*>(s.peer[q])[e0 + i] = po[i];
          }
          s.m[e0 + i] = (int8_t)((mw[i >> 2] >> (8 * (i & 3))) & 0xFFu);
          s.v[e0 + i] = (int8_t)((vw[i >> 2] >> (8 * (i & 3))) & 0xFFu);
        }
      }
    }
    stage = stage == kStages - 1 ? 0 : stage + 1;
  }
  cp_async_wait<0>();
  // the stores into other GPUs' memory are ordered before anything this
  // thread's GPU does after the kernel (the caller's barrier that tells the
  // peers their copies are complete)
  if (PUSH) __threadfence_system();
}

Hyper make_hyper(float lr, float beta1, float beta2, float eps, float bc1, float bc2, float weight_decay) {
  Hyper h{};
  h.lr = lr; h.b1 = beta1; h.b2 = beta2; h.eps = eps; h.bc1 = bc1; h.bc2 = bc2; h.wd = weight_decay;
  // host float arithmetic is IEEE round-to-nearest (SSE), as on the device
  auto two = [](float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    return ((unsigned long long)u << 32) | u;
  };
  const volatile float one = 1.0f;
  const float one_m_b1 = one - beta1, one_m_b2 = one - beta2, lr_wd = lr * weight_decay;
  const float y_bc1 = (float)(1.0 / (double)bc1), y_bc2 = (float)(1.0 / (double)bc2);
  h.pr = Pairs{two(beta1), two(one_m_b1), two(beta2), two(one_m_b2), two(-lr_wd), two(y_bc1), two(-bc1),
               two(-y_bc2), two(bc2), two(lr), two(eps), two(1.0f), two(0.5f), two(8388736.0f)};
  // Fast-path ranges: bias corrections in [2^-20, 1] (so the moments'
  // quotients stay below 2^120), eps and lr finite and below 2^40.
  const bool in_range = bc1 >= 0x1p-20f && bc1 <= 1.0f && bc2 >= 0x1p-20f && bc2 <= 1.0f && eps >= 0.0f &&
                        eps < 0x1p+40f && lr >= 0.0f && lr < 0x1p+40f && weight_decay >= 0.0f &&
                        weight_decay < 0x1p+40f;
  if (in_range) {
    h.lr_bc1 = (float)((double)lr / (double)bc1);
    h.inv_bc2 = (float)(1.0 / (double)bc2);
    h.fast_ok = 1;
  }
  return h;
}

// Self-check of the short correctly rounded sequences against CUDA's IEEE
// operations: [0] RN(1/b) for every positive normal b with a normal
// reciprocal, [1] RN(sqrt(x)) for every x in [2^-100, 2^128), [2] Markstein
// quotients a/b on pseudo-random pairs (exponents of a in [-96, 100), of b in
// [-20, 20)), [3] the whole parameter update RN(RN(lr*RN(m/bc1)) /
// RN(RN(sqrt(RN(v/bc2))) + eps)) on pseudo-random m in +-[2^-40, 2^20] and v
// in [2^-80, 2^40].
__device__ __forceinline__ uint32_t mix32(unsigned long long x) {
  x ^= x >> 33;
  x *= 0xff51afd7ed558ccdull;
  x ^= x >> 33;
  x *= 0xc4ceb9fe1a85ec53ull;
  x ^= x >> 33;
  return (uint32_t)x;
}
__device__ __forceinline__ float rand_float(uint32_t h, int emin, int espan, bool sign) {
  const uint32_t e = (uint32_t)(127 + emin + (int)((h >> 23) % (uint32_t)espan));
  return __uint_as_float((sign && (h & 1u) ? 0x80000000u : 0u) | (e << 23) | ((h * 2654435761u) & 0x7FFFFFu));
}

__global__ void selfcheck_kernel(unsigned long long* bad, const Hyper h, unsigned long long nrand) {
  const unsigned long long tid = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
  const unsigned long long nth = (unsigned long long)gridDim.x * blockDim.x;
  unsigned long long c0 = 0, c1 = 0, c2 = 0, c3 = 0;
  for (unsigned long long i = 0x00800000ull + tid; i < 0x7E800000ull; i += nth) {
    const float b = __uint_as_float((uint32_t)i);
    c0 += __float_as_uint(rcp_rn_newton(b)) != __float_as_uint(__frcp_rn(b));
  }
  for (unsigned long long i = 0x0D800000ull + tid; i < 0x7F800000ull; i += nth) {
    const float x = __uint_as_float((uint32_t)i);
    c1 += __float_as_uint(sqrt_rn_residual(x)) != __float_as_uint(__fsqrt_rn(x));
  }
  const Pairs& C = h.pr;
  for (unsigned long long i = tid; i < nrand; i += nth) {
    const uint32_t ha = mix32(4 * i), hb = mix32(4 * i + 1), hm = mix32(4 * i + 2), hv = mix32(4 * i + 3);
    const float a = rand_float(ha, -96, 196, true), b = rand_float(hb, -20, 40, false);
    const float y = rcp_rn_newton(b);
    float q0, q1;
    upk2(div_recip2(pk2(a, -a), pk2(-b, -b), pk2(y, y)), q0, q1);
    c2 += (__float_as_uint(q0) != __float_as_uint(__fdiv_rn(a, b))) + (__float_as_uint(q1) != __float_as_uint(__fdiv_rn(-a, b)));
    const float m = rand_float(hm, -40, 61, true), v = rand_float(hv, -80, 121, false);
    const float m2 = -m * 0.75f, v2 = v * 1.25f;
    const f32x2 MN = pk2(m, m2), VN = pk2(v, v2);
    float u0, u1;
    upk2(fast_update2(div_recip2(MN, C.nb1, C.yb1), neg_div_bc2(VN, C), C), u0, u1);
    auto ieee = [&](float mm, float vv) {
      const float t1 = __fdiv_rn(mm, h.bc1), t2 = __fdiv_rn(vv, h.bc2);
      return __fdiv_rn(__fmul_rn(h.lr, t1), __fadd_rn(__fsqrt_rn(t2), h.eps));
    };
    c3 += (__float_as_uint(u0) != __float_as_uint(ieee(m, v))) + (__float_as_uint(u1) != __float_as_uint(ieee(m2, v2)));
  }
  if (c0) atomicAdd(bad + 0, c0);
  if (c1) atomicAdd(bad + 1, c1);
  if (c2) atomicAdd(bad + 2, c2);
  if (c3) atomicAdd(bad + 3, c3);
}

template <bool BF16>
int launch_dtype(const packr_adam_tensor* tensors, int n_tensors, void* const* peer_p, int n_peers, const Hyper& h,
                 cudaStream_t stream) {
  // per-device cache; relaxed atomics: concurrent first calls store the same value
  static std::atomic<int> occ[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return PACKR_ERR_DEVICE;
  constexpr int kSmem = Stage<BF16>::kCtaBytes;
  int occ_dev = occ[dev].load(std::memory_order_relaxed);
  if (occ_dev == 0) {
    if (cudaFuncSetAttribute(adam8_kernel<BF16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(adam8_kernel<BF16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
            cudaSuccess)
      return launch_status();
    int o = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, adam8_kernel<BF16, false>, kThreads, kSmem) != cudaSuccess || o < 1) o = 1;
    occ[dev].store(o, std::memory_order_relaxed);
    occ_dev = o;
  }
  const int max_ctas = sm_count() * occ_dev;
  const int want_dtype = BF16 ? PACKR_DTYPE_BF16 : PACKR_DTYPE_F32;
  Launch L;
  L.n_peers = n_peers;
  int i = 0;
  while (i < n_tensors) {
    L.n = 0;
    long long blocks = 0;
    for (; i < n_tensors && L.n < kMaxTensorsPerLaunch; ++i) {
      const packr_adam_tensor& t = tensors[i];
      if (t.numel == 0 || t.dtype != want_dtype) continue;
      Slot& s = L.t[L.n];
      s.p = t.p;
      s.g = t.g;
      s.m = t.m;
      s.v = t.v;
      s.ms = t.m_scale;
      s.vs = t.v_scale;
      s.numel = t.numel;
      s.vec_ok = aligned(t.p, 16) && aligned(t.g, 16) && aligned(t.m, 4 * Geo<BF16>::kMw) &&
                 aligned(t.v, 4 * Geo<BF16>::kMw);
      s.v8_ok = aligned(t.p, 32);
      for (int q = 0; q < kMaxPeers; ++q) {
        s.peer[q] = q < n_peers ? static_cast<char*>(peer_p[(size_t)i * n_peers + q]) : nullptr;
        if (q < n_peers && !aligned(s.peer[q], 16)) s.vec_ok = 0;
        if (q < n_peers && !aligned(s.peer[q], 32)) s.v8_ok = 0;
      }
      L.block_begin[L.n] = blocks;
      blocks += (t.numel + kQuantBlock - 1) / kQuantBlock;
      ++L.n;
    }
    if (L.n == 0) break;
    L.block_begin[L.n] = blocks;
    const long long per_cta = (long long)(kThreads / 32) * Geo<BF16>::kBpw;
    const long long want = (blocks + per_cta - 1) / per_cta;
    const long long cap = (long long)max_ctas * kWaves;
    const int grid = (int)(want < cap ? want : cap);
    if (n_peers > 0)
      adam8_kernel<BF16, true><<<grid, kThreads, kSmem, stream>>>(L, h);
    else
      adam8_kernel<BF16, false><<<grid, kThreads, kSmem, stream>>>(L, h);
    const int st = launch_status();
    if (st != PACKR_OK) return st;
  }
  return PACKR_OK;
}

}  // namespace adam
}  // namespace packr

namespace packr {
namespace adam {
int multi_impl(const packr_adam_tensor* tensors, int n_tensors, void* const* peer_p, int n_peers, float lr,
               float beta1, float beta2, float eps, float bc1, float bc2, float weight_decay, void* stream) {
  if (n_tensors < 0 || (n_tensors > 0 && tensors == nullptr)) return PACKR_ERR_INVALID_ARGUMENT;
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && n_tensors > 0 && peer_p == nullptr))
    return PACKR_ERR_INVALID_ARGUMENT;
  if (n_tensors == 0) return PACKR_OK;
  int st = check_device();
  if (st != PACKR_OK) return st;
  bool any_bf16 = false, any_f32 = false;
  for (int i = 0; i < n_tensors; ++i) {
    const packr_adam_tensor& t = tensors[i];
    if (t.numel < 0) return PACKR_ERR_SHAPE;
    if (t.numel == 0) continue;
    if (!t.p || !t.g || !t.m || !t.v || !t.m_scale || !t.v_scale) return PACKR_ERR_INVALID_ARGUMENT;
    if (t.dtype != PACKR_DTYPE_BF16 && t.dtype != PACKR_DTYPE_F32) return PACKR_ERR_INVALID_ARGUMENT;
    if (t.reserved != 0) return PACKR_ERR_INVALID_ARGUMENT;
    const uintptr_t esz = t.dtype == PACKR_DTYPE_BF16 ? 2 : 4;
    if (!aligned(t.p, esz) || !aligned(t.g, esz) || !aligned(t.m_scale, 4) || !aligned(t.v_scale, 4))
      return PACKR_ERR_ALIGNMENT;
    for (int q = 0; q < n_peers; ++q) {
      const void* pq = peer_p[(size_t)i * n_peers + q];
      if (pq == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
      if (!aligned(pq, esz)) return PACKR_ERR_ALIGNMENT;
    }
    (t.dtype == PACKR_DTYPE_BF16 ? any_bf16 : any_f32) = true;
  }
  const Hyper h = make_hyper(lr, beta1, beta2, eps, bc1, bc2, weight_decay);
  cudaStream_t s = as_stream(stream);
  if (any_bf16 && (st = launch_dtype<true>(tensors, n_tensors, peer_p, n_peers, h, s)) != PACKR_OK) return st;
  if (any_f32 && (st = launch_dtype<false>(tensors, n_tensors, peer_p, n_peers, h, s)) != PACKR_OK) return st;
  return PACKR_OK;
}
}  // namespace adam
}  // namespace packr

extern "C" int packr_adam8_multi(const packr_adam_tensor* tensors, int n_tensors, float lr, float beta1,
                                 float beta2, float eps, float bc1, float bc2, float weight_decay,
                                 void* stream) {
  return packr::adam::multi_impl(tensors, n_tensors, nullptr, 0, lr, beta1, beta2, eps, bc1, bc2, weight_decay,
                                 stream);
}

extern "C" int packr_adam8_multi_push(const packr_adam_tensor* tensors, int n_tensors, void* const* peer_p,
                                      int n_peers, float lr, float beta1, float beta2, float eps, float bc1,
                                      float bc2, float weight_decay, void* stream) {
  return packr::adam::multi_impl(tensors, n_tensors, peer_p, n_peers, lr, beta1, beta2, eps, bc1, bc2,
                                 weight_decay, stream);
}

extern "C" int packr_selfcheck_rounding(unsigned long long* mismatches, void* stream) {
  using namespace packr;
  if (mismatches == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
  if (!aligned(mismatches, 8)) return PACKR_ERR_ALIGNMENT;
  int st = check_device();
  if (st != PACKR_OK) return st;
  cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(mismatches, 0, 4 * sizeof(unsigned long long), s) != cudaSuccess) return PACKR_ERR_CUDA;
  // lr 2e-5, bc1 = 1 - 0.9, bc2 = 1 - 0.999 (first step), eps 1e-8
  const adam::Hyper h = adam::make_hyper(2e-5f, 0.9f, 0.999f, 1e-8f, 0.1f, 0.001f, 0.0f);
  adam::selfcheck_kernel<<<sm_count() * 8, 256, 0, s>>>(mismatches, h, 1ull << 30);
  return launch_status();
}
