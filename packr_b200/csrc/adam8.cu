// Multi-tensor 8-bit block-absmax AdamW for sm_100a.
//
// Algorithm: reference packr/cuda_adam_kernel.cu:19-69 (one 256-thread CTA per
// 256-element quantisation block, one element per thread, scalar loads).
// Here one WARP owns one quantisation block: each lane moves 8 contiguous
// elements with 128-bit loads (bf16 p/g: 16 B each, int8 m/v: 8 B each), the
// block absmax is a 5-step xor-shuffle with no shared memory and no
// __syncthreads, and one launch walks every tensor of a parameter group
// through a block-offset table passed as a __grid_constant__ parameter.
//
// Arithmetic is written with explicit round-to-nearest intrinsics so that the
// compiler cannot re-associate or contract it differently from the oracle:
//   wd decay  p  = fma(-(lr*wd), p, p)                     (cuda_adam_kernel.cu:34)
//   m_new     = fma(1-b1, g, b1*(m*ms))                    (:36)
//   v_new     = fma((1-b2)*g, g, b2*(v*vs))                (:37)
//   scales    = max(absmax/127, 1e-14)                     (:48)
//   m code    = trunc(clamp(m_new/ms' +- 0.5, -127, 127))  (:53)
//   v code    = trunc(clamp(v_new/vs' + 0.5, 1, 127))      (:54)
//   p_new     = p - (lr*(m_new/bc1)) / (sqrt(v_new/bc2) + eps)   (:55)
//   bf16 store: integer round-to-nearest-even              (:62-64)
// The fused multiply-adds are where nvcc's default -fmad=true contracts the
// reference's source expressions (checked bit for bit against the reference
// kernel's outputs).
#include "common.cuh"

namespace packr {
namespace {

constexpr int kQuantBlock = 256;
constexpr int kMaxTensorsPerLaunch = 96;
constexpr int kThreads = 256;

struct AdamSlot {
  void* p;
  const void* g;
  int8_t* m;
  int8_t* v;
  float* ms;
  float* vs;
  long long numel;
  int bf16;
  int vec_ok;  // every base pointer allows the 128/64-bit lane accesses
};

struct AdamLaunch {
  int n;
  long long block_begin[kMaxTensorsPerLaunch + 1];
  AdamSlot t[kMaxTensorsPerLaunch];
};

struct AdamHyper {
  float lr, b1, b2, eps, bc1, bc2, wd;
};

__device__ __forceinline__ void unpack_bf16x8(const uint4& q, float* f) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// int8 -> float without the conversion unit: (x ^ 0x80) is x + 128 in
// [0, 255]; placed in the low byte of 2^23 (0x4B000000) it forms the float
// 2^23 + 128 + x exactly, and subtracting 2^23 + 128 leaves x exactly.
__device__ __forceinline__ void unpack_i8x8(const uint2& q, float* f) {
  const uint32_t w[2] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t bits = __byte_perm(w[i], 0x4B000000u, 0x7440u + j);
      f[4 * i + j] = __fsub_rn(__uint_as_float(bits), 8388736.0f);
    }
  }
}

// Division by Markstein's correction (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990; Muller et al., Handbook of Floating-Point Arithmetic,
// ch. 4): given y = RN(1/b), q = RN(a*y); r = a - b*q is exact by FMA; and
// RN(q + r*y) equals RN(a/b) when every intermediate stays in the normal range.

// Packed pairs of f32 (first element in the low half) and the sm_100
// f32x2 arithmetic: each operation rounds both halves exactly as the scalar
// instruction would (round to nearest, denormals kept).
typedef unsigned long long f32x2;
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
// Markstein's correction on pairs (see div_recip): q = RN(a*y), r = a - b*q
// (exact: fma with -b), RN(q + r*y).  For a = +0 it returns +0 like the IEEE
// quotient; a = -0 does not occur for the moments (m_new = fma(1-b1, g,
// b1*mf) and v_new are never -0 because b1*mf and b2*vf are +0 when zero).
__device__ __forceinline__ f32x2 div_recip2(f32x2 a, f32x2 neg_b, f32x2 y) {
  const f32x2 q = mul2(a, y);
  const f32x2 r = fma2(q, neg_b, a);
  return fma2(r, y, q);
}

__global__ void __launch_bounds__(kThreads, 2) adam8_multi_kernel(const __grid_constant__ AdamLaunch L,
                                                               const AdamHyper h) {
  const int lane = threadIdx.x & 31;
  const long long warp0 = ((long long)blockIdx.x * kThreads + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * kThreads) >> 5;
  const long long total = L.block_begin[L.n];

  const float one_m_b1 = __fsub_rn(1.0f, h.b1);
  const float one_m_b2 = __fsub_rn(1.0f, h.b2);
  const float lr_wd = __fmul_rn(h.lr, h.wd);
  // bc1, bc2 lie in (0, 1]: their reciprocals are normal numbers.
  const float y_bc1 = __frcp_rn(h.bc1);
  const float y_bc2 = __frcp_rn(h.bc2);

  // Raw 128-bit loads of one block plus its two scales.  The loads of the
  // warp's next block are issued before the current block is computed.
  struct Raw {
    uint4 p0, p1, g0, g1;
    uint2 m, v;
    float ms, vs;
    int t;
    long long blk;
    int my_n;
    bool vec;
  };
  auto fetch = [&](long long b, Raw& r) {
    // Largest tensor index t with block_begin[t] <= b (warp-uniform).
    int lo = 0, hi = L.n - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (L.block_begin[mid] <= b) lo = mid; else hi = mid - 1;
    }
    const AdamSlot& s = L.t[lo];
    r.t = lo;
    r.blk = b - L.block_begin[lo];
    const long long e0 = r.blk * kQuantBlock + lane * 8;
    const long long rem = s.numel - e0;
    r.my_n = rem >= 8 ? 8 : (rem > 0 ? (int)rem : 0);
    r.vec = s.vec_ok && r.my_n == 8;
    if (r.vec) {
      if (s.bf16) {
        r.p0 = __ldcs(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(s.p) + e0));
        r.g0 = __ldcs(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(s.g) + e0));
      } else {
        const uint4* pp = reinterpret_cast<const uint4*>(static_cast<const float*>(s.p) + e0);
        const uint4* gp = reinterpret_cast<const uint4*>(static_cast<const float*>(s.g) + e0);
        r.p0 = __ldcs(pp);
        r.p1 = __ldcs(pp + 1);
        r.g0 = __ldcs(gp);
        r.g1 = __ldcs(gp + 1);
      }
      r.m = __ldcs(reinterpret_cast<const uint2*>(s.m + e0));
      r.v = __ldcs(reinterpret_cast<const uint2*>(s.v + e0));
    }
    r.ms = s.ms[r.blk];
    r.vs = s.vs[r.blk];
  };

  Raw cur, nxt;
  long long b = warp0;
  if (b < total) fetch(b, cur);
  while (b < total) {
    const long long bn = b + nwarps;
    if (bn < total) fetch(bn, nxt);
    const AdamSlot& s = L.t[cur.t];
    const long long blk = cur.blk;
    const long long e0 = blk * kQuantBlock + lane * 8;
    const int my_n = cur.my_n;
    const bool vec = cur.vec;

    float pv[8], gv[8], mq[8], vq[8];
    if (vec) {
      if (s.bf16) {
        unpack_bf16x8(cur.p0, pv);
        unpack_bf16x8(cur.g0, gv);
      } else {
        const uint32_t pw[8] = {cur.p0.x, cur.p0.y, cur.p0.z, cur.p0.w, cur.p1.x, cur.p1.y, cur.p1.z, cur.p1.w};
        const uint32_t gw[8] = {cur.g0.x, cur.g0.y, cur.g0.z, cur.g0.w, cur.g1.x, cur.g1.y, cur.g1.z, cur.g1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          pv[i] = __uint_as_float(pw[i]);
          gv[i] = __uint_as_float(gw[i]);
        }
      }
      unpack_i8x8(cur.m, mq);
      unpack_i8x8(cur.v, vq);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        pv[i] = gv[i] = mq[i] = vq[i] = 0.0f;
        if (i < my_n) {
          if (s.bf16) {
            pv[i] = bf16_to_f32(static_cast<const uint16_t*>(s.p)[e0 + i]);
            gv[i] = bf16_to_f32(static_cast<const uint16_t*>(s.g)[e0 + i]);
          } else {
            pv[i] = static_cast<const float*>(s.p)[e0 + i];
            gv[i] = static_cast<const float*>(s.g)[e0 + i];
          }
          mq[i] = (float)s.m[e0 + i];
          vq[i] = (float)s.v[e0 + i];
        }
      }
    }

    const float ms = cur.ms;
    const float vs = cur.vs;
    // Lanes past the end of the tensor hold p = g = m = v = 0, so their
    // moments come out as +0 and do not change the block absmax.
    f32x2 P[4], G[4], MN[4], VN[4];
    float amax_m = 0.0f, amax_v = 0.0f, amin = 0x1p+127f;
    {
      const f32x2 ms2 = pk2(ms, ms), vs2 = pk2(vs, vs);
      const f32x2 b1_2 = pk2(h.b1, h.b1), c1_2 = pk2(one_m_b1, one_m_b1);
      const f32x2 b2_2 = pk2(h.b2, h.b2), c2_2 = pk2(one_m_b2, one_m_b2);
      const f32x2 nlrwd = pk2(-lr_wd, -lr_wd);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        P[j] = pk2(pv[2 * j], pv[2 * j + 1]);
        G[j] = pk2(gv[2 * j], gv[2 * j + 1]);
        const f32x2 mf = mul2(pk2(mq[2 * j], mq[2 * j + 1]), ms2);
        const f32x2 vf = mul2(pk2(vq[2 * j], vq[2 * j + 1]), vs2);
        if (h.wd > 0.0f) P[j] = fma2(nlrwd, P[j], P[j]);
        MN[j] = fma2(c1_2, G[j], mul2(b1_2, mf));
        VN[j] = fma2(mul2(c2_2, G[j]), G[j], mul2(b2_2, vf));
        float a0, a1, c0, c1;
        upk2(MN[j], a0, a1);
        upk2(VN[j], c0, c1);
        amax_m = fmaxf(amax_m, fmaxf(fabsf(a0), fabsf(a1)));
        amax_v = fmaxf(amax_v, fmaxf(c0, c1));
        amin = fminf(amin, fminf(fminf(fabsf(a0), fabsf(a1)), fminf(c0, c1)));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      amax_m = fmaxf(amax_m, __shfl_xor_sync(0xFFFFFFFFu, amax_m, o));
      amax_v = fmaxf(amax_v, __shfl_xor_sync(0xFFFFFFFFu, amax_v, o));
    }
    const float nms = fmaxf(__fdiv_rn(amax_m, 127.0f), 1e-14f);
    const float nvs = fmaxf(__fdiv_rn(amax_v, 127.0f), 1e-14f);
    if (lane == 0) {
      s.ms[blk] = nms;
      s.vs[blk] = nvs;
    }
    // Warp-uniform reciprocals of this block's divisors (the divisors are
    // >= 1e-14 and finite, so RN(1/b) is a normal number).  Markstein's
    // correction needs every dividend in [2^-96, 2^100); a block with a
    // smaller (or zero) or larger moment takes the IEEE divisions instead.
    const bool fast = __all_sync(0xFFFFFFFFu, amin >= 0x1p-96f) && amax_m < 0x1p+100f && amax_v < 0x1p+100f;
    f32x2 QM[4], QV[4], T1[4], T2[4];
    if (fast) {
      const float y_ms = __frcp_rn(nms), y_vs = __frcp_rn(nvs);
      const f32x2 yms = pk2(y_ms, y_ms), yvs = pk2(y_vs, y_vs), yb1 = pk2(y_bc1, y_bc1), yb2 = pk2(y_bc2, y_bc2);
      const f32x2 nms2 = pk2(-nms, -nms), nvs2 = pk2(-nvs, -nvs), nb1 = pk2(-h.bc1, -h.bc1), nb2 = pk2(-h.bc2, -h.bc2);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        QM[j] = div_recip2(MN[j], nms2, yms);
        QV[j] = div_recip2(VN[j], nvs2, yvs);
        T1[j] = div_recip2(MN[j], nb1, yb1);
        T2[j] = div_recip2(VN[j], nb2, yb2);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float a0, a1, c0, c1;
        upk2(MN[j], a0, a1);
        upk2(VN[j], c0, c1);
        QM[j] = pk2(__fdiv_rn(a0, nms), __fdiv_rn(a1, nms));
        QV[j] = pk2(__fdiv_rn(c0, nvs), __fdiv_rn(c1, nvs));
        T1[j] = pk2(__fdiv_rn(a0, h.bc1), __fdiv_rn(a1, h.bc1));
        T2[j] = pk2(__fdiv_rn(c0, h.bc2), __fdiv_rn(c1, h.bc2));
      }
    }
    // Codes.  m: trunc(clamp(q +- 0.5, -127, 127)) = sign(m_new) * floor(min(|q| + 0.5, 127));
    // v: trunc(clamp(q + 0.5, 1, 127)).  floor(y) for 0 <= y < 2^22 is the
    // low mantissa of RZ(2^23 + y); for a negative m code the byte -floor(y)
    // is the low mantissa of 2^24 + 256 - RZ(2^23 + y) (exact).
    float cmf[8], cvf[8], pn[8];
    const f32x2 half2 = pk2(0.5f, 0.5f), lr2 = pk2(h.lr, h.lr), eps2 = pk2(h.eps, h.eps);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float qm0, qm1, rv0, rv1, m0, m1, st0, st1;
      upk2(add2(QM[j] & 0x7FFFFFFF7FFFFFFFull, half2), qm0, qm1);
      upk2(add2(QV[j], half2), rv0, rv1);
      upk2(MN[j], m0, m1);
      const float t0 = __fadd_rz(fminf(qm0, 127.0f), 8388608.0f);
      const float t1 = __fadd_rz(fminf(qm1, 127.0f), 8388608.0f);
      // (m_new >= 0 selects the positive branch, as in the reference; NaN takes the negative one)
      cmf[2 * j] = m0 >= 0.0f ? t0 : __fsub_rn(16777472.0f, t0);
      cmf[2 * j + 1] = m1 >= 0.0f ? t1 : __fsub_rn(16777472.0f, t1);
      cvf[2 * j] = __fadd_rz(fminf(fmaxf(rv0, 1.0f), 127.0f), 8388608.0f);
      cvf[2 * j + 1] = __fadd_rz(fminf(fmaxf(rv1, 1.0f), 127.0f), 8388608.0f);
      // p_new = p - (lr * (m_new/bc1)) / (sqrt(v_new/bc2) + eps)
      float s0, s1;
      upk2(T2[j], s0, s1);
      float d0, d1;
      upk2(add2(pk2(__fsqrt_rn(s0), __fsqrt_rn(s1)), eps2), d0, d1);
      upk2(mul2(lr2, T1[j]), st0, st1);
      upk2(sub2(P[j], pk2(__fdiv_rn(st0, d0), __fdiv_rn(st1, d1))), pn[2 * j], pn[2 * j + 1]);
    }
    uint32_t mw[2], vw[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      mw[k] = __byte_perm(__byte_perm(__float_as_uint(cmf[4 * k]), __float_as_uint(cmf[4 * k + 1]), 0x0040u),
                          __byte_perm(__float_as_uint(cmf[4 * k + 2]), __float_as_uint(cmf[4 * k + 3]), 0x0040u),
                          0x5410u);
      vw[k] = __byte_perm(__byte_perm(__float_as_uint(cvf[4 * k]), __float_as_uint(cvf[4 * k + 1]), 0x0040u),
                          __byte_perm(__float_as_uint(cvf[4 * k + 2]), __float_as_uint(cvf[4 * k + 3]), 0x0040u),
                          0x5410u);
    }

    if (vec) {
      if (s.bf16) {
        uint4 q;
        q.x = pack_bf16x2_rne(pn[0], pn[1]);
        q.y = pack_bf16x2_rne(pn[2], pn[3]);
        q.z = pack_bf16x2_rne(pn[4], pn[5]);
        q.w = pack_bf16x2_rne(pn[6], pn[7]);
        __stcs(reinterpret_cast<uint4*>(static_cast<uint16_t*>(s.p) + e0), q);
      } else {
        float4* pp = reinterpret_cast<float4*>(static_cast<float*>(s.p) + e0);
        __stcs(pp, make_float4(pn[0], pn[1], pn[2], pn[3]));
        __stcs(pp + 1, make_float4(pn[4], pn[5], pn[6], pn[7]));
      }
      __stcs(reinterpret_cast<uint2*>(s.m + e0), make_uint2(mw[0], mw[1]));
      __stcs(reinterpret_cast<uint2*>(s.v + e0), make_uint2(vw[0], vw[1]));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < my_n) {
          if (s.bf16)
            static_cast<uint16_t*>(s.p)[e0 + i] = (uint16_t)f32_to_bf16_rne(pn[i]);
          else
            static_cast<float*>(s.p)[e0 + i] = pn[i];
          s.m[e0 + i] = (int8_t)((mw[i >> 2] >> (8 * (i & 3))) & 0xFFu);
          s.v[e0 + i] = (int8_t)((vw[i >> 2] >> (8 * (i & 3))) & 0xFFu);
        }
      }
    }
    cur = nxt;
    b = bn;
  }
}

}  // namespace
}  // namespace packr

extern "C" int packr_adam8_multi(const packr_adam_tensor* tensors, int n_tensors, float lr, float beta1,
                                 float beta2, float eps, float bc1, float bc2, float weight_decay,
                                 void* stream) {
  using namespace packr;
  if (n_tensors < 0 || (n_tensors > 0 && tensors == nullptr)) return PACKR_ERR_INVALID_ARGUMENT;
  if (n_tensors == 0) return PACKR_OK;
  int st = check_device();
  if (st != PACKR_OK) return st;
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
  }
  AdamHyper h{lr, beta1, beta2, eps, bc1, bc2, weight_decay};
  const int max_ctas = sm_count() * 8;
  AdamLaunch L;
  int i = 0;
  while (i < n_tensors) {
    L.n = 0;
    long long blocks = 0;
    for (; i < n_tensors && L.n < kMaxTensorsPerLaunch; ++i) {
      const packr_adam_tensor& t = tensors[i];
      if (t.numel == 0) continue;
      AdamSlot& s = L.t[L.n];
      s.p = t.p;
      s.g = t.g;
      s.m = t.m;
      s.v = t.v;
      s.ms = t.m_scale;
      s.vs = t.v_scale;
      s.numel = t.numel;
      s.bf16 = t.dtype == PACKR_DTYPE_BF16;
      s.vec_ok = aligned(t.p, 16) && aligned(t.g, 16) && aligned(t.m, 8) && aligned(t.v, 8);
      L.block_begin[L.n] = blocks;
      blocks += (t.numel + kQuantBlock - 1) / kQuantBlock;
      ++L.n;
    }
    if (L.n == 0) break;
    L.block_begin[L.n] = blocks;
    const long long want = (blocks + (kThreads / 32) - 1) / (kThreads / 32);
    const int grid = (int)(want < max_ctas ? want : max_ctas);
    adam8_multi_kernel<<<grid, kThreads, 0, as_stream(stream)>>>(L, h);
    st = launch_status();
    if (st != PACKR_OK) return st;
  }
  return PACKR_OK;
}
