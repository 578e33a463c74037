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

// floor(y) for 0 <= y < 2^22 without the conversion unit: 2^23 + y rounded
// toward zero is 2^23 + floor(y), whose low mantissa bits hold floor(y).
__device__ __forceinline__ int floor_small(float y) {
  return (int)(__float_as_uint(__fadd_rz(y, 8388608.0f)) - 0x4B000000u);
}

// a / b rounded to nearest, given y = RN(1/b), by Markstein's correction
// (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990; Muller et al.,
// Handbook of Floating-Point Arithmetic, ch. 4): q = RN(a*y); r = a - b*q is
// exact by FMA; RN(q + r*y) equals RN(a/b) when y = RN(1/b) and every
// intermediate stays in the normal range.  A zero dividend returns q (its
// sign is right); dividends outside [2^-96, 2^100) take the IEEE division.
__device__ __forceinline__ float div_recip(float a, float b, float y) {
  const float q = __fmul_rn(a, y);
  const float r = __fmaf_rn(-q, b, a);
  const float q2 = __fmaf_rn(r, y, q);
  return a == 0.0f ? q : q2;
}
__device__ __forceinline__ bool div_recip_ok(float a) {
  const float m = fabsf(a);
  return a == 0.0f || (m >= 0x1p-96f && m < 0x1p+100f);
}

__device__ __forceinline__ uint32_t pack_i8x4(const int* c) {
  return (uint32_t)(c[0] & 0xFF) | ((uint32_t)(c[1] & 0xFF) << 8) | ((uint32_t)(c[2] & 0xFF) << 16) |
         ((uint32_t)(c[3] & 0xFF) << 24);
}

__global__ void __launch_bounds__(kThreads, 3) adam8_multi_kernel(const __grid_constant__ AdamLaunch L,
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

  for (long long b = warp0; b < total; b += nwarps) {
    // Largest tensor index t with block_begin[t] <= b (warp-uniform).
    int lo = 0, hi = L.n - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (L.block_begin[mid] <= b) lo = mid; else hi = mid - 1;
    }
    const AdamSlot& s = L.t[lo];
    const long long blk = b - L.block_begin[lo];
    const long long e0 = blk * kQuantBlock + lane * 8;
    long long rem = s.numel - e0;
    const int my_n = rem >= 8 ? 8 : (rem > 0 ? (int)rem : 0);
    const bool vec = s.vec_ok && my_n == 8;

    float pv[8], gv[8], mq[8], vq[8];
    if (vec) {
      if (s.bf16) {
        unpack_bf16x8(__ldcs(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(s.p) + e0)), pv);
        unpack_bf16x8(__ldcs(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(s.g) + e0)), gv);
      } else {
        const float4* pp = reinterpret_cast<const float4*>(static_cast<const float*>(s.p) + e0);
        const float4* gp = reinterpret_cast<const float4*>(static_cast<const float*>(s.g) + e0);
        float4 a = __ldcs(pp), c = __ldcs(pp + 1), d = __ldcs(gp), e = __ldcs(gp + 1);
        pv[0] = a.x; pv[1] = a.y; pv[2] = a.z; pv[3] = a.w; pv[4] = c.x; pv[5] = c.y; pv[6] = c.z; pv[7] = c.w;
        gv[0] = d.x; gv[1] = d.y; gv[2] = d.z; gv[3] = d.w; gv[4] = e.x; gv[5] = e.y; gv[6] = e.z; gv[7] = e.w;
      }
      unpack_i8x8(__ldcs(reinterpret_cast<const uint2*>(s.m + e0)), mq);
      unpack_i8x8(__ldcs(reinterpret_cast<const uint2*>(s.v + e0)), vq);
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

    const float ms = s.ms[blk];
    const float vs = s.vs[blk];
    float mn[8], vn[8];
    float amax_m = 0.0f, amax_v = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < my_n) {
        const float mf = __fmul_rn(mq[i], ms);
        const float vf = __fmul_rn(vq[i], vs);
        if (h.wd > 0.0f) pv[i] = __fmaf_rn(-lr_wd, pv[i], pv[i]);
        mn[i] = __fmaf_rn(one_m_b1, gv[i], __fmul_rn(h.b1, mf));
        vn[i] = __fmaf_rn(__fmul_rn(one_m_b2, gv[i]), gv[i], __fmul_rn(h.b2, vf));
      } else {
        mn[i] = 0.0f;
        vn[i] = 0.0f;
      }
      amax_m = fmaxf(amax_m, fabsf(mn[i]));
      amax_v = fmaxf(amax_v, fabsf(vn[i]));
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
    // >= 1e-14 and finite, so RN(1/b) is a normal number).
    const float y_ms = __frcp_rn(nms);
    const float y_vs = __frcp_rn(nvs);

    int mc[8], vc[8];
    float qm[8], qv[8], t1[8], t2[8];
    bool fast = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      qm[i] = div_recip(mn[i], nms, y_ms);
      qv[i] = div_recip(vn[i], nvs, y_vs);
      t1[i] = div_recip(mn[i], h.bc1, y_bc1);
      t2[i] = div_recip(vn[i], h.bc2, y_bc2);
      fast = fast && div_recip_ok(mn[i]) && div_recip_ok(vn[i]);
    }
    if (__any_sync(0xFFFFFFFFu, !fast)) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        qm[i] = __fdiv_rn(mn[i], nms);
        qv[i] = __fdiv_rn(vn[i], nvs);
        t1[i] = __fdiv_rn(mn[i], h.bc1);
        t2[i] = __fdiv_rn(vn[i], h.bc2);
      }
    }
    float pn[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // m code: trunc(clamp(q +- 0.5, -127, 127)) = sign(m_new) * floor(min(|q| + 0.5, 127))
      const int cm = floor_small(fminf(__fadd_rn(fabsf(qm[i]), 0.5f), 127.0f));
      mc[i] = mn[i] >= 0.0f ? cm : -cm;
      // v code: trunc(clamp(q + 0.5, 1, 127))
      vc[i] = floor_small(fminf(fmaxf(__fadd_rn(qv[i], 0.5f), 1.0f), 127.0f));
      const float step = __fmul_rn(h.lr, t1[i]);
      const float denom = __fadd_rn(__fsqrt_rn(t2[i]), h.eps);
      pn[i] = __fsub_rn(pv[i], __fdiv_rn(step, denom));
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
      __stcs(reinterpret_cast<uint2*>(s.m + e0), make_uint2(pack_i8x4(mc), pack_i8x4(mc + 4)));
      __stcs(reinterpret_cast<uint2*>(s.v + e0), make_uint2(pack_i8x4(vc), pack_i8x4(vc + 4)));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < my_n) {
          if (s.bf16)
            static_cast<uint16_t*>(s.p)[e0 + i] = (uint16_t)f32_to_bf16_rne(pn[i]);
          else
            static_cast<float*>(s.p)[e0 + i] = pn[i];
          s.m[e0 + i] = (int8_t)mc[i];
          s.v[e0 + i] = (int8_t)vc[i];
        }
      }
    }
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
