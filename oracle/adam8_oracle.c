/*
 * CPU oracle for the 8-bit block-absmax AdamW step — TEST INFRASTRUCTURE ONLY.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it,
 * as the checker; the product path never calls it.
 *
 * Restates reference packr/cuda_adam_kernel.cu:19-69 (one quantisation block
 * of 256 elements at a time) in plain C with the same operation order:
 *   :21-31  load p, g (bf16 widened by <<16), mf = m*ms, vf = v*vs
 *   :34     if wd > 0: p -= (lr*wd)*p            (one fused multiply-add)
 *   :36-37  m_new = fma(1-b1, g, b1*mf),  v_new = fma((1-b2)*g, g, b2*vf)
 *           (the second product of each source expression fused into the
 *            add: the contraction nvcc's default -fmad applies to the
 *            reference, confirmed bit-for-bit against the reference kernel's
 *            outputs in tests/golden/adam8_golden.npz)
 *   :39-48  block absmax; ms' = max(amax/127, 1e-14), same for v
 *   :53-54  codes: truncate(clamp(m_new/ms' +- 0.5, -127, 127)),
 *                  truncate(clamp(v_new/vs' + 0.5, 1, 127))
 *   :55     p_new = p - (lr*(m_new/bc1)) / (sqrt(v_new/bc2) + eps)
 *   :62-64  bf16 store by integer round-to-nearest-even
 * Padding lanes of a partial last block contribute 0 to the absmax (:19-32).
 * Built with -ffp-contract=off so the only fused operations are the explicit
 * fmaf() calls; float arithmetic is IEEE single (SSE), sqrtf correctly rounded.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

void oracle_adam8_step(void* p_raw, const void* g_raw, int8_t* m, int8_t* v, float* ms, float* vs,
                       int64_t n, int is_bf16, float lr, float b1, float b2, float eps, float bc1,
                       float bc2, float wd) {
  const float one_m_b1 = 1.0f - b1;
  const float one_m_b2 = 1.0f - b2;
  const float lr_wd = lr * wd;
  float mn[256], vn[256], pv[256];
  const int64_t nblocks = (n + 255) / 256;
  for (int64_t b = 0; b < nblocks; ++b) {
    const int64_t base = b * 256;
    const int cnt = (int)((n - base) < 256 ? (n - base) : 256);
    const float s_m = ms[b], s_v = vs[b];
    float amax_m = 0.0f, amax_v = 0.0f;
    for (int i = 0; i < cnt; ++i) {
      const int64_t k = base + i;
      float p, g;
      if (is_bf16) {
        p = bf16_to_f32(((const uint16_t*)p_raw)[k]);
        g = bf16_to_f32(((const uint16_t*)g_raw)[k]);
      } else {
        p = ((const float*)p_raw)[k];
        g = ((const float*)g_raw)[k];
      }
      const float mf = (float)m[k] * s_m;
      const float vf = (float)v[k] * s_v;
      if (wd > 0.0f) p = fmaf(-lr_wd, p, p);
      mn[i] = fmaf(one_m_b1, g, b1 * mf);
      vn[i] = fmaf(one_m_b2 * g, g, b2 * vf);
      pv[i] = p;
      amax_m = fmaxf(amax_m, fabsf(mn[i]));
      amax_v = fmaxf(amax_v, fabsf(vn[i]));
    }
    const float nms = fmaxf(amax_m / 127.0f, 1e-14f);
    const float nvs = fmaxf(amax_v / 127.0f, 1e-14f);
    ms[b] = nms;
    vs[b] = nvs;
    for (int i = 0; i < cnt; ++i) {
      const int64_t k = base + i;
      const float qm = mn[i] / nms;
      const float rm = mn[i] >= 0.0f ? qm + 0.5f : qm - 0.5f;
      m[k] = (int8_t)(int)fminf(fmaxf(rm, -127.0f), 127.0f);
      const float rv = vn[i] / nvs + 0.5f;
      v[k] = (int8_t)(int)fminf(fmaxf(rv, 1.0f), 127.0f);
      const float step = lr * (mn[i] / bc1);
      const float denom = sqrtf(vn[i] / bc2) + eps;
      const float pn = pv[i] - step / denom;
      if (is_bf16)
        ((uint16_t*)p_raw)[k] = f32_to_bf16_rne(pn);
      else
        ((float*)p_raw)[k] = pn;
    }
  }
}
