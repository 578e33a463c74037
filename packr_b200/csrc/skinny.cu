// Few-token (up to 128) GEMMs of the forward and of dX on the tensor cores,
// where streaming W from HBM is the bound ("skinny" GEMMs):
//   FWD  out^T[n, m] = W^T[n, k] . x^T[k, m]      (kernel.py:133-139 transposed)
//   DX   dX^T[k, m]  = W[k, n] . bf16(dY)^T[n, m] (autograd.py:70 transposed)
// One CTA per SM (no cluster), tcgen05.mma.cta_group::1 with M = 128 output
// features (weight columns for FWD, weight rows for DX) and N = the padded
// token count, so no MMA row is wasted on absent tokens.  The A operand is
// this CTA's 128-feature slice of W, staged by TMA (W_f straight into its
// 128-byte-swizzled layout, MN-major for FWD and K-major for DX, W_p beside
// it) and decoded in place by the same routine as the large GEMMs; the B
// operand is the K-major activation tile (x, or bf16(dY) for DX).  Work units
// are (128-feature tile, reduction split) pairs, walked by a persistent grid;
// each unit's f32 accumulator (one of two TMEM slots, so a unit's epilogue
// overlaps the next unit's mainloop) goes to partial[split][m][feature] and a
// reduce kernel adds the splits in a fixed order (FWD: plus the bias, f32
// out; DX: rounded to bf16 like the large dX GEMM).  Every wait is bounded
// like the large GEMMs'.
#include "common.cuh"

namespace packr {
namespace gemm {

// Stage slots of the barrier block.
constexpr int kSkMaxStages = 6;

template <int MODE, int NPAD>
struct SkCfg {
  // as many stages as shared memory holds: under full load a stage's TMA
  // takes ~2.3 us to land, so the ring's depth sets the streaming rate.  (A
  // 16-token MMA width with a lut of two bf16 entries per shared-memory word,
  // which fits 8 stages, measured 14 % slower at 16 tokens on a B200.)
  static constexpr int kStages = NPAD <= 64 ? 6 : NPAD <= 128 ? 4 : 3;
  static constexpr int kWBytes = BN_CTA * BK * 2;  // W_f / decoded A tile: 128 features x 64 reduction
  static constexpr int kXBytes = NPAD * BK * 2;    // x tile: NPAD tokens x 64 k, K-major
  static constexpr int kPBytes = BN_CTA * BK;      // W_p tile, u8 row-major (FWD 64 x 128, DX 128 x 64)
  static constexpr int kStageBytes = kWBytes + kXBytes + kPBytes;
  static constexpr int kEpiWarps = 4;
  // 16 decode warps (two 8-column chunks per thread and stage): a stage is
  // ready for the MMA when its slowest decode warp is done, and that wait is
  // part of every ring round trip (traced on B200 at 16 tokens: 8 warps took
  // up to 1.4 us per stage against a ~3.2 us TMA landing; 16 measured 5-7 %
  // faster from 8 to 128 tokens)
  static constexpr int kDecWarps = 16;
  static constexpr int kDecWarp0 = 2 + kEpiWarps;
  static constexpr int kThreads = (2 + kEpiWarps + kDecWarps) * 32;
  static constexpr int kTmemCols = 2 * NPAD;  // two accumulator slots
  static constexpr int kLutBytes = LUT_BYTES;
  static constexpr int kBarOff = kStages * kStageBytes + kLutBytes;
  static constexpr int kSmemBytes = kBarOff + 256 + 1024;
  // A: W^T (FWD: the tile's rows of W are K, so A is MN-major) or W (DX:
  // W's rows are the output features and the reduction runs along them: K-major)
  static constexpr uint32_t kIdesc = idesc_bf16_f32(128, NPAD, /*A MN-major*/ MODE == FWD, /*B MN-major*/ false);
  static constexpr uint32_t kTxBytes = kWBytes + kXBytes + kPBytes;
};

struct SkBars {
  uint64_t full[kSkMaxStages];    // W_f, W_p and x tiles landed            (count 1 + tx)
  uint64_t bfull[kSkMaxStages];   // A tile decoded                         (count decode warps)
  uint64_t empty[kSkMaxStages];   // MMAs done with the stage               (count 1)
  uint64_t tfull[2];   // accumulator complete                   (count 1)
  uint64_t tempty[2];  // accumulator drained                    (count epilogue warps)
  uint32_t tmem_base;
  int abort;
};

struct SkParams {
  int M, N, K;                            // tokens, output features, reduction length
  int n_tiles, k_blocks, splits, kb_per;  // split s: k-blocks [s * kb_per, min(k_blocks, (s + 1) * kb_per))
  float* partial;                         // [splits][M][N]
  Params dec;                             // W bounds for the decode (w_rows = K, w_cols = N)
};

struct SkMaps {
  CUtensorMap wf, wp, x;
};

template <int MODE, int NPAD>
__global__ void __launch_bounds__(SkCfg<MODE, NPAD>::kThreads, 1)
    skinny_kernel(const SkParams P, const __grid_constant__ SkMaps maps) {
  static_assert(MODE == FWD || MODE == DX, "forward or dX");
  using C = SkCfg<MODE, NPAD>;
  constexpr int S = C::kStages;
  static_assert(S <= kSkMaxStages, "barrier slots");
  static_assert(C::kBarOff + (int)sizeof(SkBars) <= C::kSmemBytes - 1024, "barrier block");
  static_assert(C::kSmemBytes <= 227 * 1024, "shared memory per CTA");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint32_t* lut_s = reinterpret_cast<uint32_t*>(smem + S * C::kStageBytes);
  SkBars* bars = reinterpret_cast<SkBars*>(smem + C::kBarOff);
  volatile int* abort_flag = &bars->abort;
  auto w_tile = [&](int s) { return smem + s * C::kStageBytes; };
  auto x_tile = [&](int s) { return smem + s * C::kStageBytes + C::kWBytes; };
  auto p_tile = [&](int s) { return smem + s * C::kStageBytes + C::kWBytes + C::kXBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = P.n_tiles * P.splits;
  auto unit_range = [&](int u, int& n0, int& split, int& kb0, int& kb1) {
    n0 = (u % P.n_tiles) * BN_CTA;
    split = u / P.n_tiles;
    kb0 = split * P.kb_per;
    kb1 = min(P.k_blocks, kb0 + P.kb_per);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->bfull[s], C::kDecWarps);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->tfull[a], 1);
      mbar_init(&bars->tempty[a], C::kEpiWarps);
    }
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&maps.wf);
    prefetch_tmap(&maps.wp);
    prefetch_tmap(&maps.x);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp >= C::kDecWarp0) {
    const int dw = warp - C::kDecWarp0;
    for (int e = dw; e < 256; e += C::kDecWarps) lut_s[e * 32 + lane] = f32_to_bf16_rne(__ldg(P.dec.lut + e));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int n0, split, kb0, kb1;
        unit_range(u, n0, split, kb0, kb1);
        for (int kk = kb0; kk < kb1; ++kk, ++it) {
          const int s = it % S;
          const uint32_t ph = (uint32_t)(it / S) & 1u;
          if (!mbar_wait(&bars->empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
          PACKR_TRACE_EVENT(0, it);
          const int k0 = kk * BK;
          mbar_arrive_expect_tx(&bars->full[s], C::kTxBytes);
          if (MODE == FWD) {  // W rows k0.., columns n0..n0+127: two 64-column boxes
            tma_load_2d(w_tile(s), &maps.wf, &bars->full[s], n0, k0);
            tma_load_2d(w_tile(s) + 8192, &maps.wf, &bars->full[s], n0 + 64, k0);
            tma_load_2d(p_tile(s), &maps.wp, &bars->full[s], n0, k0);
          } else {            // W rows n0..n0+127, columns k0..k0+63: one box each
            tma_load_2d(w_tile(s), &maps.wf, &bars->full[s], k0, n0);
            tma_load_2d(p_tile(s), &maps.wp, &bars->full[s], k0, n0);
          }
          tma_load_2d(x_tile(s), &maps.x, &bars->full[s], k0, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, t_local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++t_local) {
        int n0, split, kb0, kb1;
        unit_range(u, n0, split, kb0, kb1);
        const int acc = t_local & 1;
        const uint32_t aph = (uint32_t)(t_local >> 1) & 1u;
        if (!mbar_wait(&bars->tempty[acc], aph ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int kk = kb0; kk < kb1; ++kk, ++it) {
          const int s = it % S;
          const uint32_t ph = (uint32_t)(it / S) & 1u;
          // the x tile: full; the decoded W tile: bfull
          if (!mbar_wait(&bars->full[s], ph, abort_flag)) { ok = false; break; }
          if (!mbar_wait(&bars->bfull[s], ph, abort_flag)) { ok = false; break; }
          PACKR_TRACE_EVENT(2, it);
          tc_fence_after();
          const uint32_t a_s = smem_u32(w_tile(s)), b_s = smem_u32(x_tile(s));
#pragma unroll
          for (int k = 0; k < BK / UK; ++k) {
            const uint64_t ad = MODE == FWD ? sdesc_sw128(a_s + k * 2048, 8192, 1024) : sdesc_sw128(a_s + k * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b_s + k * 32, 16, 1024);
            umma_bf16_ss(tmem_base + (uint32_t)(acc * NPAD), ad, bd, C::kIdesc, (kk != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit(&bars->empty[s]);
        }
        if (!ok) break;
        umma_commit(&bars->tfull[acc]);
      }
    }
  } else if (warp < C::kDecWarp0) {
    // ------------------------------------------------ epilogue: partial[split][m][n]
    const int q = warp & 3;  // TMEM lane quarter = output features q*32 .. q*32+31 of the tile
    int t_local = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++t_local) {
      int n0, split, kb0, kb1;
      unit_range(u, n0, split, kb0, kb1);
      const int acc = t_local & 1;
      const uint32_t aph = (uint32_t)(t_local >> 1) & 1u;
      if (!mbar_wait_warp(&bars->tfull[acc], aph, abort_flag, kEpilogueSleepNs)) break;
      tc_fence_after();
      const long long n = (long long)n0 + q * 32 + lane;
      float* dst = P.partial + (long long)split * P.M * P.N + n;
#pragma unroll
      for (int c = 0; c < NPAD / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + (uint32_t)(acc * NPAD + c * 32) + ((uint32_t)(q * 32) << 16), v);
        tmem_ld_wait();
        if (n < P.N) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = c * 32 + j;
            if (m < P.M) __stcg(dst + (long long)m * P.N, __uint_as_float(v[j]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tempty[acc]);
    }
  } else {
    // ------------------------------------------------ weight decode, in place
    const int t = threadIdx.x - C::kDecWarp0 * 32;
    const uint32_t* lut_lane = lut_s + lane;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int n0, split, kb0, kb1;
      unit_range(u, n0, split, kb0, kb1);
      for (int kk = kb0; kk < kb1; ++kk, ++it) {
        const int s = it % S;
        const uint32_t ph = (uint32_t)(it / S) & 1u;
        if (!mbar_wait_warp(&bars->full[s], ph, abort_flag)) { ok = false; break; }
        if (t == 0) PACKR_TRACE_EVENT(6, it);
        decode_in_place<MODE, C::kDecWarps * 32>(P.dec, w_tile(s), p_tile(s), lut_lane, t, n0, kk * BK);
        fence_proxy_async_smem();
        __syncwarp();
        if (t == 0) PACKR_TRACE_EVENT(7, it);
        if (lane == 0) mbar_arrive(&bars->bfull[s]);
      }
    }
  }
  // every MMA has completed before the accumulator memory is released: the
  // epilogue waited on the last tfull (or the CTA gave up)
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// Padded MMA width for the token count (the skinny route serves up to 128).
inline int skinny_npad(long long M) {
  return M <= 32 ? 32 : M <= 64 ? 64 : 128;
}

struct SkPlan {
  int npad, n_tiles, k_blocks, splits, kb_per, grid;
};

// Reduction splits (R = reduction length, Out = output features): the fewest
// waves of units over the resident CTAs (one per SM), each unit at least 4
// k-blocks, the partial sums at most 1/8 of W's bytes.
inline SkPlan skinny_plan(long long M, long long R, long long Out) {
  SkPlan p{};
  p.npad = skinny_npad(M);
  p.n_tiles = (int)((Out + BN_CTA - 1) / BN_CTA);
  p.k_blocks = (int)((R + BK - 1) / BK);
  const int sms = sm_count();
  long long cap = (3 * R) / (32 * M);  // splits * M * Out * 4 <= 3 * R * Out / 8
  const long long cap_k = p.k_blocks / 4 > 0 ? p.k_blocks / 4 : 1;
  if (cap > cap_k) cap = cap_k;
  if (cap < 1) cap = 1;
  double best = 1e30;
  p.splits = 1;
  for (long long s = 1; s <= cap; ++s) {
    const long long per = (p.k_blocks + s - 1) / s;
    const long long units = (long long)p.n_tiles * s;
    const long long waves = (units + sms - 1) / sms;
    const double t = (double)waves * (per + 2);  // + drain / ramp of a unit
    if (t < best - 1e-9) {
      best = t;
      p.splits = (int)s;
    }
  }
  p.kb_per = (p.k_blocks + p.splits - 1) / p.splits;
  p.splits = (p.k_blocks + p.kb_per - 1) / p.kb_per;
  const long long units = (long long)p.n_tiles * p.splits;
  p.grid = (int)(units < sms ? units : sms);
  return p;
}

inline size_t skinny_partial_bytes(long long M, long long R, long long Out) {
  const SkPlan p = skinny_plan(M, R, Out);
  return (size_t)p.splits * M * Out * sizeof(float);
}

template <int MODE, int NPAD>
int skinny_launch(const SkParams& P, const SkMaps& maps, int grid, cudaStream_t st) {
  using C = SkCfg<MODE, NPAD>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  int rc = 0;
  std::call_once(once[dev & 63], [&] {
    rc = cudaFuncSetAttribute(skinny_kernel<MODE, NPAD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              C::kSmemBytes) != cudaSuccess;
  });
  if (rc) return PACKR_ERR_CUDA;
  skinny_kernel<MODE, NPAD><<<grid, C::kThreads, C::kSmemBytes, st>>>(P, maps);
  return launch_status();
}

// The skinny GEMM's main launch: act_bf16 [M, ld_act] (x for FWD, bf16(dY)
// for DX; ld_act % 8 == 0), W [K, N] as for the TMA-staged decode (wtma_ok),
// partial [splits][M][Out].
template <int MODE>
int skinny_run(const uint16_t* act_bf16, long long ld_act, const uint8_t* W_p, const uint16_t* W_f, const float* lut,
               long long M, long long K, long long N, float* partial, SkPlan& pl, cudaStream_t st) {
  const long long R = MODE == FWD ? K : N, Out = MODE == FWD ? N : K;
  if (M < 1 || M > 128) return PACKR_ERR_SHAPE;
  pl = skinny_plan(M, R, Out);
  SkMaps maps;
  int rc = MODE == FWD ? make_map(&maps.wf, W_f, N, K, N * 2, BK) : make_map(&maps.wf, W_f, N, K, N * 2, BN_CTA);
  if (rc == PACKR_OK)
    rc = MODE == FWD ? make_map_u8(&maps.wp, W_p, N, K, N, BN_CTA, BK) : make_map_u8(&maps.wp, W_p, N, K, N, BK, BN_CTA);
  if (rc == PACKR_OK) rc = make_map(&maps.x, act_bf16, R, M, ld_act * 2, pl.npad);
  if (rc != PACKR_OK) return rc;
  SkParams P{};
  P.M = (int)M;
  P.N = (int)Out;
  P.K = (int)R;
  P.n_tiles = pl.n_tiles;
  P.k_blocks = pl.k_blocks;
  P.splits = pl.splits;
  P.kb_per = pl.kb_per;
  P.partial = partial;
  P.dec.W_p = W_p;
  P.dec.W_f = W_f;
  P.dec.lut = lut;
  P.dec.ldw = N;
  P.dec.w_rows = (int)K;
  P.dec.w_cols = (int)N;
  return pl.npad == 32   ? skinny_launch<MODE, 32>(P, maps, pl.grid, st)
         : pl.npad == 64 ? skinny_launch<MODE, 64>(P, maps, pl.grid, st)
                         : skinny_launch<MODE, 128>(P, maps, pl.grid, st);
}

// dX[m, k] = bf16(sum over splits of partial[split][m][k]), summed in split
// order, stored as bf16 or as the f32 value of that bf16 (f32 x).  One
// thread per 4 consecutive k of one row (16-byte loads when K % 4 == 0).
__global__ void __launch_bounds__(256) skinny_reduce_dx_kernel(const float* __restrict__ partial, int splits, int M,
                                                               int Kout, void* __restrict__ dX, int out_f32) {
  const long long qpr = (Kout + 3) / 4;
  const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= (long long)M * qpr) return;
  const int m = (int)(q / qpr);
  const int k = (int)(q - (long long)m * qpr) * 4;
  const int nv = min(4, Kout - k);
  const long long step = (long long)M * Kout;
  const float* p = partial + (long long)m * Kout + k;
  float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (nv == 4 && (Kout & 3) == 0) {
    for (int sp = 0; sp < splits; ++sp) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(p + sp * step));
      s[0] = __fadd_rn(s[0], v.x);
      s[1] = __fadd_rn(s[1], v.y);
      s[2] = __fadd_rn(s[2], v.z);
      s[3] = __fadd_rn(s[3], v.w);
    }
  } else {
    for (int sp = 0; sp < splits; ++sp)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j < nv) s[j] = __fadd_rn(s[j], __ldcs(p + sp * step + j));
  }
  const long long o = (long long)m * Kout + k;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j < nv) {
      const uint32_t h = pack_bf16x2_rne(s[j], 0.0f) & 0xFFFFu;
      if (out_f32)
        static_cast<float*>(dX)[o + j] = bf16_to_f32(h);
      else
        static_cast<uint16_t*>(dX)[o + j] = (uint16_t)h;
    }
  }
}

// dX of few tokens: dY_bf16 [M, ldd] (ldd % 8 == 0), dX [M, K] bf16 or f32;
// partial: skinny_partial_bytes(M, N, K).
int skinny_dx(const uint16_t* dY_bf16, long long ldd, const uint8_t* W_p, const uint16_t* W_f, const float* lut,
              void* dX, int out_f32, long long M, long long K, long long N, float* partial, cudaStream_t st) {
  SkPlan pl;
  int rc = skinny_run<DX>(dY_bf16, ldd, W_p, W_f, lut, M, K, N, partial, pl, st);
  if (rc != PACKR_OK) return rc;
  skinny_reduce_dx_kernel<<<gemv::reduce_blocks(M, K), 256, 0, st>>>(partial, pl.splits, (int)M, (int)K, dX, out_f32);
  return launch_status();
}

// x_bf16: [M, ldx] bf16 with ldx % 8 == 0; W as for the TMA-staged decode
// (wtma_ok); partial: skinny_partial_bytes(M, K, N).
int skinny_forward(const uint16_t* x_bf16, long long ldx, const uint8_t* W_p, const uint16_t* W_f, const float* lut,
                   const void* bias, int bias_f32, float* out, long long M, long long K, long long N, float* partial,
                   cudaStream_t st) {
  SkPlan pl;
  int rc = skinny_run<FWD>(x_bf16, ldx, W_p, W_f, lut, M, K, N, partial, pl, st);
  if (rc != PACKR_OK) return rc;
  gemv::gemv_reduce_kernel<<<gemv::reduce_blocks(M, N), 256, 0, st>>>(partial, pl.splits, (int)M, (int)N, bias,
                                                                       bias_f32, out, N);
  return launch_status();
}

}  // namespace gemm
}  // namespace packr
