// C-ABI entry points of the PackRLinear forward and backward: argument
// checks, workspace carving, tensor-map encoding and the launch sequence.
#include "common.cuh"

namespace packr {
namespace linear {

constexpr size_t kAlign = 256;

inline size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }
inline long long round8(long long v) { return (v + 7) & ~7ll; }

// Bump allocator over the caller's workspace.
struct Carve {
  uint8_t* base;
  size_t off = 0;
  template <class T>
  T* take(size_t count) {
    if (count == 0) return nullptr;
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off = align_up(off + count * sizeof(T));
    return p;
  }
};

bool x_needs_copy(int x_dtype, long long K) { return x_dtype == PACKR_DTYPE_F32 || (K & 7) != 0; }

// Forward token counts served by the skinny tcgen05 GEMM (W as the 128-row
// MMA operand, tokens as N): measured on the Llama-7B FFN shapes, the
// CUDA-core GEMV streams W fastest up to 4 tokens, the skinny GEMM from 5 to
// 128 (at 128 tokens: 86 vs 81 us for 4096 -> 11008 and 67 vs 186 us for
// 11008 -> 4096, whose 16 column tiles leave most SMs idle in the 256-row
// tile GEMM), the 256-row tile GEMMs beyond.
#ifndef PACKR_SKINNY_MIN_M
#define PACKR_SKINNY_MIN_M 5
#endif
constexpr long long kSkinnyMaxM = 128;
inline bool skinny_eligible(long long M, long long N) {
  return M >= PACKR_SKINNY_MIN_M && M <= kSkinnyMaxM && (N & 15) == 0;
}
// dX of up to 128 tokens takes the skinny GEMM (W rows as the MMA's 128-row
// operand, split over N): the 256 x 256 tile GEMM has only K / 256 output
// tiles there (16 for a 4096-wide layer), which leaves most SMs idle.
inline bool skinny_dx_eligible(long long M, long long N) { return M >= 1 && M <= kSkinnyMaxM && (N & 15) == 0; }

// FWD / DX take the predecode + plain GEMM route for M >= PACKR_PREDECODE_MIN_M
// (129: above the skinny GEMM's range) when W's layout allows TMA (N % 16 ==
// 0, 16-byte aligned W_p / W_f) and the workspace holds the decoded W;
// otherwise the fused-decode GEMM runs.
inline bool predecode_eligible(long long M, long long N) { return M >= PACKR_PREDECODE_MIN_M && (N & 15) == 0; }

// Stream-K scratch (partial tiles and flags) for up to this many CTA pairs.
inline int sk_pairs() { return sm_count() / 2; }
inline int plain_msub(long long M) { return M >= PACKR_PLAIN_MSUB2_MIN_M ? 2 : 1; }

struct FwdPlan {
  uint16_t* xh;
  uint16_t* wd;  // decoded W [K, N] (predecode route only)
  float* skp;    // stream-K partials / flags (predecode route only)
  int* skf;
};

size_t plan_forward(Carve& c, FwdPlan& p, long long M, long long K, long long N, int x_dtype, bool pre,
                    bool sk = false) {
  p.xh = x_needs_copy(x_dtype, K) ? c.take<uint16_t>((size_t)M * round8(K)) : nullptr;
  p.wd = pre ? c.take<uint16_t>((size_t)K * N) : nullptr;
  const bool use_sk = pre && sk;
  p.skp = use_sk ? c.take<float>(gemm::sk_partial_bytes(sk_pairs(), plain_msub(M)) / sizeof(float)) : nullptr;
  p.skf = use_sk ? c.take<int>(gemm::sk_flag_bytes(sk_pairs()) / sizeof(int)) : nullptr;
  return c.off;
}

struct BwdPlan {
  uint16_t *dh, *dl, *xh, *xl;
  uint16_t* wd;  // decoded W [K, N] (predecode route for dX only)
  float* skdx;   // split partial sums of the skinny dX GEMM (few tokens)
  float* skp;    // stream-K partials / flags of the plain dX GEMM
  int* skf;
  float *colsum, *dlut_sum;
  int32_t* counts;
};

size_t plan_backward(Carve& c, BwdPlan& p, long long M, long long K, long long N, int x_dtype, int flags,
                     bool want_dx, bool want_dw, bool want_dlut, bool want_dbias, bool have_counts, bool pre,
                     bool sk = false, bool wd_given = false, bool skdx = false) {
  const bool split = (flags & PACKR_BWD_DW_SPLIT) != 0 && (want_dw || want_dlut);
  p.wd = pre && want_dx && !wd_given ? c.take<uint16_t>((size_t)K * N) : nullptr;
  p.skdx = skdx && want_dx ? c.take<float>(gemm::skinny_partial_bytes(M, N, K) / sizeof(float)) : nullptr;
  const bool use_sk = sk && pre && want_dx;  // only the plain dX GEMM splits tiles (stream-K)
  const int msub = pre && want_dx ? plain_msub(M) : 1;
  p.skp = use_sk ? c.take<float>(gemm::sk_partial_bytes(sk_pairs(), msub) / sizeof(float)) : nullptr;
  p.skf = use_sk ? c.take<int>(gemm::sk_flag_bytes(sk_pairs()) / sizeof(int)) : nullptr;
  p.dh = c.take<uint16_t>((size_t)M * round8(N));
  p.dl = split ? c.take<uint16_t>((size_t)M * round8(N)) : nullptr;
  const bool need_x = want_dw || want_dlut;
  p.xh = need_x && x_needs_copy(x_dtype, K) ? c.take<uint16_t>((size_t)M * round8(K)) : nullptr;
  p.xl = need_x && split && x_dtype == PACKR_DTYPE_F32 ? c.take<uint16_t>((size_t)M * round8(K)) : nullptr;
  p.colsum = want_dbias ? c.take<float>((size_t)N) : nullptr;
  p.dlut_sum = want_dlut ? c.take<float>(256) : nullptr;
  p.counts = want_dlut && !have_counts ? c.take<int32_t>(256) : nullptr;
  return c.off;
}

int check_common(const void* x, int x_dtype, const uint8_t* W_p, const uint16_t* W_f, const float* lut, long long M,
                 long long K, long long N) {
  if (M < 0 || K <= 0 || N <= 0) return PACKR_ERR_SHAPE;
  if (M > 0x7FFFFFFFll || K > 0x7FFFFFFFll || N > 0x7FFFFFFFll) return PACKR_ERR_SHAPE;
  if (x_dtype != PACKR_DTYPE_F32 && x_dtype != PACKR_DTYPE_BF16) return PACKR_ERR_INVALID_ARGUMENT;
  if ((M > 0 && x == nullptr) || W_p == nullptr || W_f == nullptr || lut == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
  if (!aligned(W_f, 2) || !aligned(lut, 4) || (x && !aligned(x, x_dtype == PACKR_DTYPE_F32 ? 4 : 2)))
    return PACKR_ERR_ALIGNMENT;
  return PACKR_OK;
}

}  // namespace linear
}  // namespace packr

using namespace packr;
using namespace packr::linear;

extern "C" size_t packr_forward_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype) {
  Carve c{nullptr};
  FwdPlan p;
  M = M > 0 ? M : 0;
  K = K > 0 ? K : 0;
  N = N > 0 ? N : 0;
  const bool pre = predecode_eligible(M, N);
  size_t need = plan_forward(c, p, M, K, N, x_dtype, pre, pre);
  if (M >= 1 && K > 0 && N > 0) {
    // few rows: the split partial sums of the skinny GEMM (plus its bf16 x);
    // the CUDA-core route needs none
    if (skinny_eligible(M, N)) {
      Carve c2{nullptr};
      FwdPlan p2;
      const size_t g = plan_forward(c2, p2, M, K, N, x_dtype, false) +
                       align_up(gemm::skinny_partial_bytes(M, K, N));
      if (g > need) need = g;
    }
  }
  return need;
}

extern "C" int packr_forward(const void* x, int x_dtype, const uint8_t* W_p, const uint16_t* W_f, const float* lut,
                             const void* bias, int bias_dtype, float* out, int64_t M, int64_t K, int64_t N, void* workspace,
                             size_t workspace_bytes, void* stream) {
  int st = check_common(x, x_dtype, W_p, W_f, lut, M, K, N);
  if (st != PACKR_OK) return st;
  if (out == nullptr && M > 0) return PACKR_ERR_INVALID_ARGUMENT;
  if (bias != nullptr && bias_dtype != PACKR_DTYPE_BF16 && bias_dtype != PACKR_DTYPE_F32)
    return PACKR_ERR_INVALID_ARGUMENT;
  if (bias != nullptr && !aligned(bias, bias_dtype == PACKR_DTYPE_F32 ? 4 : 2)) return PACKR_ERR_ALIGNMENT;
  if ((st = check_device()) != PACKR_OK) return st;
  if (M == 0) return PACKR_OK;
  cudaStream_t s = as_stream(stream);
  // few tokens: the skinny tcgen05 GEMM (W streamed once as the MMA's
  // 128-row operand, split over K), when the workspace holds its partials
  if (skinny_eligible(M, N) && gemm::wtma_ok(W_p, W_f, N) && workspace != nullptr && aligned(workspace, kAlign)) {
    Carve c2{static_cast<uint8_t*>(workspace)};
    FwdPlan p2;
    plan_forward(c2, p2, M, K, N, x_dtype, false);
    float* partial = c2.take<float>(gemm::skinny_partial_bytes(M, K, N) / sizeof(float));
    if (workspace_bytes >= c2.off) {
      const uint16_t* xb = static_cast<const uint16_t*>(x);
      long long ldx = K;
      if (p2.xh != nullptr) {
        st = prep::split_rows(x, x_dtype == PACKR_DTYPE_F32, K, M, K, p2.xh, nullptr, round8(K), nullptr, s);
        if (st != PACKR_OK) return st;
        xb = p2.xh;
        ldx = round8(K);
      }
      return gemm::skinny_forward(xb, ldx, W_p, W_f, lut, bias, bias_dtype == PACKR_DTYPE_F32, out, M, K, N,
                                  partial, s);
    }
  }
  // few rows: stream W once through the CUDA cores (fp16-lut decode of the
  // reference's forward, f32 accumulation, one launch, no workspace)
  if (gemv::eligible(M, K, N, W_p, W_f)) {
    return gemv::forward(x, x_dtype == PACKR_DTYPE_F32, W_p, W_f, lut, bias, bias_dtype == PACKR_DTYPE_F32, out, M,
                         K, N, static_cast<float*>(workspace), s);
  }
  // the richest route the workspace holds: predecode + stream-K, predecode,
  // fused decode
  const bool pre_ok = predecode_eligible(M, N) && gemm::wtma_ok(W_p, W_f, N);
  Carve c{static_cast<uint8_t*>(workspace)};
  FwdPlan p;
  bool pre = false;
  size_t need = 0;
  const bool tries[3][2] = {{true, true}, {true, false}, {false, false}};
  for (const auto& t : tries) {
    if (t[0] && !pre_ok) continue;
    c = Carve{static_cast<uint8_t*>(workspace)};
    need = plan_forward(c, p, M, K, N, x_dtype, t[0], t[1]);
    pre = t[0];
    if (workspace_bytes >= need) break;
  }
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned(workspace, kAlign)))
    return PACKR_ERR_WORKSPACE;
  const void* a_ptr = x;
  long long lda = K;
  if (p.xh != nullptr) {
    st = prep::split_rows(x, x_dtype == PACKR_DTYPE_F32, K, M, K, p.xh, nullptr, round8(K), nullptr, s);
    if (st != PACKR_OK) return st;
    a_ptr = p.xh;
    lda = round8(K);
  }
  gemm::Maps maps;
  st = gemm::make_map(&maps.a[0], a_ptr, K, M, lda * 2, gemm::BM);
  if (st != PACKR_OK) return st;
  gemm::Params P{};
  P.Mg = (int)M;
  P.Ng = (int)N;
  P.Kg = (int)K;
  P.nseg = 1;
  P.W_p = W_p;
  P.W_f = W_f;
  P.lut = lut;
  P.ldw = N;
  P.w_rows = (int)K;
  P.w_cols = (int)N;
  P.out = out;
  P.ld_out = N;
  P.bias = bias;
  P.bias_f32 = bias_dtype == PACKR_DTYPE_F32;
  P.sk_partial = p.skp;
  P.sk_flags = p.skf;
  P.sk_slots = p.skp != nullptr ? sk_pairs() : 0;
  if (pre) {
    if ((st = gemm::predecode(W_p, W_f, lut, p.wd, K, N, s)) != PACKR_OK) return st;
    if ((st = gemm::make_map(&maps.b[0], p.wd, N, K, N * 2, 64)) != PACKR_OK) return st;
    return gemm::launch_plain<gemm::FWD>(P, maps, s);
  }
  return gemm::launch<gemm::FWD>(P, maps, s);
}

extern "C" size_t packr_forward_decoded_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype) {
  Carve c{nullptr};
  FwdPlan p;
  return plan_forward(c, p, M > 0 ? M : 0, K > 0 ? K : 0, N > 0 ? N : 0, x_dtype, false);
}

extern "C" int packr_forward_decoded(const void* x, int x_dtype, const uint16_t* Wd, const void* bias, int bias_dtype,
                                     float* out, int64_t M, int64_t K, int64_t N, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  if (M < 0 || K <= 0 || N <= 0 || M > 0x7FFFFFFFll || K > 0x7FFFFFFFll || N > 0x7FFFFFFFll) return PACKR_ERR_SHAPE;
  if ((N & 7) != 0) return PACKR_ERR_SHAPE;  // Wd rows must be 16-byte multiples for TMA
  if (x_dtype != PACKR_DTYPE_F32 && x_dtype != PACKR_DTYPE_BF16) return PACKR_ERR_INVALID_ARGUMENT;
  if (Wd == nullptr || (M > 0 && (x == nullptr || out == nullptr))) return PACKR_ERR_INVALID_ARGUMENT;
  if (bias != nullptr && bias_dtype != PACKR_DTYPE_BF16 && bias_dtype != PACKR_DTYPE_F32)
    return PACKR_ERR_INVALID_ARGUMENT;
  if (!aligned(Wd, 16) || (x && !aligned(x, x_dtype == PACKR_DTYPE_F32 ? 4 : 2)) || !aligned(out, 4) ||
      (bias != nullptr && !aligned(bias, bias_dtype == PACKR_DTYPE_F32 ? 4 : 2)))
    return PACKR_ERR_ALIGNMENT;
  int st = check_device();
  if (st != PACKR_OK) return st;
  if (M == 0) return PACKR_OK;
  cudaStream_t s = as_stream(stream);
  Carve c{static_cast<uint8_t*>(workspace)};
  FwdPlan p;
  const size_t need = plan_forward(c, p, M, K, N, x_dtype, false);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned(workspace, kAlign)))
    return PACKR_ERR_WORKSPACE;
  const void* a_ptr = x;
  long long lda = K;
  if (p.xh != nullptr) {
    st = prep::split_rows(x, x_dtype == PACKR_DTYPE_F32, K, M, K, p.xh, nullptr, round8(K), nullptr, s);
    if (st != PACKR_OK) return st;
    a_ptr = p.xh;
    lda = round8(K);
  }
  gemm::Maps maps;
  if ((st = gemm::make_map(&maps.a[0], a_ptr, K, M, lda * 2, gemm::BM)) != PACKR_OK) return st;
  if ((st = gemm::make_map(&maps.b[0], Wd, N, K, N * 2, 64)) != PACKR_OK) return st;
  gemm::Params P{};
  P.Mg = (int)M;
  P.Ng = (int)N;
  P.Kg = (int)K;
  P.nseg = 1;
  P.out = out;
  P.ld_out = N;
  P.bias = bias;
  P.bias_f32 = bias_dtype == PACKR_DTYPE_F32;
  return gemm::launch_plain<gemm::FWD>(P, maps, s);
}

extern "C" size_t packr_backward_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype, int flags) {
  Carve c{nullptr};
  BwdPlan p;
  M = M > 0 ? M : 0;
  K = K > 0 ? K : 0;
  N = N > 0 ? N : 0;
  return plan_backward(c, p, M, K, N, x_dtype, flags, true, true, true, true, false, predecode_eligible(M, N), true,
                       false, M > 0 && K > 0 && skinny_dx_eligible(M, N));
}

namespace packr {
namespace linear {
// The backward launch sequence; wd_given (nullable) is W decoded by the
// caller exactly as packr_predecode_bf16 decodes it, used instead of a
// predecode of its own by the plain dX GEMM.
static int backward_impl(const float* dY, const void* x, int x_dtype, const uint8_t* W_p, const uint16_t* W_f,
                         const float* lut, const uint16_t* wd_given, const int32_t* lut_counts, void* dX,
                         uint16_t* dW_f, float* dlut, uint16_t* dbias, int64_t M, int64_t K, int64_t N, int flags,
                         void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_common(x, x_dtype, W_p, W_f, lut, M, K, N);
  if (st != PACKR_OK) return st;
  if (M > 0 && dY == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
  if ((flags & ~PACKR_BWD_DW_SPLIT) != 0) return PACKR_ERR_INVALID_ARGUMENT;
  if ((dY && !aligned(dY, 4)) || (dX && !aligned(dX, x_dtype == PACKR_DTYPE_F32 ? 4 : 2)) ||
      (dW_f && !aligned(dW_f, 2)) || (dlut && !aligned(dlut, 4)) || (dbias && !aligned(dbias, 2)) ||
      (lut_counts && !aligned(lut_counts, 4)))
    return PACKR_ERR_ALIGNMENT;
  if ((st = check_device()) != PACKR_OK) return st;
  cudaStream_t s = as_stream(stream);
  const bool want_dx = dX != nullptr, want_dw = dW_f != nullptr, want_dlut = dlut != nullptr,
             want_dbias = dbias != nullptr;
  if (M == 0) {  // empty batch: every gradient is zero
    if (want_dw && cudaMemsetAsync(dW_f, 0, (size_t)K * N * 2, s) != cudaSuccess) return PACKR_ERR_CUDA;
    if (want_dlut && cudaMemsetAsync(dlut, 0, 256 * 4, s) != cudaSuccess) return PACKR_ERR_CUDA;
    if (want_dbias && cudaMemsetAsync(dbias, 0, (size_t)N * 2, s) != cudaSuccess) return PACKR_ERR_CUDA;
    return PACKR_OK;
  }
  // the richest route the workspace holds (for dX: predecode with stream-K,
  // predecode, or the skinny GEMM for few tokens; else the fused decode)
  const bool pre_ok = want_dx && predecode_eligible(M, N) && gemm::wtma_ok(W_p, W_f, N);
  const bool skdx_ok = want_dx && skinny_dx_eligible(M, N) && gemm::wtma_ok(W_p, W_f, N);
  Carve c{static_cast<uint8_t*>(workspace)};
  BwdPlan p;
  bool pre = false;
  size_t need = 0;
  const bool tries[4][3] = {{true, true, false}, {true, false, false}, {false, false, true}, {false, false, false}};
  for (const auto& t : tries) {
    if ((t[0] && !pre_ok) || (t[2] && !skdx_ok)) continue;
    c = Carve{static_cast<uint8_t*>(workspace)};
    need = plan_backward(c, p, M, K, N, x_dtype, flags, want_dx, want_dw, want_dlut, want_dbias,
                         lut_counts != nullptr, t[0], t[1], wd_given != nullptr, t[2]);
    pre = t[0];
    if (workspace_bytes >= need) break;
  }
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, kAlign)) return PACKR_ERR_WORKSPACE;
  if (p.colsum && cudaMemsetAsync(p.colsum, 0, (size_t)N * 4, s) != cudaSuccess) return PACKR_ERR_CUDA;
  if (p.dlut_sum && cudaMemsetAsync(p.dlut_sum, 0, 256 * 4, s) != cudaSuccess) return PACKR_ERR_CUDA;
  const long long ldN = round8(N), ldK = round8(K);
  // bf16(dY) (+ its residual for the split dW) and the bias gradient sums
  st = prep::split_rows(dY, 1, N, M, N, p.dh, p.dl, ldN, p.colsum, s);
  if (st != PACKR_OK) return st;
  if (want_dx && p.skdx != nullptr) {
    st = gemm::skinny_dx(p.dh, ldN, W_p, W_f, lut, dX, x_dtype == PACKR_DTYPE_F32, M, K, N, p.skdx, s);
    if (st != PACKR_OK) return st;
  } else if (want_dx) {
    gemm::Maps maps;
    if ((st = gemm::make_map(&maps.a[0], p.dh, N, M, ldN * 2, gemm::BM)) != PACKR_OK) return st;
    gemm::Params P{};
    P.Mg = (int)M;
    P.Ng = (int)K;
    P.Kg = (int)N;
    P.nseg = 1;
    P.W_p = W_p;
    P.W_f = W_f;
    P.lut = lut;
    P.ldw = N;
    P.w_rows = (int)K;
    P.w_cols = (int)N;
    P.out = dX;
    P.ld_out = K;
    P.out_f32 = x_dtype == PACKR_DTYPE_F32;
    P.sk_partial = p.skp;
    P.sk_flags = p.skf;
    P.sk_slots = p.skp != nullptr ? sk_pairs() : 0;
    if (pre) {
      const uint16_t* wd = wd_given;
      if (wd == nullptr) {
        if ((st = gemm::predecode(W_p, W_f, lut, p.wd, K, N, s)) != PACKR_OK) return st;
        wd = p.wd;
      }
      if ((st = gemm::make_map(&maps.b[0], wd, N, K, N * 2, gemm::BN_CTA)) != PACKR_OK) return st;
      st = gemm::launch_plain<gemm::DX>(P, maps, s);
    } else {
      st = gemm::launch<gemm::DX>(P, maps, s);
    }
    if (st != PACKR_OK) return st;
  }
  if (want_dw || want_dlut) {
    const void* xa = x;
    long long ldx = K;
    if (p.xh != nullptr) {
      st = prep::split_rows(x, x_dtype == PACKR_DTYPE_F32, K, M, K, p.xh, p.xl, ldK, nullptr, s);
      if (st != PACKR_OK) return st;
      xa = p.xh;
      ldx = ldK;
    }
    // reduction segments: x.dh  [+ x.dl  [+ xl.dh]]
    gemm::Maps maps;
    int nseg = 0;
    auto add_seg = [&](const void* a, long long lda, const void* b) -> int {
      int r = gemm::make_map(&maps.a[nseg], a, K, M, lda * 2, 64);
      if (r == PACKR_OK) r = gemm::make_map(&maps.b[nseg], b, N, M, ldN * 2, 64);
      ++nseg;
      return r;
    };
    if ((st = add_seg(xa, ldx, p.dh)) != PACKR_OK) return st;
    if (p.dl != nullptr) {
      if ((st = add_seg(xa, ldx, p.dl)) != PACKR_OK) return st;
      if (p.xl != nullptr && (st = add_seg(p.xl, ldK, p.dh)) != PACKR_OK) return st;
    }
    gemm::Params P{};
    P.Mg = (int)K;
    P.Ng = (int)N;
    P.Kg = (int)M;
    P.nseg = nseg;
    P.out = dW_f;
    P.ld_out = N;
    P.hist_idx = want_dlut ? W_p : nullptr;
    P.dlut_sum = p.dlut_sum;
    P.sk_partial = p.skp;
    P.sk_flags = p.skf;
    P.sk_slots = p.skp != nullptr ? sk_pairs() : 0;
    if ((st = gemm::launch<gemm::DW>(P, maps, s)) != PACKR_OK) return st;
  }
  const int32_t* counts = lut_counts;
  if (want_dlut && counts == nullptr) {
    if ((st = prep::bincount256(W_p, K * N, p.counts, s)) != PACKR_OK) return st;
    counts = p.counts;
  }
  return prep::finalize(dlut, p.dlut_sum, counts, dbias, p.colsum, N, s);
}
}  // namespace linear
}  // namespace packr

extern "C" int packr_backward(const float* dY, const void* x, int x_dtype, const uint8_t* W_p, const uint16_t* W_f,
                              const float* lut, const int32_t* lut_counts, void* dX, uint16_t* dW_f, float* dlut,
                              uint16_t* dbias, int64_t M, int64_t K, int64_t N, int flags, void* workspace,
                              size_t workspace_bytes, void* stream) {
  return backward_impl(dY, x, x_dtype, W_p, W_f, lut, nullptr, lut_counts, dX, dW_f, dlut, dbias, M, K, N, flags,
                       workspace, workspace_bytes, stream);
}

extern "C" size_t packr_backward_decoded_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype, int flags) {
  Carve c{nullptr};
  BwdPlan p;
  M = M > 0 ? M : 0;
  K = K > 0 ? K : 0;
  N = N > 0 ? N : 0;
  return plan_backward(c, p, M, K, N, x_dtype, flags, true, true, true, true, false, predecode_eligible(M, N), true,
                       true);
}

extern "C" int packr_backward_decoded(const float* dY, const void* x, int x_dtype, const uint8_t* W_p,
                                      const uint16_t* W_f, const float* lut, const uint16_t* Wd,
                                      const int32_t* lut_counts, void* dX, uint16_t* dW_f, float* dlut,
                                      uint16_t* dbias, int64_t M, int64_t K, int64_t N, int flags, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  if (Wd == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
  if (!aligned(Wd, 16)) return PACKR_ERR_ALIGNMENT;
  return backward_impl(dY, x, x_dtype, W_p, W_f, lut, Wd, lut_counts, dX, dW_f, dlut, dbias, M, K, N, flags,
                       workspace, workspace_bytes, stream);
}

extern "C" int packr_predecode_route(int64_t M, int64_t K, int64_t N, const uint8_t* W_p, const uint16_t* W_f) {
  (void)K;
  return predecode_eligible(M, N) && gemm::wtma_ok(W_p, W_f, N) ? 1 : 0;
}

extern "C" int packr_bincount256(const uint8_t* W_p, int64_t n, int32_t* counts, void* stream) {
  if (n < 0) return PACKR_ERR_SHAPE;
  if ((n > 0 && W_p == nullptr) || counts == nullptr) return PACKR_ERR_INVALID_ARGUMENT;
  if (!aligned(counts, 4)) return PACKR_ERR_ALIGNMENT;
  int st = check_device();
  if (st != PACKR_OK) return st;
  return prep::bincount256(W_p, n, counts, as_stream(stream));
}

extern "C" int packr_lut_finalize(float* dlut, const float* dlut_sum, const int32_t* counts, void* stream) {
  if (!dlut || !dlut_sum || !counts) return PACKR_ERR_INVALID_ARGUMENT;
  int st = check_device();
  if (st != PACKR_OK) return st;
  return prep::finalize(dlut, dlut_sum, counts, nullptr, nullptr, 0, as_stream(stream));
}

extern "C" int packr_predecode_bf16(const uint8_t* W_p, const uint16_t* W_f, const float* lut, uint16_t* out,
                                    int64_t K, int64_t N, void* stream) {
  if (K < 0 || N < 0 || K > 0x7FFFFFFFll || N > 0x7FFFFFFFll) return PACKR_ERR_SHAPE;
  if (K * N == 0) return PACKR_OK;
  if (!W_p || !W_f || !lut || !out) return PACKR_ERR_INVALID_ARGUMENT;
  if ((N & 15) != 0) return PACKR_ERR_SHAPE;
  if (!aligned(lut, 4)) return PACKR_ERR_ALIGNMENT;
  int st = check_device();
  if (st != PACKR_OK) return st;
  return gemm::predecode(W_p, W_f, lut, out, K, N, as_stream(stream));
}

extern "C" int packr_decode_bf16(const uint8_t* W_p, const uint16_t* W_f, const float* lut, uint16_t* out, int64_t K,
                                 int64_t N, void* stream) {
  if (K < 0 || N < 0 || K > 0x7FFFFFFFll || N > 0x7FFFFFFFll) return PACKR_ERR_SHAPE;
  if (K * N == 0) return PACKR_OK;
  if (!W_p || !W_f || !lut || !out) return PACKR_ERR_INVALID_ARGUMENT;
  if (!aligned(W_f, 2) || !aligned(out, 2) || !aligned(lut, 4)) return PACKR_ERR_ALIGNMENT;
  int st = check_device();
  if (st != PACKR_OK) return st;
  return gemm::decode_check(W_p, W_f, lut, out, K, N, as_stream(stream));
}
