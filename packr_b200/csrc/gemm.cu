// tcgen05 GEMMs of the PackRLinear forward and backward, with the weight
// decode fused into the operand pipeline (or read predecoded) and the lut
// gradient folded into the dW epilogue.
//
// One persistent, warp-specialised kernel template serves three GEMMs
// (K = in_features, N = out_features, T = tokens):
//   FWD  out[T,N]  (f32)  = x[T,K] . W[K,N]           + bias      (kernel.py:133-139, layer.py:96-97)
//   DX   dX[T,K]   (bf16) = bf16(dY)[T,N] . W[K,N]^T             (autograd.py:70)
//   DW   dW_f[K,N] (bf16) = x^T[K,T] . dY[T,N], fp32 accumulate   (autograd.py:73-75)
//        + dlut_sum[W_p[k,n]] += dW[k,n]                          (autograd.py:77-82)
// with W = bf16(W_f + bf16(lut[W_p])) (autograd.py:66-67).  The weight
// operand of FWD / DX comes from one of three sources (BSrc): W_f / W_p tiles
// staged by TMA and decoded in place in shared memory (B_WTMA), the same
// decode fed by a register ring of global loads when W's rows are not 16-byte
// multiples (B_RING), or a bf16 W decoded once by predecode_kernel and read by
// TMA (B_PLAIN, large T).  The decode looks the 256-entry lut up in a
// lane-replicated shared-memory copy (bank-conflict free) and adds in bf16
// (add.rn.bf16x2: the reference's fp32 add then bf16 rounding gives the same
// bits because 24 >= 2*8+2).  Activations (x, bf16(dY)) arrive by TMA.
//
// Tiles and roles.  A cluster of two CTAs (one per SM) runs
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16 per instruction): each
// CTA holds 128 rows of A and 128 columns of B in its own shared memory, and
// its TMEM holds its 128 output rows x 256 columns per accumulator.  MSUB = 2
// stacks two such M-subtiles in one 512 x 256 tile that shares every B stage.
// Per CTA:
//   warp 0      TMA producer (activation tiles; both operands for DW and
//               B_PLAIN; W_f / W_p for B_WTMA); loads of the pair complete on
//               the even CTA's mbarrier (.cta_group::2, no multicast)
//   warp 1      TMEM owner; in the even CTA also the single-thread MMA issuer
//   warps 2..   epilogue (4 or 8 warps): tcgen05.ld of the f32 accumulator,
//               bias / rounding / lut-gradient histogram / stream-K partials,
//               row-coalesced stores through a per-warp staging buffer
//   then        weight decode warps (B_WTMA, B_RING) and, for B_RING, the
//               decode-completion signal warp
// TMEM: two 256-column accumulators — double buffered across tiles for
// MSUB = 1, one per subtile for MSUB = 2.  Every mbarrier and flag wait is
// bounded (2 s); a wait that gives up sets the CTA abort word and the device
// timeout word, every role drains and the kernel returns.
#include <cudaTypedefs.h>

#include <mutex>

#include "sm100.cuh"

namespace packr {
namespace gemm {

using namespace sm100;

// Event trace for pipeline studies: compiled to nothing unless the library is
// built with -DPACKR_TRACE, in which case the build provides
// packr_trace(kind, index) recording timestamps of CTA pair 0.
#ifdef PACKR_TRACE
__device__ void packr_trace(int kind, int index);
#define PACKR_TRACE_EVENT(kind, index) \
  do {                                 \
    if (blockIdx.x < 2) packr_trace((kind), (index)); \
  } while (0)
#else
#define PACKR_TRACE_EVENT(kind, index) \
  do {                                 \
  } while (0)
#endif

constexpr int BM = 128;          // A rows per CTA (MMA M = 256 per pair)
constexpr int BN = 256;          // MMA N (output columns per tile)
constexpr int BN_CTA = 128;      // B columns held by each CTA
constexpr int BK = 64, UK = 16;
constexpr int MAX_STAGES = 6;
constexpr int TILE_Q = 4;        // dynamic-tile queue slots
constexpr int BARS_BYTES = 512;  // shared memory reserved for struct Bars
constexpr int A_BYTES = BM * BK * 2;      // 16 KB
constexpr int B_BYTES = BN_CTA * BK * 2;  // 16 KB
constexpr int DEC_WARPS = 8;           // decode warps, register-ring path (and the decode check)
constexpr int DEC_WARPS_TMA = 8;       // decode warps, TMA-staged path
constexpr int DEC_THREADS = DEC_WARPS * 32;
constexpr int CHUNKS = BN_CTA * BK / 8 / DEC_THREADS;  // chunks of 8 weights per thread per stage (ring path)
constexpr int LUT_BYTES = 256 * 32 * 4;  // one u32 per (entry, lane)
// lut-gradient histogram of the DW epilogue, in fixed point.  Shared f32
// atomics retire ~1.7 elements per clock per SM on B200 against ~6.5 for
// 32-bit integer ones (measured), so each tile's f32 dW values are scaled to
// integers of at most 2^21 relative to the tile's largest |dW| (one shared
// exponent per tile, agreed by the epilogue warps at a named barrier),
// added by red.shared.add.u32 into lane-interleaved integer copies (bin b of
// lane l is word b*32 + l: the 32 lanes of a red always hit 32 banks;
// epilogue warps 2-5 share copy 0, warps 6-9 copy 1), and after the tile
// folded into a per-CTA f32 sum per bin (lane l of epilogue warp w owns bin
// 32w + l).  A word takes at most 512 values per tile (4 warps x 4 chunks x
// 32), so |word| <= 2^30.  Tiles holding Inf / NaN or only values below
// 2^-106 add their f32 values to the per-CTA sums directly.
constexpr int HIST_COPIES = 2;
constexpr int HIST_COPY_BYTES = 256 * 32 * 4;
constexpr int HIST_SUM_BYTES = 256 * 4;   // per-CTA f32 bin sums
constexpr int HIST_XCHG_BYTES = 2 * 8 * 4;  // tile maxima: [tile parity][epilogue warp]
constexpr int ACC_COLS = BN;
// Epilogue warps wait a whole mainloop for their accumulator: they poll
// with the hardware's suspend hint (ns) so their polls do not take issue
// slots from the roles on the critical path.
constexpr uint32_t kEpilogueSleepNs = 1000;
// FWD / DX switch from the fused decode to predecode + plain GEMM at this
// many output rows (tokens), the first count above the skinny GEMM's range.
// Measured on the Llama-7B FFN layers (fwd+bwd of gate/up/down, same box):
// M = 129, 192, 256, 512 take 0.97, 0.98, 0.98, 1.09 ms that way against
// 1.22, 1.23, 1.22, 1.54 ms with the shared-memory decode, whose 256-row
// tiles number only N / 256 (16 to 43 here) and leave most SMs idle.
#ifndef PACKR_PREDECODE_MIN_M
#define PACKR_PREDECODE_MIN_M 129
#endif
// Stream-K work split for the GEMMs without a fused decode (1: on).
#ifndef PACKR_STREAM_K
#define PACKR_STREAM_K 1
#endif
// Stream-K over the last waves when the last wave of whole tiles would be at
// most this full (percent of the pairs).
#ifndef PACKR_SK_LAST_WAVE_PCT
#define PACKR_SK_LAST_WAVE_PCT 50
#endif
// Whole tiles of those GEMMs taken from a launch-wide counter (1: on).
#ifndef PACKR_DYN_TILES
#define PACKR_DYN_TILES 1
#endif
// Plain GEMMs use 512-row pair tiles from this many rows on.
#ifndef PACKR_PLAIN_MSUB2_MIN_M
#define PACKR_PLAIN_MSUB2_MIN_M 1024
#endif
constexpr int TMEM_COLS = 2 * ACC_COLS;
constexpr uint16_t PAIR_MASK = 0x3;

enum Mode { FWD = 0, DX = 1, DW = 2 };
// Where the B operand of FWD / DX comes from: decoded on the fly from W_f /
// W_p loaded through a register ring (B_RING) or by TMA (B_WTMA), or read by
// TMA from a bf16 array the predecode kernel wrote (B_PLAIN).
enum BSrc { B_RING = 0, B_WTMA = 1, B_PLAIN = 2 };

// B_WTMA (decode modes): W_f and W_p tiles arrive by TMA into shared memory
// and are decoded in place; B_RING (rows of W_p not a multiple of 16 bytes):
// the decode warps load them into a register ring.  B_PLAIN: no decode.
// MSUB: output rows per pair tile = 256 * MSUB.  With MSUB = 2 every decoded
// B stage feeds two pair MMAs (two 256-row subtiles), halving the decode and
// lut traffic per FLOP; the two subtiles' accumulators then fill TMEM (no
// double buffering across tiles, but each subtile is released separately).
template <int MODE, int BSRC, int MSUB>
struct Cfg {
  static constexpr bool kDecode = MODE != DW && BSRC != B_PLAIN;
  static constexpr bool kWtma = kDecode && BSRC == B_WTMA;
  static constexpr bool kPlainB = MODE != DW && BSRC == B_PLAIN;  // FWD / DX with B by TMA
  static constexpr int kMSub = MSUB;
  static constexpr int kStages = kWtma ? (MSUB == 2 ? 3 : 4) : (kPlainB && MSUB == 2 ? 4 : (MODE == DW ? 4 : 6));
  static constexpr int kABytes = MSUB * A_BYTES;            // A subtiles per stage
  static constexpr int kWpBytes = kWtma ? BN_CTA * BK : 0;  // u8 W_p tile per stage
  static constexpr int kStageBytes = kABytes + B_BYTES + kWpBytes;
  // DW's histogram epilogue is the heavier one: two warps per TMEM lane
  // quarter, each taking half of the tile's columns.
  static constexpr int kEpiWarps = kDecode ? 4 : 8;
  // The TMA-fed modes and DW pass each 32-row output block through a 4 KB
  // per-warp shared-memory buffer, so that global stores cover whole rows
  // segments of 128 (f32) or 64 (bf16) bytes instead of 16 bytes per row
  // (for DW at few tokens, where its epilogue is the bound, the row-per-lane
  // stores made two half-sector L2 writes per 32 bytes of dW_f).
  static constexpr bool kStageOut = kWtma || kPlainB || MODE == DW;
  // stream-K code compiled in (used when Params::sk): the plain FWD / DX
  // GEMMs only (for DW the split-tile fix-up measured slower than the wave
  // quantisation it removes)
  static constexpr bool kStreamK = kPlainB;
  static constexpr int kStgBytes = kStageOut ? kEpiWarps * 4096 : 0;
  static constexpr int kChunksPerEpiWarp = (BN / 32) / (kEpiWarps / 4);
  static constexpr int kDecWarp0 = 2 + kEpiWarps;             // first decode warp
  static constexpr int kDecWarps = kWtma ? DEC_WARPS_TMA : DEC_WARPS;
  static constexpr int kSignalWarp = kDecWarp0 + kDecWarps;   // decode-completion signaller (register ring only)
  static constexpr int kWarps = 2 + kEpiWarps + (kDecode ? kDecWarps + (kWtma ? 0 : 1) : 0);
  static constexpr int kThreads = kWarps * 32;
  static constexpr bool kAmn = MODE == DW;   // A stored MN-major in smem
  static constexpr bool kBmn = MODE != DX;   // B stored MN-major in smem
  static constexpr int kHistBytes = HIST_COPIES * HIST_COPY_BYTES + HIST_SUM_BYTES + HIST_XCHG_BYTES;
  static constexpr int kLutBytes = kDecode ? LUT_BYTES : 0;
  static constexpr int kStgOff = MODE == DW ? kHistBytes : kLutBytes;  // staging buffers in the aux region
  static constexpr int kAuxBytes = kStgOff + kStgBytes;
  static constexpr int kBarOff = kStages * kStageBytes + kAuxBytes;
  static constexpr int kSmemBytes = kBarOff + BARS_BYTES + 1024;  // barriers + alignment slack
  // dynamic-tile queue consumers: the odd CTA's producer, the MMA issuer and
  // every epilogue warp of both CTAs
  static constexpr int kQConsumers = 2 + 2 * kEpiWarps;
  static constexpr uint32_t kIdesc = idesc_bf16_f32(2 * BM, BN, kAmn, kBmn);
  static constexpr uint32_t kTxBytes = 2 * (kDecode ? kABytes : kABytes + B_BYTES);  // both CTAs
  static constexpr uint32_t kWTxBytes = B_BYTES + kWpBytes;                          // this CTA's W tiles
  static constexpr uint32_t kBfullCount = kWtma ? 2 * kDecWarps : 2;
};

struct Params {
  int Mg, Ng;          // output tile space: D[Mg, Ng]
  int Kg;              // reduction length of one segment
  int nseg;            // reduction segments (1..3), each with its own A/B maps
  int m_tiles, n_tiles, k_blocks;
  // decoded operand W[w_rows, w_cols] row-major with leading dimension ldw
  const uint8_t* W_p;
  const uint16_t* W_f;
  const float* lut;
  long long ldw;
  int w_rows, w_cols;
  int w_vec;                 // W_f 16-B / W_p 8-B aligned rows: vector loads allowed
  // epilogue
  void* out;
  long long ld_out;
  int out_f32;               // DX: 1 -> f32(bf16(acc)), 0 -> bf16
  const void* bias;          // FWD, nullable
  int bias_f32;              // bias dtype: 1 f32, 0 bf16
  const uint8_t* hist_idx;   // DW: W_p (same indexing as dW_f), nullable
  float* dlut_sum;           // DW: [256], nullable
  int out_vec;               // out base 16-B aligned
  int idx_vec;               // hist_idx base 16-B aligned
  // stream-K (sk = 1): the (tile, k-block) iteration space is cut into equal
  // contiguous ranges, one per CTA pair.  A tile split between pairs p and
  // p+1 (.. p+h when the tiles are fewer than the pairs): each later pair
  // computes its share of the tile's k-blocks first ("head") and leaves the
  // f32 partial in its own sk_partial slot; p computes the tile's first
  // k-blocks last ("tail"), adds the partials in pair order and runs the
  // epilogue.
  int sk;
  float* sk_partial;         // [pairs][MSUB][2 ranks][256 cols][128 rows]
  int* sk_flags;             // [pairs][2 ranks][epilogue warps], zeroed before the launch
  int sk_slots;              // pairs the two buffers above have room for (0: no stream-K)
  int sk_dp_tiles;           // with sk: tiles [0, sk_dp_tiles) go round-robin first (whole tiles)
  // dynamic tiles (plain FWD / DX without stream-K): each pair takes its next
  // whole tile from this counter (zeroed before the launch), so that pairs
  // that start late (SMs held by a kernel on another stream, e.g. a
  // collective) take fewer tiles instead of ending the launch late
  int dyn;
  int* tile_counter;
};

// Workspace for stream-K: partial slots and flags for up to `pairs` CTA pairs.
inline size_t sk_partial_bytes(int pairs, int msub) { return (size_t)pairs * msub * 2 * BN * BM * sizeof(float); }
inline size_t sk_flag_bytes(int pairs) { return (size_t)pairs * 2 * 8 * sizeof(int); }

// One unit of a pair's work: k-blocks [k0, k1) of one tile.
struct Unit {
  int tile, k0, k1;
  int kind;  // 0 whole tile, 1 head (partial to the workspace), 2 tail (adds the next pair's head)
};

// The sequence of units of one CTA pair; every role walks the same sequence:
// whole tiles round-robin (tile = pair + i * pairs) below dp_tiles, then, with
// stream-K, this pair's contiguous share of the remaining (tile, k-block)
// iterations.  Round-robin keeps the tiles in flight at once adjacent (shared
// operands stay in L2); the stream-K tail balances the last wave.
struct Sched {
  long long g, g_end;  // stream-K iteration range (tile * kb_total + k-block)
  int tile, step, dp_end, kb_total;
  bool sk;
};

__device__ __forceinline__ Sched make_sched(const Params& P, int pair, int npairs) {
  Sched s;
  s.kb_total = P.nseg * P.k_blocks;
  const int num_tiles = P.m_tiles * P.n_tiles;
  s.sk = P.sk != 0;
  s.dp_end = s.sk ? P.sk_dp_tiles : num_tiles;
  const long long T = (long long)(num_tiles - s.dp_end) * s.kb_total;
  const long long base = (long long)s.dp_end * s.kb_total;
  s.g = base + T * pair / npairs;
  s.g_end = base + T * (pair + 1) / npairs;
  s.tile = pair;
  s.step = npairs;
  return s;
}

// First (tile, k-block) iteration of pair q's stream-K range (make_sched).
__device__ __forceinline__ long long sk_start(const Params& P, int q, int npairs) {
  const long long kbt = (long long)P.nseg * P.k_blocks;
  const long long num_tiles = (long long)P.m_tiles * P.n_tiles;
  const long long base = (long long)P.sk_dp_tiles * kbt;
  return base + (num_tiles - P.sk_dp_tiles) * kbt * q / npairs;
}

__device__ __forceinline__ bool next_unit(Sched& s, Unit& u) {
  if (s.tile < s.dp_end) {
    u.tile = s.tile;
    u.k0 = 0;
    u.k1 = s.kb_total;
    u.kind = 0;
    s.tile += s.step;
    return true;
  }
  if (!s.sk || s.g >= s.g_end) return false;
  const long long tile = s.g / s.kb_total;
  const long long t0 = tile * s.kb_total, t1 = t0 + s.kb_total;
  const long long e = s.g_end < t1 ? s.g_end : t1;
  u.tile = (int)tile;
  u.k0 = (int)(s.g - t0);
  u.k1 = (int)(e - t0);
  u.kind = u.k0 > 0 ? 1 : (u.k1 < s.kb_total ? 2 : 0);
  s.g = e;
  return true;
}

struct Maps {
  CUtensorMap a[3];
  CUtensorMap b[3];
  CUtensorMap wf;  // W_f (bf16), decode modes with TMA-staged weights
  CUtensorMap wp;  // W_p (u8)
};

// Barriers live at the same offset in both CTAs of a pair.  full / bfull /
// tempty are used in the even CTA only (the odd CTA's producers arrive there
// remotely); empty / tfull / drain receive the even CTA's multicast commits.
struct Bars {
  uint64_t full[MAX_STAGES];    // A (DW: A and B) bytes of both CTAs landed  (count 1 + tx)
  uint64_t bfull[MAX_STAGES];   // decoded B written by both CTAs              (count kBfullCount)
  uint64_t empty[MAX_STAGES];   // MMAs done reading the stage                 (count 1)
  uint64_t wfull[MAX_STAGES];   // this CTA's W_f / W_p tiles landed           (count 1 + tx)
  uint64_t tfull[2];        // accumulator complete                 (count 1)
  uint64_t tempty[2];       // accumulator drained by both CTAs     (count 2*epilogue warps)
  uint64_t drain;           // every MMA complete                   (count 1)
  // dynamic tiles: the even CTA's producer writes tile numbers into qtile of
  // both CTAs and arrives on both CTAs' qfull; every other role reads its own
  // CTA's copy and arrives on the even CTA's qempty
  uint64_t qfull[TILE_Q];   // tile number published                 (count 1)
  uint64_t qempty[TILE_Q];  // read by every consumer of both CTAs    (count kQConsumers)
  int qtile[TILE_Q];        // tile number, or -1 after the last tile
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Bars) <= BARS_BYTES, "barrier region");

__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// ------------------------------------------------------------------ decode
// One decode thread moves CHUNKS chunks of 8 consecutive weights per stage.
struct Chunks {
  uint4 wf[CHUNKS];
  uint2 wp[CHUNKS];
  uint32_t nvalid;  // 4 bits per chunk: number of valid weights (0..8)
};

// FWD: the CTA's B half is 64 reduction rows x 128 columns: chunk i of
//      thread t (of NT decode threads) covers row k = t/16 + (NT/16)*i and
//      columns 8*(t%16) .. +7 (W row = k, W columns = n).
// DX : the B half is 128 output columns (W rows) x 64 reduction columns:
//      chunk i covers B row r = t/8 + (NT/8)*i and reduction columns
//      8*(t%8) .. +7.
template <int MODE, int NT = DEC_THREADS>
__device__ __forceinline__ void chunk_coords(int t, int i, int& brow, int& bcol8) {
  if (MODE == FWD) {
    brow = (t >> 4) + (NT / 16) * i;
    bcol8 = t & 15;
  } else {
    brow = (t >> 3) + (NT / 8) * i;
    bcol8 = t & 7;
  }
}

// Shared-memory byte offset of a chunk inside the CTA's B stage (128-byte
// swizzle: 16-byte chunk index XOR row-within-8).
template <int MODE>
__device__ __forceinline__ uint32_t chunk_smem_off(int brow, int bcol8) {
  if (MODE == FWD)  // MN-major: two 64-column blocks of 64 rows x 128 B
    return (uint32_t)((bcol8 >> 3) * 8192 + brow * 128 + (((bcol8 & 7) ^ (brow & 7)) << 4));
  return (uint32_t)(brow * 128 + ((bcol8 ^ (brow & 7)) << 4));  // K-major: one 128 B row per column
}

template <int MODE>
__device__ __forceinline__ void decode_load(Chunks& c, const Params& P, int t, int nb0, int k0) {
  c.nvalid = 0;
  const bool vec_ok = P.w_vec != 0;
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    int brow, bcol8;
    chunk_coords<MODE>(t, i, brow, bcol8);
    long long wr, wc;
    if (MODE == FWD) {
      wr = (long long)k0 + brow;
      wc = (long long)nb0 + 8 * bcol8;
    } else {
      wr = (long long)nb0 + brow;
      wc = (long long)k0 + 8 * bcol8;
    }
    int nv = 0;
    if (wr < P.w_rows && wc < P.w_cols) nv = (int)min(8ll, (long long)P.w_cols - wc);
    c.nvalid |= (uint32_t)nv << (4 * i);
    const long long off = wr * P.ldw + wc;
    if (nv == 8 && vec_ok) {
      c.wf[i] = __ldg(reinterpret_cast<const uint4*>(P.W_f + off));
      c.wp[i] = __ldg(reinterpret_cast<const uint2*>(P.W_p + off));
    } else {
      uint32_t f[4] = {0, 0, 0, 0}, p[2] = {0, 0};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < nv) {
          f[j >> 1] |= (uint32_t)__ldg(P.W_f + off + j) << (16 * (j & 1));
          p[j >> 2] |= (uint32_t)__ldg(P.W_p + off + j) << (8 * (j & 3));
        }
      }
      c.wf[i] = make_uint4(f[0], f[1], f[2], f[3]);
      c.wp[i] = make_uint2(p[0], p[1]);
    }
  }
}

// lut_lane = shared address of this lane's column of the replicated lut:
// entry e lives at lut_lane + 128*e.
__device__ __forceinline__ uint32_t lut_fetch(uint32_t lut_lane, uint32_t idx_byte_shifted7) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(lut_lane + idx_byte_shifted7));
  return v;
}

template <int MODE>
__device__ __forceinline__ void decode_store(const Chunks& c, uint32_t b_stage, uint32_t lut_lane, int t) {
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    int brow, bcol8;
    chunk_coords<MODE>(t, i, brow, bcol8);
    const uint32_t off = chunk_smem_off<MODE>(brow, bcol8);
    const uint32_t w[2] = {c.wp[i].x, c.wp[i].y};
    const uint32_t f[4] = {c.wf[i].x, c.wf[i].y, c.wf[i].z, c.wf[i].w};
    uint32_t r[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t word = w[p >> 1];
      const int sh = 16 * (p & 1);
      const uint32_t e0 = ((word >> sh) & 0xFFu) << 7;
      const uint32_t e1 = ((word >> (sh + 8)) & 0xFFu) << 7;
      const uint32_t l = prmt(lut_fetch(lut_lane, e0), lut_fetch(lut_lane, e1), 0x5410u);
      r[p] = bf16x2_add(f[p], l);
    }
    const int nv = (c.nvalid >> (4 * i)) & 15;
    if (nv < 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j >= nv) r[j >> 1] &= (j & 1) ? 0x0000FFFFu : 0xFFFF0000u;
    }
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(b_stage + off), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
  }
}

// Decode of a TMA-staged stage in place: W_f already sits in the B tile in
// its swizzled layout, W_p in a row-major u8 tile (FWD: 64 rows x 128,
// DX: 128 rows x 64).  Elements outside W (zero-filled by TMA) are stored as
// zero rather than decoded.
template <int MODE, int NT>
__device__ __forceinline__ void decode_in_place(const Params& P, uint8_t* b_stage, const uint8_t* wp_stage,
                                                const uint32_t* lut_lane, int t, int nb0, int k0) {
  constexpr int NCH = BN_CTA * BK / 8 / NT;
  uint4 f[NCH];
  uint2 w[NCH];
  int nv[NCH];
  uint32_t off[NCH];
#pragma unroll
  for (int i = 0; i < NCH; ++i) {  // all loads of the stage first
    int brow, bcol8;
    chunk_coords<MODE, NT>(t, i, brow, bcol8);
    off[i] = chunk_smem_off<MODE>(brow, bcol8);
    const int wpoff = brow * (MODE == FWD ? BN_CTA : BK) + 8 * bcol8;
    long long wr, wc;
    if (MODE == FWD) {
      wr = (long long)k0 + brow;
      wc = (long long)nb0 + 8 * bcol8;
    } else {
      wr = (long long)nb0 + brow;
      wc = (long long)k0 + 8 * bcol8;
    }
    nv[i] = (wr < P.w_rows && wc < P.w_cols) ? (int)min(8ll, (long long)P.w_cols - wc) : 0;
    f[i] = *reinterpret_cast<const uint4*>(b_stage + off[i]);
    w[i] = *reinterpret_cast<const uint2*>(wp_stage + wpoff);
  }
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const uint32_t ww[2] = {w[i].x, w[i].y};
    const uint32_t ff[4] = {f[i].x, f[i].y, f[i].z, f[i].w};
    uint32_t r[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t word = ww[p >> 1];
      const int sh = 16 * (p & 1);
      const uint32_t l0 = lut_lane[((word >> sh) & 0xFFu) * 32];
      const uint32_t l1 = lut_lane[((word >> (sh + 8)) & 0xFFu) * 32];
      r[p] = bf16x2_add(ff[p], prmt(l0, l1, 0x5410u));
    }
    if (nv[i] < 8) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j >= nv[i]) r[j >> 1] &= (j & 1) ? 0x0000FFFFu : 0xFFFF0000u;
    }
    *reinterpret_cast<uint4*>(b_stage + off[i]) = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

// Row-coalesced store of a warp's 32 x 32 output block.  On entry lane l
// holds row r0 + l: 32 values of ESIZE bytes packed in v (ESIZE 4: 32 words,
// ESIZE 2: 16 words of bf16 pairs).  The rows are written to the warp's
// staging buffer (RB = 32 * ESIZE bytes per row, 16-byte chunks XOR-swizzled
// by row so both phases are free of bank conflicts), then read back so that
// RB / 16 consecutive lanes store one row segment and each store instruction
// writes 512 contiguous-by-row bytes (4 rows of 128 B or 8 rows of 64 B).
// Rows at or beyond m_limit are skipped;
// columns gn0 .. gn0 + 31 must lie inside the output.
template <int ESIZE>
__device__ __forceinline__ void store_rows_staged(uint32_t stg, const float* v, void* out, int r0, int m_limit,
                                                  long long ld, int gn0) {
  constexpr int RB = 32 * ESIZE;      // bytes per row
  constexpr int CPR = RB / 16;        // 16-byte chunks per row (8 or 4)
  constexpr int RPI = 32 / CPR;       // rows per store instruction (4 or 8)
  const int lane = threadIdx.x & 31;
  const int sw = ESIZE == 4 ? (lane & 7) : ((lane >> 1) & 3);
#pragma unroll
  for (int j = 0; j < CPR; ++j)
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(stg + (uint32_t)(lane * RB + ((j ^ sw) << 4))),
                 "r"(__float_as_uint(v[4 * j])), "r"(__float_as_uint(v[4 * j + 1])), "r"(__float_as_uint(v[4 * j + 2])),
                 "r"(__float_as_uint(v[4 * j + 3]))
                 : "memory");
  __syncwarp();
  const int jc = lane % CPR;
#pragma unroll
  for (int i = 0; i < CPR; ++i) {
    const int r = i * RPI + lane / CPR;
    const int rsw = ESIZE == 4 ? (r & 7) : ((r >> 1) & 3);
    uint4 d;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(d.x), "=r"(d.y), "=r"(d.z), "=r"(d.w)
                 : "r"(stg + (uint32_t)(r * RB + ((jc ^ rsw) << 4)))
                 : "memory");
    const long long gr = (long long)r0 + r;
    if (gr < m_limit)
      __stcs(reinterpret_cast<uint4*>(static_cast<uint8_t*>(out) + (gr * ld + gn0) * ESIZE + jc * 16), d);
  }
  __syncwarp();
}

// Bounded wait for a stream-K flag written by another CTA pair of the same
// launch (all pairs are resident at once).  Lane 0 polls with acquire loads
// and decides; the result is the same in every lane, and the warp barrier
// orders the other lanes' later loads after lane 0's acquire.  Gives up like
// mbar_wait.
__device__ __forceinline__ bool wait_flag(const int* f, volatile int* abort_flag) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0;; ++i) {
      int v;
      asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (v != 0) {
        ok = 1;
        break;
      }
      if ((i & 63u) == 63u) {
        if (*abort_flag) break;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          *abort_flag = 1;
          atomicExch(&g_wait_timeout, 1u);
          break;
        }
        __nanosleep(200);
      }
    }
  }
  ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
  __syncwarp();
  return ok != 0;
}

// ------------------------------------------------------------------ kernel
template <int MODE, int BSRC, int MSUB>
__global__ void __launch_bounds__(Cfg<MODE, BSRC, MSUB>::kThreads, 1)
    packr_gemm_kernel(const Params P, const __grid_constant__ Maps maps) {
  using C = Cfg<MODE, BSRC, MSUB>;
  constexpr int STAGES = C::kStages;
  static_assert(C::kSmemBytes <= 227 * 1024, "shared memory per CTA");
  static_assert(MODE != DW || MSUB == 1, "the DW epilogue's histogram runs per 256-row tile");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base for the 128-byte-swizzled tiles; offsetting the
  // __shared__ array keeps the compiler emitting shared-memory accesses.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::kABytes;
  uint8_t* sWp = sB + STAGES * B_BYTES;
  uint8_t* sAux = smem + STAGES * C::kStageBytes;
  Bars* bars = reinterpret_cast<Bars*>(smem + C::kBarOff);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs, 1: its peer
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int num_tiles = P.m_tiles * P.n_tiles;
  const int kb_total = P.nseg * P.k_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->bfull[s], C::kBfullCount);
      mbar_init(&bars->empty[s], 1);
      mbar_init(&bars->wfull[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->tfull[a], 1);
      mbar_init(&bars->tempty[a], 2 * C::kEpiWarps);
    }
    mbar_init(&bars->drain, 1);
    for (int r = 0; r < TILE_Q; ++r) {
      mbar_init(&bars->qfull[r], 1);
      mbar_init(&bars->qempty[r], C::kQConsumers);
    }
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < P.nseg; ++s) {
      prefetch_tmap(&maps.a[s]);
      if (MODE == DW || C::kPlainB) prefetch_tmap(&maps.b[s]);
    }
    if (C::kWtma) {
      prefetch_tmap(&maps.wf);
      prefetch_tmap(&maps.wp);
    }
  }
  if (MODE == DW && warp >= 2 && warp < C::kDecWarp0) {
    uint32_t* hist = reinterpret_cast<uint32_t*>(sAux);
    for (int i = threadIdx.x - 64; i < C::kHistBytes / 4; i += C::kEpiWarps * 32) hist[i] = 0u;
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (C::kDecode && warp >= C::kDecWarp0 && warp < C::kDecWarp0 + C::kDecWarps) {
    // Lane-replicated bf16 lut: word (e*32 + l) holds bf16_rne(lut[e]) for lane l.
    uint32_t* lut_s = reinterpret_cast<uint32_t*>(sAux);
    const int dw = warp - C::kDecWarp0;
    for (int e = dw; e < 256; e += C::kDecWarps) lut_s[e * 32 + lane] = f32_to_bf16_rne(__ldg(P.lut + e));
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  // Dynamic tiles (one thread per role).  Entry i of the pair's sequence sits
  // in queue slot i % TILE_Q, phase (i / TILE_Q) & 1.
  const bool dyn = C::kPlainB && P.dyn != 0;
  // the even CTA's producer: takes the next tile (-1 past the last) and
  // publishes it to both CTAs; -2 if the kernel aborted
  auto q_push = [&](int i) -> int {
    const int slot = i % TILE_Q;
    const uint32_t ph = (uint32_t)(i / TILE_Q) & 1u;
    if (!mbar_wait_cluster(&bars->qempty[slot], ph ^ 1u, abort_flag)) return -2;
    int t = atomicAdd(P.tile_counter, 1);
    if (t >= num_tiles) t = -1;
    bars->qtile[slot] = t;
    st_shared_cluster_u32(mapa(smem_u32(&bars->qtile[slot]), 1), (uint32_t)t);
    mbar_arrive_release_cluster(mapa(smem_u32(&bars->qfull[slot]), 0));
    mbar_arrive_release_cluster(mapa(smem_u32(&bars->qfull[slot]), 1));
    return t;
  };
  // any other role: reads entry i from its own CTA's queue and releases the
  // slot on the even CTA; false if the kernel aborted
  auto q_pop = [&](int i, int& t) -> bool {
    const int slot = i % TILE_Q;
    const uint32_t ph = (uint32_t)(i / TILE_Q) & 1u;
    if (!mbar_wait_cluster(&bars->qfull[slot], ph, abort_flag)) return false;
    t = *reinterpret_cast<volatile int*>(&bars->qtile[slot]);
    mbar_arrive_release_cluster(mapa(smem_u32(&bars->qempty[slot]), 0));
    return true;
  };
  auto whole_tile = [&](int t, Unit& x) {
    x.tile = t;
    x.k0 = 0;
    x.k1 = kb_total;
    x.kind = 0;
  };

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      Sched sc = make_sched(P, pair, npairs);
      Unit u;
      for (int qi = 0; ok; ++qi) {
        if (dyn) {
          int t = -1;
          if (rank == 0) {
            t = q_push(qi);
            if (t == -2) break;
          } else if (!q_pop(qi, t)) {
            break;
          }
          if (t < 0) break;
          whole_tile(t, u);
        } else if (!next_unit(sc, u)) {
          break;
        }
        const int tile = u.tile;
        const int m0 = (tile % P.m_tiles) * (2 * BM * MSUB) + (int)rank * BM;
        const int n0 = (tile / P.m_tiles) * BN + (int)rank * BN_CTA;
        for (int kk = u.k0; kk < u.k1; ++kk, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!mbar_wait(&bars->empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
          PACKR_TRACE_EVENT(0, it);
          const int seg = kk / P.k_blocks;
          const int k0 = (kk % P.k_blocks) * BK;
          if (rank == 0) mbar_arrive_expect_tx(&bars->full[s], C::kTxBytes);
          const uint32_t fbar = mapa(smem_u32(&bars->full[s]), 0);
          uint8_t* a_dst = sA + s * C::kABytes;
          if (MODE == DW) {
            tma_load_2d_pair(a_dst, &maps.a[seg], fbar, m0, k0);
            tma_load_2d_pair(a_dst + 8192, &maps.a[seg], fbar, m0 + 64, k0);
            uint8_t* b_dst = sB + s * B_BYTES;
            tma_load_2d_pair(b_dst, &maps.b[seg], fbar, n0, k0);
            tma_load_2d_pair(b_dst + 8192, &maps.b[seg], fbar, n0 + 64, k0);
          } else {
#pragma unroll
            for (int sub = 0; sub < MSUB; ++sub)
              tma_load_2d_pair(a_dst + sub * A_BYTES, &maps.a[seg], fbar, k0, m0 + sub * 2 * BM);
            if (C::kPlainB) {
              // this CTA's 128 columns of the predecoded B
              uint8_t* b_dst = sB + s * B_BYTES;
              if (MODE == FWD) {  // W [K, N]: MN-major, two 64-column blocks
                tma_load_2d_pair(b_dst, &maps.b[seg], fbar, n0, k0);
                tma_load_2d_pair(b_dst + 8192, &maps.b[seg], fbar, n0 + 64, k0);
              } else {            // W rows are dX columns: K-major
                tma_load_2d_pair(b_dst, &maps.b[seg], fbar, k0, n0);
              }
            }
            if (C::kWtma) {
              // this CTA's W_f / W_p tiles (its 128 columns of B) onto its own wfull
              const int nb0 = (tile / P.m_tiles) * BN + (int)rank * BN_CTA;
              uint8_t* b_dst = sB + s * B_BYTES;
              uint8_t* p_dst = sWp + s * C::kWpBytes;
              mbar_arrive_expect_tx(&bars->wfull[s], C::kWTxBytes);
              if (MODE == FWD) {
                tma_load_2d(b_dst, &maps.wf, &bars->wfull[s], nb0, k0);
                tma_load_2d(b_dst + 8192, &maps.wf, &bars->wfull[s], nb0 + 64, k0);
                tma_load_2d(p_dst, &maps.wp, &bars->wfull[s], nb0, k0);
              } else {
                tma_load_2d(b_dst, &maps.wf, &bars->wfull[s], k0, nb0);
                tma_load_2d(p_dst, &maps.wp, &bars->wfull[s], k0, nb0);
              }
            }
          }
        }
      }
      (void)ok;
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      int it = 0, t_local = 0;
      bool ok = true;
      const uint32_t sA0 = smem_u32(sA), sB0 = smem_u32(sB);
      Sched sc = make_sched(P, pair, npairs);
      Unit u;
      for (; ok; ++t_local) {
        if (dyn) {
          int t = -1;
          if (!q_pop(t_local, t) || t < 0) break;
          whole_tile(t, u);
        } else if (!next_unit(sc, u)) {
          break;
        }
        // accumulator slots (256 TMEM columns each): MSUB = 1 alternates the
        // two slots between tiles; MSUB = 2 uses slot `sub` for subtile `sub`
        const int acc = MSUB == 1 ? (t_local & 1) : 0;
        const uint32_t aph = MSUB == 1 ? ((uint32_t)(t_local >> 1) & 1u) : ((uint32_t)t_local & 1u);
        if (!mbar_wait(&bars->tempty[acc], aph ^ 1u, abort_flag)) { ok = false; break; }
        PACKR_TRACE_EVENT(3, t_local);
        tc_fence_after();
        for (int kk = u.k0; kk < u.k1; ++kk, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!mbar_wait(&bars->full[s], ph, abort_flag)) { ok = false; break; }
          PACKR_TRACE_EVENT(1, it);
          if (C::kDecode && !mbar_wait(&bars->bfull[s], ph, abort_flag)) { ok = false; break; }
          PACKR_TRACE_EVENT(2, it);
          tc_fence_after();
          const uint32_t a_s = sA0 + s * C::kABytes, b_s = sB0 + s * B_BYTES;
#pragma unroll
          for (int sub = 0; sub < MSUB; ++sub) {
            if (sub == 1 && kk == u.k0) {  // subtile 1's accumulator is released after subtile 0's
              if (!mbar_wait(&bars->tempty[1], aph ^ 1u, abort_flag)) { ok = false; break; }
              tc_fence_after();
            }
            const uint32_t a_sub = a_s + sub * A_BYTES;
            const uint32_t d_tmem = tmem_base + (uint32_t)((MSUB == 1 ? acc : sub) * ACC_COLS);
#pragma unroll
            for (int k = 0; k < BK / UK; ++k) {
              const uint64_t bd = C::kBmn ? sdesc_sw128(b_s + k * 2048, 8192, 1024) : sdesc_sw128(b_s + k * 32, 16, 1024);
              const uint64_t ad = C::kAmn ? sdesc_sw128(a_sub + k * 2048, 8192, 1024) : sdesc_sw128(a_sub + k * 32, 16, 1024);
              umma_bf16_pair(d_tmem, ad, bd, C::kIdesc, (kk != u.k0 || k != 0) ? 1u : 0u);
            }
            // subtile 0 complete: its drain overlaps subtile 1's last MMAs
            if (MSUB == 2 && sub == 0 && kk == u.k1 - 1) umma_commit_pair(&bars->tfull[0], PAIR_MASK);
          }
          if (!ok) break;
          umma_commit_pair(&bars->empty[s], PAIR_MASK);
          PACKR_TRACE_EVENT(10, it);
        }
        if (!ok) break;
        if (MSUB == 1) {
          umma_commit_pair(&bars->tfull[acc], PAIR_MASK);
        } else {
          umma_commit_pair(&bars->tfull[1], PAIR_MASK);
        }
      }
      umma_commit_pair(&bars->drain, PAIR_MASK);
    }
  } else if (warp < C::kDecWarp0) {
    // ------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;                    // TMEM lane quarter this warp may access
    const int cc0 = ((warp - 2) >> 2) * C::kChunksPerEpiWarp;  // first 32-column chunk
    const int row = q * 32 + lane;
    const uint32_t tempty0 = mapa(smem_u32(&bars->tempty[0]), 0);
    const uint32_t tempty1 = mapa(smem_u32(&bars->tempty[1]), 0);
    const uint32_t hist_lane = smem_u32(sAux) + (uint32_t)(((warp - 2) >> 2) * HIST_COPY_BYTES + lane * 4);
    const uint32_t stg = smem_u32(sAux) + (uint32_t)(C::kStgOff + (warp - 2) * 4096);
    // DW: the W_p bytes of the next tile's chunks are fetched before its
    // accumulator is ready (they do not depend on it)
    uint4 wpa[C::kChunksPerEpiWarp], wpb[C::kChunksPerEpiWarp];
    auto fetch_idx = [&](int tile) {
      const long long gm = (long long)((tile % P.m_tiles) * (2 * BM * MSUB) + (int)rank * BM + row);
      const int n0 = (tile / P.m_tiles) * BN;
#pragma unroll
      for (int c = 0; c < C::kChunksPerEpiWarp; ++c) {
        const int gn0 = n0 + (cc0 + c) * 32;
        if (gn0 + 32 <= P.Ng && (P.ld_out & 15) == 0 && P.idx_vec) {
          // straight into the registers (a row past W_p reads row 0, whose
          // values the histogram skips): no merge with zeros, so the loads
          // stay in flight until the histogram needs them
          const uint8_t* ip = P.hist_idx + (gm < P.Mg ? gm : 0) * P.ld_out + gn0;
          wpa[c] = __ldg(reinterpret_cast<const uint4*>(ip));
          wpb[c] = __ldg(reinterpret_cast<const uint4*>(ip + 16));
          continue;
        }
        uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (gm < P.Mg && gn0 < P.Ng) {
          const uint8_t* ip = P.hist_idx + gm * P.ld_out + gn0;
          const int nval = min(32, P.Ng - gn0);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nval) w[j >> 2] |= (uint32_t)__ldg(ip + j) << (8 * (j & 3));
        }
        wpa[c] = make_uint4(w[0], w[1], w[2], w[3]);
        wpb[c] = make_uint4(w[4], w[5], w[6], w[7]);
      }
    };
    const bool want_hist = MODE == DW && P.hist_idx != nullptr;
    const int ew = warp - 2;  // epilogue warp index
    Sched sc = make_sched(P, pair, npairs);
    Unit u, un;
    bool alive = true;
    int qi = 0;
    // the warp's next unit: lane 0 reads the queue (dynamic tiles), every
    // lane gets the same answer
    auto next_any = [&](Unit& x) -> bool {
      if (!dyn) return next_unit(sc, x);
      int t = -1, got = 1;
      if (lane == 0) got = q_pop(qi, t) ? 1 : 0;
      got = __shfl_sync(0xFFFFFFFFu, got, 0);
      t = __shfl_sync(0xFFFFFFFFu, t, 0);
      ++qi;
      if (!got) alive = false;
      if (!got || t < 0) return false;
      whole_tile(t, x);
      return true;
    };
    bool have = next_any(u);
    if (want_hist && have) fetch_idx(u.tile);
    int t_local = 0;
    int n_heads = 0;  // stream-K: head partials the current tail tile adds
    // With the histogram, every epilogue warp takes the per-tile named
    // barriers of every tile of its schedule, also after an abort (then
    // without waiting on or reading the accumulator), so that the barrier
    // sequence of the eight warps always matches.
    for (; have && (alive || want_hist); ++t_local) {
    // static schedules look one unit ahead (DW fetches the next tile's W_p
    // early); the queue is read after the tile, so that this warp never
    // waits for the producer to start a tile while it holds an accumulator
    bool have_next = dyn ? false : next_unit(sc, un);
    const int tile = u.tile;
    for (int sub = 0; sub < MSUB; ++sub) {
      const int acc = MSUB == 1 ? (t_local & 1) : sub;
      const uint32_t aph = MSUB == 1 ? ((uint32_t)(t_local >> 1) & 1u) : ((uint32_t)t_local & 1u);
      // one lane polls; the warp proceeds only if every lane saw the phase
      const bool ready = alive && mbar_wait_warp(&bars->tfull[acc], aph, abort_flag, kEpilogueSleepNs);
      if (!ready) {
        alive = false;
        if (!want_hist) break;
      }
      uint32_t hmax = 0;  // DW: this lane's largest |dW| bits of the tile
      if (ready) {
      if (warp == 2 && lane == 0) PACKR_TRACE_EVENT(4, t_local);
      tc_fence_after();
      const int m0 = (tile % P.m_tiles) * (2 * BM * MSUB) + sub * 2 * BM + (int)rank * BM;
      const int n0 = (tile / P.m_tiles) * BN;
      const long long gm = (long long)m0 + row;
      const bool row_ok = gm < P.Mg;
      // stream-K partial slots ([col][row] f32, this CTA rank's 128 rows)
      float* const my_slot = P.sk_partial + (((size_t)pair * MSUB + sub) * 2 + rank) * (size_t)(BN * BM);
      if (C::kStreamK && u.kind == 2 && sub == 0) {
        // tail: every following pair whose range starts inside this tile
        // left a head partial (one pair, or several when a tile spans more
        // than two ranges); wait until all of them are published
        const long long tile_end = (long long)(tile + 1) * kb_total;
        n_heads = 0;
        for (int q2 = pair + 1; q2 < npairs && sk_start(P, q2, npairs) < tile_end; ++q2) {
          if (!wait_flag(P.sk_flags + (q2 * 2 + (int)rank) * C::kEpiWarps + ew, abort_flag)) {
            alive = false;
            break;
          }
          ++n_heads;
        }
        if (!alive) break;
      }
#pragma unroll
      for (int c = 0; c < C::kChunksPerEpiWarp; ++c) {
        const int cc = cc0 + c;
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + (uint32_t)(acc * ACC_COLS + cc * 32) + ((uint32_t)(q * 32) << 16), v);
        tmem_ld_wait();
        if (warp == 2 && lane == 0) PACKR_TRACE_EVENT(12, (t_local * 2 + sub) * 8 + c);
        const int gn0 = n0 + cc * 32;
        // warp-uniform skip; the staged stores are collective, the others per row
        if (gn0 >= P.Ng || m0 + q * 32 >= P.Mg) continue;
        if (C::kStreamK && u.kind == 1) {  // head: raw partial, coalesced along rows
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(my_slot + (cc * 32 + j) * BM + row, __uint_as_float(v[j]));
          continue;
        }
        if (C::kStreamK && u.kind == 2) {  // the heads' partials, added in pair order
          for (int h = 1; h <= n_heads; ++h) {
            const float* const slot =
                P.sk_partial + (((size_t)(pair + h) * MSUB + sub) * 2 + rank) * (size_t)(BN * BM);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              v[j] = __float_as_uint(__fadd_rn(__uint_as_float(v[j]), __ldcg(slot + (cc * 32 + j) * BM + row)));
          }
        }
        if (!C::kStageOut && !row_ok) continue;
        const int nval = min(32, P.Ng - gn0);
        if (MODE == FWD) {
          float* o = static_cast<float*>(P.out) + gm * P.ld_out + gn0;
          float f[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
          if (P.bias != nullptr) {
            if (P.bias_f32) {
              const float* bp = static_cast<const float*>(P.bias) + gn0;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < nval) f[j] = __fadd_rn(f[j], __ldg(bp + j));
            } else {
              const uint16_t* bp = static_cast<const uint16_t*>(P.bias) + gn0;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < nval) f[j] = __fadd_rn(f[j], bf16_to_f32(__ldg(bp + j)));
            }
          }
          if (C::kStageOut && nval == 32 && (P.ld_out & 3) == 0 && P.out_vec) {
            store_rows_staged<4>(stg, f, P.out, m0 + q * 32, P.Mg, P.ld_out, gn0);
          } else if (!row_ok) {
          } else if (nval == 32 && (P.ld_out & 3) == 0 && P.out_vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) __stcs(reinterpret_cast<float4*>(o + j), make_float4(f[j], f[j + 1], f[j + 2], f[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nval) o[j] = f[j];
          }
        } else {  // DX: bf16(acc) as bf16 or f32;  DW: bf16(acc) (+ histogram)
          uint32_t h[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) h[j] = pack_bf16x2_rne(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
          if (P.out != nullptr) {
            if (MODE == DX && P.out_f32) {
              float* o = static_cast<float*>(P.out) + gm * P.ld_out + gn0;
              if (C::kStageOut && nval == 32 && (P.ld_out & 3) == 0 && P.out_vec) {
                float f[32];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  f[2 * j] = __uint_as_float(h[j] << 16);
                  f[2 * j + 1] = __uint_as_float(h[j] & 0xFFFF0000u);
                }
                store_rows_staged<4>(stg, f, P.out, m0 + q * 32, P.Mg, P.ld_out, gn0);
              } else if (!row_ok) {
              } else if (nval == 32 && (P.ld_out & 3) == 0 && P.out_vec) {
#pragma unroll
                for (int j = 0; j < 16; j += 2)
                  __stcs(reinterpret_cast<float4*>(o + 2 * j),
                         make_float4(__uint_as_float(h[j] << 16), __uint_as_float(h[j] & 0xFFFF0000u),
                                     __uint_as_float(h[j + 1] << 16), __uint_as_float(h[j + 1] & 0xFFFF0000u)));
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < nval) o[j] = bf16_to_f32((h[j >> 1] >> (16 * (j & 1))) & 0xFFFFu);
              }
            } else {
              uint16_t* o = static_cast<uint16_t*>(P.out) + gm * P.ld_out + gn0;
              if (C::kStageOut && nval == 32 && (P.ld_out & 7) == 0 && P.out_vec) {
                store_rows_staged<2>(stg, reinterpret_cast<const float*>(h), P.out, m0 + q * 32, P.Mg, P.ld_out, gn0);
              } else if (!row_ok) {
              } else if (nval == 32 && (P.ld_out & 7) == 0 && P.out_vec) {
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                  __stcs(reinterpret_cast<uint4*>(o + 2 * j), make_uint4(h[j], h[j + 1], h[j + 2], h[j + 3]));
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < nval) o[j] = (uint16_t)(h[j >> 1] >> (16 * (j & 1)));
              }
            }
          }
          if (warp == 2 && lane == 0) PACKR_TRACE_EVENT(13, (t_local * 2 + sub) * 8 + c);
          if (MODE == DW && want_hist && row_ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nval) hmax = max(hmax, v[j] & 0x7FFFFFFFu);  // NaN and Inf order above every finite value
          }
        }
      }
      }  // ready
      if constexpr (MODE == DW) {
        if (want_hist) {
          // tile max |dW| over the eight epilogue warps
          uint32_t* xchg = reinterpret_cast<uint32_t*>(sAux + HIST_COPIES * HIST_COPY_BYTES + HIST_SUM_BYTES) +
                           (t_local & 1) * 8;
          const uint32_t wmax = __reduce_max_sync(0xFFFFFFFFu, hmax);
          if (lane == 0) xchg[ew] = wmax;
          asm volatile("bar.sync 1, %0;" ::"n"(C::kEpiWarps * 32) : "memory");
          uint32_t tmax = 0;
#pragma unroll
          for (int i = 0; i < 8; ++i) tmax = max(tmax, xchg[i]);
          const uint32_t E = tmax >> 23;  // biased exponent of the tile max
          const bool fixed = tmax != 0 && tmax < 0x7F800000u && E >= 21;
          float* bin_sum = reinterpret_cast<float*>(sAux + HIST_COPIES * HIST_COPY_BYTES);
          if (ready && tmax != 0) {
            // q = RN(dW * 2^(20 - e)) for a tile max in [2^e, 2^(e+1)): |q| <= 2^21,
            // rounded by adding 1.5 * 2^23 (exact for |dW * scale| < 2^22)
            const float scale = __int_as_float((int)((274u - E) << 23));
            const int m0 = (tile % P.m_tiles) * (2 * BM * MSUB) + sub * 2 * BM + (int)rank * BM;
            const int n0 = (tile / P.m_tiles) * BN;
#pragma unroll
            for (int c = 0; c < C::kChunksPerEpiWarp; ++c) {
              const int cc = cc0 + c;
              uint32_t v[32];
              tmem_ld_32x32b_x32(tmem_base + (uint32_t)(acc * ACC_COLS + cc * 32) + ((uint32_t)(q * 32) << 16), v);
              tmem_ld_wait();
              const int gn0 = n0 + cc * 32;
              if (gn0 >= P.Ng || m0 + q * 32 >= P.Mg) continue;
              const int nval = (int)(m0 + q * 32 + lane) < P.Mg ? min(32, P.Ng - gn0) : 0;  // rows past dW: none
              const uint32_t w[8] = {wpa[c].x, wpa[c].y, wpa[c].z, wpa[c].w, wpb[c].x, wpb[c].y, wpb[c].z, wpb[c].w};
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (j < nval) {
                  const uint32_t bin = (w[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                  if (fixed) {
                    const int qv = __float_as_int(__fmaf_rn(__uint_as_float(v[j]), scale, 12582912.0f)) - 0x4B400000;
                    asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(hist_lane + bin * 128), "r"(qv) : "memory");
                  } else {
                    asm volatile("red.shared.add.f32 [%0], %1;" ::"r"(smem_u32(bin_sum + bin)),
                                 "f"(__uint_as_float(v[j]))
                                 : "memory");
                  }
                }
              }
            }
          }
          if (ready) {
            tc_fence_before();
            __syncwarp();
            if (warp == 2 && lane == 0) PACKR_TRACE_EVENT(5, t_local);
            if (lane == 0) mbar_arrive_cluster(acc ? tempty1 : tempty0);
          }
          asm volatile("bar.sync 1, %0;" ::"n"(C::kEpiWarps * 32) : "memory");
          if (fixed) {
            // bin 32 * ew + lane: its 64 integer words (read skewed by lane,
            // so the warp's loads hit 32 banks), cleared for the next tile
            uint32_t* words = reinterpret_cast<uint32_t*>(sAux);
            const int b = ew * 32 + lane;
            long long sum = 0;
#pragma unroll 8
            for (int i = 0; i < HIST_COPIES * 32; ++i) {
              const int wi = (i >> 5) * (HIST_COPY_BYTES / 4) + b * 32 + ((i + lane) & 31);
              sum += (int)words[wi];
              words[wi] = 0u;
            }
            const float inv = __int_as_float((int)((E - 20u) << 23));  // 2^(e - 20)
            bin_sum[b] = __fadd_rn(bin_sum[b], __fmul_rn(__ll2float_rn(sum), inv));
          }
        }
      }
      if (!(MODE == DW && want_hist) && ready) {
        tc_fence_before();
        __syncwarp();
        if (warp == 2 && lane == 0) PACKR_TRACE_EVENT(5, t_local);
        if (lane == 0) mbar_arrive_cluster(acc ? tempty1 : tempty0);
      }
    }
    if (C::kStreamK && alive && u.kind == 1) {  // publish this warp's part of the head partial
      __threadfence();
      __syncwarp();
      if (lane == 0) {
        int* f = P.sk_flags + (pair * 2 + (int)rank) * C::kEpiWarps + ew;
        asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(1) : "memory");
      }
    }
    if (dyn) have_next = alive && next_any(un);
    if (want_hist && have_next) fetch_idx(un.tile);
    u = un;
    have = have_next;
    }
    if (MODE == DW && want_hist && P.dlut_sum != nullptr) {
      asm volatile("bar.sync 1, %0;" ::"n"(C::kEpiWarps * 32) : "memory");
      // this CTA's bin sums (bin 32 * ew + lane) into the launch's
      const float s = reinterpret_cast<const float*>(sAux + HIST_COPIES * HIST_COPY_BYTES)[ew * 32 + lane];
      if (alive && s != 0.0f) atomicAdd(P.dlut_sum + ew * 32 + lane, s);
    }
  } else if (C::kDecode && !C::kWtma && warp == C::kSignalWarp) {
    // ------------------------------------------------ decode-completion signaller
    // The decode warps keep global loads of later stages in flight; a memory
    // fence issued by them would wait for those loads.  They hand each
    // finished stage (after fence.proxy.async) to this warp through a named
    // barrier instead, and this warp (no loads outstanding) arrives on the
    // even CTA's bfull.
    const int my_tiles = pair < num_tiles ? (num_tiles - 1 - pair) / npairs + 1 : 0;
    const int total = my_tiles * kb_total;
    for (int it = 0; it < total; ++it) {
      const int s = it % STAGES;
      asm volatile("bar.sync %0, %1;" ::"r"(2 + s), "n"(DEC_THREADS + 32) : "memory");
      if (lane == 0) PACKR_TRACE_EVENT(8, it);
      if (lane == 0 && !*abort_flag) mbar_arrive_cluster(mapa(smem_u32(&bars->bfull[s]), 0));
      if (lane == 0) PACKR_TRACE_EVENT(9, it);
    }
  } else if (C::kWtma) {
    // ------------------------------------------------ weight decode, TMA-staged (both CTAs)
    const int t = threadIdx.x - C::kDecWarp0 * 32;
    const uint32_t* lut_lane = reinterpret_cast<const uint32_t*>(sAux) + lane;
    const int my_tiles = pair < num_tiles ? (num_tiles - 1 - pair) / npairs + 1 : 0;
    const int total = my_tiles * kb_total;
    for (int it = 0; it < total; ++it) {
      const int s = it % STAGES;
      const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
      if (!mbar_wait_warp(&bars->wfull[s], ph, abort_flag)) break;
      if (t == 0) PACKR_TRACE_EVENT(6, it);
      const int tile = pair + (it / kb_total) * npairs;
      const int nb0 = (tile / P.m_tiles) * BN + (int)rank * BN_CTA;
      decode_in_place<MODE, C::kDecWarps * 32>(P, sB + s * B_BYTES, sWp + s * C::kWpBytes, lut_lane, t, nb0,
                                               ((it % kb_total) % P.k_blocks) * BK);
      fence_proxy_async_smem();
      __syncwarp();
      if (t == 0) PACKR_TRACE_EVENT(7, it);
      if (lane == 0) mbar_arrive_cluster(mapa(smem_u32(&bars->bfull[s]), 0));
    }
  } else if (C::kDecode) {
    // ------------------------------------------------ weight decode, register ring (both CTAs)
    const int t = threadIdx.x - C::kDecWarp0 * 32;
    const uint32_t lut_lane = smem_u32(sAux) + (uint32_t)lane * 4u;
    const uint32_t sB0 = smem_u32(sB);
    const int my_tiles = pair < num_tiles ? (num_tiles - 1 - pair) / npairs + 1 : 0;
    const int total = my_tiles * kb_total;
    auto load = [&](Chunks& c, int it) {
      const int tl = it / kb_total;
      const int kk = it % kb_total;
      const int tile = pair + tl * npairs;
      // this CTA's half of the decoded operand: 128 output columns of the tile
      const int nb0 = (tile / P.m_tiles) * BN + (int)rank * BN_CTA;
      decode_load<MODE>(c, P, t, nb0, (kk % P.k_blocks) * BK);
    };
    // Every decode thread arrives on the hand-off barrier for every item, also
    // after an abort (then without decoding), so the signal warp's bar.sync
    // always completes.
    auto process = [&](const Chunks& c, int it) {
      const int s = it % STAGES;
      const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
      const bool go = __shfl_sync(0xFFFFFFFFu, *abort_flag ? 0 : 1, 0) != 0;  // warp-uniform
      if (go && mbar_wait_warp(&bars->empty[s], ph ^ 1u, abort_flag)) {
        if (t == 0) PACKR_TRACE_EVENT(6, it);
        decode_store<MODE>(c, sB0 + s * B_BYTES, lut_lane, t);
        fence_proxy_async_smem();
        if (t == 0) PACKR_TRACE_EVENT(7, it);
      }
      __syncwarp();
      asm volatile("bar.arrive %0, %1;" ::"r"(2 + s), "n"(DEC_THREADS + 32) : "memory");
    };
    // 3-deep ring: loads for items it+1 and it+2 are in flight while item it
    // is decoded.
    Chunks r0, r1, r2;
    if (total > 0) load(r0, 0);
    if (total > 1) load(r1, 1);
    for (int it = 0; it < total; it += 3) {
      if (it + 2 < total) load(r2, it + 2);
      if (t == 0) PACKR_TRACE_EVENT(11, it);
      process(r0, it);
      if (it + 1 >= total) break;
      if (it + 3 < total) load(r0, it + 3);
      process(r1, it + 1);
      if (it + 2 >= total) break;
      if (it + 4 < total) load(r1, it + 4);
      process(r2, it + 2);
    }
  }

  // Every MMA issued must complete before TMEM is released (both CTAs wait
  // for the even CTA's final multicast commit).
  if (warp == 1 && lane == 0) {
    volatile int no_abort = 0;
    mbar_wait(&bars->drain, 0, &no_abort);
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 2-D map over [rows, inner] with the given row stride, 128-byte swizzle,
// box {64, box_rows}.  Out-of-range elements read as zero.
int make_map(CUtensorMap* m, const void* base, long long inner, long long rows, long long row_stride_bytes,
             int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return PACKR_ERR_CUDA;
  if (!aligned(base, 16) || (row_stride_bytes & 15) != 0) return PACKR_ERR_ALIGNMENT;
  if (inner <= 0 || rows <= 0) return PACKR_ERR_SHAPE;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride_bytes};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PACKR_OK : PACKR_ERR_INVALID_ARGUMENT;
}

// u8 2-D map over [rows, inner] (row stride in bytes), no swizzle, box
// {box_inner, box_rows}; out-of-range elements read as zero.
int make_map_u8(CUtensorMap* m, const void* base, long long inner, long long rows, long long row_stride_bytes,
                int box_inner, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return PACKR_ERR_CUDA;
  if (!aligned(base, 16) || (row_stride_bytes & 15) != 0) return PACKR_ERR_ALIGNMENT;
  if (inner <= 0 || rows <= 0) return PACKR_ERR_SHAPE;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PACKR_OK : PACKR_ERR_INVALID_ARGUMENT;
}

template <int MODE, int BSRC, int MSUB = 1>
int launch_impl(Params P, const Maps& maps, cudaStream_t stream) {
  using C = Cfg<MODE, BSRC, MSUB>;
  static std::once_flag attr_once[64];
  static int resident_pairs[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int attr_rc = 0;
  std::call_once(attr_once[dev & 63], [&] {
    attr_rc = cudaFuncSetAttribute(packr_gemm_kernel<MODE, BSRC, MSUB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   C::kSmemBytes) != cudaSuccess;
    // CTA pairs that can be resident at once (a cluster needs two free SMs
    // of one GPC): the persistent grid is never larger
    cudaLaunchConfig_t q = cfg;
    q.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, packr_gemm_kernel<MODE, BSRC, MSUB>, &q) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = sm_count() / 2;
    }
    resident_pairs[dev & 63] = n;
  });
  if (attr_rc) return PACKR_ERR_CUDA;
  P.m_tiles = (P.Mg + 2 * BM * MSUB - 1) / (2 * BM * MSUB);
  const int tiles = P.m_tiles * P.n_tiles;
  if (tiles == 0) return PACKR_OK;
  const int max_pairs = resident_pairs[dev & 63];
  const long long kbt = (long long)P.nseg * P.k_blocks;
  // Fewer tiles than resident pairs (few output tiles, a long reduction):
  // every pair takes an equal share of the (tile, k-block) iterations, a
  // tile's share spanning several pairs whose partials its first pair adds
  // (measured: the plain forward and dX at 256 rows, 16-43 tiles of the
  // Llama FFN layers, otherwise leave most SMs idle).
  const bool sk_all = C::kStreamK && PACKR_STREAM_K && P.sk_partial != nullptr && P.sk_flags != nullptr &&
                      tiles < max_pairs && max_pairs > 1 && max_pairs <= P.sk_slots && kbt >= 2 &&
                      (long long)tiles * kbt >= max_pairs;  // every pair a non-empty range (it publishes a flag)
  const int pairs = sk_all ? max_pairs : (tiles < max_pairs ? tiles : max_pairs);
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  // stream-K when every pair gets at least one tile's worth of k-blocks (so a
  // tile is split between two pairs at most) and the workspace has the slots
  P.sk = 0;
  if (sk_all) {
    P.sk = 1;
    P.sk_dp_tiles = 0;
    if (cudaMemsetAsync(P.sk_flags, 0, (size_t)pairs * 2 * C::kEpiWarps * sizeof(int), stream) != cudaSuccess)
      return PACKR_ERR_CUDA;
  } else if (C::kStreamK && PACKR_STREAM_K && P.sk_partial != nullptr && P.sk_flags != nullptr && pairs > 1 &&
             pairs <= P.sk_slots) {
    // Only when the last wave of whole tiles would be less than half full:
    // a split tile costs an extra accumulator drain and a partial read, more
    // than a fuller last wave wastes.  Whole waves but the last go
    // round-robin; the stream-K share of the rest is at least one tile per
    // pair.
    const int waves = tiles / pairs, rem = tiles % pairs;
    P.sk_dp_tiles = waves >= 2 ? (waves - 1) * pairs : 0;
    if (waves >= 1 && rem != 0 && rem * 100 <= pairs * PACKR_SK_LAST_WAVE_PCT &&
        (long long)(tiles - P.sk_dp_tiles) * kbt / pairs >= kbt) {
      P.sk = 1;
      if (cudaMemsetAsync(P.sk_flags, 0, (size_t)pairs * 2 * C::kEpiWarps * sizeof(int), stream) != cudaSuccess)
        return PACKR_ERR_CUDA;
    }
  }
  // whole tiles from a counter when there is no stream-K split (the counter
  // is the first word of the stream-K flags, unused then)
  P.dyn = 0;
  P.tile_counter = nullptr;
  if (C::kPlainB && PACKR_DYN_TILES && !P.sk && P.sk_flags != nullptr && tiles > pairs) {
    P.dyn = 1;
    P.tile_counter = P.sk_flags;
    if (cudaMemsetAsync(P.tile_counter, 0, sizeof(int), stream) != cudaSuccess) return PACKR_ERR_CUDA;
  }
  if (cudaLaunchKernelEx(&cfg, packr_gemm_kernel<MODE, BSRC, MSUB>, P, maps) != cudaSuccess) {
    cudaGetLastError();
    return PACKR_ERR_LAUNCH;
  }
  return launch_status();
}

// W_f / W_p can be staged by TMA: rows of W_p a multiple of 16 bytes and both
// bases 16-byte aligned.
inline bool wtma_ok(const uint8_t* W_p, const uint16_t* W_f, long long ldw) {
  return (ldw & 15) == 0 && aligned(W_f, 16) && aligned(W_p, 16);
}

// Launches one GEMM.  Decode modes stage W_f / W_p by TMA when W's rows are
// 16-byte multiples of u8 (N % 16 == 0) and both bases are 16-byte aligned;
// otherwise the decode warps load them through a register ring.  TMA-staged
// decode with more than 256 output rows uses 512-row pair tiles.
template <int MODE>
int launch(Params P, Maps maps, cudaStream_t stream) {
  P.w_vec = (P.ldw & 7) == 0 && aligned(P.W_f, 16) && aligned(P.W_p, 8);
  P.out_vec = aligned(P.out, 16);
  P.idx_vec = aligned(P.hist_idx, 16);
  P.n_tiles = (P.Ng + BN - 1) / BN;
  P.k_blocks = (P.Kg + BK - 1) / BK;
  if constexpr (MODE == DW) {
    return launch_impl<MODE, B_RING>(P, maps, stream);
  } else {
  if (!wtma_ok(P.W_p, P.W_f, P.ldw)) return launch_impl<MODE, B_RING>(P, maps, stream);
  int st = make_map(&maps.wf, P.W_f, P.w_cols, P.w_rows, P.ldw * 2, MODE == FWD ? BK : BN_CTA);
  if (st == PACKR_OK)
    st = MODE == FWD ? make_map_u8(&maps.wp, P.W_p, P.w_cols, P.w_rows, P.ldw, BN_CTA, BK)
                     : make_map_u8(&maps.wp, P.W_p, P.w_cols, P.w_rows, P.ldw, BK, BN_CTA);
  if (st != PACKR_OK) return st;
  // more than one 256-row pair tile: two subtiles share each decoded stage
  if (P.Mg > 2 * BM) return launch_impl<MODE, B_WTMA, 2>(P, maps, stream);
  return launch_impl<MODE, B_WTMA, 1>(P, maps, stream);
  }
}

// FWD / DX over a predecoded bf16 W (maps.b[0] set by the caller: FWD an
// [K, N] map with 64-row boxes, DX an [K, N] map with 128-row boxes).
template <int MODE>
int launch_plain(Params P, const Maps& maps, cudaStream_t stream) {
  static_assert(MODE != DW, "DW has its own operands");
  P.out_vec = aligned(P.out, 16);
  P.idx_vec = 0;
  P.n_tiles = (P.Ng + BN - 1) / BN;
  P.k_blocks = (P.Kg + BK - 1) / BK;
  if (P.Mg >= PACKR_PLAIN_MSUB2_MIN_M) return launch_impl<MODE, B_PLAIN, 2>(P, maps, stream);
  return launch_impl<MODE, B_PLAIN, 1>(P, maps, stream);
}

}  // namespace gemm
}  // namespace packr

namespace packr {
namespace gemm {

// Stand-alone decode of W = bf16(W_f + bf16(lut[W_p])) into a row-major
// [K, N] bf16 array, through exactly the load / lookup / add / swizzled store
// routines the FWD GEMM's decode warps run, one 64 x 128 half-tile at a time.
__global__ void __launch_bounds__(DEC_THREADS) decode_check_kernel(const Params P, uint16_t* __restrict__ out,
                                                                  int k_tiles, int n_tiles) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint32_t* lut_s = reinterpret_cast<uint32_t*>(smem);
  uint8_t* tile = smem + LUT_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = threadIdx.x;
  for (int e = warp; e < 256; e += DEC_WARPS) lut_s[e * 32 + lane] = f32_to_bf16_rne(__ldg(P.lut + e));
  __syncthreads();
  const uint32_t lut_lane = smem_u32(lut_s) + (uint32_t)lane * 4u;
  for (int idx = blockIdx.x; idx < k_tiles * n_tiles; idx += gridDim.x) {
    const int k0 = (idx % k_tiles) * BK, n0 = (idx / k_tiles) * BN_CTA;
    Chunks c;
    decode_load<FWD>(c, P, t, n0, k0);
    decode_store<FWD>(c, smem_u32(tile), lut_lane, t);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < CHUNKS; ++i) {
      int brow, bcol8;
      chunk_coords<FWD>(t, i, brow, bcol8);
      const uint32_t off = chunk_smem_off<FWD>(brow, bcol8);
      const uint4 q = *reinterpret_cast<const uint4*>(tile + off);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      const long long r = (long long)k0 + brow, c0 = (long long)n0 + 8 * bcol8;
      if (r >= P.w_rows) continue;
      for (int j = 0; j < 8 && c0 + j < P.w_cols; ++j)
        out[r * P.ldw + c0 + j] = (uint16_t)(w[j >> 1] >> (16 * (j & 1)));
    }
    __syncthreads();
  }
}

int decode_check(const uint8_t* W_p, const uint16_t* W_f, const float* lut, uint16_t* out, long long K, long long N,
                 cudaStream_t st) {
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = LUT_BYTES + B_BYTES + 1024;
  int rc = 0;
  std::call_once(once[dev & 63], [&] {
    rc = cudaFuncSetAttribute(decode_check_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess;
  });
  if (rc) return PACKR_ERR_CUDA;
  Params P{};
  P.W_p = W_p;
  P.W_f = W_f;
  P.lut = lut;
  P.ldw = N;
  P.w_rows = (int)K;
  P.w_cols = (int)N;
  P.w_vec = (N & 7) == 0 && aligned(W_f, 16) && aligned(W_p, 8);
  const long long kt = (K + BK - 1) / BK, nt = (N + BN_CTA - 1) / BN_CTA;
  if (kt * nt == 0) return PACKR_OK;
  const long long grid = kt * nt < 4 * sm_count() ? kt * nt : 4 * sm_count();
  decode_check_kernel<<<(int)grid, DEC_THREADS, smem, st>>>(P, out, (int)kt, (int)nt);
  return launch_status();
}

}  // namespace gemm
}  // namespace packr
