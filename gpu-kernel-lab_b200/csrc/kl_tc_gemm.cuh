// Kernel template of the persistent tcgen05 weight-only GEMM, shared by the
// translation units that instantiate it (kl_tc_gemm.cu: the bf16-MMA formats;
// kl_tc_i8.cu: the int8-MMA row format).
#pragma once
// tcgen05 weight-only quantized GEMM for B200 (sm_100a): decode (M <= 64),
// prefill (M > 64) and grouped launches of independent GEMMs, in one
// warp-specialised persistent kernel.
//
//   y[m, n] = sum_k x[m, k] * dequant(w)[n, k]      (f32 accumulate, bf16/f16 out)
//
// Swap-AB mapping: the MMA's M dimension is 128 WEIGHT rows and its N
// dimension is a tile of n_mma TOKENS, so a single decode token still uses a
// legal 128 x 16 MMA and the weight stream -- the quantity that sets the speed
// at small M -- is read exactly once per tile.
//
// Data path per 128-element K block (one pipeline unit):
//   HBM --TMA--> smem int8/int4 tile (swizzled)          [W producer warp]
//   L2  --TMA--> smem x tile (swizzled, MMA B operand)    [X producer warp]
//   smem --ld.shared--> regs --exact int->bf16--> tcgen05.st --> TMEM
//                                                         [8 converter warps]
//   tcgen05.mma.kind::f16  D[tmem] += A[tmem] * X[smem]    [1 MMA thread]
//   TMEM --tcgen05.ld--> regs --> scale / SwiGLU --> global [4 epilogue warps]
// The weight ring is released by the converters as soon as a tile is in TMEM,
// independently of the MMA, so its depth (up to 16 x 16 KB per SM) is what
// covers HBM latency.  Converting straight into tensor memory keeps the bf16
// copy of the weights out of shared memory entirely.
//
// The integer codes are exact in bf16 (|q| <= 127 for int8, |q - z| <= 15 for
// int4) and the per-row / per-group scales are applied to the f32 accumulator,
// so the dequantised weights the tensor core multiplies are bit-exact and the
// only rounding is f32 accumulation plus the final cast.
//   KL_W8_ROW  : one f32 accumulation per (tile, K range); scale in epilogue.
//   KL_W4_ASYM / KL_W4_SYM (group 128 = one K block): every K block is a
//   separate accumulation that the epilogue scales and adds in registers.
//
// Work partition (stream-K): the (problem, tile, k-block) units of all
// problems are split into `grid` contiguous ranges.  A tile covered by one CTA
// is finished in place; a tile split between CTAs is finished by the last CTA
// to arrive (an atomic counter), which sums every contributor's f32 partial in
// CTA order -- deterministic, with no spin-wait on another CTA.  Every
// mbarrier wait is bounded (see kl_common.cuh).
#include "kl_common.cuh"
#include "kl_internal.h"

#include <atomic>
#include <type_traits>

namespace kl {

namespace {

// A single thread issues one small-N tcgen05.mma every ~27 ns regardless of
// its size, so at decode shapes the MMA issue rate -- not the tensor core --
// bounds the weight stream.  Each K block's 8 MMAs are therefore split across
// NI issuing threads (separate warps), each accumulating into its own TMEM
// region; the epilogue adds the NI partial accumulators.
template <int NMMA, int KBL>
struct TcCfg {
  static constexpr int NI = NMMA <= 64 ? 2 : 1;                        // MMA issuer warps
  static constexpr int ACOLS = KBL / 2;                      // TMEM columns of one A stage (bf16 pairs)
  static constexpr int D_PITCH = NMMA < 32 ? 32 : NMMA;     // columns per D accumulator
  static constexpr int A_STAGES_FIT = (512 - 2 * NI * D_PITCH) / ACOLS;
  static constexpr int A_STAGES = A_STAGES_FIT > 4 ? 4 : A_STAGES_FIT;
  static constexpr int D_COL0 = ACOLS * A_STAGES;            // A stages first
  static constexpr int TMEM_COLS = 512;
  static constexpr int NDB = 2;                              // accumulator buffers
  static_assert(A_STAGES >= 2 && D_COL0 + 2 * NI * D_PITCH <= TMEM_COLS, "TMEM budget");
  // D accumulator of buffer b (0/1) and issuer w
  static constexpr uint32_t d_col(int b, int w) { return D_COL0 + (b * NI + w) * D_PITCH; }
  static constexpr int KSTEPS = KBL / 16;                    // MMAs (K = 16 each) per stage
  static constexpr int X_ATOM = NMMA * 128;                  // bytes: NMMA rows x 64 bf16
  static constexpr int X_ATOMS = KBL / 64;
  static constexpr int X_STAGE = X_ATOMS * X_ATOM;
};

template <int FMT> constexpr bool is_w4() { return FMT == KL_W4_SYM || FMT == KL_W4_ASYM || FMT == kFmtI8W4; }
template <int FMT> constexpr bool is_i8() { return FMT == kFmtI8; }
template <int FMT> constexpr bool is_i8w4() { return FMT == kFmtI8W4; }
// bf16 group scales and zero points (the asymmetric format's data)
template <int FMT> constexpr bool asym4() { return FMT == KL_W4_ASYM || FMT == kFmtI8W4; }

// Int8-MMA row format (kFmtI8): the weights are the MMA's A operand straight
// from the TMA-filled shared-memory stage (int8, K-major, 128B swizzle), and
// B is the tile's activations as three int8 digit planes [h; m; l] of T
// tokens each (x = s_t * (65536 h + 256 m + l), see kl_tc_i8.cu), so one
// tcgen05.mma.kind::i8 of N = i8_tile_rows(T) produces all digit sums in
// int32.  No conversion, no A stages in TMEM; a K block of 128 is 4 MMAs of
// K = 32.
template <int T, int KBL>
struct TcCfgI8 {
  static constexpr int NI = 1;
  static constexpr int ACOLS = 0;
  static constexpr int A_STAGES = 0;
  static constexpr int ROWS = i8_tile_rows(T);               // MMA N: h [0, T), m [T, 2T), l [2T, 3T), padding
  static constexpr int D_PITCH = ROWS;
  static constexpr int D_COL0 = 0;
  static constexpr int TMEM_COLS = 2 * ROWS <= 32 ? 32 : 2 * ROWS <= 64 ? 64 : 2 * ROWS <= 128 ? 128
                                 : 2 * ROWS <= 256 ? 256 : 512;   // two accumulator buffers, a power of two
  static constexpr int NDB = 2;
  static constexpr uint32_t d_col(int b, int w) { return D_COL0 + (b * NI + w) * D_PITCH; }
  static constexpr int KSTEPS = KBL / 32;                    // MMAs (K = 32 each) per stage
  static constexpr int X_ATOM = ROWS * 128;                  // bytes: the tile's digit rows x 128
  static constexpr int X_ATOMS = KBL / 128;
  static constexpr int X_STAGE = X_ATOMS * X_ATOM;
  static_assert(X_ATOM % 1024 == 0, "digit atoms stay 1024-byte aligned for the 128-byte swizzle");
};
// Int8-MMA 4-bit format (kFmtI8W4): the converters turn each 128-group of
// nibbles into int8 (q - z) -- exact, four per TMEM column -- as the A operand
// of tcgen05.mma.kind::i8 against the same digit planes as kFmtI8.  Every
// group is its own accumulation (the epilogue applies its bf16 scale), so the
// accumulator ring is deep: int8 A stages take half the TMEM of bf16 ones,
// which leaves room for 8 accumulators and lets the epilogue trail the MMAs
// by several groups instead of holding them every second stage.
template <int T, int KBL>
struct TcCfgI8W4 {
  static_assert(KBL == 128, "one 128-group per stage");
  static constexpr int NI = 1;
  static constexpr int ACOLS = KBL / 4;                      // int8: four per 32-bit column
  static constexpr int A_STAGES = 4;
  static constexpr int ROWS = i8_tile_rows(T);
  static constexpr int D_PITCH = ROWS;
  static constexpr int D_COL0 = ACOLS * A_STAGES;
  static constexpr int NDB_FIT = (512 - D_COL0) / D_PITCH;
  static constexpr int NDB = NDB_FIT > 8 ? 8 : NDB_FIT;
  static constexpr int TMEM_COLS = 512;
  static_assert(NDB >= 2, "TMEM budget");
  static constexpr uint32_t d_col(int b, int w) { return D_COL0 + (b * NI + w) * D_PITCH; }
  static constexpr int KSTEPS = KBL / 32;                    // MMAs (K = 32 each) per stage
  static constexpr int X_ATOM = ROWS * 128;
  static constexpr int X_ATOMS = KBL / 128;
  static constexpr int X_STAGE = X_ATOMS * X_ATOM;
};
// Two-group bf16 4-bit stages (K block 256, 16-token tiles): every stage is two
// accumulations that the epilogue must scale before the MMA may reuse their
// buffer, so the ring trades one of the three A stages for two more
// accumulator buffers (2 x 128 A columns + 4 x 64 D columns).
template <int NMMA, int KBL>
struct TcCfgW4Pair : TcCfg<NMMA, KBL> {
  static constexpr int A_STAGES = 2;
  static constexpr int D_COL0 = TcCfg<NMMA, KBL>::ACOLS * A_STAGES;
  static constexpr int NDB = 4;
  static_assert(D_COL0 + NDB * TcCfg<NMMA, KBL>::NI * TcCfg<NMMA, KBL>::D_PITCH <= 512, "TMEM budget");
  static constexpr uint32_t d_col(int b, int w) {
    return D_COL0 + (b * TcCfg<NMMA, KBL>::NI + w) * TcCfg<NMMA, KBL>::D_PITCH;
  }
};
template <int FMT, int NMMA, int KBL>
constexpr bool w4_pair_stage() { return (FMT == KL_W4_SYM || FMT == KL_W4_ASYM) && KBL == 256 && NMMA == 16; }
template <int FMT, int NMMA, int KBL>
using TcCfgOf = std::conditional_t<
    is_i8<FMT>(), TcCfgI8<NMMA, KBL>,
    std::conditional_t<is_i8w4<FMT>(), TcCfgI8W4<NMMA, KBL>,
                       std::conditional_t<w4_pair_stage<FMT, NMMA, KBL>(), TcCfgW4Pair<NMMA, KBL>, TcCfg<NMMA, KBL>>>>;

// s * (65536 h + 256 m + l) from the three int32 digit-plane sums, one rounding
KL_DEVICE float digits3(uint32_t h, uint32_t m, uint32_t l) {
  return fmaf(65536.0f, static_cast<float>(static_cast<int>(h)),
              fmaf(256.0f, static_cast<float>(static_cast<int>(m)), static_cast<float>(static_cast<int>(l))));
}

// Warp roles: 0 W-TMA, 1 MMA issuer 0 (+ TMEM owner), 2 X-TMA, then CW
// converter warps (CW/4 per TMEM lane quadrant, each converting a 1/(CW/4)
// slice of the K block), 4 epilogue warps, then the NI-1 other MMA issuers,
// then (optional) a second epilogue group that owns accumulator buffer 1 and
// finishes every other tile.  The int -> bf16 conversion is latency-bound at
// two warps per scheduler, so the 256-element stages with small token tiles
// get four converter warps per scheduler.  The two-group 4-bit stages use 8
// converter warps in CG = 2 groups of 4 that take alternate units, each thread
// converting a whole 256-wide row of its TMEM lane.  With 16 warps on one unit
// (768 threads, 80 registers and epilogue spills) a unit took ~1750 cycles and
// under half the issue slots were used; 512 threads leave every role 128
// registers, and two units in flight overlap one group's waits with the
// other's conversion.
// The int8-MMA mode has no converters: W-TMA, MMA issuer, X-TMA, 4 epilogue warps.
template <int FMT, int NMMA, int KBL>
struct TcRoles {
  static constexpr int NI = TcCfgOf<FMT, NMMA, KBL>::NI;
  static constexpr int CW = is_i8<FMT>() ? 0
                          : (KBL == 256 && NMMA == 16 && !(FMT == KL_W4_SYM || FMT == KL_W4_ASYM)) ? 16 : 8;
  // two converter groups on alternate units: two-group 4-bit stages, and the
  // int8 4-bit format (a thread converts a whole 128-wide row per unit)
  static constexpr int CG = (is_i8w4<FMT>() || (KBL == 256 && NMMA == 16 && (FMT == KL_W4_SYM || FMT == KL_W4_ASYM)))
                                ? 2 : 1;
  static constexpr int CWG = is_i8<FMT>() ? 4 : CW / CG;    // converter warps per group (per unit)
  static constexpr int CONV0 = 3;
  static constexpr int EPI0_WARP0 = CONV0 + CW;
  static constexpr int ISS1_WARP0 = EPI0_WARP0 + 4;
  static constexpr int EPI_GROUPS = 1;
  static constexpr int EPI1_WARP0 = ISS1_WARP0 + NI - 1;
  static constexpr int WARPS = EPI1_WARP0 + 4 * (EPI_GROUPS - 1);
  static constexpr int THREADS = WARPS * 32;
  static constexpr int EPT = KBL / (CWG / 4);               // K elements per converter thread and stage
};
// Weight stage: 128 rows x KBL elements, stored as column blocks of one
// swizzle span (128 B of int8 / 64 B of packed int4) by 128 rows.
template <int FMT, int KBL> constexpr int w_row_bytes() { return is_w4<FMT>() ? KBL / 2 : KBL; }
template <int FMT, int KBL> constexpr int w_stage_bytes() { return 128 * w_row_bytes<FMT, KBL>(); }
// Two-group asymmetric 4-bit stages also carry the tile's zero points: the W
// producer copies a box of 8 groups x 128 rows of the bf16 zeros [N, K/128]
// (two 64-row halves, 1 KB each) behind the weights with the same barrier, so
// the converters read each row's zero from shared memory instead of walking
// the units themselves.  Needs K % 1024 == 0 (16-byte rows of zeros).
template <int FMT, int KBL> constexpr bool zeros_in_stage() { return FMT == KL_W4_ASYM && KBL == 256; }
constexpr int kZeroStageBytes = 2048;
template <int FMT, int KBL> constexpr int w_stage_pitch() {
  return w_stage_bytes<FMT, KBL>() + (zeros_in_stage<FMT, KBL>() ? kZeroStageBytes : 0);
}
template <int FMT> constexpr bool grouped() { return is_w4<FMT>(); }

constexpr int kXchFloats = 64 * 16;               // SwiGLU up-value exchange: 64 rows x 16 cols f32
constexpr int kXchBytes = 2 * kXchFloats * 4;      // one exchange area per epilogue group
constexpr int kUnitCacheBytes = 8 * kMaxGroup;    // problem unit_begin cache (grouped launches)

struct SmemLayout {
  uint32_t w, x, xch, ucache, zoff, bars, misc, total;
};
__host__ __device__ constexpr SmemLayout smem_layout(int wsb, int x_stage, int a_stages, int sw, int sx, int ndb = 2) {
  SmemLayout l{};
  l.w = 0;
  l.x = l.w + sw * wsb;
  l.xch = l.x + sx * x_stage;
  l.ucache = l.xch + kXchBytes;
  l.zoff = l.ucache + kUnitCacheBytes;       // per weight stage: zero-point offset in its box (4 B each)
  l.bars = l.zoff + 4 * kMaxWStages;
  // w_full, w_empty [sw]; x_full, x_empty [sx]; a_full, a_empty [A]; d_full, d_empty [ndb]; done
  l.misc = l.bars + 8 * (2 * sw + 2 * sx + 2 * a_stages + 2 * ndb + 1);
  l.total = l.misc + 16 + 1024;           // + slack to align the base to 1024 B
  return l;
}

struct Pipe {
  int idx, n;
  uint32_t phase;
  KL_DEVICE void next() {
    if (++idx == n) { idx = 0; phase ^= 1u; }
  }
};

KL_DEVICE bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        record_error(status, KL_ERR_TIMEOUT);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// wait_bar executed by every lane of a warp, with a warp-uniform result.
KL_DEVICE bool wait_bar_warp(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  const bool ok = wait_bar(bar, parity, abort_flag, status);
  return __all_sync(0xFFFFFFFFu, ok);
}

// Abort path of a TMA producer: wait (time-bounded) until the last copy issued
// into every stage of a ring has landed, so no copy is in flight when the
// CTA's shared memory is released.  Stage s was last filled by issue number
// s + n*((issued-1-s)/n), whose barrier phase parity is ((that)/n) & 1.
template <typename BarFn>
KL_DEVICE void drain_ring(BarFn full, int n, int issued) {
  for (int s = 0; s < n && s < issued; ++s) {
    const int last = s + n * ((issued - 1 - s) / n);
    mbar_wait_time(full(s), static_cast<uint32_t>((last / n) & 1));
  }
}

// Barrier among the 4 warps of one epilogue group (ids 1 and 2; 0 is __syncthreads).
KL_DEVICE void named_bar_epi(int g) { asm volatile("bar.sync %0, 128;" :: "r"(1 + g) : "memory"); }

struct Problems {
  const TcParams* p;
  const long long* ucache;            // smem copy of unit_begin (count > 1)
  KL_DEVICE const TcProblem& get(int i) const { return p->count == 1 ? p->single : p->table[i]; }
  KL_DEVICE int find(long long u) const {
    if (p->count == 1) return 0;
    int lo = 0, hi = p->count - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (ucache[mid] <= u) lo = mid; else hi = mid - 1;
    }
    return lo;
  }
};

// Walks a CTA's contiguous range of (problem, m-tile, n-tile, k-block) units
// incrementally: one division at start-up, none per unit (64-bit division is
// a long instruction sequence on the GPU and sat on every role's critical path).
struct Cursor {
  const Problems* ps;
  const TcProblem* pr;
  long long u, u_lo, u_hi, tile_u0;
  int prob, mt, nt, kb, kb_total, n_tiles, m_tiles;
  KL_DEVICE void load() {
    pr = &ps->get(prob);
    kb_total = pr->kb_total;
    n_tiles = pr->n_tiles;
    m_tiles = pr->m_tiles;
  }
  KL_DEVICE void init(const Problems& P, long long lo, long long hi) {
    ps = &P;
    u_lo = lo;
    u_hi = hi;
    u = lo;
    prob = 0;
    mt = nt = kb = 0;
    tile_u0 = lo;
    if (lo >= hi) return;
    prob = P.find(lo);
    load();
    const int rel = static_cast<int>(lo - pr->unit_begin);   // < 2^31 units per problem
    const int tile = rel / kb_total;
    kb = rel - tile * kb_total;
    mt = tile / n_tiles;
    nt = tile - mt * n_tiles;
    tile_u0 = lo - kb;
  }
  KL_DEVICE bool seg_start() const { return u == u_lo || kb == 0; }
  KL_DEVICE bool seg_end() const { return u == u_hi - 1 || kb == kb_total - 1; }
  KL_DEVICE void next() {
    ++u;
    if (++kb == kb_total) {
      kb = 0;
      tile_u0 = u;
      if (++nt == n_tiles) {
        nt = 0;
        if (++mt == m_tiles) {
          mt = 0;
          ++prob;
          if (u < u_hi) load();
        }
      }
    }
  }
};

// 32-bit sort key of a candidate within a 128-row tile: the order-preserving
// bits of the value rounded to bf16 (the logit the layer would output; zero of
// either sign as +0) in the high half, the inverted row within the tile in the
// low half.  A larger key is the larger value and, on ties, the lower row; the
// value is exact in the key because a bf16 value has 16 bits.  Key 0 is below
// every real candidate.
KL_DEVICE uint32_t topk_key(float v_bf16, int row_in_tile) {
  uint32_t u = __float_as_uint(v_bf16);
  if ((u & 0x7FFFFFFFu) == 0u) u = 0u;
  const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (ord & 0xFFFF0000u) | (0xFFFFu - static_cast<uint32_t>(row_in_tile));
}
// The merge kernel's packed form: (index << 32) | f32 value bits.
KL_DEVICE unsigned long long topk_packed(uint32_t key, int row0, long long index_offset) {
  if (key == 0u) return (0x7FFFFFFFull << 32) | __float_as_uint(-INFINITY);   // no candidate
  const uint32_t ord = key & 0xFFFF0000u;
  const uint32_t u = (ord & 0x80000000u) ? (ord & 0x7FFF0000u) : (~ord & 0xFFFF0000u);
  const long long row = row0 + static_cast<long long>(0xFFFFu - (key & 0xFFFFu));
  return (static_cast<unsigned long long>(row + index_offset) << 32) | u;
}
// Bitonic sorts of J independent keys per lane across the warp, descending
// (lane 0 holds the largest of each).  The J networks run stage by stage side
// by side, so their shuffles overlap instead of each sort waiting out fifteen
// dependent shuffle round trips.
template <int J>
KL_DEVICE void warp_sort_desc(uint32_t (&key)[J]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const bool desc = size == 32 || (lane & size) == 0;
      const bool keep_max = ((lane & stride) == 0) == desc;
      uint32_t other[J];
#pragma unroll
      for (int j = 0; j < J; ++j) other[j] = __shfl_xor_sync(0xFFFFFFFFu, key[j], stride);
#pragma unroll
      for (int j = 0; j < J; ++j) key[j] = keep_max ? max(key[j], other[j]) : min(key[j], other[j]);
    }
  }
}

template <int FMT, int NMMA, int EPI, bool XBF16>
struct Epi {
  static constexpr bool SWIGLU = EPI == kEpiSwiglu;
  static constexpr bool TOPK = EPI == kEpiTopk;
  // Physical weight row of tile row r (0..127) of n-tile nt.
  KL_DEVICE static int phys_row(const TcProblem& pr, int nt, int r) {
    if constexpr (SWIGLU) return r < 64 ? nt * 64 + r : pr.n_out + nt * 64 + (r - 64);
    else return nt * 128 + r;
  }
  KL_DEVICE static float row_scale(const TcProblem& pr, int prow) {
    if constexpr (FMT == KL_W8_ROW || FMT == kFmtI8) {
      const int r = prow < pr.n ? prow : pr.n - 1;
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(pr.scales)[r]);
    } else {
      return 1.0f;
    }
  }
  // Emit 16 token columns [cb*16, cb*16+16) of tile row r.
  KL_DEVICE static void emit16(const TcProblem& pr, int mt, int nt, int r, int cb, const float (&v)[16], float* xch,
                               int g) {
    const int m0 = mt * NMMA + cb * 16;
    if constexpr (TOPK) {
      // per token, the tile's top-k rows: each warp sorts its 32 rows, then the
      // four warps merge the four warps' best, warp w taking tokens w, w + 4, ...
      // (all 128 threads call this)
      static_assert(XBF16, "the top-k epilogue keys bf16 logits");
      const int n = nt * 128 + r;
      const bool valid = n < pr.n_out;
      const int lane = r & 31, wq = r >> 5, kk = pr.topk;
      uint32_t* xk = reinterpret_cast<uint32_t*>(xch);   // [4 warps][16 tokens][8]
      const int mv = pr.m - m0;                          // tokens of these 16 that exist
      // sorts of tokens j0 .. j0 + J - 1 side by side (as many as exist, rounded up)
      auto sort_rows = [&](auto jc, auto j0c) {
        constexpr int J = decltype(jc)::value, j0 = decltype(j0c)::value;   // compile time: v[] stays in registers
        uint32_t key[J];
#pragma unroll
        for (int jj = 0; jj < J; ++jj)
          key[jj] = (valid && j0 + jj < mv) ? topk_key(round_act<XBF16>(v[j0 + jj]), r) : 0u;
        warp_sort_desc<J>(key);
#pragma unroll
        for (int jj = 0; jj < J; ++jj)
          if (j0 + jj < mv && lane < kk) xk[(wq * 16 + j0 + jj) * 8 + lane] = key[jj];
      };
      using C0 = std::integral_constant<int, 0>;
      using C8 = std::integral_constant<int, 8>;
      if (NMMA == 16 && mv <= 1) {            // the narrow forms only where M <= 16 makes them common
        sort_rows(std::integral_constant<int, 1>{}, C0{});
      } else if (NMMA == 16 && mv <= 4) {
        sort_rows(std::integral_constant<int, 4>{}, C0{});
      } else {
        sort_rows(C8{}, C0{});
        if (mv > 8) sort_rows(C8{}, C8{});
      }
      named_bar_epi(g);
      // the four warps merge the four warps' best: warp wq takes tokens wq, wq + 4, ...;
      // lane l reads candidate l % kk of warp l / kk
      auto merge_rows = [&](auto tc) {
        constexpr int T = decltype(tc)::value;
        const int src = lane < 4 * kk ? (lane / kk) * 16 * 8 + lane % kk : 0;
        uint32_t key[T];
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const int j = wq + 4 * t;
          key[t] = (j < mv && lane < 4 * kk) ? xk[src + j * 8] : 0u;
        }
        warp_sort_desc<T>(key);
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const int j = wq + 4 * t;
          if (j < mv && lane < kk)
            pr.cand[static_cast<long long>(m0 + j) * pr.cand_ld + nt * kk + lane] =
                topk_packed(key[t], nt * 128, pr.index_offset);
        }
      };
      if (wq < mv) {
        if (NMMA == 16 && mv <= 4) merge_rows(std::integral_constant<int, 1>{});
        else merge_rows(std::integral_constant<int, 4>{});
      }
      named_bar_epi(g);
      return;
    }
    if constexpr (!SWIGLU) {
      // a warp's 32 rows x 16 tokens in range of a row-major output: stage them
      // [token][row] in this warp's 1 KB of the (otherwise idle) exchange area
      // and store 64 contiguous bytes per token as 16-byte vectors
      const int n0 = nt * 128 + (r & ~31), lane = r & 31;
      if (pr.vec_store == 1 && n0 + 32 <= pr.n_out && m0 + 16 <= pr.m) {
        uint8_t* st = reinterpret_cast<uint8_t*>(xch + (r >> 5) * 256);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 16; ++j) store_act<XBF16>(st, j * 32 + lane, v[j]);
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 2; ++it) {
          const int vi = it * 32 + lane, t = vi >> 2, part = vi & 3;
          const uint4 val = *reinterpret_cast<const uint4*>(st + t * 64 + part * 16);
          *reinterpret_cast<uint4*>(static_cast<uint8_t*>(pr.y) +
                                    ((static_cast<long long>(m0 + t) * pr.ldy + n0 + part * 8) << 1)) = val;
        }
        return;
      }
      const int n = nt * 128 + r;
      if (pr.vec_store == 2 && n < pr.n_out && m0 + 16 <= pr.m) {
        // transposed output: this row's 16 tokens are contiguous, two 16-byte stores
        uint32_t pk[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) pk[j] = XBF16 ? pack_bf16x2(v[2 * j], v[2 * j + 1]) : pack_f16x2(v[2 * j], v[2 * j + 1]);
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(pr.y) + ((static_cast<long long>(n) * pr.ldy + m0) << 1));
        dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        return;
      }
      if (n < pr.n_out) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + j;
          if (m < pr.m) {
            const long long yi = pr.y_transposed ? static_cast<long long>(n) * pr.ldy + m
                                                 : static_cast<long long>(m) * pr.ldy + n;
            store_act<XBF16>(pr.y, yi, v[j]);
          }
        }
      }
    } else {
      if (r >= 64) {
#pragma unroll
        for (int j = 0; j < 16; ++j) xch[(r - 64) * 16 + ((j + r) & 15)] = v[j];
      }
      named_bar_epi(g);
      if (r < 64) {
        const int n = nt * 64 + r;
        if (n < pr.n_out) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + j;
            if (m < pr.m) {
              const float up = xch[r * 16 + ((j + r + 64) & 15)];
              const long long yi = pr.y_transposed ? static_cast<long long>(n) * pr.ldy + m
                                                   : static_cast<long long>(m) * pr.ldy + n;
              store_act<XBF16>(pr.y, yi, swiglu_model_ordered<XBF16>(v[j], up));
            }
          }
        }
      }
      named_bar_epi(g);
    }
  }
};

template <int FMT, int NMMA, int KBL, int EPI, bool XBF16>
__global__ void __launch_bounds__(TcRoles<FMT, NMMA, KBL>::THREADS, 1)
tc_qgemm_kernel(const __grid_constant__ TcParams p) {
  constexpr bool SWIGLU = EPI == kEpiSwiglu;
  using Cfg = TcCfgOf<FMT, NMMA, KBL>;
  constexpr bool I8 = is_i8<FMT>();
  constexpr bool DIG = is_i8<FMT>() || is_i8w4<FMT>();   // B operand = activation digit planes
  using Roles = TcRoles<FMT, NMMA, KBL>;
  using E = Epi<FMT, NMMA, EPI, XBF16>;
  static_assert(!grouped<FMT>() || KBL == 128 || (KBL == 256 && NMMA == 16), "4-bit group mode: one or two groups of 128 per stage");
  constexpr int WSB = w_stage_bytes<FMT, KBL>();
  constexpr bool ZST = zeros_in_stage<FMT, KBL>();
  constexpr int WSP = w_stage_pitch<FMT, KBL>();                // stage pitch: weights (+ zeros)
  static_assert(WSP % 1024 == 0, "stages stay 1024-byte aligned for the 128-byte swizzle");
  constexpr int ROW_BYTES = w_row_bytes<FMT, KBL>();      // bytes of one tile row per stage
  constexpr int SPAN = (is_w4<FMT>() && KBL == 128) ? 64 : 128;   // swizzle span = TMA box inner bytes
  constexpr int NBLK = ROW_BYTES / SPAN;                  // column blocks per stage
  constexpr int BLK = 128 * SPAN;                         // bytes of one column block
  constexpr int A = Cfg::A_STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int SW = p.w_stages, SX = p.x_stages;
  constexpr int NDB = Cfg::NDB;
  const SmemLayout L = smem_layout(WSP, Cfg::X_STAGE, A, SW, SX, NDB);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t s_w = s_base + L.w, s_x = s_base + L.x, s_bars = s_base + L.bars;
  float* xch = reinterpret_cast<float*>(smem + L.xch);
  long long* ucache = reinterpret_cast<long long*>(smem + L.ucache);
  volatile uint32_t* zoff = reinterpret_cast<volatile uint32_t*>(smem + L.zoff);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L.misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc + 4);
  volatile int* fix_flags = reinterpret_cast<volatile int*>(smem + L.misc + 8);   // one per epilogue group
  auto w_full = [&](int i) { return s_bars + 8u * i; };
  auto w_empty = [&](int i) { return s_bars + 8u * (SW + i); };
  auto x_full = [&](int i) { return s_bars + 8u * (2 * SW + i); };
  auto x_empty = [&](int i) { return s_bars + 8u * (2 * SW + SX + i); };
  auto a_full = [&](int i) { return s_bars + 8u * (2 * SW + 2 * SX + i); };
  auto a_empty = [&](int i) { return s_bars + 8u * (2 * SW + 2 * SX + A + i); };
  auto d_full = [&](int i) { return s_bars + 8u * (2 * SW + 2 * SX + 2 * A + i); };
  auto d_empty = [&](int i) { return s_bars + 8u * (2 * SW + 2 * SX + 2 * A + NDB + i); };
  const uint32_t done_bar = s_bars + 8u * (2 * SW + 2 * SX + 2 * A + 2 * NDB);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long G = gridDim.x, c = blockIdx.x;
  const long long u_lo = unit_lo(c, p.units, G), u_hi = unit_lo(c + 1, p.units, G);
  const int n_local = static_cast<int>(u_hi - u_lo);
  Problems probs{&p, ucache};

  if (p.count > 1) {
    for (int i = threadIdx.x; i < p.count; i += blockDim.x) ucache[i] = p.table[i].unit_begin;
    __syncthreads();                        // unit cache visible before any unit decoding
  }
  // Thread 0 initialises the barriers and starts streaming weights at once
  // (before TMEM allocation and the block-wide barrier): weights are static, so
  // this also runs ahead of the previous kernel in the stream (PDL).
  Pipe pw{0, SW, 0};
  int w_pre = 0;
  Cursor cw;
  auto issue_w = [&]() {
    const TcProblem& pr = *cw.pr;
    const uint32_t dst = s_w + pw.idx * WSP;
    // zeros box: 8 groups from a 16-byte-aligned group index; the stage's pair
    // starts at (2 kb) & 7 within it (published with the barrier's release)
    if constexpr (ZST) zoff[pw.idx] = static_cast<uint32_t>((cw.kb * 2) & 7);
    mbar_arrive_expect_tx(w_full(pw.idx), ZST ? WSB + kZeroStageBytes : WSB);
    const int y0 = SWIGLU ? cw.nt * 64 : cw.nt * 128;
    const int y1 = SWIGLU ? pr.n_out + cw.nt * 64 : cw.nt * 128 + 64;
#pragma unroll
    for (int b = 0; b < NBLK; ++b) {
      tma_load_2d(dst + b * BLK, &pr.tmap_w, cw.kb * ROW_BYTES + b * SPAN, y0, w_full(pw.idx));
      tma_load_2d(dst + b * BLK + BLK / 2, &pr.tmap_w, cw.kb * ROW_BYTES + b * SPAN, y1, w_full(pw.idx));
    }
    if constexpr (ZST) {
      const int gx = (cw.kb * 2) & ~7;
      tma_load_2d(dst + WSB, &pr.tmap_z, gx, y0, w_full(pw.idx));
      tma_load_2d(dst + WSB + kZeroStageBytes / 2, &pr.tmap_z, gx, y1, w_full(pw.idx));
    }
    cw.next();
  };
  if (threadIdx.x == 0) {
    // a weight stage is released by its converters, or (int8 MMA) by the MMAs that read it
    for (int i = 0; i < SW; ++i) { mbar_init(w_full(i), 1); mbar_init(w_empty(i), I8 ? Cfg::NI : Roles::CWG); }
    for (int i = 0; i < SX; ++i) { mbar_init(x_full(i), 1); mbar_init(x_empty(i), Cfg::NI); }
    for (int i = 0; i < A; ++i) { mbar_init(a_full(i), Roles::CWG); mbar_init(a_empty(i), Cfg::NI); }
    for (int i = 0; i < NDB; ++i) { mbar_init(d_full(i), Cfg::NI); mbar_init(d_empty(i), 4); }
    mbar_init(done_bar, Cfg::NI);
    *abort_flag = 0;
    fix_flags[0] = 0;
    fix_flags[1] = 0;
    fence_mbar_init();
    cw.init(probs, u_lo, u_hi);
    if (n_local > 0) prefetch_tmap(&cw.pr->tmap_w);
    w_pre = n_local < SW ? n_local : SW;
    for (int i = 0; i < w_pre; ++i) { issue_w(); pw.next(); }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ W producer
    if (lane == 0) {
      bool ok = true;
      int last_prob = cw.prob, issued = w_pre;
      for (int i = w_pre; i < n_local; ++i) {
        if (!(ok = wait_bar(w_empty(pw.idx), pw.phase ^ 1u, abort_flag, p.status))) break;
        if (cw.prob != last_prob) { prefetch_tmap(&cw.pr->tmap_w); last_prob = cw.prob; }
        issue_w();
        pw.next();
        ++issued;
      }
      if (!ok) drain_ring(w_full, SW, issued);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ X producer
    if (lane == 0) {
      pdl_wait();                          // activations come from the previous kernel
      Pipe px{0, SX, 0};
      bool ok = true;
      int last_prob = -1, issued = 0;
      Cursor cx;
      cx.init(probs, u_lo, u_hi);
      for (int i = 0; i < n_local; ++i, cx.next()) {
        if (!(ok = wait_bar(x_empty(px.idx), px.phase ^ 1u, abort_flag, p.status))) break;
        const TcProblem& pr = *cx.pr;
        if (cx.prob != last_prob) { prefetch_tmap(&pr.tmap_x); last_prob = cx.prob; }
        const uint32_t dst = s_x + px.idx * Cfg::X_STAGE;
        mbar_arrive_expect_tx(x_full(px.idx), Cfg::X_STAGE);
#pragma unroll
        for (int a = 0; a < Cfg::X_ATOMS; ++a)
          tma_load_2d(dst + a * Cfg::X_ATOM, &pr.tmap_x, cx.kb * KBL + (DIG ? 128 : 64) * a,
                      cx.mt * (DIG ? i8_tile_rows(NMMA) : NMMA), x_full(px.idx));
        px.next();
        ++issued;
      }
      if (!ok) drain_ring(x_full, SX, issued);
    }
  } else if (warp == 1 || (warp >= Roles::ISS1_WARP0 && warp < Roles::EPI1_WARP0)) {
    // ------------------------------------------------------------ MMA issuers
    // The whole warp runs the loop (so operands stay warp-uniform) and one
    // elected lane issues the MMAs and commits.
    if constexpr (I8) {
      // A = the weight stage itself (int8, 128B swizzle, 128-byte column
      // blocks of 128 rows), B = the digit stage; the MMAs' commit releases both.
      constexpr uint32_t idesc = make_idesc_i8(128, Cfg::ROWS);
      constexpr int NBLK_W = KBL / 128;
      static_assert(Cfg::KSTEPS == 4 * NBLK_W, "four K = 32 steps per 128-byte column block");
      const uint32_t w_desc0 = smem_desc_sw128_lo(s_w), x_desc0 = smem_desc_sw128_lo(s_x);
      Pipe pwm{0, SW, 0}, px{0, SX, 0}, pd{0, NDB, 0};
      bool ok = true;
      Cursor cm;
      cm.init(probs, u_lo, u_hi);
      for (int i = 0; i < n_local && ok; ++i, cm.next()) {
        const bool chunk_start = cm.seg_start();
        const bool chunk_end = cm.seg_end();
        if (chunk_start && !(ok = wait_bar_warp(d_empty(pd.idx), pd.phase ^ 1u, abort_flag, p.status))) break;
        if (!(ok = wait_bar_warp(x_full(px.idx), px.phase, abort_flag, p.status))) break;
        if (!(ok = wait_bar_warp(w_full(pwm.idx), pwm.phase, abort_flag, p.status))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + Cfg::d_col(pd.idx, 0);
        const uint32_t wd = w_desc0 + static_cast<uint32_t>((pwm.idx * WSP) >> 4);
        const uint32_t xd = x_desc0 + static_cast<uint32_t>(px.idx * (Cfg::X_STAGE >> 4));
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < Cfg::KSTEPS; ++j)
            tc_mma_ss_i8(d_tmem, wd + static_cast<uint32_t>(((j >> 2) * BLK + (j & 3) * 32) >> 4),
                         xd + static_cast<uint32_t>(((j >> 2) * Cfg::X_ATOM + (j & 3) * 32) >> 4), idesc,
                         (chunk_start && j == 0) ? 0u : 1u);
          tc_commit(x_empty(px.idx));
          tc_commit(w_empty(pwm.idx));
          if (chunk_end) tc_commit(d_full(pd.idx));
        }
        __syncwarp();
        px.next();
        pwm.next();
        if (chunk_end) pd.next();
      }
      if (elect_one()) tc_commit(done_bar);
      __syncwarp();
      mbar_wait_time(done_bar, 0);
    } else {
      constexpr uint32_t idesc = is_i8w4<FMT>() ? make_idesc_i8(128, i8_tile_rows(NMMA)) : make_idesc_f16(128, NMMA, XBF16);
      constexpr int JPER = Cfg::KSTEPS / Cfg::NI;    // K steps (of 16, or 32 for int8) per issuer and stage
      const int w = warp == 1 ? 0 : warp - Roles::ISS1_WARP0 + 1;
      // Descriptor and TMEM offsets of this issuer's K steps, computed once:
      // the issue loop then costs one add per operand per MMA.
      const uint32_t x_desc0 = smem_desc_sw128_lo(s_x);
      uint32_t b_off[JPER];
#pragma unroll
      for (int jj = 0; jj < JPER; ++jj) {
        const int j = w * JPER + jj;
        b_off[jj] = static_cast<uint32_t>((j >> 2) * Cfg::X_ATOM + (j & 3) * 32) >> 4;
      }
      const uint32_t a_off = 8u * static_cast<uint32_t>(w * JPER);
      Pipe px{0, SX, 0}, pa{0, A, 0}, pd{0, NDB, 0};
      bool ok = true;
      Cursor cm;
      cm.init(probs, u_lo, u_hi);
      for (int i = 0; i < n_local && ok; ++i, cm.next()) {
        const bool chunk_start = grouped<FMT>() ? true : cm.seg_start();
        const bool chunk_end = grouped<FMT>() ? true : cm.seg_end();
        if (chunk_start && !(ok = wait_bar_warp(d_empty(pd.idx), pd.phase ^ 1u, abort_flag, p.status))) break;
        if (!(ok = wait_bar_warp(x_full(px.idx), px.phase, abort_flag, p.status))) break;
        if (!(ok = wait_bar_warp(a_full(pa.idx), pa.phase, abort_flag, p.status))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + Cfg::d_col(pd.idx, w);
        const uint32_t a_tmem = tmem + static_cast<uint32_t>(Cfg::ACOLS) * pa.idx + a_off;
        const uint32_t xd = x_desc0 + static_cast<uint32_t>(px.idx * (Cfg::X_STAGE >> 4));
        if (elect_one()) {
#pragma unroll
          for (int jj = 0; jj < JPER; ++jj) {
            if constexpr (is_i8w4<FMT>())
              tc_mma_ts_i8_lo(d_tmem, a_tmem + 8u * jj, xd + b_off[jj], idesc, (chunk_start && jj == 0) ? 0u : 1u);
            else
              tc_mma_ts_lo(d_tmem, a_tmem + 8u * jj, xd + b_off[jj], idesc, (chunk_start && jj == 0) ? 0u : 1u);
          }
          tc_commit(x_empty(px.idx));
          tc_commit(a_empty(pa.idx));
          if (chunk_end) tc_commit(d_full(pd.idx));
        }
        __syncwarp();
        px.next();
        pa.next();
        if (chunk_end) pd.next();
      }
      // Make sure no MMA is still reading/writing TMEM when the CTA tears down.
      if (elect_one()) tc_commit(done_bar);
      __syncwarp();
      mbar_wait_time(done_bar, 0);
    }
  } else if (warp < Roles::EPI0_WARP0) {
    // -------------------------------------------------------------- converters
   if constexpr (!I8) {
    const int q = warp & 3;                 // TMEM lane quadrant of this warp
    const int cg = (warp - Roles::CONV0) / Roles::CWG;          // converter group: units cg, cg + CG, ...
    const int h = ((warp - Roles::CONV0) % Roles::CWG) >> 2;    // which slice of the K block
    const int r = q * 32 + lane;            // tile row owned by this thread
    Pipe pwc{0, SW, 0}, pa{0, A, 0};
    // this group's first unit; every pass then steps CG units
    auto step = [&](Cursor& cu, Pipe* pw, Pipe* pp) {
#pragma unroll
      for (int s = 0; s < Roles::CG; ++s) {
        cu.next();
        if (pw) pw->next();
        if (pp) pp->next();
      }
    };
    Cursor cc_;
    cc_.init(probs, u_lo, u_hi);
    for (int s = 0; s < cg; ++s) { cc_.next(); pwc.next(); pa.next(); }
    // 4-bit zero point of this thread's row for a unit (a global load, issued
    // one unit ahead so its latency overlaps the previous unit's conversion)
    auto load_zero = [&](const Cursor& cu) -> float {
      if constexpr (asym4<FMT>()) {
        const TcProblem& pz = *cu.pr;
        int zr = E::phys_row(pz, cu.nt, r);
        zr = zr < pz.n ? zr : pz.n - 1;
        // groups of 128 along K; this thread's slice of the stage lies in one group
        constexpr int GPS = KBL / 128;
        const int grp = cu.kb * GPS + (h * Roles::EPT) / 128;
        return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(pz.zeros)[static_cast<long long>(zr) * cu.kb_total * GPS + grp]);
      } else {
        return 8.0f;
      }
    };
    // zeros carried in the stage: this thread's row within the box (two 64-row halves)
    const uint32_t zrow = static_cast<uint32_t>(r) * 16u;
    float z_cur = 8.0f;
    if constexpr (is_w4<FMT>() && !ZST) { if (cg < n_local) z_cur = load_zero(cc_); }
    for (int i = cg; i < n_local; i += Roles::CG) {
      float z_next = 8.0f;
      if constexpr (is_w4<FMT>() && !ZST) {
        if (i + Roles::CG < n_local) {
          Cursor nx = cc_;
          step(nx, nullptr, nullptr);
          z_next = load_zero(nx);
        }
      }
      if (!wait_bar(w_full(pwc.idx), pwc.phase, abort_flag, p.status)) break;
      if (!wait_bar(a_empty(pa.idx), pa.phase ^ 1u, abort_flag, p.status)) break;
      constexpr int EPT = Roles::EPT;              // elements per thread (a slice of the stage row)
      const uint8_t* wstage = smem + L.w + pwc.idx * WSP;
      // zero points of the stage's two groups (slices that lie in one group use one)
      float zg0 = z_cur, zg1 = z_cur;
      if constexpr (ZST) {
        const uint32_t zz = *reinterpret_cast<const uint32_t*>(wstage + WSB + zrow + zoff[pwc.idx] * 2u);
        zg0 = __uint_as_float(zz << 16);
        zg1 = __uint_as_float(zz & 0xFFFF0000u);
      }
      if constexpr (!is_w4<FMT>()) {
        // EPT int8 = EPT/16 chunks of 16 B; chunk g of the stage row sits in column
        // block g/8 at position (g%8) ^ (r & 7) (128B swizzle).  All chunks are
        // loaded first; then each pair of chunks (16 TMEM columns) is converted and
        // stored, so at most 16 converted words are live at a time.
        uint4 v[EPT / 16];
#pragma unroll
        for (int cc = 0; cc < EPT / 16; ++cc) {
          const int g = h * (EPT / 16) + cc;
          v[cc] = *reinterpret_cast<const uint4*>(wstage + (g >> 3) * BLK + r * 128 + (((g & 7) ^ (r & 7)) << 4));
        }
        const uint32_t a_tmem = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(Cfg::ACOLS) * pa.idx +
                                static_cast<uint32_t>(EPT / 2) * h;
#pragma unroll
        for (int j = 0; j < EPT / 32; ++j) {
          uint32_t part[16];
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            const uint4 vv = v[2 * j + c2];
            const uint32_t wd[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              if constexpr (XBF16) s8x4_to_bf16x4_fma(wd[t], part[c2 * 8 + 2 * t], part[c2 * 8 + 2 * t + 1]);
              else s8x4_to_f16x4(wd[t], part[c2 * 8 + 2 * t], part[c2 * 8 + 2 * t + 1]);
            }
          }
          tmem_st16(a_tmem + 16u * j, part);
        }
      } else if constexpr (is_i8w4<FMT>()) {
        // EPT nibbles of row r = EPT/32 chunks of 16 B (64B swizzle: chunk g at
        // g ^ ((r >> 1) & 3)) -> EPT int8 (q - z) in K order, EPT/4 TMEM columns.
        // Per 8 nibbles: the even and odd codes as bytes 128 + c (one lop3
        // each), interleaved back into K order (two byte permutes), minus z in
        // every byte (no borrow: 128 + c - z >= 113), then ^ 0x80 leaves the
        // two's-complement int8 q - z.
        static_assert(EPT % 64 == 0, "whole 16-column TMEM stores");
        const uint32_t z4 = static_cast<uint32_t>(__float2int_rn(zg0)) * 0x01010101u;
        uint4 v[EPT / 32];
#pragma unroll
        for (int cc = 0; cc < EPT / 32; ++cc) {
          const int g = h * (EPT / 32) + cc;
          v[cc] = *reinterpret_cast<const uint4*>(wstage + r * 64 + ((g ^ ((r >> 1) & 3)) << 4));
        }
#pragma unroll
        for (int c2 = 0; c2 < EPT / 64; ++c2) {
          uint32_t part[16];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t wd[4] = {v[2 * c2 + c].x, v[2 * c2 + c].y, v[2 * c2 + c].z, v[2 * c2 + c].w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const uint32_t lo = lop3<0xEA>(wd[t], 0x0F0F0F0Fu, 0x80808080u);
              const uint32_t hi = lop3<0xEA>(wd[t] >> 4, 0x0F0F0F0Fu, 0x80808080u);
              part[c * 8 + 2 * t] = (prmt(lo, hi, 0x5140u) - z4) ^ 0x80808080u;
              part[c * 8 + 2 * t + 1] = (prmt(lo, hi, 0x7362u) - z4) ^ 0x80808080u;
            }
          }
          tmem_st16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(Cfg::ACOLS) * pa.idx +
                        static_cast<uint32_t>(EPT / 4) * h + 16u * c2,
                    part);
        }
      } else {
        // EPT nibbles = EPT/32 chunks of 16 B; 64B swizzle: chunk g at g ^ ((r >> 1) & 3)
        auto bias_of = [&](float z) {
          return XBF16 ? pack_bf16x2(-(128.0f + z), -(128.0f + z)) : pack_f16x2(-(1024.0f + z), -(1024.0f + z));
        };
        const uint32_t bias0 = bias_of(zg0), bias1 = bias_of(zg1);
        constexpr uint32_t magic = XBF16 ? (FMT == KL_W4_SYM ? 0x43084308u : 0x43004300u)
                                         : (FMT == KL_W4_SYM ? 0x64086408u : 0x64006400u);
        // each 16-byte chunk (32 nibbles) is 16 TMEM columns: convert and store it at once
        const uint32_t a_tmem4 = tmem + (static_cast<uint32_t>(q * 32) << 16) +
                                 static_cast<uint32_t>(Cfg::ACOLS) * pa.idx + static_cast<uint32_t>(EPT / 2) * h;
#pragma unroll
        for (int cc = 0; cc < EPT / 32; ++cc) {
          const int g = h * (EPT / 32) + cc;
          // this chunk's group within the stage (32 nibbles per chunk, 128 per group)
          const uint32_t bias = (KBL == 256 && (g >> 2)) ? bias1 : bias0;
          uint32_t part[16];
          // 64-byte rows (64B swizzle) for 128-wide stages, 128-byte rows (128B swizzle) for 256
          const uint4 v = KBL == 128 ? *reinterpret_cast<const uint4*>(wstage + r * 64 + ((g ^ ((r >> 1) & 3)) << 4))
                                     : *reinterpret_cast<const uint4*>(wstage + r * 128 + ((g ^ (r & 7)) << 4));
          const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint32_t sh = wd[t] >> 4;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              part[t * 4 + b] = XBF16 ? u4x2_to_bf16x2(wd[t], sh, nib_sel(b), magic, bias)
                                      : u4x2_to_f16x2(wd[t], sh, nib_sel(b), magic, bias);
            }
          }
          tmem_st16(a_tmem4 + 16u * cc, part);
        }
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(a_full(pa.idx));
        mbar_arrive(w_empty(pwc.idx));
      }
      step(cc_, &pwc, &pa);
      if constexpr (!ZST) z_cur = z_next;
    }
   }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int eg = warp >= Roles::EPI1_WARP0 ? 1 : 0;          // epilogue group
    const int first_thread = (eg ? Roles::EPI1_WARP0 : Roles::EPI0_WARP0) * 32;
    volatile int* fix_flag = fix_flags + eg;
    float* xg = xch + eg * kXchFloats;
    pdl_wait();                             // outputs / workspace written only after the previous kernel
    // chunk c uses accumulator buffer c % 2; with two groups, group g takes the
    // chunks with c % 2 == g, i.e. always buffer g
    Pipe pd{eg, NDB, 0};
    int chunk = 0;
    constexpr int NCHG = (NMMA + 15) / 16;   // 16-column chunks of a token tile
    float acc[grouped<FMT>() ? NCHG * 16 : 1];
    int seg_kb0 = 0;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    // 16 columns of the accumulator: the sum of the NI issuers' partial D regions
    auto load_d16 = [&](uint32_t d0, int cb, float (&v)[16]) {
      if constexpr (Cfg::NI == 2) {
        // both issuers' partial regions in flight before one wait
        uint32_t t0[16], t1[16];
        tmem_ld16(d0 + 16u * cb, t0);
        tmem_ld16(d0 + static_cast<uint32_t>(Cfg::D_PITCH) + 16u * cb, t1);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(t0[j]) + __uint_as_float(t1[j]);
      } else {
        uint32_t t[16];
        tmem_ld16(d0 + 16u * cb, t);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(t[j]);
#pragma unroll
        for (int w = 1; w < Cfg::NI; ++w) {
          tmem_ld16(d0 + static_cast<uint32_t>(w * Cfg::D_PITCH) + 16u * cb, t);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += __uint_as_float(t[j]);
        }
      }
    };
    Cursor ce;
    ce.init(probs, u_lo, u_hi);
    const long long first_tile_u0 = ce.tile_u0;
    // int8 4-bit format: every unit is one group whose scale the epilogue needs
    // right after the accumulator wait; a cursor running kAhead units ahead
    // loads the scales early (a ring in registers) so that their latency is
    // not paid once per unit
    constexpr int kAhead = is_i8w4<FMT>() ? 3 : 0;
    float gring[kAhead + 1];
    Cursor cs = ce;
    auto scale_at = [&](const Cursor& cu) -> float {
      const TcProblem& pz = *cu.pr;
      int zr = E::phys_row(pz, cu.nt, r);
      zr = zr < pz.n ? zr : pz.n - 1;
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(pz.scales)[static_cast<long long>(zr) * cu.kb_total + cu.kb]);
    };
    if constexpr (kAhead > 0) {
#pragma unroll
      for (int a = 0; a < kAhead; ++a) {
        gring[a] = a < n_local ? scale_at(cs) : 0.0f;
        if (a < n_local) cs.next();
      }
    }
    bool ok = true;
    for (int i = 0; i < n_local && ok; ++i, ce.next()) {
      const TcProblem& pr = *ce.pr;
      const int mt = ce.mt, nt = ce.nt;
      float g_cur = 1.0f;
      if constexpr (kAhead > 0) {
        gring[kAhead] = i + kAhead < n_local ? scale_at(cs) : 0.0f;
        if (i + kAhead < n_local) cs.next();
        g_cur = gring[0];
#pragma unroll
        for (int a = 0; a < kAhead; ++a) gring[a] = gring[a + 1];
      }
      const bool seg_end = ce.seg_end();
      if (ce.seg_start()) {
        seg_kb0 = ce.kb;
        if constexpr (grouped<FMT>()) {
#pragma unroll
          for (int j = 0; j < NCHG * 16; ++j) acc[j] = 0.f;
        }
      }
      const bool chunk_end = grouped<FMT>() ? true : seg_end;
      if (!chunk_end) continue;
      const int my_chunk = chunk++;
      if (Roles::EPI_GROUPS == 2 && (my_chunk & 1) != eg) continue;
      const int prow = E::phys_row(pr, nt, r);
      constexpr int GPS = grouped<FMT>() ? KBL / 128 : 1;    // 128-groups per stage
      float gs[GPS];                           // group scales, loaded before the wait
#pragma unroll
      for (int gi = 0; gi < GPS; ++gi) gs[gi] = 1.0f;
      if constexpr (is_i8w4<FMT>()) {
        gs[0] = g_cur;
      } else if constexpr (grouped<FMT>()) {
        const int pr_row = prow < pr.n ? prow : pr.n - 1;
        const long long sbase = static_cast<long long>(pr_row) * ce.kb_total * GPS + ce.kb * GPS;
#pragma unroll
        for (int gi = 0; gi < GPS; ++gi) {
          if constexpr (asym4<FMT>())
            gs[gi] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(pr.scales)[sbase + gi]);
          else
            gs[gi] = reinterpret_cast<const float*>(pr.scales)[sbase + gi];
        }
      }
      if (!(ok = wait_bar(d_full(pd.idx), pd.phase, abort_flag, p.status))) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem + lane_base + Cfg::d_col(pd.idx, 0);
      const bool full_tile = seg_end && seg_kb0 == 0 && ce.kb == ce.kb_total - 1;
      float* part_base = nullptr;
      const int mrem = pr.m - mt * NMMA;      // token columns of this tile that exist
      if (seg_end && !full_tile) {
        const int slot = (ce.tile_u0 == first_tile_u0) ? 0 : 1;
        part_base = p.partials + (c * 2 + slot) * static_cast<long long>(NMMA) * 128;
      }
      if constexpr (grouped<FMT>()) {
        if constexpr (is_i8w4<FMT>()) {
          // the group's three int32 digit sums -> f32 times the group scale; the
          // token scales (one per tile) are applied where the tile is finished
          const float s = gs[0];
          if constexpr (NMMA == 8) {
            uint32_t t0[16], t1[16];             // columns 0-7 h, 8-15 m, 16-23 l
            tmem_ld16(d_tmem, t0);
            tmem_ld16(d_tmem + 16u, t1);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = fmaf(s, digits3(t0[j], t0[8 + j], t1[j]), acc[j]);
          } else {
#pragma unroll
            for (int cb = 0; cb < NMMA / 16; ++cb) {
              uint32_t th[16], tm[16], tl[16];
              tmem_ld16(d_tmem + 16u * cb, th);
              tmem_ld16(d_tmem + static_cast<uint32_t>(NMMA) + 16u * cb, tm);
              tmem_ld16(d_tmem + static_cast<uint32_t>(2 * NMMA) + 16u * cb, tl);
              tc_wait_ld();
#pragma unroll
              for (int j = 0; j < 16; ++j) acc[cb * 16 + j] = fmaf(s, digits3(th[j], tm[j], tl[j]), acc[cb * 16 + j]);
            }
          }
        } else if constexpr (GPS == 1) {
          const float s = gs[0];
#pragma unroll
          for (int cb = 0; cb < NMMA / 16; ++cb) {
            float v[16];
            load_d16(d_tmem, cb, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[cb * 16 + j] = fmaf(s, v[j], acc[cb * 16 + j]);
          }
        } else {
          // two groups per stage: issuer 0 holds group 0 (K steps 0-7), issuer 1 group 1
          static_assert(GPS == 2 && Cfg::NI == 2, "two-group stages use one issuer per group");
#pragma unroll
          for (int cb = 0; cb < NMMA / 16; ++cb) {
            uint32_t t0[16], t1[16];
            tmem_ld16(d_tmem + 16u * cb, t0);
            tmem_ld16(d_tmem + static_cast<uint32_t>(Cfg::D_PITCH) + 16u * cb, t1);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j)
              acc[cb * 16 + j] = fmaf(gs[1], __uint_as_float(t1[j]), fmaf(gs[0], __uint_as_float(t0[j]), acc[cb * 16 + j]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty(pd.idx));
        if (Roles::EPI_GROUPS == 2) pd.phase ^= 1u; else pd.next();
        if (!seg_end) continue;
        if constexpr (is_i8w4<FMT>()) {
          const float* tsp = pr.tscale + static_cast<long long>(mt) * NMMA;
#pragma unroll
          for (int j = 0; j < NMMA; ++j) acc[j] *= tsp[j];
        }
        if (full_tile) {
#pragma unroll
          for (int cb = 0; cb < NCHG; ++cb) {
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = acc[cb * 16 + j];
            E::emit16(pr, mt, nt, r, cb, o, xg, eg);
          }
          continue;
        }
        const int mvg = min(mrem, NMMA);
#pragma unroll
        for (int cb = 0; cb < NCHG; ++cb)
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (cb * 16 + j < mvg) part_base[(cb * 16 + j) * 128 + r] = acc[cb * 16 + j];
      } else if constexpr (I8) {
        // int32 digit sums -> f32: v = s_t * (65536 h + 256 m + l) per token
        // (s_t a power of two, so the only roundings are the two f32 adds); the
        // row scale is applied where the tile is finished.  The buffer goes
        // back to the MMA before the stores.
        constexpr int NCH = (NMMA + 15) / 16;
        const float s = E::row_scale(pr, prow);
        const float* tsp = pr.tscale + static_cast<long long>(mt) * NMMA;
        auto digits3 = [](uint32_t h, uint32_t m, uint32_t l) {
          return fmaf(65536.0f, static_cast<float>(static_cast<int>(h)),
                      fmaf(256.0f, static_cast<float>(static_cast<int>(m)), static_cast<float>(static_cast<int>(l))));
        };
        float v[NCH * 16];
        if constexpr (NMMA == 8) {
          uint32_t t0[16], t1[16];                 // columns 0-7 h, 8-15 m, 16-23 l
          tmem_ld16(d_tmem, t0);
          tmem_ld16(d_tmem + 16u, t1);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            v[j] = digits3(t0[j], t0[8 + j], t1[j]) * tsp[j];
            v[8 + j] = 0.0f;
          }
        } else {
#pragma unroll
          for (int cb = 0; cb < NMMA / 16; ++cb) {
            uint32_t th[16], tm[16], tl[16];
            tmem_ld16(d_tmem + 16u * cb, th);
            tmem_ld16(d_tmem + static_cast<uint32_t>(NMMA) + 16u * cb, tm);
            tmem_ld16(d_tmem + static_cast<uint32_t>(2 * NMMA) + 16u * cb, tl);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[cb * 16 + j] = digits3(th[j], tm[j], tl[j]) * tsp[cb * 16 + j];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty(pd.idx));
        pd.next();
        const int mv = min(mrem, NMMA);
#pragma unroll
        for (int cb = 0; cb < NCH; ++cb) {
          if (full_tile) {
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = v[cb * 16 + j] * s;
            E::emit16(pr, mt, nt, r, cb, o, xg, eg);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (cb * 16 + j < mv) part_base[(cb * 16 + j) * 128 + r] = v[cb * 16 + j];
          }
        }
        if (full_tile) continue;
      } else if constexpr (NMMA <= 64) {
        // Pull the whole accumulator into registers and hand the TMEM buffer
        // back to the MMA issuers before the (slower) global stores.
        const float s = E::row_scale(pr, prow);
        float v[NMMA];
#pragma unroll
        for (int cb = 0; cb < NMMA / 16; ++cb) {
          float t[16];
          load_d16(d_tmem, cb, t);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[cb * 16 + j] = t[j];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty(pd.idx));
        if (Roles::EPI_GROUPS == 2) pd.phase ^= 1u; else pd.next();
#pragma unroll
        for (int cb = 0; cb < NMMA / 16; ++cb) {
          if (full_tile) {
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = v[cb * 16 + j] * s;
            E::emit16(pr, mt, nt, r, cb, o, xg, eg);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (cb * 16 + j < mrem) part_base[(cb * 16 + j) * 128 + r] = v[cb * 16 + j];
          }
        }
        if (full_tile) continue;
      } else {
        const float s = E::row_scale(pr, prow);
        for (int cb = 0; cb < NMMA / 16; ++cb) {
          float v[16];
          load_d16(d_tmem, cb, v);
          if (full_tile) {
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = v[j] * s;
            E::emit16(pr, mt, nt, r, cb, o, xg, eg);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (cb * 16 + j < mrem) part_base[(cb * 16 + j) * 128 + r] = v[j];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty(pd.idx));
        if (Roles::EPI_GROUPS == 2) pd.phase ^= 1u; else pd.next();
        if (full_tile) continue;
      }
      // ---- split tile: publish the partial, the last contributor finishes it.
      const long long c_first = unit_owner(ce.tile_u0, p.units, G);
      const long long c_last = unit_owner(ce.tile_u0 + ce.kb_total - 1, p.units, G);
      __threadfence();
      named_bar_epi(eg);
      if (threadIdx.x == first_thread) {
        const int old = atomicAdd(p.counters + c_first, 1);
        const int last = (old == static_cast<int>(c_last - c_first));
        if (last) p.counters[c_first] = 0;   // ready for the next launch
        *fix_flag = last;
      }
      named_bar_epi(eg);
      const bool last = *fix_flag != 0;
      named_bar_epi(eg);                      // everyone read fix_flag before it is reused
      if (!last) continue;
      __threadfence();
      const float s = grouped<FMT>() ? 1.0f : E::row_scale(pr, prow);
      for (int cb = 0; cb < (NMMA + 15) / 16; ++cb) {
        // partials hold only the token columns that exist; the contributors are
        // summed in CTA order whatever the number of columns
        const int nv = min(mrem, NMMA) - cb * 16;
        if (nv <= 0) break;
        float o[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = 0.f;
        // slot 0 holds a contributor's first tile: the one its range starts in
        auto part_src = [&](long long cc) {
          const int sl = unit_lo(cc, p.units, G) >= ce.tile_u0 ? 0 : 1;
          return p.partials + (cc * 2 + sl) * static_cast<long long>(NMMA) * 128 + cb * 16 * 128 + r;
        };
        if (nv == 1) {
          // one token: eight contributors' loads in flight at a time
#pragma unroll 8
          for (long long cc = c_first; cc <= c_last; ++cc) o[0] += __ldcg(part_src(cc));
        } else {
#pragma unroll 4
          for (long long cc = c_first; cc <= c_last; ++cc) {
            const float* src = part_src(cc);
            float t[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) t[j] = j < nv ? __ldcg(src + j * 128) : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] += t[j];
          }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] *= s;
        E::emit16(pr, mt, nt, r, cb, o, xg, eg);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

template <int FMT, int NMMA, int KBL, int EPI, bool XBF16>
cudaError_t launch_one(const TcParams& p, const TcPlan& plan, bool pdl, cudaStream_t s) {
  auto kern = tc_qgemm_kernel<FMT, NMMA, KBL, EPI, XBF16>;
  static std::atomic<int> smem_set[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (smem_set[dev].load(std::memory_order_acquire) < plan.smem) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, plan.smem);
    if (e != cudaSuccess) return e;
    int cur = smem_set[dev].load();
    while (cur < plan.smem && !smem_set[dev].compare_exchange_weak(cur, plan.smem)) {
    }
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(TcRoles<FMT, NMMA, KBL>::THREADS);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace
}  // namespace kl
