// tcgen05 weight-only quantized GEMM for B200 (sm_100a): decode (M <= 64) and
// prefill (M > 64) in one warp-specialised kernel.
//
//   y[m, n] = sum_k x[m, k] * dequant(w)[n, k]      (f32 accumulate, bf16/f16 out)
//
// Swap-AB mapping: the MMA's M dimension is 128 WEIGHT rows and its N
// dimension is a tile of n_mma TOKENS, so a single decode token still uses a
// legal 128 x 16 MMA and the weight stream -- the quantity that sets the speed
// at small M -- is read exactly once per tile.
//
// Data path per 128-element K block (one pipeline stage):
//   HBM --TMA--> smem int8/int4 tile (swizzled)       [producer warp]
//   smem --ld.shared--> registers --exact int->bf16--> tcgen05.st --> TMEM
//                                                       [4 converter warps]
//   tcgen05.mma.kind::f16  D[tmem] += A[tmem] * X[smem]  [1 MMA thread]
//   TMEM --tcgen05.ld--> registers --> scale / SwiGLU --> global
//                                                       [4 epilogue warps]
// Converting straight into tensor memory keeps the bf16 copy of the weights
// out of shared memory entirely: smem only carries the compressed tile once.
//
// The integer codes are exact in bf16 (|q| <= 127 for int8, |q - z| <= 15 for
// int4) and the per-row / per-group scales are applied to the f32 accumulator,
// so the dequantised weights the tensor core multiplies are bit-exact and the
// only rounding is f32 accumulation plus the final cast.
//   KL_W8_ROW  : one f32 accumulation per (tile, K range); scale in epilogue.
//   KL_W4_ASYM / KL_W4_SYM (group 128 = one K block): every K block is a
//   separate accumulation that the epilogue scales and adds in registers.
//
// Work partition (stream-K): the (tile, k-block) units are split into `grid`
// contiguous ranges.  A tile covered by one CTA is finished in place; a tile
// split between CTAs is finished by the last CTA to arrive (an atomic counter),
// which sums every contributor's f32 partial in CTA order -- deterministic,
// with no spin-wait on another CTA.  Every mbarrier wait is bounded (see
// kl_common.cuh).
#include "kl_common.cuh"
#include "kl_internal.h"

#include <atomic>

namespace kl {

namespace {

template <int NMMA>
struct TcCfg {
  static constexpr int A_STAGES = NMMA == 128 ? 4 : (NMMA == 64 ? 2 : 3);
  static constexpr int D_PITCH = NMMA < 32 ? 32 : NMMA;     // columns per D buffer
  static constexpr int D_COL0 = 64 * A_STAGES;               // A stages first (64 cols each)
  static constexpr int USED = D_COL0 + 2 * D_PITCH;
  static constexpr int TMEM_COLS = USED <= 64 ? 64 : USED <= 128 ? 128 : USED <= 256 ? 256 : 512;
  static constexpr int X_ATOM = NMMA * 128;                  // bytes: NMMA rows x 64 bf16
  static constexpr int X_STAGE = 2 * X_ATOM;
};

template <int FMT> constexpr bool is_w4() { return FMT == KL_W4_SYM || FMT == KL_W4_ASYM; }
template <int FMT> constexpr int w_stage_bytes() { return is_w4<FMT>() ? 8192 : 16384; }
template <int FMT> constexpr bool grouped() { return is_w4<FMT>(); }

constexpr int kXchBytes = 64 * 16 * 4;   // SwiGLU up-value exchange: 64 rows x 16 cols f32

struct SmemLayout {
  uint32_t w, x, xch, bars, misc, total;
};
template <int FMT, int NMMA>
__host__ __device__ constexpr SmemLayout smem_layout(int stages) {
  SmemLayout l{};
  l.w = 0;
  l.x = l.w + stages * w_stage_bytes<FMT>();
  l.xch = l.x + stages * TcCfg<NMMA>::X_STAGE;
  l.bars = l.xch + kXchBytes;
  // w_full, x_full, w_empty, x_empty [stages]; a_full, a_empty [A]; d_full, d_empty [2]; done
  l.misc = l.bars + 8 * (4 * stages + 2 * TcCfg<NMMA>::A_STAGES + 5);
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

KL_DEVICE void named_bar_epi() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Unit bookkeeping shared by all roles.
struct UnitInfo {
  int tile, kb;
  bool seg_start, seg_end;
};
KL_DEVICE UnitInfo unit_info(long long u, long long u_lo, long long u_hi, int kb_total) {
  UnitInfo r;
  r.tile = static_cast<int>(u / kb_total);
  r.kb = static_cast<int>(u % kb_total);
  r.seg_start = (u == u_lo) || (r.kb == 0);
  r.seg_end = (u == u_hi - 1) || (r.kb == kb_total - 1);
  return r;
}

template <int FMT, int NMMA, bool SWIGLU, bool XBF16>
struct Epi {
  // Physical weight row of tile row r (0..127) of n-tile nt.
  KL_DEVICE static int phys_row(const TcParams& p, int nt, int r) {
    if constexpr (SWIGLU) return r < 64 ? nt * 64 + r : p.n_out + nt * 64 + (r - 64);
    else return nt * 128 + r;
  }
  KL_DEVICE static float row_scale(const TcParams& p, int prow) {
    if constexpr (FMT == KL_W8_ROW) {
      const int pr = prow < p.n ? prow : p.n - 1;
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.scales)[pr]);
    } else {
      return 1.0f;
    }
  }
  // Emit 16 token columns [cb*16, cb*16+16) of tile row r.
  KL_DEVICE static void emit16(const TcParams& p, int mt, int nt, int r, int cb, const float (&v)[16],
                               float* xch) {
    const int m0 = mt * NMMA + cb * 16;
    if constexpr (!SWIGLU) {
      const int n = nt * 128 + r;
      if (n < p.n_out) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + j;
          if (m < p.m) {
            const long long yi = p.y_transposed ? static_cast<long long>(n) * p.ldy + m
                                                : static_cast<long long>(m) * p.ldy + n;
            store_act<XBF16>(p.y, yi, v[j]);
          }
        }
      }
    } else {
      if (r >= 64) {
#pragma unroll
        for (int j = 0; j < 16; ++j) xch[(r - 64) * 16 + ((j + r) & 15)] = v[j];
      }
      named_bar_epi();
      if (r < 64) {
        const int n = nt * 64 + r;
        if (n < p.n_out) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + j;
            if (m < p.m) {
              const float up = xch[r * 16 + ((j + r + 64) & 15)];
              const long long yi = p.y_transposed ? static_cast<long long>(n) * p.ldy + m
                                                  : static_cast<long long>(m) * p.ldy + n;
              store_act<XBF16>(p.y, yi, swiglu_model_ordered<XBF16>(v[j], up));
            }
          }
        }
      }
      named_bar_epi();
    }
  }
};

template <int FMT, int NMMA, bool SWIGLU, bool XBF16>
__global__ void __launch_bounds__(kTcThreads, 1)
tc_qgemm_kernel(const __grid_constant__ TcParams p, const int stages) {
  using Cfg = TcCfg<NMMA>;
  using E = Epi<FMT, NMMA, SWIGLU, XBF16>;
  constexpr int WSB = w_stage_bytes<FMT>();
  constexpr int ROW_BYTES = is_w4<FMT>() ? 64 : 128;     // bytes of one tile row per stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SmemLayout L = smem_layout<FMT, NMMA>(stages);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t s_w = s_base + L.w, s_x = s_base + L.x, s_bars = s_base + L.bars;
  float* xch = reinterpret_cast<float*>(smem + L.xch);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L.misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc + 4);
  volatile int* fix_flag = reinterpret_cast<volatile int*>(smem + L.misc + 8);
  const int S = stages;
  auto w_full = [&](int i) { return s_bars + 8u * i; };
  auto x_full = [&](int i) { return s_bars + 8u * (S + i); };
  auto w_empty = [&](int i) { return s_bars + 8u * (2 * S + i); };
  auto x_empty = [&](int i) { return s_bars + 8u * (3 * S + i); };
  auto a_full = [&](int i) { return s_bars + 8u * (4 * S + i); };
  auto a_empty = [&](int i) { return s_bars + 8u * (4 * S + Cfg::A_STAGES + i); };
  auto d_full = [&](int i) { return s_bars + 8u * (4 * S + 2 * Cfg::A_STAGES + i); };
  auto d_empty = [&](int i) { return s_bars + 8u * (4 * S + 2 * Cfg::A_STAGES + 2 + i); };
  const uint32_t done_bar = s_bars + 8u * (4 * S + 2 * Cfg::A_STAGES + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long G = gridDim.x, c = blockIdx.x;
  const long long u_lo = unit_lo(c, p.units, G), u_hi = unit_lo(c + 1, p.units, G);
  const int n_local = static_cast<int>(u_hi - u_lo);
  const int KB = p.kb_total;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(w_full(i), 1);
      mbar_init(x_full(i), 1);
      mbar_init(w_empty(i), 4);
      mbar_init(x_empty(i), 1);
    }
    for (int i = 0; i < Cfg::A_STAGES; ++i) {
      mbar_init(a_full(i), 4);
      mbar_init(a_empty(i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(d_full(i), 1);
      mbar_init(d_empty(i), 4);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    *fix_flag = 0;
    fence_mbar_init();
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
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tmap_w);
      prefetch_tmap(&p.tmap_x);
      Pipe pw{0, S, 0}, px{0, S, 0};
      bool ok = true;
      bool issued_w[8] = {}, issued_x[8] = {};
      uint32_t last_w[8] = {}, last_x[8] = {};
      auto issue_w = [&](int i) {
        issued_w[pw.idx] = true;
        last_w[pw.idx] = pw.phase;
        const UnitInfo ui = unit_info(u_lo + i, u_lo, u_hi, KB);
        const int nt = ui.tile % p.n_tiles;
        const uint32_t dst = s_w + pw.idx * WSB;
        mbar_arrive_expect_tx(w_full(pw.idx), WSB);
        const int y0 = SWIGLU ? nt * 64 : nt * 128;
        const int y1 = SWIGLU ? p.n_out + nt * 64 : nt * 128 + 64;
        tma_load_2d(dst, &p.tmap_w, ui.kb * ROW_BYTES, y0, w_full(pw.idx));
        tma_load_2d(dst + WSB / 2, &p.tmap_w, ui.kb * ROW_BYTES, y1, w_full(pw.idx));
      };
      auto issue_x = [&](int i) {
        issued_x[px.idx] = true;
        last_x[px.idx] = px.phase;
        const UnitInfo ui = unit_info(u_lo + i, u_lo, u_hi, KB);
        const int mt = ui.tile / p.n_tiles;
        const uint32_t dst = s_x + px.idx * Cfg::X_STAGE;
        mbar_arrive_expect_tx(x_full(px.idx), Cfg::X_STAGE);
        tma_load_2d(dst, &p.tmap_x, ui.kb * kTcKBlock, mt * NMMA, x_full(px.idx));
        tma_load_2d(dst + Cfg::X_ATOM, &p.tmap_x, ui.kb * kTcKBlock + 64, mt * NMMA, x_full(px.idx));
      };
      const int pre = n_local < S ? n_local : S;
      // Weights are static: stream the first stages before waiting on the
      // previous kernel in the stream (programmatic dependent launch).
      for (int i = 0; i < pre; ++i) { issue_w(i); pw.next(); }
      pdl_wait();
      for (int i = 0; i < n_local && ok; ++i) {
        if (i >= pre) {
          if (!(ok = wait_bar(w_empty(pw.idx), pw.phase ^ 1u, abort_flag, p.status))) break;
          issue_w(i);
          pw.next();
        }
        if (!(ok = wait_bar(x_empty(px.idx), px.phase ^ 1u, abort_flag, p.status))) break;
        issue_x(i);
        px.next();
      }
      if (!ok) {
        // Abort path: let every copy already issued land before smem is released.
        for (int s = 0; s < S; ++s) {
          if (issued_w[s]) mbar_wait_time(w_full(s), last_w[s]);
          if (issued_x[s]) mbar_wait_time(x_full(s), last_x[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(128, NMMA, XBF16);
      Pipe px{0, S, 0}, pa{0, Cfg::A_STAGES, 0}, pd{0, 2, 0};
      bool ok = true;
      for (int i = 0; i < n_local && ok; ++i) {
        const UnitInfo ui = unit_info(u_lo + i, u_lo, u_hi, KB);
        const bool chunk_start = grouped<FMT>() ? true : ui.seg_start;
        const bool chunk_end = grouped<FMT>() ? true : ui.seg_end;
        if (chunk_start && !(ok = wait_bar(d_empty(pd.idx), pd.phase ^ 1u, abort_flag, p.status))) break;
        if (!(ok = wait_bar(x_full(px.idx), px.phase, abort_flag, p.status))) break;
        if (!(ok = wait_bar(a_full(pa.idx), pa.phase, abort_flag, p.status))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + Cfg::D_COL0 + pd.idx * Cfg::D_PITCH;
        const uint32_t a_tmem = tmem + 64u * pa.idx;
        const uint32_t xs = s_x + px.idx * Cfg::X_STAGE;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint64_t bdesc = smem_desc_sw128(xs + (j >> 2) * Cfg::X_ATOM + (j & 3) * 32);
          tc_mma_ts(d_tmem, a_tmem + 8u * j, bdesc, idesc, (chunk_start && j == 0) ? 0u : 1u);
        }
        tc_commit(x_empty(px.idx));
        tc_commit(a_empty(pa.idx));
        px.next();
        pa.next();
        if (chunk_end) {
          tc_commit(d_full(pd.idx));
          pd.next();
        }
      }
      // Make sure no MMA is still reading/writing TMEM when the CTA tears down.
      tc_commit(done_bar);
      mbar_wait_time(done_bar, 0);
    }
  } else if (warp < 6) {
    // -------------------------------------------------------------- converters
    const int q = warp & 3;                 // TMEM lane quadrant of this warp
    const int r = q * 32 + lane;            // tile row owned by this thread
    Pipe pw{0, S, 0}, pa{0, Cfg::A_STAGES, 0};
    for (int i = 0; i < n_local; ++i) {
      const UnitInfo ui = unit_info(u_lo + i, u_lo, u_hi, KB);
      if (!wait_bar(w_full(pw.idx), pw.phase, abort_flag, p.status)) break;
      if (!wait_bar(a_empty(pa.idx), pa.phase ^ 1u, abort_flag, p.status)) break;
      const uint8_t* wrow = smem + L.w + pw.idx * WSB + r * ROW_BYTES;
      uint32_t out[64];
      if constexpr (!is_w4<FMT>()) {
        // 128 int8 = 8 chunks of 16 B; 128B swizzle: chunk c at c ^ (r & 7)
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const uint4 v = *reinterpret_cast<const uint4*>(wrow + ((cc ^ (r & 7)) << 4));
          const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            if constexpr (XBF16) s8x4_to_bf16x4(wd[t], out[cc * 8 + 2 * t], out[cc * 8 + 2 * t + 1]);
            else s8x4_to_f16x4(wd[t], out[cc * 8 + 2 * t], out[cc * 8 + 2 * t + 1]);
          }
        }
      } else {
        // 128 nibbles = 4 chunks of 16 B; 64B swizzle: chunk c at c ^ ((r >> 1) & 3)
        const int nt = ui.tile % p.n_tiles;
        int prow = E::phys_row(p, nt, r);
        prow = prow < p.n ? prow : p.n - 1;
        float z = 8.0f;
        if constexpr (FMT == KL_W4_ASYM)
          z = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.zeros)[static_cast<long long>(prow) * KB + ui.kb]);
        const uint32_t bias = XBF16 ? pack_bf16x2(-(128.0f + z), -(128.0f + z))
                                    : pack_f16x2(-(1024.0f + z), -(1024.0f + z));
        constexpr uint32_t magic = XBF16 ? (FMT == KL_W4_SYM ? 0x43084308u : 0x43004300u)
                                         : (FMT == KL_W4_SYM ? 0x64086408u : 0x64006400u);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const uint4 v = *reinterpret_cast<const uint4*>(wrow + ((cc ^ ((r >> 1) & 3)) << 4));
          const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint32_t sh = wd[t] >> 4;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              out[cc * 16 + t * 4 + b] = XBF16 ? u4x2_to_bf16x2(wd[t], sh, nib_sel(b), magic, bias)
                                               : u4x2_to_f16x2(wd[t], sh, nib_sel(b), magic, bias);
            }
          }
        }
      }
      const uint32_t a_tmem = tmem + (static_cast<uint32_t>(q * 32) << 16) + 64u * pa.idx;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t part[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) part[t] = out[16 * j + t];
        tmem_st16(a_tmem + 16u * j, part);
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(a_full(pa.idx));
        mbar_arrive(w_empty(pw.idx));
      }
      pw.next();
      pa.next();
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;
    pdl_wait();                             // outputs / workspace written only after the previous kernel
    Pipe pd{0, 2, 0};
    float acc[grouped<FMT>() ? NMMA : 1];
    int seg_kb0 = 0;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    bool ok = true;
    for (int i = 0; i < n_local && ok; ++i) {
      const UnitInfo ui = unit_info(u_lo + i, u_lo, u_hi, KB);
      const int mt = ui.tile / p.n_tiles, nt = ui.tile % p.n_tiles;
      if (ui.seg_start) {
        seg_kb0 = ui.kb;
        if constexpr (grouped<FMT>()) {
#pragma unroll
          for (int j = 0; j < NMMA; ++j) acc[j] = 0.f;
        }
      }
      const bool chunk_end = grouped<FMT>() ? true : ui.seg_end;
      if (!chunk_end) continue;
      if (!(ok = wait_bar(d_full(pd.idx), pd.phase, abort_flag, p.status))) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem + lane_base + Cfg::D_COL0 + pd.idx * Cfg::D_PITCH;
      const int prow = E::phys_row(p, nt, r);
      const bool full_tile = ui.seg_end && seg_kb0 == 0 && ui.kb == KB - 1;
      float* part_base = nullptr;
      if (ui.seg_end && !full_tile) {
        const long long first_tile = unit_lo(c, p.units, G) / KB;
        const int slot = (ui.tile == first_tile) ? 0 : 1;
        part_base = p.partials + (c * 2 + slot) * static_cast<long long>(NMMA) * 128;
      }
      if constexpr (grouped<FMT>()) {
        const int pr = prow < p.n ? prow : p.n - 1;
        float s;
        if constexpr (FMT == KL_W4_ASYM)
          s = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.scales)[static_cast<long long>(pr) * KB + ui.kb]);
        else
          s = reinterpret_cast<const float*>(p.scales)[static_cast<long long>(pr) * KB + ui.kb];
#pragma unroll
        for (int cb = 0; cb < NMMA / 16; ++cb) {
          uint32_t v[16];
          tmem_ld16(d_tmem + 16u * cb, v);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[cb * 16 + j] = fmaf(s, __uint_as_float(v[j]), acc[cb * 16 + j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty(pd.idx));
        pd.next();
        if (!ui.seg_end) continue;
        if (full_tile) {
#pragma unroll
          for (int cb = 0; cb < NMMA / 16; ++cb) {
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = acc[cb * 16 + j];
            E::emit16(p, mt, nt, r, cb, o, xch);
          }
          continue;
        }
#pragma unroll
        for (int cb = 0; cb < NMMA / 16; ++cb)
#pragma unroll
          for (int j = 0; j < 16; ++j) part_base[(cb * 16 + j) * 128 + r] = acc[cb * 16 + j];
      } else {
        const float s = E::row_scale(p, prow);
        for (int cb = 0; cb < NMMA / 16; ++cb) {
          uint32_t v[16];
          tmem_ld16(d_tmem + 16u * cb, v);
          tc_wait_ld();
          if (full_tile) {
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = __uint_as_float(v[j]) * s;
            E::emit16(p, mt, nt, r, cb, o, xch);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) part_base[(cb * 16 + j) * 128 + r] = __uint_as_float(v[j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty(pd.idx));
        pd.next();
        if (full_tile) continue;
      }
      // ---- split tile: publish the partial, the last contributor finishes it.
      const long long t_first_unit = static_cast<long long>(ui.tile) * KB;
      const long long c_first = unit_owner(t_first_unit, p.units, G);
      const long long c_last = unit_owner(t_first_unit + KB - 1, p.units, G);
      __threadfence();
      named_bar_epi();
      if (threadIdx.x == 6 * 32) {
        const int old = atomicAdd(p.counters + c_first, 1);
        const int last = (old == static_cast<int>(c_last - c_first));
        if (last) p.counters[c_first] = 0;   // ready for the next launch
        *fix_flag = last;
      }
      named_bar_epi();
      const bool last = *fix_flag != 0;
      named_bar_epi();                        // everyone read fix_flag before it is reused
      if (!last) continue;
      __threadfence();
      const float s = grouped<FMT>() ? 1.0f : E::row_scale(p, prow);
      for (int cb = 0; cb < NMMA / 16; ++cb) {
        float o[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = 0.f;
        for (long long cc = c_first; cc <= c_last; ++cc) {
          const long long ft = unit_lo(cc, p.units, G) / KB;
          const int sl = (ui.tile == ft) ? 0 : 1;
          const float* src = p.partials + (cc * 2 + sl) * static_cast<long long>(NMMA) * 128;
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] += __ldcg(src + (cb * 16 + j) * 128 + r);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] *= s;
        E::emit16(p, mt, nt, r, cb, o, xch);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

template <int FMT, int NMMA, bool SWIGLU, bool XBF16>
cudaError_t launch_one(const TcParams& p, const TcPlan& plan, bool pdl, cudaStream_t s) {
  auto kern = tc_qgemm_kernel<FMT, NMMA, SWIGLU, XBF16>;
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
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p, plan.stages);
}

template <int FMT, bool SWIGLU, bool XBF16>
cudaError_t launch_nmma(const TcParams& p, const TcPlan& plan, bool pdl, cudaStream_t s) {
  switch (plan.n_mma) {
    case 16: return launch_one<FMT, 16, SWIGLU, XBF16>(p, plan, pdl, s);
    case 32: return launch_one<FMT, 32, SWIGLU, XBF16>(p, plan, pdl, s);
    case 64: return launch_one<FMT, 64, SWIGLU, XBF16>(p, plan, pdl, s);
    default:
      if constexpr (grouped<FMT>()) return cudaErrorInvalidValue;   // group mode keeps <= 64 columns in registers
      else return launch_one<FMT, 128, SWIGLU, XBF16>(p, plan, pdl, s);
  }
}

template <bool SWIGLU, bool XBF16>
cudaError_t launch_fmt(const TcParams& p, const TcPlan& plan, int fmt, bool pdl, cudaStream_t s) {
  switch (fmt) {
    case KL_W8_ROW: return launch_nmma<KL_W8_ROW, SWIGLU, XBF16>(p, plan, pdl, s);
    case KL_W4_ASYM: return launch_nmma<KL_W4_ASYM, SWIGLU, XBF16>(p, plan, pdl, s);
    case KL_W4_SYM: return launch_nmma<KL_W4_SYM, SWIGLU, XBF16>(p, plan, pdl, s);
    default: return cudaErrorInvalidValue;
  }
}

int tc_stage_bytes(int fmt, int nmma) {
  return ((fmt == KL_W4_SYM || fmt == KL_W4_ASYM) ? 8192 : 16384) + 2 * nmma * 128;
}
int tc_fixed_bytes(int nmma) {
  const int a = nmma == 128 ? 4 : (nmma == 64 ? 2 : 3);
  return kXchBytes + 8 * (2 * a + 5) + 16 + 1024;
}

}  // namespace

TcPlan plan_tc(int m, int n, int k, int fmt, bool swiglu, int sm_count) {
  TcPlan t{};
  t.ok = false;
  const bool w4 = fmt == KL_W4_SYM || fmt == KL_W4_ASYM;
  if (!(fmt == KL_W8_ROW || w4)) return t;
  if (m <= 0 || n <= 0 || k <= 0) return t;
  if (swiglu && (n % 2)) return t;
  t.n_mma = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128;
  if (w4 && t.n_mma > 64) t.n_mma = 64;      // group mode: host splits M into 64-token launches
  const int n_out = swiglu ? n / 2 : n;
  t.m_tiles = (m + t.n_mma - 1) / t.n_mma;
  if (w4) t.m_tiles = 1;
  t.n_tiles = swiglu ? (n_out + 63) / 64 : (n + 127) / 128;
  t.kb_total = (k + kTcKBlock - 1) / kTcKBlock;
  t.units = static_cast<long long>(t.m_tiles) * t.n_tiles * t.kb_total;
  t.grid = static_cast<int>(std::min<long long>(t.units, sm_count));
  const int per_stage = tc_stage_bytes(fmt, t.n_mma);
  const int budget = (t.n_mma == 128 ? 200 : 104) * 1024 - tc_fixed_bytes(t.n_mma);
  t.stages = std::max(2, std::min(6, budget / per_stage));
  t.a_stages = t.n_mma == 128 ? 4 : (t.n_mma == 64 ? 2 : 3);
  t.smem = t.stages * per_stage + tc_fixed_bytes(t.n_mma) + 8 * 4 * t.stages;
  t.tmem_cols = t.n_mma == 128 ? 512 : 256;
  t.workspace = kCounterBytes + static_cast<size_t>(t.grid) * 2 * t.n_mma * 128 * sizeof(float);
  if (t.grid > kCounterBytes / 4) return t;
  t.ok = true;
  return t;
}

cudaError_t launch_tc(const TcParams& p, const TcPlan& plan, int fmt, bool swiglu, bool xbf16, bool pdl, cudaStream_t s) {
  if (swiglu) return xbf16 ? launch_fmt<true, true>(p, plan, fmt, pdl, s) : launch_fmt<true, false>(p, plan, fmt, pdl, s);
  return xbf16 ? launch_fmt<false, true>(p, plan, fmt, pdl, s) : launch_fmt<false, false>(p, plan, fmt, pdl, s);
}

}  // namespace kl
