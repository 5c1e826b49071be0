// Prefill (many-token) int8 row-scale linear on CTA pairs:
//   y[m, n] = s[n] * sum_k q[n, k] * x[m, k]      (optionally SwiGLU-fused)
//
// Each 2-CTA cluster computes a tile of 256 weight rows x 192 tokens with one
// tcgen05 MMA stream of shape M = 256 (128 weight rows per CTA) x N = 192
// (tokens; 96 in each CTA's shared memory) x K = 16:
//   * every CTA converts ITS 128 weight rows of a 64-wide K block from int8 to
//     bf16 (exact) into its own TMEM: the MMA's A operand;
//   * every CTA loads ITS 96 tokens of the block with TMA: half of the B
//     operand; both halves complete on the leader CTA's barrier;
//   * the leader issues the pair's MMAs; the f32 accumulators (2 buffers of
//     192 columns) live in each CTA's TMEM for its 128 rows;
//   * 4 epilogue warps per CTA apply the row scale (and SwiGLU), round to the
//     activation type and store.
// Per SM and 64-wide K step this moves 8 KB of weights and 12 KB of tokens
// into shared memory for 3.1 MFLOP, against 16 KB + 16 KB per 2.1 MFLOP for
// a single-CTA 128 x 128 tile: the pair halves both the shared-memory traffic
// and the conversion work per FLOP.  A pipeline stage is 128 wide in K (two
// such steps): the per-stage barrier round trips between converters, MMA and
// TMA are paid once per 6.3 MFLOP per SM.
//
// Warp roles (15 warps per CTA): 0 weight TMA, 1 token TMA, 2 TMEM owner and
// (leader) MMA issuer, 3-10 converters (two per TMEM lane quadrant, each one
// half of the K block), 11-14 epilogue.  Cross-CTA signalling uses mbarriers
// only; every wait is bounded (kWaitLimitNs) and records KL_ERR_TIMEOUT.
#include <cuda.h>

#include <algorithm>
#include <cstring>

#include "kl_common.cuh"
#include "kl_internal.h"

namespace kl {
namespace {

constexpr int kPfKb = 128;                       // K elements per stage
constexpr int kPfKAlign = 64;                    // K granularity the kernel takes (a last half stage is zero-filled)
constexpr int kPfXAtomK = 64;                    // K elements of one 128-byte token row (bf16)
constexpr int kPfRows = 128;                     // weight rows per CTA
constexpr int kPfMaxTokens = 192;                // tokens per tile (MMA N): 192, 128 or 64
constexpr int kPfW = 6;                          // weight stages (16 KB each)
constexpr int kPfX = 4;                          // token stages (two 64-wide atoms each)
constexpr int kPfAMax = 4;                       // TMEM A stages (at most)
constexpr int kPfWStage = kPfRows * kPfKb;       // 16 KB of int8
// token stage of one CTA: half the tile's tokens x 64 bf16 (12 KB at 192 tokens)
__host__ __device__ constexpr int pf_xatom(int tok) { return (tok / 2) * kPfXAtomK * 2; }
__host__ __device__ constexpr int pf_xstage(int tok) { return (kPfKb / kPfXAtomK) * pf_xatom(tok); }
constexpr int kPfACols = kPfKb / 2;              // TMEM columns per A stage
// A stages fill the TMEM the two accumulator buffers leave: 2 at 192-token
// tiles (the same K depth as 4 stages of 64), 4 at 128 or 64
__host__ __device__ constexpr int pf_a_stages(int tok) {
  return (512 - 2 * tok) / kPfACols < kPfAMax ? (512 - 2 * tok) / kPfACols : kPfAMax;
}
constexpr int kPfConv = 8;
constexpr int kPfEpi0 = 3 + kPfConv;
constexpr int kPfThreads = (kPfEpi0 + 4) * 32;   // 480
constexpr int kPfChunk = 32;                     // tokens per epilogue step
constexpr int kPfXchHalf = 64 * (kPfChunk / 2 + 1);  // one direction of the SwiGLU exchange (padded rows)
constexpr int kPfXchFloats = 2 * kPfXchHalf;
constexpr int kPfStageBytes = 32 * kPfChunk * 2; // per epilogue warp: 32 rows x 32 tokens, bf16
static_assert(pf_a_stages(kPfMaxTokens) >= 2 && pf_a_stages(kPfMaxTokens) * kPfACols + 2 * kPfMaxTokens <= 512,
              "TMEM budget");

struct PfLayout {
  uint32_t w, x, xch, stage, tcache, bars, misc, total;
};
constexpr PfLayout pf_layout(int tok) {
  PfLayout l{};
  l.w = 0;
  l.x = l.w + kPfW * kPfWStage;
  l.xch = l.x + kPfX * pf_xstage(tok);
  l.stage = l.xch + kPfXchFloats * 4;
  l.tcache = l.stage + 4 * kPfStageBytes;        // grouped launches: each problem's first tile
  l.bars = l.tcache + 4 * kMaxGroup;
  // w_full, w_empty [W]; x_full, x_empty [X]; a_full, a_empty [A]; d_full, d_empty [2]; done
  l.misc = l.bars + 8 * (2 * kPfW + 2 * kPfX + 2 * pf_a_stages(tok) + 5);
  l.total = l.misc + 16 + 1024;
  return l;
}

struct PfPipe {
  int idx, n;
  uint32_t phase;
  KL_DEVICE void next() {
    if (++idx == n) { idx = 0; phase ^= 1u; }
  }
};

// Bounded wait on a local barrier that remote CTAs may arrive on (acquire at
// cluster scope).  Returns false after the limit; records the timeout.
KL_DEVICE bool pf_wait(uint32_t bar, uint32_t parity, int* status) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((spin & 63u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
      record_error(status, KL_ERR_TIMEOUT);
      return false;
    }
  }
}
KL_DEVICE bool pf_wait_warp(uint32_t bar, uint32_t parity, int* status) {
  return __all_sync(0xFFFFFFFFu, pf_wait(bar, parity, status));
}

// Store one epilogue step of one warp: output columns col0 .. col0+31 (lane =
// column) for tokens m0 .. m0+31 (o[j] = token m0 + j).  A block that is fully
// in range in a row-major output (p.vec_store) goes through the warp's staging
// tile [token][column] and leaves as 16-byte stores, 64 contiguous bytes per
// token; ragged edges and the transposed layout are stored element by element.
template <bool XBF16, int T>
KL_DEVICE void pf_emit(const PfParams& p, uint8_t* stage, int col0, int ncols, int m0, int lane, const float (&o)[T]) {
  if (p.vec_store == 2 && col0 + lane < ncols && m0 + T <= p.m) {
    // transposed output: this column's T tokens are contiguous, 16-byte stores
    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.y) +
                                          ((static_cast<long long>(col0 + lane) * p.ldy + m0) << 1));
#pragma unroll
    for (int v4 = 0; v4 < T / 8; ++v4) {
      uint32_t pk[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        pk[j] = XBF16 ? pack_bf16x2(o[8 * v4 + 2 * j], o[8 * v4 + 2 * j + 1]) : pack_f16x2(o[8 * v4 + 2 * j], o[8 * v4 + 2 * j + 1]);
      dst[v4] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    return;
  }
  if (p.vec_store == 1 && col0 + 32 <= ncols && m0 + T <= p.m) {
    __syncwarp();                                    // previous step's reads of the tile are done
#pragma unroll
    for (int j = 0; j < T; ++j) store_act<XBF16>(stage, j * 32 + lane, o[j]);
    __syncwarp();
#pragma unroll
    for (int it = 0; it < T * 64 / 16 / 32; ++it) {
      const int v = it * 32 + lane, t = v >> 2, part = v & 3;
      const uint4 val = *reinterpret_cast<const uint4*>(stage + t * 64 + part * 16);
      *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.y) +
                                ((static_cast<long long>(m0 + t) * p.ldy + col0 + part * 8) << 1)) = val;
    }
    return;
  }
  const int col = col0 + lane;
  if (col >= ncols) return;
#pragma unroll
  for (int j = 0; j < T; ++j) {
    const int m = m0 + j;
    if (m < p.m)
      store_act<XBF16>(p.y, p.y_transposed ? static_cast<long long>(col) * p.ldy + m
                                           : static_cast<long long>(m) * p.ldy + col, o[j]);
  }
}

// Walks one role's tiles (increasing global tile index) through the problems
// of a launch: the problem of tile t is the last one whose first tile is <= t.
struct PfCursor {
  const PfLaunch* l;
  const int* tbegin;                   // shared-memory copy of the problems' tile_begin
  int prob;
  KL_DEVICE const PfParams& get() const { return l->count == 1 ? l->single : l->table[prob]; }
  KL_DEVICE void seek(int t) {
    while (prob + 1 < l->count && tbegin[prob + 1] <= t) ++prob;
  }
};

template <bool SWIGLU, bool XBF16, int TOK>
__global__ void __launch_bounds__(kPfThreads, 1) tc_prefill_kernel(const __grid_constant__ PfLaunch pl) {
  constexpr int kPfTokens = TOK;                 // tokens per tile (MMA N)
  constexpr int kPfHalf = TOK / 2;               // tokens per CTA
  constexpr int kPfXStage = pf_xstage(TOK);
  constexpr int kPfXAtom = pf_xatom(TOK);
  constexpr int kPfA = pf_a_stages(TOK);         // TMEM A stages
  constexpr int kPfDCol0 = kPfA * kPfACols;      // accumulators after the A stages
  static_assert(kPfXAtom % 1024 == 0, "token atoms stay 1024-byte aligned for the 128-byte swizzle");
  static_assert(TOK % kPfChunk == 0 && TOK <= kPfMaxTokens, "token tile");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr PfLayout L = pf_layout(TOK);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int tiles = pl.tiles;
  int* const status = pl.status;
  int my_tiles = 0;
  if (pair < tiles) my_tiles = (tiles - 1 - pair) / pairs + 1;
  int* tbegin = reinterpret_cast<int*>(smem + L.tcache);
  if (pl.count > 1)
    for (int i = threadIdx.x; i < pl.count; i += blockDim.x) tbegin[i] = pl.table[i].tile_begin;
  // (visible to every role after the cluster barrier below)

  const uint32_t s_w = smem_u32(smem + L.w), s_x = smem_u32(smem + L.x);
  const uint32_t bars = smem_u32(smem + L.bars);
  auto w_full = [&](int i) { return bars + 8u * i; };
  auto w_empty = [&](int i) { return bars + 8u * (kPfW + i); };
  auto x_full = [&](int i) { return bars + 8u * (2 * kPfW + i); };
  auto x_empty = [&](int i) { return bars + 8u * (2 * kPfW + kPfX + i); };
  auto a_full = [&](int i) { return bars + 8u * (2 * kPfW + 2 * kPfX + i); };
  auto a_empty = [&](int i) { return bars + 8u * (2 * kPfW + 2 * kPfX + kPfA + i); };
  auto d_full = [&](int i) { return bars + 8u * (2 * kPfW + 2 * kPfX + 2 * kPfA + i); };
  auto d_empty = [&](int i) { return bars + 8u * (2 * kPfW + 2 * kPfX + 2 * kPfA + 2 + i); };
  const uint32_t done_bar = bars + 8u * (2 * kPfW + 2 * kPfX + 2 * kPfA + 4);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L.misc);
  float* xch = reinterpret_cast<float*>(smem + L.xch);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPfW; ++i) { mbar_init(w_full(i), 1); mbar_init(w_empty(i), kPfConv); }
    for (int i = 0; i < kPfX; ++i) { mbar_init(x_full(i), 1); mbar_init(x_empty(i), 1); }
    for (int i = 0; i < kPfA; ++i) { mbar_init(a_full(i), 2 * kPfConv); mbar_init(a_empty(i), 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(d_full(i), 1); mbar_init(d_empty(i), 8); }
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc_pair(smem_u32(tmem_holder), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();                              // barrier inits and TMEM allocation visible to the pair
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------------------------------------------------- weight TMA
    if (lane == 0 && my_tiles > 0) {
      PfPipe pw{0, kPfW, 0};
      PfCursor cur{&pl, tbegin, 0};
      int last_prob = -1;
      for (int it = 0; it < my_tiles; ++it) {
        const int t = pair + it * pairs;
        cur.seek(t);
        const PfParams& p = cur.get();
        if (cur.prob != last_prob) { prefetch_tmap(&p.tmap_w); last_prob = cur.prob; }
        const int nt = (t - p.tile_begin) % p.n_tiles;
        const int kbs = p.kb_total;
        const int y0 = SWIGLU ? nt * 128 + static_cast<int>(rank) * 64 : nt * 256 + static_cast<int>(rank) * 128;
        const int y1 = SWIGLU ? p.n_out + y0 : y0 + 64;
        for (int kb = 0; kb < kbs; ++kb) {
          if (!pf_wait(w_empty(pw.idx), pw.phase ^ 1u, status)) { it = my_tiles; break; }
          const uint32_t dst = s_w + pw.idx * kPfWStage;
          mbar_arrive_expect_tx(w_full(pw.idx), kPfWStage);
          tma_load_2d(dst, &p.tmap_w, kb * kPfKb, y0, w_full(pw.idx));
          tma_load_2d(dst + kPfWStage / 2, &p.tmap_w, kb * kPfKb, y1, w_full(pw.idx));
          pw.next();
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- token TMA
    if (lane == 0 && my_tiles > 0) {
      pdl_wait();                              // tokens come from the previous kernel
      const uint32_t lead_full0 = mapa_shared(x_full(0), 0);
      PfPipe px{0, kPfX, 0};
      PfCursor cur{&pl, tbegin, 0};
      int last_prob = -1;
      for (int it = 0; it < my_tiles; ++it) {
        const int t = pair + it * pairs;
        cur.seek(t);
        const PfParams& p = cur.get();
        if (cur.prob != last_prob) { prefetch_tmap(&p.tmap_x); last_prob = cur.prob; }
        const int mt = (t - p.tile_begin) / p.n_tiles;
        const int kbs = p.kb_total;
        const int row = mt * kPfTokens + static_cast<int>(rank) * kPfHalf;
        for (int kb = 0; kb < kbs; ++kb) {
          if (!pf_wait(x_empty(px.idx), px.phase ^ 1u, status)) { it = my_tiles; break; }
          if (leader) mbar_arrive_expect_tx(x_full(px.idx), 2 * kPfXStage);
#pragma unroll
          for (int a = 0; a < kPfKb / kPfXAtomK; ++a)
            tma_load_2d_pair(s_x + px.idx * kPfXStage + a * kPfXAtom, &p.tmap_x, kb * kPfKb + a * kPfXAtomK, row,
                             lead_full0 + 8u * px.idx);
          px.next();
        }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------- MMA issuer (leader)
    if (leader) {
      constexpr uint32_t idesc = make_idesc_f16(256, kPfTokens, XBF16);
      const uint32_t x_desc0 = smem_desc_sw128_lo(s_x);
      PfPipe px{0, kPfX, 0}, pa{0, kPfA, 0}, pd{0, 2, 0};
      PfCursor cur{&pl, tbegin, 0};
      bool ok = true;
      for (int it = 0; it < my_tiles && ok; ++it) {
        cur.seek(pair + it * pairs);
        const int kbs = cur.get().kb_total;
        if (!(ok = pf_wait_warp(d_empty(pd.idx), pd.phase ^ 1u, status))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + kPfDCol0 + pd.idx * kPfTokens;
        for (int kb = 0; kb < kbs; ++kb) {
          if (!(ok = pf_wait_warp(x_full(px.idx), px.phase, status))) break;
          if (!(ok = pf_wait_warp(a_full(pa.idx), pa.phase, status))) break;
          tc_fence_after();
          const uint32_t a_tmem = tmem + pa.idx * kPfACols;
          const uint32_t xd = x_desc0 + static_cast<uint32_t>(px.idx * (kPfXStage >> 4));
          if (elect_one()) {
#pragma unroll
            for (int j = 0; j < kPfKb / 16; ++j)
              tc_mma_pair_ts(d_tmem, a_tmem + 8u * j,
                             xd + static_cast<uint32_t>(((j >> 2) * kPfXAtom + (j & 3) * 32) >> 4), idesc,
                             (kb == 0 && j == 0) ? 0u : 1u);
            tc_commit_pair_mc(x_empty(px.idx), 0x3);
            tc_commit_pair_mc(a_empty(pa.idx), 0x3);
            if (kb == kbs - 1) tc_commit_pair_mc(d_full(pd.idx), 0x3);
          }
          __syncwarp();
          px.next();
          pa.next();
        }
        pd.next();
      }
      if (elect_one()) tc_commit_pair_mc(done_bar, 0x3);
      __syncwarp();
    }
  } else if (warp < kPfEpi0) {
    // ----------------------------------------------------------- converters
    const int q = warp & 3;
    const int h = (warp - 3) >> 2;             // which 64-wide half of the K block
    const int r = q * 32 + lane;               // weight row of this CTA's 128
    const uint32_t lead_a_full0 = mapa_shared(a_full(0), 0);
    PfPipe pw{0, kPfW, 0}, pa{0, kPfA, 0};
    PfCursor cur{&pl, tbegin, 0};
    for (int it = 0; it < my_tiles; ++it) {
      bool ok = true;
      cur.seek(pair + it * pairs);
      const int kbs = cur.get().kb_total;
      for (int kb = 0; kb < kbs; ++kb) {
        if (!(ok = pf_wait(w_full(pw.idx), pw.phase, status))) break;
        if (!(ok = pf_wait(a_empty(pa.idx), pa.phase ^ 1u, status))) break;
        tc_fence_after();
        const uint8_t* ws = smem + L.w + pw.idx * kPfWStage;
        uint4 vv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int g = 4 * h + c;             // 16-byte chunk of the 128-byte row (128B swizzle)
          vv[c] = *reinterpret_cast<const uint4*>(ws + r * 128 + ((g ^ (r & 7)) << 4));
        }
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t part[16];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint4 v = vv[2 * c2 + c];
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
              if constexpr (XBF16) s8x4_to_bf16x4_fma(wd[t4], part[c * 8 + 2 * t4], part[c * 8 + 2 * t4 + 1]);
              else s8x4_to_f16x4(wd[t4], part[c * 8 + 2 * t4], part[c * 8 + 2 * t4 + 1]);
            }
          }
          tmem_st16(tmem + (static_cast<uint32_t>(q * 32) << 16) + pa.idx * kPfACols + 32u * h + 16u * c2, part);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_cluster(lead_a_full0 + 8u * pa.idx);
          mbar_arrive(w_empty(pw.idx));
        }
        pw.next();
        pa.next();
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;               // weight row of this CTA's 128
    const uint32_t lead_d_empty0 = mapa_shared(d_empty(0), 0);
    uint8_t* stg = smem + L.stage + (warp - kPfEpi0) * kPfStageBytes;
    pdl_wait();                                // y is written only after the previous kernel
    PfPipe pd{0, 2, 0};
    PfCursor cur{&pl, tbegin, 0};
    for (int it = 0; it < my_tiles; ++it) {
      const int t = pair + it * pairs;
      cur.seek(t);
      const PfParams& p = cur.get();
      const int lt = t - p.tile_begin;
      const int nt = lt % p.n_tiles, mt = lt / p.n_tiles;
      // the 4 epilogue warps take the same decision (they share named barriers)
      const bool got = pf_wait(d_full(pd.idx), pd.phase, status);
      uint32_t all_got;
      asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, 2, 128, q;\n selp.u32 %0, 1, 0, p;\n}"
                   : "=r"(all_got) : "r"(got ? 1u : 0u) : "memory");
      if (!all_got) break;
      tc_fence_after();
      // this warp's 32 output columns (gate rows for SwiGLU) and this thread's row
      const int col0 = SWIGLU ? nt * 128 + static_cast<int>(rank) * 64 + (q & 1) * 32
                              : nt * 256 + static_cast<int>(rank) * 128 + q * 32;
      const int ncols = SWIGLU ? p.n_out : p.n;
      const int col = col0 + lane;
      const int wrow = SWIGLU ? (r < 64 ? col : p.n_out + col) : col;
      const float s = col < ncols ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.scales)[wrow]) : 0.0f;
      const int m0 = mt * kPfTokens;
      const uint32_t d_tmem = tmem + (static_cast<uint32_t>(q * 32) << 16) + kPfDCol0 + pd.idx * kPfTokens;
#pragma unroll 1
      for (int c = 0; c < kPfTokens / kPfChunk; ++c) {
        uint32_t lo[16], hi[16];
        tmem_ld16(d_tmem + kPfChunk * c, lo);
        tmem_ld16(d_tmem + kPfChunk * c + 16u, hi);
        tc_wait_ld();
        if (c == kPfTokens / kPfChunk - 1) {
          // accumulator buffer fully read: release it to the leader's MMA
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(lead_d_empty0 + 8u * pd.idx);
        }
        float v[kPfChunk];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          v[j] = __uint_as_float(lo[j]) * s;
          v[16 + j] = __uint_as_float(hi[j]) * s;
        }
        if constexpr (SWIGLU) {
          // gate rows (r < 64) finish tokens 0..15 of the step, up rows (r >= 64)
          // tokens 16..31; each hands the other half to its partner row r ^ 64
          constexpr int H = kPfChunk / 2;
          const bool gate = r < 64;
          const int pr = r & 63;
          asm volatile("bar.sync 1, 128;" ::: "memory");        // previous step's reads done
#pragma unroll
          for (int j = 0; j < H; ++j) xch[(gate ? 0 : kPfXchHalf) + pr * (H + 1) + j] = gate ? v[H + j] : v[j];
          asm volatile("bar.sync 1, 128;" ::: "memory");
          float o[H];
#pragma unroll
          for (int j = 0; j < H; ++j) {
            const float other = xch[(gate ? kPfXchHalf : 0) + pr * (H + 1) + j];
            const float g_val = gate ? v[j] : other;
            const float u_val = gate ? other : v[H + j];
            o[j] = swiglu_model_ordered_fast<XBF16>(g_val, u_val);
          }
          pf_emit<XBF16, H>(p, stg, col0, ncols, m0 + c * kPfChunk + (gate ? 0 : H), lane, o);
        } else {
          pf_emit<XBF16, kPfChunk>(p, stg, col0, ncols, m0 + c * kPfChunk, lane, v);
        }
      }
      pd.next();
    }
  }

  // ---- teardown: every MMA of the pair has completed before TMEM is freed
  if (warp == 2) {
    if (my_tiles > 0 && !mbar_wait_time(done_bar, 0)) record_error(status, KL_ERR_TIMEOUT);
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (warp == 2) tmem_dealloc_pair(tmem, 512);
}

template <bool SWIGLU, bool XBF16, int TOK>
cudaError_t launch_pf(const PfLaunch& p, int grid, bool pdl, cudaStream_t s) {
  auto kern = tc_prefill_kernel<SWIGLU, XBF16, TOK>;
  constexpr int smem = static_cast<int>(pf_layout(TOK).total);
  static bool attr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < kMaxDevices && !attr[dev]) {
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
    attr[dev] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kPfThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  // no more pairs than can be resident at once (a GPC with an odd number of
  // SMs holds fewer 2-CTA clusters than SMs / 2)
  static int max_pairs[kMaxDevices] = {};
  if (dev >= 0 && dev < kMaxDevices) {
    if (max_pairs[dev] == 0) {
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = grid / 2;
      }
      max_pairs[dev] = n;
    }
    if (grid / 2 > max_pairs[dev]) cfg.gridDim = dim3(static_cast<unsigned>(2 * max_pairs[dev]));
  }
  // programmatic dependent launch: the set-up and the weight stream overlap the
  // previous kernel on the stream; token loads and output stores wait for it
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace

int prefill_threads() { return kPfThreads; }
int prefill_smem_bytes(int tok) { return static_cast<int>(pf_layout(tok).total); }
int prefill_k_block() { return kPfKAlign; }
int prefill_w_stages() { return kPfW; }

// Tokens per tile: the tile count of each choice is spread over the CTA pairs
// in waves; a tile costs about (tile tokens + 48) token-steps of MMA and
// epilogue, but never less than 192, because converting the tile's weights
// takes the same time per K block whatever the token count (measured: 128-token
// tiles ran at about the pace of 192-token ones).  The lowest waves x cost wins,
// the larger tile on ties.
int prefill_choose_tokens(int m, int n_tiles, int sm_count) {
  const int pairs = std::max(1, sm_count / 2);
  int best = kPfMaxTokens;
  long long best_cost = -1;
  for (int tok : {192, 128, 64}) {
    const long long tiles = static_cast<long long>(n_tiles) * ((m + tok - 1) / tok);
    const long long waves = (tiles + pairs - 1) / pairs;
    const long long cost = waves * std::max(tok + 48, 192);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = tok;
    }
  }
  return best;
}

void prefill_tiles(PfParams& p, bool swiglu, int sm_count) {
  p.n_tiles = swiglu ? (p.n_out + 127) / 128 : (p.n + 255) / 256;
  p.tok = prefill_choose_tokens(p.m, p.n_tiles, sm_count);
  p.m_tiles = (p.m + p.tok - 1) / p.tok;
  p.kb_total = (p.k + kPfKb - 1) / kPfKb;
}

int prefill_grid(const PfParams& p, int sm_count) {
  const int tiles = p.n_tiles * p.m_tiles;
  const int pairs = std::max(1, std::min(tiles, sm_count / 2));
  return 2 * pairs;
}

template <bool SWIGLU, bool XBF16>
cudaError_t launch_tok(const PfLaunch& l, int tok, int grid, bool pdl, cudaStream_t s) {
  switch (tok) {
    case 192: return launch_pf<SWIGLU, XBF16, 192>(l, grid, pdl, s);
    case 128: return launch_pf<SWIGLU, XBF16, 128>(l, grid, pdl, s);
    case 64: return launch_pf<SWIGLU, XBF16, 64>(l, grid, pdl, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_prefill_group(const PfLaunch& l, int grid, bool swiglu, bool xbf16, bool pdl, cudaStream_t s) {
  const int tok = l.single.tok;
  if (swiglu) return xbf16 ? launch_tok<true, true>(l, tok, grid, pdl, s) : launch_tok<true, false>(l, tok, grid, pdl, s);
  return xbf16 ? launch_tok<false, true>(l, tok, grid, pdl, s) : launch_tok<false, false>(l, tok, grid, pdl, s);
}

cudaError_t launch_prefill(const PfParams& p, int grid, bool swiglu, bool xbf16, bool pdl, cudaStream_t s) {
  PfLaunch l;
  std::memset(&l, 0, sizeof(l));
  l.single = p;
  l.single.tile_begin = 0;
  l.table = nullptr;
  l.count = 1;
  l.tiles = p.n_tiles * p.m_tiles;
  l.status = p.status;
  return launch_prefill_group(l, grid, swiglu, xbf16, pdl, s);
}

// Token tile for a group: every problem gets the same tile; the choice
// minimises (tile-K-blocks per pair, rounded up) x the per-K-block cost of a
// tile, max(tok + 48, 192) token-steps (see prefill_choose_tokens).
int prefill_group_tiles(PfParams* probs, int count, bool swiglu, int sm_count) {
  const int pairs = std::max(1, sm_count / 2);
  int best = kPfMaxTokens;
  long long best_cost = -1;
  for (int tok : {192, 128, 64}) {
    long long work = 0;                  // tile x K-block units
    for (int i = 0; i < count; ++i) {
      const int n_tiles = swiglu ? (probs[i].n_out + 127) / 128 : (probs[i].n + 255) / 256;
      work += static_cast<long long>(n_tiles) * ((probs[i].m + tok - 1) / tok) * ((probs[i].k + kPfKb - 1) / kPfKb);
    }
    const long long cost = ((work + pairs - 1) / pairs) * std::max(tok + 48, 192);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = tok;
    }
  }
  int tiles = 0;
  for (int i = 0; i < count; ++i) {
    PfParams& p = probs[i];
    p.n_tiles = swiglu ? (p.n_out + 127) / 128 : (p.n + 255) / 256;
    p.tok = best;
    p.m_tiles = (p.m + best - 1) / best;
    p.kb_total = (p.k + kPfKb - 1) / kPfKb;
    p.tile_begin = tiles;
    tiles += p.n_tiles * p.m_tiles;
  }
  return tiles;
}

}  // namespace kl
