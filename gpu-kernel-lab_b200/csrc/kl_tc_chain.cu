// Latency-first tcgen05 GEMM for ONE decode-size int8 linear (M <= 64 tokens)
// that runs inside a dependent chain -- a model forward, where every linear
// waits for the op that produced its input (reference call pattern:
// profiling/decode_stage2_ablation.py:78-143 around the op of
// learning/10_cuda_decode/warp_gemv.cu:56-90).
//
//   y[m, n] = scale[n] * sum_k x[m, k] * q[n, k]      (f32 accumulate, bf16/f16 out)
//
// In a chain the time of a small linear is latency, not bandwidth: a 4 MB QKV
// streams in 0.65 us, but a persistent stream-K launch that starts, fetches,
// converts, multiplies and fixes up split tiles through global memory only
// after the previous kernel has finished costs several microseconds.  This
// kernel moves everything that does not depend on the input in front of the
// programmatic-dependent-launch wait and keeps what follows it short:
//
//   * Grid = tiles x K splits.  A thread-block cluster of `csize` CTAs owns one
//     128-row weight tile; CTA `rank` owns K blocks [rank*bpc, rank*bpc + bpc)
//     (128 elements each).  Nothing is persistent and nothing is shared
//     between tiles.
//   * Before the wait: the CTA's weight blocks (16 KB each) are copied by TMA
//     into shared memory and converted exactly to bf16/f16 into tensor memory
//     (the MMA's A operand).  TMEM use is 256 columns and shared memory under
//     100 KB, so a CTA of the next linear fits beside one of this linear on an
//     SM and fetches its weights while this one finishes.
//   * After the wait: one TMA copy of the activations, 4 MMAs per issuer warp
//     and K block (two issuers accumulate separately), one TMEM read, and a
//     reduce-scatter of the K-split partial sums through distributed shared
//     memory: each CTA owns a slice of the tile's rows.  The partials are
//     staged token-major per owning CTA in this CTA's (by then idle) weight
//     and activation buffers and sent with one bulk copy per peer, counted on
//     the owner's mbarrier; the owner sums them in CTA order (deterministic),
//     applies the row scales it loaded before the wait, and stores coalesced.
//   * TMEM is allocated before the dependents are triggered and released as
//     soon as the accumulators are read, so a blocked allocation can only wait
//     for a CTA that is already running (no cycle between chained kernels).
//
// Every mbarrier wait is bounded (kl_common.cuh); on expiry the kernel records
// KL_ERR_TIMEOUT, waits (bounded) for its own copies, frees TMEM and returns.
#include "kl_common.cuh"
#include "kl_internal.h"

#include <algorithm>
#include <atomic>
#include <mutex>

namespace kl {

namespace {

constexpr int kThreads = 256;                 // warps: 0 W-TMA, 1-2 MMA, 3 X-TMA, 4-7 convert + epilogue
constexpr int kTmemCols = 256;
constexpr int kKbl = 128;                     // K elements per block / A stage
constexpr int kWBlock = 128 * kKbl;           // bytes of one int8 weight block
constexpr int kChainMaxSmem = 227 * 1024;

__host__ __device__ constexpr int d_pitch(int nmma) { return nmma < 32 ? 32 : nmma; }
__host__ __device__ constexpr int a_stages(int nmma) { return (kTmemCols - 2 * d_pitch(nmma)) / 64; }

__host__ __device__ constexpr int pad4(int v) { return (v + 3) & ~3; }

struct Layout {
  uint32_t w, x, stage, recv, scale, bars, misc, total;
  int u_own_max, own_pad_max;
};
// Shared memory: weight blocks | activation atoms, reused after the MMAs as the
// staging area of the partial sums | receive area | row scales | barriers.
__host__ __device__ inline Layout layout(int nmma, int bpc, int csize, bool swiglu) {
  Layout l{};
  const int U = swiglu ? 64 : 128, H = swiglu ? 2 : 1;
  l.w = 0;
  l.x = static_cast<uint32_t>(bpc * kWBlock);                  // 1024-aligned
  const uint32_t wx_end = l.x + static_cast<uint32_t>(bpc * 2 * nmma * 128);
  l.u_own_max = (U + csize - 1) / csize;
  l.own_pad_max = pad4(l.u_own_max * H);
  // staging: every owner's block, token-major, rows padded to 16 bytes
  int stage_floats = 0;
  for (int j = 0; j < csize; ++j) {
    const int own = (((j + 1) * U + csize - 1) / csize) - ((j * U + csize - 1) / csize);
    stage_floats += pad4(own * H);
  }
  const uint32_t stage_end = static_cast<uint32_t>(stage_floats * nmma * 4);
  l.stage = 0;
  l.recv = ((wx_end > stage_end ? wx_end : stage_end) + 127u) & ~127u;
  l.scale = l.recv + static_cast<uint32_t>(csize * nmma * l.own_pad_max * 4);
  l.bars = (l.scale + static_cast<uint32_t>(l.own_pad_max * 4) + 15u) & ~15u;
  l.misc = l.bars + 8u * (kChainMaxBlocks + 12);
  l.total = l.misc + 16u + 1024u;                              // + slack to align the base to 1024 B
  return l;
}

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
KL_DEVICE bool wait_bar_warp(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  const bool ok = wait_bar(bar, parity, abort_flag, status);
  return __all_sync(0xFFFFFFFFu, ok);
}
// The receive barrier completes through other CTAs' st.async: acquire at cluster scope.
KL_DEVICE bool wait_bar_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
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

template <int NMMA, bool SWIGLU, bool XBF16>
__global__ void __launch_bounds__(kThreads, 2)
tc_chain_kernel(const __grid_constant__ ChainParams p) {
  constexpr int NI = 2;                                  // MMA issuer warps
  constexpr int DP = d_pitch(NMMA);
  constexpr int S = a_stages(NMMA);                      // A stages of 64 TMEM columns
  constexpr int D_COL0 = 64 * S;
  constexpr int X_ATOM = NMMA * 128;                     // NMMA rows x 64 elements, 128B swizzle
  constexpr int U = SWIGLU ? 64 : 128;                   // reduction units: rows, or gate/up row pairs
  constexpr int H = SWIGLU ? 2 : 1;
  static_assert(D_COL0 + NI * DP <= kTmemCols && S >= 2, "TMEM budget");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int C = p.csize, bpc = p.bpc;
  const Layout L = layout(NMMA, bpc, C, SWIGLU);
  const int rank = static_cast<int>(cluster_ctarank());
  const int nt = blockIdx.y;
  const int kb0 = rank * bpc;
  const int nb = min(bpc, p.kb_total - kb0);             // >= 1: the host sizes csize so
  const uint32_t s_base = smem_u32(smem);
  const uint32_t s_w = s_base + L.w, s_x = s_base + L.x, s_bars = s_base + L.bars;
  constexpr int WB = kChainMaxBlocks;
  auto w_full = [&](int i) { return s_bars + 8u * i; };
  const uint32_t x_full = s_bars + 8u * WB;
  auto a_full = [&](int i) { return s_bars + 8u * (WB + 1 + i); };
  auto a_empty = [&](int i) { return s_bars + 8u * (WB + 4 + i); };
  const uint32_t d_full = s_bars + 8u * (WB + 7), recv_bar = s_bars + 8u * (WB + 8),
                 done_bar = s_bars + 8u * (WB + 9), tmem_free = s_bars + 8u * (WB + 10);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L.misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.misc + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mv = p.m < NMMA ? p.m : NMMA;                // token columns that exist
  auto ubegin = [&](int j) { return (j * U + C - 1) / C; };   // first unit reduced by CTA j

  if (threadIdx.x == 0) {
    for (int i = 0; i < nb; ++i) mbar_init(w_full(i), 1);
    mbar_init(x_full, 1);
    for (int i = 0; i < S; ++i) {
      mbar_init(a_full(i), 4);
      mbar_init(a_empty(i), NI);
    }
    mbar_init(d_full, NI);
    mbar_init(recv_bar, 1);
    mbar_init(done_bar, NI);
    mbar_init(tmem_free, 4);
    *abort_flag = 0;
    fence_mbar_init();
    // Weights are static: stream them at once, before anything waits.
    prefetch_tmap(&p.tmap_w);
    const int y0 = SWIGLU ? nt * 64 : nt * 128;
    const int y1 = SWIGLU ? p.n_out + nt * 64 : nt * 128 + 64;
    for (int i = 0; i < nb; ++i) {
      const int kx = (kb0 + i) * kKbl;
      mbar_arrive_expect_tx(w_full(i), kWBlock);
      tma_load_2d(s_w + i * kWBlock, &p.tmap_w, kx, y0, w_full(i));
      tma_load_2d(s_w + i * kWBlock + kWBlock / 2, &p.tmap_w, kx, y1, w_full(i));
    }
    // bytes the other CTAs of the cluster will send for this CTA's units
    const int own = ubegin(rank + 1) - ubegin(rank);
    mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>((C - 1) * mv * pad4(own * H) * 4));
    prefetch_tmap(&p.tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  cluster_arrive();                     // phase 0: this CTA's barriers exist for the peers
  pdl_launch_dependents();              // after the TMEM allocation (see the header comment)

  if (warp == 0 || warp == 3) {
    if (warp == 3 && lane == 0) {
      // ---------------------------------------------------------- X producer
      pdl_wait();                       // activations come from the previous kernel
      mbar_arrive_expect_tx(x_full, static_cast<uint32_t>(nb * 2 * X_ATOM));
      for (int a = 0; a < 2 * nb; ++a)
        tma_load_2d(s_x + a * X_ATOM, &p.tmap_x, kb0 * kKbl + 64 * a, 0, x_full);
      mbar_wait_time(x_full, 0);        // no copy in flight at teardown
    }
    if (warp == 0 && lane == 0)
      for (int i = 0; i < nb; ++i) mbar_wait_time(w_full(i), 0);   // weight copies landed before teardown
    cluster_wait();
    cluster_arrive();
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuers
    const int w = warp - 1;
    constexpr uint32_t idesc = make_idesc_f16(128, NMMA, XBF16);
    const uint32_t d_tmem = tmem + static_cast<uint32_t>(D_COL0 + w * DP);
    bool ok = wait_bar_warp(x_full, 0, abort_flag, p.status);
    for (int i = 0; i < nb && ok; ++i) {
      const int st = i % S;
      if (!(ok = wait_bar_warp(a_full(st), static_cast<uint32_t>((i / S) & 1), abort_flag, p.status))) break;
      tc_fence_after();
      if (elect_one()) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = w * 4 + jj;                        // K step of 16 within the block
          const int e = i * kKbl + j * 16;                 // element offset in this CTA's K range
          const uint32_t b_lo = smem_desc_sw128_lo(s_x + static_cast<uint32_t>((e >> 6) * X_ATOM + (e & 63) * 2));
          tc_mma_ts_lo(d_tmem, tmem + static_cast<uint32_t>(st * 64 + j * 8), b_lo, idesc, (i | jj) ? 1u : 0u);
        }
        tc_commit(a_empty(st));
        if (i == nb - 1) tc_commit(d_full);
      }
      __syncwarp();
    }
    if (elect_one()) tc_commit(done_bar);
    __syncwarp();
    mbar_wait_time(done_bar, 0);        // no MMA reads or writes TMEM any more
    if (warp == 1) {
      // TMEM goes back as soon as the epilogue has read the accumulators
      mbar_wait_time(tmem_free, 0);
      tc_fence_after();
      tmem_dealloc(tmem, kTmemCols);
    }
    cluster_wait();
    cluster_arrive();
  } else {
    // ------------------------------------------------- converters, then epilogue
    const int q = warp - 4;             // TMEM lane quadrant
    const int r = q * 32 + lane;        // tile row of this thread
    bool ok = true;
    for (int i = 0; i < nb; ++i) {
      const int st = i % S;
      if (!(ok = wait_bar(w_full(i), 0, abort_flag, p.status))) break;
      if (!(ok = wait_bar(a_empty(st), static_cast<uint32_t>(((i / S) & 1) ^ 1), abort_flag, p.status))) break;
      const uint8_t* wb = smem + L.w + i * kWBlock;
      uint4 v[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) v[g] = *reinterpret_cast<const uint4*>(wb + r * 128 + ((g ^ (r & 7)) << 4));
      const uint32_t a_tmem = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(st * 64);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
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
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(a_full(st));
    }
    // ---- row scales of the units this CTA reduces: static, loaded before the accumulators
    const int u0 = ubegin(rank), own = ubegin(rank + 1) - u0;
    float* s_scale = reinterpret_cast<float*>(smem + L.scale);
    {
      const int t = threadIdx.x - 128;
      if (t < own * H) {
        const int lu = t / H, hh = t - lu * H;
        const int prow = SWIGLU ? (hh ? p.n_out : 0) + nt * 64 + u0 + lu : nt * 128 + u0 + lu;
        s_scale[t] = prow < p.n ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.scales)[prow]) : 0.f;
      }
    }
    // ---- exchange geometry, all before the accumulators are ready.  Unit u of
    // the tile is reduced by CTA (u * C) / U; the staging area holds one block
    // per owner, [token][unit * H + half], rows padded to 16 bytes.
    const int t = threadIdx.x - 128;
    const int u = SWIGLU ? (r & 63) : r;
    const int half = SWIGLU ? (r >> 6) : 0;
    const int owner = (u * C) / U;
    int blk = 0, bj = 0, bme = 0;       // floats per token before the owner's, peer t's and this CTA's block
    for (int i = 0; i < C; ++i) {
      const int pi = pad4((ubegin(i + 1) - ubegin(i)) * H);
      if (i < owner) blk += pi;
      if (i < t) bj += pi;
      if (i < rank) bme += pi;
    }
    const int opad = pad4((ubegin(owner + 1) - ubegin(owner)) * H);
    const int lu_row = u - ubegin(owner);
    const int padj = t < C ? pad4((ubegin(t + 1) - ubegin(t)) * H) : 0;
    const int mypad = pad4(own * H);
    // reduction work: unit l = t % own, tokens t / own, t / own + step, ...
    const int tstep = 128 / own;
    const int tl = t % own, tm0 = t / own;
    // the output parameters in registers now: a first read of the kernel
    // parameters at the end would wait on a constant-cache miss
    void* y_ptr = p.y;
    long long ldy = p.ldy;
    int n_out = p.n_out, y_tr = p.y_transposed;
    asm volatile("" : "+l"(y_ptr), "+l"(ldy), "+r"(n_out), "+r"(y_tr));
    cluster_wait();                     // phase 0: every peer's receive barrier is initialised
    // ---- the two issuers' accumulators of this row
    float acc[NMMA];
#pragma unroll
    for (int j = 0; j < NMMA; ++j) acc[j] = 0.f;
    const bool have = ok && wait_bar(d_full, 0, abort_flag, p.status);
    if (have) {
      tc_fence_after();
      const uint32_t d0 = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(D_COL0);
#pragma unroll
      for (int cb = 0; cb < NMMA / 16; ++cb) {
        uint32_t t0[16], t1[16];
        tmem_ld16(d0 + 16u * cb, t0);
        tmem_ld16(d0 + static_cast<uint32_t>(DP) + 16u * cb, t1);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[cb * 16 + j] = __uint_as_float(t0[j]) + __uint_as_float(t1[j]);
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(tmem_free);
    float* stage = reinterpret_cast<float*>(smem + L.stage);
    if (C == 1) {
      // ---- one CTA per tile: no partial sums to exchange; scale and store from
      // registers (the up rows of a SwiGLU tile hand their values to the gate
      // rows' threads through shared memory)
      if constexpr (SWIGLU) {
        if (have && r >= 64) {
#pragma unroll
          for (int m = 0; m < NMMA; ++m)
            if (m < mv) stage[m * 64 + (r - 64)] = acc[m];
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");   // scales (and up values) in place
      const int n = SWIGLU ? nt * 64 + r : nt * 128 + r;
      if (have && (!SWIGLU || r < 64) && n < n_out) {
        const float sc0 = s_scale[r * H], sc1 = SWIGLU ? s_scale[r * H + 1] : 0.f;
#pragma unroll
        for (int m = 0; m < NMMA; ++m) {
          if (m < mv) {
            const float out = SWIGLU ? swiglu_model_ordered<XBF16>(acc[m] * sc0, stage[m * 64 + r] * sc1) : acc[m] * sc0;
            const long long yi = y_tr ? static_cast<long long>(n) * ldy + m : static_cast<long long>(m) * ldy + n;
            store_act<XBF16>(y_ptr, yi, out);
          }
        }
      }
      cluster_arrive_relaxed();         // phase 1
    } else {
    // ---- stage this row's partials (the weights and activations are consumed:
    // the MMAs have completed) and send each peer its block in one bulk copy
    if (have) {
      float* dst = stage + blk * mv + lu_row * H + half;
#pragma unroll
      for (int m = 0; m < NMMA; ++m)
        if (m < mv) dst[m * opad] = acc[m];
    }
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, 128;" ::: "memory");   // every row of the tile is staged
    if (have && t < C && t != rank) {
      const uint32_t src = s_base + L.stage + static_cast<uint32_t>(bj * mv * 4);
      const uint32_t dst = mapa_shared(s_base + L.recv + static_cast<uint32_t>(rank * mv * padj * 4),
                                       static_cast<uint32_t>(t));
      bulk_copy_to_peer(dst, src, static_cast<uint32_t>(mv * padj * 4), mapa_shared(recv_bar, static_cast<uint32_t>(t)));
    }
    const bool got = have && wait_bar_cluster(recv_bar, 0, abort_flag, p.status);
    cluster_arrive_relaxed();           // phase 1: nothing more will be written into this CTA
    if (got && t < tstep * own) {
      // (the outputs follow the previous kernel: the MMAs consumed activations
      // copied after this grid's dependency wait returned)
      const float* mine = stage + bme * mv;
      const float* recv = reinterpret_cast<const float*>(smem + L.recv);
      const int n = SWIGLU ? nt * 64 + u0 + tl : nt * 128 + u0 + tl;
      const float sc0 = s_scale[tl * H], sc1 = SWIGLU ? s_scale[tl * H + 1] : 0.f;
      for (int m = tm0; m < mv; m += tstep) {
        float v0[kChainMaxCluster], v1[kChainMaxCluster];
#pragma unroll
        for (int src = 0; src < kChainMaxCluster; ++src) {
          // all peers' loads in flight, then the sum in CTA order
          const float* b = (src == rank ? mine : recv + src * mv * mypad) + m * mypad + tl * H;
          v0[src] = src < C ? b[0] : 0.f;
          v1[src] = (SWIGLU && src < C) ? b[1] : 0.f;
        }
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int src = 0; src < kChainMaxCluster; ++src) {
          s0 += v0[src];
          if constexpr (SWIGLU) s1 += v1[src];
        }
        if (n < n_out) {
          const float out = SWIGLU ? swiglu_model_ordered<XBF16>(s0 * sc0, s1 * sc1) : s0 * sc0;
          const long long yi = y_tr ? static_cast<long long>(n) * ldy + m : static_cast<long long>(m) * ldy + n;
          store_act<XBF16>(y_ptr, yi, out);
        }
      }
    }
    }
  }
  cluster_wait();                       // phase 1: no peer writes into this CTA's shared memory
}

template <int NMMA, bool SWIGLU, bool XBF16>
cudaError_t launch_one(const ChainParams& p, const ChainPlan& plan, bool pdl, cudaStream_t s) {
  auto kern = tc_chain_kernel<NMMA, SWIGLU, XBF16>;
  static std::atomic<int> configured[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (configured[dev].load(std::memory_order_acquire) == 0) {
    // the largest shared-memory request of any plan
    int max_smem = 0;
    for (int c = 1; c <= kChainMaxCluster; ++c)
      for (int b = 1; b <= kChainMaxBlocks; ++b) {
        const int sz = static_cast<int>(layout(NMMA, b, c, SWIGLU).total);
        if (sz <= kChainMaxSmem) max_smem = std::max(max_smem, sz);
      }
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)) != cudaSuccess) return e;
    configured[dev].store(1, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(plan.csize, plan.n_tiles, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = plan.csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  // Whether a cluster of this size and shared-memory footprint can be resident
  // at all on this device (checked once per configuration); if not, the caller
  // takes the persistent kernel instead.
  {
    static std::mutex mu;
    static int known[kMaxDevices][kChainMaxCluster + 1][2];   // {smem checked, fits}
    std::lock_guard<std::mutex> lock(mu);
    int* slot = known[dev][plan.csize];
    if (slot[0] != plan.smem) {
      cfg.numAttrs = 1;
      int clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
      if (e != cudaSuccess) return e;
      slot[0] = plan.smem;
      slot[1] = clusters > 0 ? 1 : 0;
      cfg.numAttrs = pdl ? 2 : 1;
    }
    if (!slot[1]) return cudaErrorNotSupported;
  }
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <bool SWIGLU, bool XBF16>
cudaError_t launch_nmma(const ChainParams& p, const ChainPlan& plan, bool pdl, cudaStream_t s) {
  switch (plan.n_mma) {
    case 16: return launch_one<16, SWIGLU, XBF16>(p, plan, pdl, s);
    case 32: return launch_one<32, SWIGLU, XBF16>(p, plan, pdl, s);
    case 64: return launch_one<64, SWIGLU, XBF16>(p, plan, pdl, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

ChainPlan plan_chain(int m, int n, int k, bool swiglu, int sm_count) {
  ChainPlan c{};
  c.ok = false;
  if (m < 1 || m > kChainMaxM || n < 1 || k < 1 || sm_count < 1) return c;
  if (swiglu && (n % 2)) return c;
  c.n_mma = m <= 16 ? 16 : m <= 32 ? 32 : 64;
  const int n_out = swiglu ? n / 2 : n;
  c.n_tiles = swiglu ? (n_out + 63) / 64 : (n + 127) / 128;
  const int kb = (k + kKbl - 1) / kKbl;
  // K blocks per CTA: the fewest from two up (one block per CTA costs more in
  // MMA issue and exchange than it saves) that keep the cluster portable
  // (<= 8 CTAs) and the grid within one CTA per SM -- two for 64-token tiles,
  // whose epilogue work grows with the tokens and is better spread -- else
  // within two CTAs per SM
  c.bpc = 0;
  const int cap0 = c.n_mma >= 64 ? 2 * sm_count : sm_count;
  for (int cap = cap0; cap <= 2 * sm_count && c.bpc == 0; cap += sm_count) {
    for (int bpc = 2; bpc <= 4; ++bpc) {
      const int cs = (kb + bpc - 1) / bpc;
      if (cs <= kChainMaxCluster && static_cast<long long>(c.n_tiles) * cs <= cap) {
        c.bpc = bpc;
        break;
      }
    }
  }
  if (c.bpc == 0) return c;
  c.bpc = kb < c.bpc ? kb : c.bpc;
  c.csize = (kb + c.bpc - 1) / c.bpc;
  c.smem = static_cast<int>(layout(c.n_mma, c.bpc, c.csize, swiglu).total);
  if (c.smem > kChainMaxSmem) return c;
  c.ok = true;
  return c;
}

cudaError_t launch_chain(const ChainParams& p, const ChainPlan& plan, bool swiglu, bool xbf16, bool pdl,
                         cudaStream_t s) {
  if (swiglu) return xbf16 ? launch_nmma<true, true>(p, plan, pdl, s) : launch_nmma<true, false>(p, plan, pdl, s);
  return xbf16 ? launch_nmma<false, true>(p, plan, pdl, s) : launch_nmma<false, false>(p, plan, pdl, s);
}

}  // namespace kl
