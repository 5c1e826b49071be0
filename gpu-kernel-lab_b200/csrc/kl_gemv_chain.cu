// CUDA-core decode linear for ONE or TWO tokens inside a dependent chain (a
// model forward: every linear waits for the op that produced its input; the
// call pattern of profiling/decode_stage2_ablation.py:78-143 around the op of
// learning/10_cuda_decode/warp_gemv.cu:56-90, whose per-row warp GEMV this
// replaces for the int8 row format, and of learning/09_int4/kernels.py:67-75
// for 4-bit weights).
//
//   int8 rows:  y[m, n] = scale[n] * sum_k x[m, k] * q[n, k]
//   4-bit:      y[m, n] = sum_g scale[n, g] * sum_{k in g} x[m, k] * (q[n, k] - zero[n, g])
//               (asymmetric: bf16 scale and zero per group; symmetric: f32
//               scale, two's-complement nibbles, i.e. zero 8 after q ^ 8)
//   f32 accumulate, bf16/f16 out.
//
// For one or two tokens the arithmetic is small (4 M multiply-adds for a 4 MB
// QKV, spread over the SMs) and the time of a dependent linear is latency.
// The tensor-core path pays, after the dependency wait, for the activation
// copy, the MMA issue, the TMEM read and a K-split exchange between CTAs; this
// kernel keeps only what must follow the wait:
//
//   * Each CTA owns `rows` output rows with all of K (gate and up rows of a
//     SwiGLU pair together), so nothing is exchanged between CTAs.
//   * Before the wait: one bulk copy of the CTA's weight rows (contiguous in
//     the [N, K] and [N, K/2] layouts) into shared memory; the row scales into
//     registers, or the group scales and zero points into shared memory.
//     The dependent kernel is triggered first, so the next linear's CTAs can
//     start and fetch their weights while this one waits and computes.
//   * After the wait: the activations (2 KB per token at K = 1024) are staged
//     in shared memory once; each warp takes its rows, each lane a strided
//     set of 16-element K chunks: exact integer -> f32 (the 2^23 magic number;
//     the zero point folds into the same packed subtract), packed f32x2
//     multiply-adds against the activations kept in registers across the
//     warp's rows (4-bit: one chunk lies in one group, whose scale multiplies
//     the chunk's sum), one transposing warp reduction, scale and store.
//
// Every wait is bounded; on expiry the kernel records KL_ERR_TIMEOUT and
// waits (bounded) for its own copy before returning.
#include "kl_common.cuh"
#include "kl_internal.h"

#include <algorithm>
#include <atomic>

namespace kl {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxRpw = 8;                       // output rows per warp (at most): 4, or 8 for wide problems

KL_DEVICE unsigned long long pack2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
KL_DEVICE float sum2(unsigned long long v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}
KL_DEVICE void ffma2(unsigned long long& acc, unsigned long long a, unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
KL_DEVICE unsigned long long fsub2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// 16 int8 weights -> 8 f32 pairs (elements 2e, 2e+1).  Byte j of
// (word ^ 0x80808080) placed under the exponent bits 0x4B00 is the f32 2^23 + u
// with u = q + 128; one packed subtract of 2^23 + 128 per pair leaves q exactly.
KL_DEVICE void w16_to_f32x2(const uint4& v, unsigned long long (&w)[8]) {
  const uint32_t wd[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
  const unsigned long long bias = pack2(8388736.0f, 8388736.0f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    unsigned long long a, b;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "r"(prmt(wd[i], 0x4B000000u, 0x7540u)), "r"(prmt(wd[i], 0x4B000000u, 0x7541u)));
    asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "r"(prmt(wd[i], 0x4B000000u, 0x7542u)), "r"(prmt(wd[i], 0x4B000000u, 0x7543u)));
    w[2 * i] = fsub2(a, bias);
    w[2 * i + 1] = fsub2(b, bias);
  }
}
// 16 nibbles (low nibble = even k) -> 8 f32 pairs (2^23 + c, c the code, with
// c ^ 8 for two's-complement codes), minus `bias` = (2^23 + zero) in both
// halves: exactly q - zero.
template <bool SYM>
KL_DEVICE void w4x16_to_f32x2(const uint2& v, unsigned long long bias, unsigned long long (&w)[8]) {
  constexpr uint32_t kFlip = SYM ? 0x08080808u : 0u;
  const uint32_t wd[2] = {v.x, v.y};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t lo = lop3<0x6A>(wd[i], 0x0F0F0F0Fu, kFlip);          // even-k codes, one per byte
    const uint32_t hi = lop3<0x6A>(wd[i] >> 4, 0x0F0F0F0Fu, kFlip);     // odd-k codes
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      unsigned long long a;
      asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "r"(prmt(lo, 0x4B000000u, 0x7540u + j)), "r"(prmt(hi, 0x4B000000u, 0x7540u + j)));
      w[4 * i + j] = fsub2(a, bias);
    }
  }
}
// 8 activations (one 16-byte chunk) -> 4 f32 pairs.
template <bool XBF16>
KL_DEVICE void x8_to_f32x2(const uint4& v, unsigned long long* out) {
  const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (XBF16) {
      out[i] = pack2(__uint_as_float(wd[i] << 16), __uint_as_float(wd[i] & 0xFFFF0000u));
    } else {
      const __half2 h = *reinterpret_cast<const __half2*>(&wd[i]);
      out[i] = pack2(__low2float(h), __high2float(h));
    }
  }
}

// s[i] for a runtime i < RPW without indexing the register array dynamically.
template <int RPW>
KL_DEVICE float sc_sel(const float (&s)[RPW], int i) {
  float r = s[0];
#pragma unroll
  for (int j = 1; j < RPW; ++j) r = i == j ? s[j] : r;
  return r;
}

// Shared memory: weight rows [H][R][rb], then (4-bit) group scales and zero
// points [H][R][G] as float pairs, then the activations [MT][K], then the
// weights' mbarrier.
struct GemvChainLayout {
  size_t groups, x, bar, total;
};
__host__ __device__ inline GemvChainLayout gemv_chain_layout(int h, int rows, int rb, int groups, int mt, int k) {
  GemvChainLayout l{};
  l.groups = static_cast<size_t>(h) * rows * rb;                            // rb is a multiple of 16
  l.x = l.groups + ((static_cast<size_t>(h) * rows * groups * 8 + 15) & ~static_cast<size_t>(15));
  l.bar = l.x + static_cast<size_t>(mt) * k * 2;
  l.total = l.bar + 16;
  return l;
}

KL_DEVICE bool wait_bounded(uint32_t bar, int* status) {
  if (mbar_try_wait(bar, 0)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, 0)) return true;
    if ((spin & 63u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
      record_error(status, KL_ERR_TIMEOUT);
      return false;
    }
  }
}

template <int FMT, int MT, int kRpw, bool SWIGLU, bool XBF16>
__global__ void __launch_bounds__(kThreads, 2) gemv_chain_kernel(const __grid_constant__ GemvChainParams p) {
  constexpr bool W4 = FMT != KL_W8_ROW;
  constexpr int H = SWIGLU ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  const int k = p.k, R = p.rows;
  const int rb = W4 ? k / 2 : k;                         // bytes of one weight row
  const int G = W4 ? k / p.group : 0;                    // groups per row (4-bit)
  const int r0 = blockIdx.x * R;
  const int nr = min(R, p.n_out - r0);                   // output rows of this CTA
  const GemvChainLayout L = gemv_chain_layout(H, R, rb, G, MT, k);
  uint8_t* wsm = smem;                                   // [H][R][rb] weight rows
  float2* gsm = reinterpret_cast<float2*>(smem + L.groups);   // [H][R][G] (scale, 2^23 + zero)
  uint8_t* xs = smem + L.x;                              // [MT][K] activations (bf16/f16)
  const uint32_t bar = smem_u32(smem + L.bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint8_t* wg = static_cast<const uint8_t*>(p.w);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    const uint32_t bytes = static_cast<uint32_t>(nr) * rb;
    mbar_arrive_expect_tx(bar, H * bytes);
    // weights are static: fetch them while the previous kernel runs
    bulk_copy_g2s(smem_u32(wsm), wg + static_cast<size_t>(r0) * rb, bytes, bar);
    if constexpr (SWIGLU)
      bulk_copy_g2s(smem_u32(wsm + static_cast<size_t>(R) * rb), wg + static_cast<size_t>(p.n_out + r0) * rb, bytes,
                    bar);
  }
  __syncthreads();                                       // barrier initialised before anyone waits on it
  pdl_launch_dependents();
  float sc[kRpw], scu[kRpw];
  if constexpr (W4) {
    // group scales and zero points of the CTA's rows (static data, read before the wait)
    const int per_h = nr * G;
    for (int e = threadIdx.x; e < H * per_h; e += kThreads) {
      const int h = e / per_h, rem = e - h * per_h, row = rem / G, g = rem - row * G;
      const long long gi = static_cast<long long>(h * p.n_out + r0 + row) * G + g;
      float sv, zv;
      if constexpr (FMT == KL_W4_ASYM) {
        sv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.scales)[gi]);
        zv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.zeros)[gi]);
      } else {
        sv = reinterpret_cast<const float*>(p.scales)[gi];
        zv = 8.0f;                                       // codes flipped by ^ 8 in the conversion
      }
      gsm[(h * R + row) * G + g] = make_float2(sv, 8388608.0f + zv);
    }
#pragma unroll
    for (int i = 0; i < kRpw; ++i) sc[i] = scu[i] = 1.0f;
  } else {
#pragma unroll
    for (int i = 0; i < kRpw; ++i) {
      const int row = warp + kWarps * i;
      const __nv_bfloat16* sp = reinterpret_cast<const __nv_bfloat16*>(p.scales);
      sc[i] = row < nr ? __bfloat162float(sp[r0 + row]) : 0.f;
      scu[i] = (SWIGLU && row < nr) ? __bfloat162float(sp[p.n_out + r0 + row]) : 0.f;
    }
  }
  void* y_ptr = p.y;
  long long ldy = p.ldy;
  int y_tr = p.y_transposed, m = p.m;
  asm volatile("" : "+l"(y_ptr), "+l"(ldy), "+r"(y_tr), "+r"(m));
  const int kc = k / 8;
  const char* xg = static_cast<const char*>(p.x);
  // Warm L2 with the activations' lines now: they are only read after the
  // dependency wait, but L2 is where global memory is coherent, so a line the
  // previous kernel rewrites in the meantime is read fresh all the same.
  for (int c = threadIdx.x * 8; c < kc; c += kThreads * 8)
    for (int t = 0; t < m; ++t)
      asm volatile("prefetch.global.L2 [%0];" :: "l"(xg + (static_cast<size_t>(t) * k + c * 8) * 2));

  pdl_wait();                                            // the activations come from the previous kernel
  // ---- stage the activations: every token row's 16-byte chunks, all loads in flight
  for (int c = threadIdx.x; c < kc; c += kThreads) {
    uint4 v[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t)
      v[t] = t < m ? __ldcg(reinterpret_cast<const uint4*>(xg + (static_cast<size_t>(t) * k + c * 8) * 2))
                   : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int t = 0; t < MT; ++t) *reinterpret_cast<uint4*>(xs + (static_cast<size_t>(t) * k + c * 8) * 2) = v[t];
  }
  __syncthreads();
  const bool ok = wait_bounded(bar, p.status);
  if (__syncthreads_and(ok) == 0) {
    if (threadIdx.x == 0) mbar_wait_time(bar, 0);       // the copy has landed before the CTA exits
    return;
  }

  // ---- per warp: rows warp, warp + 8, ...; per lane: K chunks lane, lane + 32, ...
  unsigned long long acc[kRpw][MT], accu[kRpw][MT];
#pragma unroll
  for (int i = 0; i < kRpw; ++i)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[i][t] = accu[i][t] = 0ull;
  for (int c = lane; c < k / 16; c += 32) {
    unsigned long long xv[MT][8];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const uint4* xp = reinterpret_cast<const uint4*>(xs + (static_cast<size_t>(t) * k + c * 16) * 2);
      x8_to_f32x2<XBF16>(xp[0], &xv[t][0]);
      x8_to_f32x2<XBF16>(xp[1], &xv[t][4]);
    }
    const int grp = W4 ? (c * 16) / p.group : 0;        // the chunk's group (4-bit)
#pragma unroll
    for (int i = 0; i < kRpw; ++i) {
      const int row = warp + kWarps * i;
      if (row < nr) {
#pragma unroll
        for (int h = 0; h < H; ++h) {
          unsigned long long w[8];
          unsigned long long(&a)[MT] = h ? accu[i] : acc[i];
          const uint8_t* wrow = wsm + (static_cast<size_t>(h) * R + row) * rb;
          if constexpr (W4) {
            const float2 sz = gsm[(h * R + row) * G + grp];
            w4x16_to_f32x2<FMT == KL_W4_SYM>(*reinterpret_cast<const uint2*>(wrow + c * 8), pack2(sz.y, sz.y), w);
            const unsigned long long s2 = pack2(sz.x, sz.x);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              unsigned long long d = 0ull;               // the chunk's sum, then scaled by its group's scale
#pragma unroll
              for (int e = 0; e < 8; ++e) ffma2(d, w[e], xv[t][e]);
              ffma2(a[t], d, s2);
            }
          } else {
            w16_to_f32x2(*reinterpret_cast<const uint4*>(wrow + c * 16), w);
#pragma unroll
            for (int t = 0; t < MT; ++t)
#pragma unroll
              for (int e = 0; e < 8; ++e) ffma2(a[t], w[e], xv[t][e]);
          }
        }
      }
    }
  }
  // ---- reduce all of the warp's sums at once (transposing butterfly), scale, store
  constexpr int V = kRpw * MT * H;                       // value (i, t, h) at index (i * MT + t) * H + h
  float v[V];
#pragma unroll
  for (int i = 0; i < kRpw; ++i)
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      v[(i * MT + t) * H] = sum2(acc[i][t]);
      if constexpr (SWIGLU) v[(i * MT + t) * H + 1] = sum2(accu[i][t]);
    }
  const float total = warp_reduce_multi<V>(v);
  const int idx = value_index_of_lane<V>(lane);          // the value this lane now holds in full
  constexpr int kLanesPerValue = 32 / V;
  // the lowest index bit (h) comes from lane bit 5 - log2(V): the up sum of a
  // SwiGLU pair sits on the lane that differs in that bit
  constexpr int kHBit = kLanesPerValue;
  const float up = SWIGLU ? __shfl_xor_sync(0xFFFFFFFFu, total, kHBit) : 0.f;
  const int i = idx / (MT * H), t = (idx / H) % MT, h = idx % H;
  const int row = warp + kWarps * i;
  if (lane % kLanesPerValue == 0 && h == 0 && row < nr && t < m) {
    const float g = total * sc_sel(sc, i);
    const float out = SWIGLU ? swiglu_model_ordered<XBF16>(g, up * sc_sel(scu, i)) : g;
    const int n = r0 + row;
    const long long yi = y_tr ? static_cast<long long>(n) * ldy + t : static_cast<long long>(t) * ldy + n;
    store_act<XBF16>(y_ptr, yi, out);
  }
}

template <int FMT, int MT, int RPW, bool SWIGLU, bool XBF16>
cudaError_t launch_one(const GemvChainParams& p, const GemvChainPlan& plan, bool pdl, cudaStream_t s) {
  auto kern = gemv_chain_kernel<FMT, MT, RPW, SWIGLU, XBF16>;
  static std::atomic<int> configured[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (configured[dev].load(std::memory_order_acquire) == 0) {
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvChainMaxSmem)) != cudaSuccess)
      return e;
    configured[dev].store(1, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int FMT, bool SWIGLU, bool XBF16>
cudaError_t launch_mt(const GemvChainParams& p, const GemvChainPlan& plan, bool pdl, cudaStream_t s) {
  if (plan.rpw == 4)
    return plan.mt == 1 ? launch_one<FMT, 1, 4, SWIGLU, XBF16>(p, plan, pdl, s)
                        : launch_one<FMT, 2, 4, SWIGLU, XBF16>(p, plan, pdl, s);
  if (plan.mt == 1) return launch_one<FMT, 1, 8, SWIGLU, XBF16>(p, plan, pdl, s);
  if constexpr (!SWIGLU) return launch_one<FMT, 2, 8, SWIGLU, XBF16>(p, plan, pdl, s);
  return cudaErrorInvalidConfiguration;                  // not planned: it would spill registers
}

template <int FMT>
cudaError_t launch_fmt(const GemvChainParams& p, const GemvChainPlan& plan, bool swiglu, bool xbf16, bool pdl,
                       cudaStream_t s) {
  if (swiglu) return xbf16 ? launch_mt<FMT, true, true>(p, plan, pdl, s) : launch_mt<FMT, true, false>(p, plan, pdl, s);
  return xbf16 ? launch_mt<FMT, false, true>(p, plan, pdl, s) : launch_mt<FMT, false, false>(p, plan, pdl, s);
}

}  // namespace

GemvChainPlan plan_gemv_chain(int m, int n, int k, int w_format, int group, bool swiglu, int sm_count) {
  GemvChainPlan c{};
  c.ok = false;
  const bool w4 = w_format == KL_W4_ASYM || w_format == KL_W4_SYM;
  if (!(w_format == KL_W8_ROW || w4)) return c;
  if (m < 1 || m > kGemvChainMaxM || n < 1 || k < 16 || k % 16 || sm_count < 1) return c;
  // 4-bit: a 16-element chunk lies in one group; rows of K/2 bytes are whole 16-byte units
  if (w4 && (group < 16 || group % 16 || k % group || k % 32)) return c;
  if (swiglu && (n % 2)) return c;
  const int n_out = swiglu ? n / 2 : n;
  const int h = swiglu ? 2 : 1;
  c.mt = m <= 1 ? 1 : 2;
  // about one CTA per SM, at most 4 (else 8) rows per warp
  c.rows = (n_out + sm_count - 1) / sm_count;
  if (c.rows > kWarps * kMaxRpw) return c;              // large heads stream through the tcgen05 kernel
  c.rpw = c.rows <= kWarps * 4 ? 4 : 8;
  if (c.rpw == 8 && swiglu && c.mt == 2) return c;      // 32 sums per lane: more registers than a lane has
  c.grid = (n_out + c.rows - 1) / c.rows;
  const GemvChainLayout L = gemv_chain_layout(h, c.rows, w4 ? k / 2 : k, w4 ? k / group : 0, c.mt, k);
  // at least kGemvChainMinSmem, so that at most two CTAs share an SM: the next
  // linear's CTAs sit beside this one's, and the one after waits for them
  c.smem = std::max<int>(static_cast<int>(L.total), kGemvChainMinSmem);
  if (L.total > static_cast<size_t>(kGemvChainMaxSmem)) return c;
  c.ok = true;
  return c;
}

cudaError_t launch_gemv_chain(const GemvChainParams& p, const GemvChainPlan& plan, int w_format, bool swiglu,
                              bool xbf16, bool pdl, cudaStream_t s) {
  switch (w_format) {
    case KL_W8_ROW: return launch_fmt<KL_W8_ROW>(p, plan, swiglu, xbf16, pdl, s);
    case KL_W4_ASYM: return launch_fmt<KL_W4_ASYM>(p, plan, swiglu, xbf16, pdl, s);
    case KL_W4_SYM: return launch_fmt<KL_W4_SYM>(p, plan, swiglu, xbf16, pdl, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace kl
