// CUDA-core (SIMT) quantized GEMV for small M, every weight format.
//
// This is the B200 path for the reference's own weight formats (group-scaled
// int8 with an inverse channel vector, symmetric int4 with f32 group scales),
// for BF16 weights, and for shapes the tcgen05 kernel does not take (K not a
// multiple of 16, misaligned rows).  Math per output (reference
// learning/10_cuda_decode/warp_gemv.cu:14-54 and learning/09_int4/kernels.py:7-26):
//   y[m, n] = sum_k x[m, k] * w[n, k],  w dequantised exactly in f32,
// accumulated in f32; output rounded to the activation dtype; optional
// model-ordered SwiGLU over (gate row n, up row n + N/2).
//
// Design (B200): a warp owns ROWS output rows at a time and each lane streams
// one 16-byte chunk of every row per step with a non-allocating 128-bit load,
// so a warp step moves 512 B per row, fully coalesced.  The activations (x, or
// x * inverse for the calibrated format) are staged once per CTA in shared
// memory as f32, in a lane-interleaved layout that makes the per-lane 16-byte
// reads conflict-free.  Integer codes become f32 with the 2^23 magic-number
// trick (one PRMT/LOP3 + one FADD per element), group scales are applied once
// per 16-byte chunk, and the ROWS x MT partial sums are reduced across the warp
// with a transposing butterfly (V-1+5-log2 V shuffles instead of 5V).
#include "kl_common.cuh"
#include "kl_internal.h"

namespace kl {

namespace {

// 0x4B000000 + u  ==  8388608.0f + u  for 0 <= u < 2^23.
KL_DEVICE float magic_u8(uint32_t u_word, int j) {
  // byte j of u_word -> [u, 00, 00, 4B]
  return __uint_as_float(prmt(u_word, 0x4B000000u, 0x7540u + static_cast<uint32_t>(j))) - 8388736.0f;
}

template <int FMT> struct Fmt;
// CE: elements per 16-byte chunk of one weight row
template <> struct Fmt<KL_W8_ROW>     { static constexpr int CE = 16; static constexpr bool GROUPED = false; };
template <> struct Fmt<KL_W8_GROUP>   { static constexpr int CE = 16; static constexpr bool GROUPED = true; };
template <> struct Fmt<KL_W4_SYM>     { static constexpr int CE = 32; static constexpr bool GROUPED = true; };
template <> struct Fmt<KL_W4_ASYM>    { static constexpr int CE = 32; static constexpr bool GROUPED = true; };
template <> struct Fmt<KL_BF16_DENSE> { static constexpr int CE = 8;  static constexpr bool GROUPED = false; };

// Streaming 16-byte load that does not allocate in L1 (weights are read once).
KL_DEVICE uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Decode sub-chunk q (8 elements) of a 16-byte chunk into exact f32 values.
// `zbias` is 8388608 + z for the asymmetric 4-bit format.
template <int FMT>
KL_DEVICE void decode8(const uint4& c, int q, float zbias, float (&v)[8]) {
  const uint32_t wds[4] = {c.x, c.y, c.z, c.w};
  if constexpr (FMT == KL_W8_ROW || FMT == KL_W8_GROUP) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t u = wds[2 * q + i] ^ 0x80808080u;
#pragma unroll
      for (int j = 0; j < 4; ++j) v[4 * i + j] = magic_u8(u, j);
    }
  } else if constexpr (FMT == KL_W4_SYM || FMT == KL_W4_ASYM) {
    constexpr uint32_t kMagic = (FMT == KL_W4_SYM) ? 0x4B000008u : 0x4B000000u;
    const float sub = (FMT == KL_W4_SYM) ? 8388616.0f : zbias;
    const uint32_t w = wds[q];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t t = lop3<0x6A>(w >> (4 * j), 0xFu, kMagic);   // ((w >> 4j) & 15) ^ magic
      v[j] = __uint_as_float(t) - sub;
    }
  } else {  // bf16 dense: 8 elements = the whole chunk
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(wds[i] << 16);
      v[2 * i + 1] = __uint_as_float(wds[i] & 0xFFFF0000u);
    }
  }
}

// Shared-memory index of activation element k for the lane-interleaved layout.
template <int CE>
KL_DEVICE int xs_index(int k) {
  const int c = k / CE, e = k % CE;
  return (c >> 5) * (32 * CE) + (e >> 2) * 128 + (c & 31) * 4 + (e & 3);
}

template <int FMT, int MT, int ROWS, bool SWIGLU, bool XBF16>
__global__ void __launch_bounds__(256)
gemv_vec_kernel(const GemvArgs a) {
  constexpr int CE = Fmt<FMT>::CE;
  constexpr int PHYS = SWIGLU ? 2 * ROWS : ROWS;          // weight rows per warp step
  constexpr int V = PHYS * MT;                             // accumulators per lane
  static_assert(V == 4 || V == 8 || V == 16, "V must be a power of two <= 16");
  extern __shared__ float xs[];
  const int k = a.k;
  const int kpad = a.kpad;                                 // multiple of 32*CE
  const int m0 = blockIdx.y * MT;

  // Stage x (times inverse for the calibrated int8 format) as f32.
  for (int t = 0; t < MT; ++t) {
    const int m = m0 + t;
    for (int kk = threadIdx.x; kk < k; kk += blockDim.x) {
      float xv = (m < a.m) ? load_act<XBF16>(a.x, static_cast<long long>(m) * k + kk) : 0.f;
      if constexpr (FMT == KL_W8_GROUP) xv *= a.inverse[kk];
      xs[t * kpad + xs_index<CE>(kk)] = xv;
    }
  }
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  const int nchunks = k / CE;
  const int groups = Fmt<FMT>::GROUPED ? k / a.group : 1;
  const int chunks_per_group = Fmt<FMT>::GROUPED ? a.group / CE : nchunks;
  const long long row_bytes = static_cast<long long>(nchunks) * 16;
  const char* wbase = static_cast<const char*>(a.w);

  for (int rg = blockIdx.x * (blockDim.x >> 5) + warp; rg * ROWS < a.n_out; rg += warps_total) {
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
    long long prow[PHYS];
#pragma unroll
    for (int r = 0; r < PHYS; ++r) {
      const int lr = rg * ROWS + (SWIGLU ? (r % ROWS) : r);
      const int valid_lr = lr < a.n_out ? lr : a.n_out - 1;   // clamped rows are computed, never stored
      prow[r] = (SWIGLU && r >= ROWS) ? valid_lr + a.n_out : valid_lr;
    }
    for (int c = lane; c < nchunks; c += 32) {
      uint4 chunk[PHYS];
#pragma unroll
      for (int r = 0; r < PHYS; ++r) chunk[r] = ldg_stream(wbase + prow[r] * row_bytes + 16ll * c);
      float zb[PHYS], sc[PHYS];
      const int g = c / chunks_per_group;
#pragma unroll
      for (int r = 0; r < PHYS; ++r) {
        zb[r] = 0.f;
        sc[r] = 1.f;
        if constexpr (FMT == KL_W4_ASYM) {
          const long long si = prow[r] * groups + g;
          zb[r] = 8388608.0f + __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.zeros)[si]);
          sc[r] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.scales)[si]);
        } else if constexpr (FMT == KL_W8_GROUP || FMT == KL_W4_SYM) {
          sc[r] = reinterpret_cast<const float*>(a.scales)[prow[r] * groups + g];
        }
      }
      float part[V];
#pragma unroll
      for (int i = 0; i < V; ++i) part[i] = 0.f;
      const float* xc = xs + (c >> 5) * (32 * CE) + (c & 31) * 4;
#pragma unroll
      for (int q = 0; q < CE / 8; ++q) {
        float xv[MT][8];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const float4 f0 = *reinterpret_cast<const float4*>(xc + t * kpad + (2 * q) * 128);
          const float4 f1 = *reinterpret_cast<const float4*>(xc + t * kpad + (2 * q + 1) * 128);
          xv[t][0] = f0.x; xv[t][1] = f0.y; xv[t][2] = f0.z; xv[t][3] = f0.w;
          xv[t][4] = f1.x; xv[t][5] = f1.y; xv[t][6] = f1.z; xv[t][7] = f1.w;
        }
#pragma unroll
        for (int r = 0; r < PHYS; ++r) {
          float wv[8];
          decode8<FMT>(chunk[r], q, zb[r], wv);
#pragma unroll
          for (int t = 0; t < MT; ++t)
#pragma unroll
            for (int e = 0; e < 8; ++e) part[r * MT + t] = fmaf(wv[e], xv[t][e], part[r * MT + t]);
        }
      }
#pragma unroll
      for (int r = 0; r < PHYS; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          if constexpr (Fmt<FMT>::GROUPED) acc[r * MT + t] = fmaf(sc[r], part[r * MT + t], acc[r * MT + t]);
          else acc[r * MT + t] += part[r * MT + t];
        }
    }
    const float total = warp_reduce_multi<V>(acc);
    const int idx = value_index_of_lane<V>(lane);
    constexpr int lanes_per_value = 32 / V;
    if constexpr (!SWIGLU) {
      if ((lane % lanes_per_value) == 0) {
        const int r = idx / MT, t = idx % MT;
        const int lr = rg * ROWS + r;
        const int m = m0 + t;
        float out = total;
        if constexpr (FMT == KL_W8_ROW)
          out *= __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.scales)[prow[r]]);
        if (lr < a.n_out && m < a.m) {
          const long long yi = a.y_transposed ? static_cast<long long>(lr) * a.ldy + m
                                              : static_cast<long long>(m) * a.ldy + lr;
          store_act<XBF16>(a.y, yi, out);
        }
      }
    } else {
      // gate values sit at indices [0, V/2), up values at +V/2; the butterfly
      // decided the top index bit from lane bit 4, so the partner is lane ^ 16.
      const float partner = __shfl_xor_sync(0xffffffffu, total, 16);
      if (idx < V / 2 && (lane % lanes_per_value) == 0) {
        const int r = idx / MT, t = idx % MT;
        const int lr = rg * ROWS + r;
        const int m = m0 + t;
        float gate = total, up = partner;
        if constexpr (FMT == KL_W8_ROW) {
          gate *= __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.scales)[prow[r]]);
          up *= __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.scales)[prow[r + ROWS]]);
        }
        if (lr < a.n_out && m < a.m) {
          const long long yi = a.y_transposed ? static_cast<long long>(lr) * a.ldy + m
                                              : static_cast<long long>(m) * a.ldy + lr;
          store_act<XBF16>(a.y, yi, swiglu_model_ordered<XBF16>(gate, up));
        }
      }
    }
  }
}

// General scalar kernel: any K, any group dividing K, any format.  One warp per
// output row, lanes stride over K, every token handled in turn.
template <int FMT, bool SWIGLU, bool XBF16>
__global__ void __launch_bounds__(256)
gemv_scalar_kernel(const GemvArgs a) {
  const int lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  const int k = a.k;
  const int groups = (FMT == KL_W8_ROW || FMT == KL_BF16_DENSE) ? 1 : k / a.group;
  for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < a.n_out; row += warps_total) {
    for (int m = 0; m < a.m; ++m) {
      float acc[2] = {0.f, 0.f};
#pragma unroll
      for (int h = 0; h < (SWIGLU ? 2 : 1); ++h) {
        const long long wr = row + (h ? a.n_out : 0);
        for (int kk = lane; kk < k; kk += 32) {
          float xv = load_act<XBF16>(a.x, static_cast<long long>(m) * k + kk);
          float wv;
          if constexpr (FMT == KL_W8_ROW || FMT == KL_W8_GROUP) {
            wv = static_cast<float>(static_cast<const int8_t*>(a.w)[wr * k + kk]);
            if constexpr (FMT == KL_W8_GROUP) {
              wv *= reinterpret_cast<const float*>(a.scales)[wr * groups + kk / a.group];
              xv *= a.inverse[kk];
            }
          } else if constexpr (FMT == KL_W4_SYM || FMT == KL_W4_ASYM) {
            const uint8_t b = static_cast<const uint8_t*>(a.w)[wr * (k / 2) + kk / 2];
            const int code = (kk & 1) ? (b >> 4) : (b & 15);
            const long long si = wr * groups + kk / a.group;
            if constexpr (FMT == KL_W4_SYM) {
              wv = static_cast<float>(code >= 8 ? code - 16 : code) * reinterpret_cast<const float*>(a.scales)[si];
            } else {
              const float z = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.zeros)[si]);
              wv = (static_cast<float>(code) - z) * __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.scales)[si]);
            }
          } else {
            wv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.w)[wr * k + kk]);
          }
          acc[h] = fmaf(wv, xv, acc[h]);
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) acc[h] += __shfl_down_sync(0xffffffffu, acc[h], off);
        if constexpr (FMT == KL_W8_ROW)
          acc[h] *= __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.scales)[wr]);
      }
      if (lane == 0) {
        const float out = SWIGLU ? swiglu_model_ordered<XBF16>(acc[0], acc[1]) : acc[0];
        const long long yi = a.y_transposed ? static_cast<long long>(row) * a.ldy + m
                                            : static_cast<long long>(m) * a.ldy + row;
        store_act<XBF16>(a.y, yi, out);
      }
    }
  }
}

template <int FMT, int MT, int ROWS, bool SWIGLU, bool XBF16>
cudaError_t launch_vec(const GemvArgs& a, const GemvPlan& p, cudaStream_t s) {
  auto kern = gemv_vec_kernel<FMT, MT, ROWS, SWIGLU, XBF16>;
  if (p.smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem);
    if (e != cudaSuccess) return e;
  }
  kern<<<dim3(p.grid_x, p.grid_y), p.threads, p.smem, s>>>(a);
  return cudaGetLastError();
}

template <int FMT, bool SWIGLU, bool XBF16>
cudaError_t launch_fmt(const GemvArgs& a, const GemvPlan& p, cudaStream_t s) {
  if (!p.vec) {
    gemv_scalar_kernel<FMT, SWIGLU, XBF16><<<p.grid_x, p.threads, 0, s>>>(a);
    return cudaGetLastError();
  }
  constexpr int ROWS = SWIGLU ? 2 : 4;
  switch (p.mt) {
    case 1: return launch_vec<FMT, 1, ROWS, SWIGLU, XBF16>(a, p, s);
    case 2: return launch_vec<FMT, 2, ROWS, SWIGLU, XBF16>(a, p, s);
    default: return launch_vec<FMT, 4, ROWS, SWIGLU, XBF16>(a, p, s);
  }
}

template <bool SWIGLU, bool XBF16>
cudaError_t launch_sw(const GemvArgs& a, const GemvPlan& p, int fmt, cudaStream_t s) {
  switch (fmt) {
    case KL_W8_ROW: return launch_fmt<KL_W8_ROW, SWIGLU, XBF16>(a, p, s);
    case KL_W8_GROUP: return launch_fmt<KL_W8_GROUP, SWIGLU, XBF16>(a, p, s);
    case KL_W4_SYM: return launch_fmt<KL_W4_SYM, SWIGLU, XBF16>(a, p, s);
    case KL_W4_ASYM: return launch_fmt<KL_W4_ASYM, SWIGLU, XBF16>(a, p, s);
    default: return launch_fmt<KL_BF16_DENSE, SWIGLU, XBF16>(a, p, s);
  }
}

}  // namespace

int chunk_elems(int fmt) {
  switch (fmt) {
    case KL_W4_SYM: case KL_W4_ASYM: return 32;
    case KL_BF16_DENSE: return 8;
    default: return 16;
  }
}

GemvPlan plan_gemv(int m, int n_out, int k, int fmt, int group, bool swiglu, bool aligned, int sm_count) {
  GemvPlan p{};
  const int ce = chunk_elems(fmt);
  const bool grouped = fmt == KL_W8_GROUP || fmt == KL_W4_SYM || fmt == KL_W4_ASYM;
  p.vec = aligned && k % ce == 0 && (!grouped || (group % ce == 0));
  p.threads = 256;
  const int warps_per_cta = p.threads / 32;
  if (!p.vec) {
    p.mt = 1;
    p.grid_x = std::max(1, std::min((n_out + warps_per_cta - 1) / warps_per_cta, sm_count * 8));
    p.grid_y = 1;
    p.smem = 0;
    return p;
  }
  p.kpad = ((k + 32 * ce - 1) / (32 * ce)) * (32 * ce);
  const int max_smem = 200 * 1024;
  p.mt = m >= 4 ? 4 : (m >= 2 ? 2 : 1);
  while (p.mt > 1 && static_cast<long long>(p.mt) * p.kpad * 4 > max_smem) p.mt >>= 1;
  p.smem = p.mt * p.kpad * 4;
  if (p.smem > max_smem) { p.vec = false; return plan_gemv(m, n_out, k, fmt, group, swiglu, false, sm_count); }
  p.grid_y = (m + p.mt - 1) / p.mt;
  const int rows = swiglu ? 2 : 4;
  const int row_groups = (n_out + rows - 1) / rows;
  // enough CTAs to cover every SM a few times, but never more than row groups
  const int ctas_needed = (row_groups + warps_per_cta - 1) / warps_per_cta;
  const int per_sm = p.smem <= 48 * 1024 ? 4 : (p.smem <= 100 * 1024 ? 2 : 1);
  p.grid_x = std::max(1, std::min(ctas_needed, std::max(1, sm_count * per_sm / std::max(1, p.grid_y))));
  return p;
}

cudaError_t launch_gemv(const GemvArgs& a, const GemvPlan& p, int fmt, bool swiglu, bool xbf16, cudaStream_t s) {
  if (swiglu) return xbf16 ? launch_sw<true, true>(a, p, fmt, s) : launch_sw<true, false>(a, p, fmt, s);
  return xbf16 ? launch_sw<false, true>(a, p, fmt, s) : launch_sw<false, false>(a, p, fmt, s);
}

}  // namespace kl
