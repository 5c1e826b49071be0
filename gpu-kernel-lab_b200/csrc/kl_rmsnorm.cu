// Qwen RMSNorm, optionally fused with the residual add in front of it.
//
//   c = T(x + r)                                   residual stream (stored when fused)
//   y = T( float(T(c * rsqrt(mean(c^2) + eps))) * float(w) )
//
// This is the operation order of the reference's learning/03_rmsnorm/qwen_rmsnorm.py:
// the residual kernel at :30-51, the plain kernel at :13-27, and the eager form
// at :54-63. The normalised value is rounded to the activation type BEFORE the
// weight multiply, as Qwen3RMSNorm does. The squares are summed in f32 and
// divided by n.
//
// It is HBM-bound. Each row moves n*|T| bytes per tensor: x, r and w are read;
// y and c are written.
//
// Vector path (n a multiple of 16 B / |T|, all pointers 16-byte aligned):
//   * WPR warps per row, each lane holding up to 8 chunks of 16 bytes of the
//     row in registers.
//   * Chunk index (k*WPR + warp_in_row)*32 + lane, so every warp instruction
//     moves 512 contiguous bytes.
//   * A warp-shuffle sum, plus a shared-memory combine when WPR > 1.
// Other shapes take a one-row-per-CTA strided path that reads the inputs twice.
#include "kl_common.cuh"
#include "kl_internal.h"

namespace kl {
namespace {

constexpr int kNormThreads = 256;
constexpr int kNormChunks = 8;          // most 16-byte chunks per lane (vector path)

template <typename T> KL_DEVICE float to_f(T v);
template <> KL_DEVICE float to_f<float>(float v) { return v; }
template <> KL_DEVICE float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> KL_DEVICE float to_f<__half>(__half v) { return __half2float(v); }
template <typename T> KL_DEVICE T from_f(float v);
template <> KL_DEVICE float from_f<float>(float v) { return v; }
template <> KL_DEVICE __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> KL_DEVICE __half from_f<__half>(float v) { return __float2half_rn(v); }
// round an f32 to T and back (the activation-type rounding of the model)
template <typename T> KL_DEVICE float rnd(float v) { return to_f<T>(from_f<T>(v)); }

KL_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

KL_DEVICE float inv_rms(float sumsq, int n, float eps, int precise) {
  const float var = sumsq / static_cast<float>(n) + eps;
  return precise ? 1.0f / sqrtf(var) : rsqrtf(var);
}

// CH = 16-byte chunks per lane: 4 for rows one warp covers with 4 (fewer
// registers, twice the resident warps), else kNormChunks.
template <typename T, bool RES, int CH>
__global__ void __launch_bounds__(kNormThreads, CH == 4 ? 4 : 2) rmsnorm_vec_kernel(const T* __restrict__ x, const T* __restrict__ r,
                                                                  const T* __restrict__ w, T* __restrict__ y,
                                                                  T* __restrict__ rout, int rows, int n, float eps,
                                                                  int precise, int wpr) {
  constexpr int E = 16 / static_cast<int>(sizeof(T));
  __shared__ float red[kNormThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_per_cta = (kNormThreads / 32) / wpr;
  const int row = blockIdx.x * rows_per_cta + warp / wpr;
  const int sub = warp % wpr;
  const bool active = row < rows && warp / wpr < rows_per_cta;
  const int chunks = n / E;
  const size_t base = static_cast<size_t>(row) * n;
  float c[CH * E];
  uint4 wq[CH];                    // weight chunks, loaded with the row (no second round trip)
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int ch = (k * wpr + sub) * 32 + lane;
    if (active && ch < chunks) {
      T xv[E];
      *reinterpret_cast<uint4*>(xv) = __ldcs(reinterpret_cast<const uint4*>(x + base) + ch);
      wq[k] = __ldg(reinterpret_cast<const uint4*>(w) + ch);
      if constexpr (RES) {
        T rv[E], ov[E];
        *reinterpret_cast<uint4*>(rv) = __ldcs(reinterpret_cast<const uint4*>(r + base) + ch);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          ov[e] = from_f<T>(to_f<T>(xv[e]) + to_f<T>(rv[e]));
          c[k * E + e] = to_f<T>(ov[e]);
        }
        __stcs(reinterpret_cast<uint4*>(rout + base) + ch, *reinterpret_cast<const uint4*>(ov));
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) c[k * E + e] = to_f<T>(xv[e]);
      }
#pragma unroll
      for (int e = 0; e < E; ++e) ss = fmaf(c[k * E + e], c[k * E + e], ss);
    }
  }
  ss = warp_sum(ss);
  if (wpr > 1) {                              // uniform over the CTA
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    ss = 0.0f;
    const int w0 = (warp / wpr) * wpr;
    for (int i = 0; i < wpr; ++i) ss += red[w0 + i];
  }
  if (!active) return;
  const float inv = inv_rms(ss, n, eps, precise);
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int ch = (k * wpr + sub) * 32 + lane;
    if (ch < chunks) {
      T wv[E], yv[E];
      *reinterpret_cast<uint4*>(wv) = wq[k];
#pragma unroll
      for (int e = 0; e < E; ++e) yv[e] = from_f<T>(rnd<T>(c[k * E + e] * inv) * to_f<T>(wv[e]));
      __stcs(reinterpret_cast<uint4*>(y + base) + ch, *reinterpret_cast<const uint4*>(yv));
    }
  }
}

// Any n and alignment: one row per CTA, element-strided, inputs read twice.
template <typename T, bool RES>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_any_kernel(const T* __restrict__ x, const T* __restrict__ r,
                                                                  const T* __restrict__ w, T* __restrict__ y,
                                                                  T* __restrict__ rout, int n, float eps, int precise) {
  __shared__ float red[kNormThreads / 32];
  const size_t base = static_cast<size_t>(blockIdx.x) * n;
  auto combined = [&](int i) {
    return RES ? rnd<T>(to_f<T>(x[base + i]) + to_f<T>(r[base + i])) : to_f<T>(x[base + i]);
  };
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += kNormThreads) {
    const float v = combined(i);
    if constexpr (RES) rout[base + i] = from_f<T>(v);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = 0.0f;
  for (int i = 0; i < kNormThreads / 32; ++i) ss += red[i];
  const float inv = inv_rms(ss, n, eps, precise);
  for (int i = threadIdx.x; i < n; i += kNormThreads)
    y[base + i] = from_f<T>(rnd<T>(combined(i) * inv) * to_f<T>(w[i]));
}

template <typename T, bool RES>
cudaError_t launch_norm_t(const void* x, const void* r, const void* w, void* y, void* rout, int rows, int n, float eps,
                          int precise, cudaStream_t s) {
  constexpr int E = 16 / static_cast<int>(sizeof(T));
  const bool vec = n % E == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                                   reinterpret_cast<uintptr_t>(y) | (RES ? reinterpret_cast<uintptr_t>(r) |
                                   reinterpret_cast<uintptr_t>(rout) : 0)) & 15u) == 0;
  const int per_warp = 32 * kNormChunks * E;
  int wpr = 1;
  while (wpr * per_warp < n) wpr *= 2;
  if (vec && wpr <= kNormThreads / 32) {
    const int rows_per_cta = (kNormThreads / 32) / wpr;
    const int grid = (rows + rows_per_cta - 1) / rows_per_cta;
    if (wpr == 1 && n <= 32 * 4 * E)
      rmsnorm_vec_kernel<T, RES, 4><<<grid, kNormThreads, 0, s>>>(
          static_cast<const T*>(x), static_cast<const T*>(r), static_cast<const T*>(w), static_cast<T*>(y),
          static_cast<T*>(rout), rows, n, eps, precise, wpr);
    else
      rmsnorm_vec_kernel<T, RES, kNormChunks><<<grid, kNormThreads, 0, s>>>(
          static_cast<const T*>(x), static_cast<const T*>(r), static_cast<const T*>(w), static_cast<T*>(y),
          static_cast<T*>(rout), rows, n, eps, precise, wpr);
  } else {
    rmsnorm_any_kernel<T, RES><<<rows, kNormThreads, 0, s>>>(
        static_cast<const T*>(x), static_cast<const T*>(r), static_cast<const T*>(w), static_cast<T*>(y),
        static_cast<T*>(rout), n, eps, precise);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_norm_d(const void* x, const void* r, const void* w, void* y, void* rout, int rows, int n, float eps,
                          int precise, cudaStream_t s) {
  return r ? launch_norm_t<T, true>(x, r, w, y, rout, rows, n, eps, precise, s)
           : launch_norm_t<T, false>(x, r, w, y, rout, rows, n, eps, precise, s);
}

}  // namespace

cudaError_t launch_rmsnorm(const void* x, const void* residual, const void* weight, int dtype, int rows, int n,
                           float eps, int precise, void* y, void* residual_out, cudaStream_t s) {
  switch (dtype) {
    case KL_DT_BF16: return launch_norm_d<__nv_bfloat16>(x, residual, weight, y, residual_out, rows, n, eps, precise, s);
    case KL_DT_F16: return launch_norm_d<__half>(x, residual, weight, y, residual_out, rows, n, eps, precise, s);
    default: return launch_norm_d<float>(x, residual, weight, y, residual_out, rows, n, eps, precise, s);
  }
}

}  // namespace kl
