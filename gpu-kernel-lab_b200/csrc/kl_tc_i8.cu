// Int8 tensor-core mode of the persistent weight-only GEMM for int8 row-scale
// weights (KL_W8_ROW) and asymmetric 4-bit group-128 weights (KL_W4_ASYM),
// used by grouped decode launches.
//
// The bf16 path converts every weight to bf16 on the CUDA cores before the
// MMA; at decode sizes that conversion, not HBM, sets the pace, and under the
// power cap (SM clock 1.5 GHz instead of 1.97) it falls further behind.  Here
// the weights are never touched by a CUDA core: the TMA-filled int8 stage is
// the A operand of tcgen05.mma.kind::i8, and the activations are brought to
// integers instead, once per call, by a small digits pass:
//
//   per token t:  a_t = max_k |x[t, k]|,  e_t = floor(log2 a_t),  s_t = 2^(e_t - 21)
//                 x[t, k] / s_t rounded to the nearest integer = 65536 h + 256 m + l,
//                 h in [-64, 64], m and l in [-128, 127]          (three int8 planes)
//
//   y[t, n] = scale[n] * s_t * (65536 H + 256 M + L),  H = sum_k q[n, k] h[t, k], ...
//
// One MMA of N = i8_tile_rows(T) (the h plane's T rows, the m plane's, the l
// plane's, zero padding) gives the three int32 sums; they are exact, so the
// only roundings are the digits of the very smallest activations and two f32
// adds.  Accuracy: x / s_t has 22 integer bits, so every activation within a
// factor 2^14 of the token's largest (bf16 carries 8 significant bits) is
// represented exactly, and any other is off by at most s_t / 2 <= a_t * 2^-22
// -- the size of f32 accumulation noise.  Two digit planes (a factor 2^6)
// measured here flipped SwiGLU outputs (two bf16 roundings in a row) by two
// ulps at M = 64; three do not.  A token whose largest |x| is infinite or NaN
// gets s_t = NaN (its outputs are NaN), an all-zero token s_t = 0.
//
// Work per token row of K elements: 2K bytes read, 3K bytes of digits and a
// scale written; the GEMM then streams the int8 weights exactly as the bf16
// mode does (same stream-K partition, tiles, epilogues).
#include "kl_tc_gemm.cuh"

namespace kl {

namespace {

constexpr int kDigitThreads = 256;
constexpr int kDigitChunks = 4;            // 16-byte chunks per thread held in registers (K <= 8192)

// One CTA per (problem, token row): blockIdx.y = problem, blockIdx.x = token.
// The row is read once into registers (all loads in flight together), its
// largest |x| reduced over the CTA, and the three digit planes written from
// the registers.  Rows longer than kDigitThreads * kDigitChunks * 8 elements
// take a second, strided pass over global memory.
__global__ void __launch_bounds__(kDigitThreads) act_digits_kernel(const TcProblem* __restrict__ tab,
                                                                   const __grid_constant__ TcProblem single) {
  __shared__ uint32_t red[kDigitThreads / 32];
  const TcProblem& pr = tab ? tab[blockIdx.y] : single;
  const int t = blockIdx.x;
  const int T = pr.tok;
  // the previous kernel on the stream may still read the digits (the GEMM of
  // the previous call) or write x: wait for it before touching either
  pdl_wait();
  pdl_launch_dependents();
  if (t >= pr.m_tiles * T) return;
  const int k = pr.k;
  const long long ld = pr.digits_ld;
  const int R = i8_tile_rows(T);
  int8_t* tile = pr.digits + static_cast<long long>(t / T) * R * ld;
  int8_t* hrow = tile + static_cast<long long>(t % T) * ld;
  int8_t* mrow = hrow + static_cast<long long>(T) * ld;
  int8_t* lrow = mrow + static_cast<long long>(T) * ld;
  const int kc = k / 8;                                  // 16-byte chunks of the bf16 row (K % 16 == 0)
  // the tile's padding rows (3T .. R-1: only T = 8 has them) are zeroed by the
  // CTAs of the tile's first tokens
  if (3 * T + (t % T) < R) {
    int8_t* prow = tile + static_cast<long long>(3 * T + (t % T)) * ld;
    for (int c = threadIdx.x; c < kc; c += kDigitThreads) *reinterpret_cast<uint2*>(prow + c * 8) = make_uint2(0u, 0u);
  }
  if (t >= pr.m) {                                       // padding token of the last tile: zero digits
    for (int c = threadIdx.x; c < kc; c += kDigitThreads) {
      *reinterpret_cast<uint2*>(hrow + c * 8) = make_uint2(0u, 0u);
      *reinterpret_cast<uint2*>(mrow + c * 8) = make_uint2(0u, 0u);
      *reinterpret_cast<uint2*>(lrow + c * 8) = make_uint2(0u, 0u);
    }
    if (threadIdx.x == 0) pr.tscale[t] = 0.0f;
    return;
  }
  const uint4* xr = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(pr.x_src) + static_cast<long long>(t) * k);
  // the largest |x| as f32 bits (bf16 -> f32 is a shift, ordering kept)
  auto absmax8 = [](const uint4& v, uint32_t a) {
    const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) a = max(max(a, (wd[i] << 16) & 0x7FFFFFFFu), wd[i] & 0x7FFF0000u);
    return a;
  };
  uint4 v[kDigitChunks];
  uint32_t amax = 0u;
#pragma unroll
  for (int j = 0; j < kDigitChunks; ++j) {
    const int c = threadIdx.x + j * kDigitThreads;
    v[j] = c < kc ? __ldcg(xr + c) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int j = 0; j < kDigitChunks; ++j) amax = absmax8(v[j], amax);
  for (int c = threadIdx.x + kDigitChunks * kDigitThreads; c < kc; c += kDigitThreads) amax = absmax8(__ldcg(xr + c), amax);
  amax = __reduce_max_sync(0xFFFFFFFFu, amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kDigitThreads / 32; ++w) amax = max(amax, red[w]);
  float mul, ts;
  if (amax >= 0x7F800000u) {                             // inf or NaN: no finite scale
    mul = 0.0f;
    ts = __uint_as_float(0x7FC00000u);
  } else if (amax == 0u) {
    mul = 0.0f;
    ts = 0.0f;
  } else {
    const int e = max(static_cast<int>(amax >> 23) - 127, -100);   // floor(log2 a); subnormals clamp
    mul = __uint_as_float(static_cast<uint32_t>(127 + 21 - e) << 23);   // 2^(21 - e)
    ts = __uint_as_float(static_cast<uint32_t>(127 + e - 21) << 23);    // 2^(e - 21)
  }
  auto digits8 = [&](const uint4& x8, int c) {
    const uint32_t wd[4] = {x8.x, x8.y, x8.z, x8.w};
    uint32_t hw[2] = {0u, 0u}, mw[2] = {0u, 0u}, lw[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t bits = (i & 1) ? (wd[i >> 1] & 0xFFFF0000u) : (wd[i >> 1] << 16);
      const int xi = __float2int_rn(__uint_as_float(bits) * mul);   // |xi| <= 2^22, exact products
      const int r1 = (xi + 128) >> 8;                    // xi = 256 r1 + l, l in [-128, 127]
      const int l = xi - (r1 << 8);
      const int h = (r1 + 128) >> 8;                     // r1 = 256 h + m, |h| <= 64
      const int mm = r1 - (h << 8);
      hw[i >> 2] |= (static_cast<uint32_t>(h) & 0xFFu) << (8 * (i & 3));
      mw[i >> 2] |= (static_cast<uint32_t>(mm) & 0xFFu) << (8 * (i & 3));
      lw[i >> 2] |= (static_cast<uint32_t>(l) & 0xFFu) << (8 * (i & 3));
    }
    *reinterpret_cast<uint2*>(hrow + c * 8) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(mrow + c * 8) = make_uint2(mw[0], mw[1]);
    *reinterpret_cast<uint2*>(lrow + c * 8) = make_uint2(lw[0], lw[1]);
  };
#pragma unroll
  for (int j = 0; j < kDigitChunks; ++j) {
    const int c = threadIdx.x + j * kDigitThreads;
    if (c < kc) digits8(v[j], c);
  }
  for (int c = threadIdx.x + kDigitChunks * kDigitThreads; c < kc; c += kDigitThreads) digits8(__ldcg(xr + c), c);
  if (threadIdx.x == 0) pr.tscale[t] = ts;
}

template <int T, int EPI>
cudaError_t launch_kblk(const TcParams& p, const TcPlan& plan, bool pdl, cudaStream_t s) {
  if (plan.kblk == 256) return launch_one<kFmtI8, T, 256, EPI, true>(p, plan, pdl, s);
  if (plan.kblk == 128) return launch_one<kFmtI8, T, 128, EPI, true>(p, plan, pdl, s);
  return cudaErrorInvalidValue;
}

template <int EPI>
cudaError_t launch_tokens(const TcParams& p, const TcPlan& plan, bool pdl, cudaStream_t s) {
  switch (plan.n_mma) {
    case 8: return launch_kblk<8, EPI>(p, plan, pdl, s);
    case 16: return launch_kblk<16, EPI>(p, plan, pdl, s);
    case 32: return launch_kblk<32, EPI>(p, plan, pdl, s);
    case 64: return launch_kblk<64, EPI>(p, plan, pdl, s);
    default: return cudaErrorInvalidValue;
  }
}

// 4-bit asymmetric weights: one 128-group per stage, token tiles of 8 or 16
template <int EPI>
cudaError_t launch_tokens_w4(const TcParams& p, const TcPlan& plan, bool pdl, cudaStream_t s) {
  if (plan.kblk != 128) return cudaErrorInvalidValue;
  switch (plan.n_mma) {
    case 8: return launch_one<kFmtI8W4, 8, 128, EPI, true>(p, plan, pdl, s);
    case 16: return launch_one<kFmtI8W4, 16, 128, EPI, true>(p, plan, pdl, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int tc_choose_tokens_i8(int m) { return m <= 8 ? 8 : m <= 16 ? 16 : m <= 32 ? 32 : 64; }

int tc_threads_i8() { return TcRoles<kFmtI8, 16, 128>::THREADS; }

cudaError_t launch_act_digits(const TcProblem* dev_tab, const TcProblem& single, int count, int rows_max, bool pdl,
                              cudaStream_t s) {
  if (count < 1 || rows_max < 1) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(rows_max, count);
  cfg.blockDim = dim3(kDigitThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, act_digits_kernel, count > 1 ? dev_tab : nullptr, single);
}

cudaError_t launch_tc_i8(const TcParams& p, const TcPlan& plan, int fmt, int epi, bool pdl, cudaStream_t s) {
  if (fmt == kFmtI8W4) {
    if (epi == kEpiSwiglu) return launch_tokens_w4<kEpiSwiglu>(p, plan, pdl, s);
    if (epi == kEpiPlain) return launch_tokens_w4<kEpiPlain>(p, plan, pdl, s);
    return cudaErrorInvalidValue;
  }
  if (fmt != kFmtI8) return cudaErrorInvalidValue;
  if (epi == kEpiSwiglu) return launch_tokens<kEpiSwiglu>(p, plan, pdl, s);
  if (epi == kEpiPlain) return launch_tokens<kEpiPlain>(p, plan, pdl, s);
  return cudaErrorInvalidValue;
}

}  // namespace kl
