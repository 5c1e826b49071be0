// Host side of the persistent tcgen05 weight-only GEMM (kernel template in
// kl_tc_gemm.cuh): instantiation and launch for the bf16-MMA formats, and the
// planning helpers shared with the int8-MMA mode.
#include "kl_tc_gemm.cuh"

namespace kl {

namespace {

template <int FMT, int SWIGLU, bool XBF16>
cudaError_t launch_nmma(const TcParams& p, const TcPlan& plan, bool pdl, cudaStream_t s) {
  if constexpr (FMT == KL_W8_ROW) {
    if (plan.kblk == 256) {
      switch (plan.n_mma) {
        case 16: return launch_one<FMT, 16, 256, SWIGLU, XBF16>(p, plan, pdl, s);
        case 32: return launch_one<FMT, 32, 256, SWIGLU, XBF16>(p, plan, pdl, s);
        case 64: return launch_one<FMT, 64, 256, SWIGLU, XBF16>(p, plan, pdl, s);
        default: return cudaErrorInvalidValue;
      }
    }
  } else if constexpr (grouped<FMT>()) {
    if (plan.kblk == 256)   // two 128-groups per stage: 16-token tiles only
      return plan.n_mma == 16 ? launch_one<FMT, 16, 256, SWIGLU, XBF16>(p, plan, pdl, s) : cudaErrorInvalidValue;
  }
  if (plan.kblk != 128) return cudaErrorInvalidValue;
  switch (plan.n_mma) {
    case 16: return launch_one<FMT, 16, 128, SWIGLU, XBF16>(p, plan, pdl, s);
    case 32: return launch_one<FMT, 32, 128, SWIGLU, XBF16>(p, plan, pdl, s);
    case 64: return launch_one<FMT, 64, 128, SWIGLU, XBF16>(p, plan, pdl, s);
    default:
      if constexpr (grouped<FMT>()) return cudaErrorInvalidValue;   // group mode keeps <= 64 columns in registers
      else return launch_one<FMT, 128, 128, SWIGLU, XBF16>(p, plan, pdl, s);
  }
}

template <int SWIGLU, bool XBF16>
cudaError_t launch_fmt(const TcParams& p, const TcPlan& plan, int fmt, bool pdl, cudaStream_t s) {
  switch (fmt) {
    case KL_W8_ROW: return launch_nmma<KL_W8_ROW, SWIGLU, XBF16>(p, plan, pdl, s);
    case KL_W4_ASYM: return launch_nmma<KL_W4_ASYM, SWIGLU, XBF16>(p, plan, pdl, s);
    case KL_W4_SYM: return launch_nmma<KL_W4_SYM, SWIGLU, XBF16>(p, plan, pdl, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int tc_threads(int fmt, int n_mma, int kblk) {
  const bool w4 = fmt == KL_W4_SYM || fmt == KL_W4_ASYM;
  if (kblk == 256) {
    switch (n_mma) {
      case 16: return w4 ? TcRoles<KL_W4_ASYM, 16, 256>::THREADS : TcRoles<KL_W8_ROW, 16, 256>::THREADS;
      case 32: return TcRoles<KL_W8_ROW, 32, 256>::THREADS;
      default: return TcRoles<KL_W8_ROW, 64, 256>::THREADS;
    }
  }
  switch (n_mma) {
    case 16: return TcRoles<KL_W8_ROW, 16, 128>::THREADS;
    case 32: return TcRoles<KL_W8_ROW, 32, 128>::THREADS;
    case 64: return w4 ? TcRoles<KL_W4_ASYM, 64, 128>::THREADS : TcRoles<KL_W8_ROW, 64, 128>::THREADS;
    default: return TcRoles<KL_W8_ROW, 128, 128>::THREADS;
  }
}

static int tc_a_stages(int n_mma, int kblk) {
  if (kblk == 256) return n_mma <= 32 ? TcCfg<16, 256>::A_STAGES : TcCfg<64, 256>::A_STAGES;
  return n_mma <= 32 ? TcCfg<16, 128>::A_STAGES : (n_mma == 64 ? TcCfg<64, 128>::A_STAGES : TcCfg<128, 128>::A_STAGES);
}

int tc_choose_kblk(int fmt, int n_mma, long long units_at_256, int sm_count) {
  if (fmt == KL_W4_SYM || fmt == KL_W4_ASYM)   // callers also require K % 256 == 0
    return (n_mma == 16 && units_at_256 >= 2ll * sm_count) ? 256 : 128;
  if (!(fmt == KL_W8_ROW || fmt == kFmtI8) || n_mma > 64) return 128;
  if (fmt == kFmtI8 && n_mma == 64) return 128;     // 192 digit rows: 256-wide stages would not fit twice
  return units_at_256 >= 2ll * sm_count ? 256 : 128;
}

int tc_choose_nmma(int m, int fmt) {
  const bool w4 = fmt == KL_W4_SYM || fmt == KL_W4_ASYM;
  const int n = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128;
  return (w4 && n > 64) ? 64 : n;     // group mode: the host splits M into 64-token launches
}

long long tc_problem_tiles(TcProblem& pr, int n_mma, int kblk, bool swiglu) {
  pr.m_tiles = (pr.m + n_mma - 1) / n_mma;
  pr.n_tiles = swiglu ? (pr.n_out + 63) / 64 : (pr.n + 127) / 128;
  pr.kb_total = (pr.k + kblk - 1) / kblk;
  return static_cast<long long>(pr.m_tiles) * pr.n_tiles * pr.kb_total;
}

TcPlan plan_tc(int n_mma, int kblk, long long units, int fmt, int sm_count) {
  TcPlan t{};
  t.ok = false;
  if (units <= 0 || sm_count <= 0) return t;
  const bool i8w4 = fmt == kFmtI8W4;
  const bool w4 = fmt == KL_W4_SYM || fmt == KL_W4_ASYM || i8w4;
  const bool i8 = fmt == kFmtI8;
  if (i8 && !(n_mma == 8 || n_mma == 16 || n_mma == 32 || n_mma == 64)) return t;
  if (i8w4 && !((n_mma == 8 || n_mma == 16) && kblk == 128)) return t;
  if (!(kblk == 128 || (kblk == 256 && (fmt == KL_W8_ROW || i8) && n_mma <= 64) || (kblk == 256 && w4 && n_mma == 16)))
    return t;
  t.n_mma = n_mma;
  t.kblk = kblk;
  t.units = units;
  t.grid = static_cast<int>(std::min<long long>(units, sm_count));
  // weight stage pitch (the two-group asymmetric 4-bit stages carry their zeros)
  const int wsb = 128 * (w4 ? kblk / 2 : kblk) + ((fmt == KL_W4_ASYM && kblk == 256) ? kZeroStageBytes : 0);
  // x stage: bf16 tiles of n_mma tokens, or (int8 MMA) two digit planes of n_mma tokens
  const int x_stage = (i8 || i8w4) ? (kblk / 128) * i8_tile_rows(n_mma) * 128 : (kblk / 64) * n_mma * 128;
  const bool w4_pair = (fmt == KL_W4_SYM || fmt == KL_W4_ASYM) && kblk == 256 && n_mma == 16;
  const int a_stages = i8 ? 0 : i8w4 ? 4 : w4_pair ? 2 : tc_a_stages(n_mma, kblk);
  const int ndb = i8w4 ? std::min(8, (512 - 4 * (kblk / 4)) / i8_tile_rows(n_mma)) : w4_pair ? 4 : 2;
  t.x_stages = n_mma == 128 ? 3 : (x_stage > 16384 ? 3 : 4);
  // digit stages are small and come from L2 (written by the digits pass):
  // keep about 48 KB of them in flight so that L2 latency does not pace the MMAs
  if (i8 || i8w4) t.x_stages = std::max(t.x_stages, std::min(12, (48 * 1024) / x_stage));
  // ~128 KB of weights in flight per SM: deeper rings over-subscribe HBM
  const int budget = 220 * 1024;
  int sw = std::max(2, std::min(kMaxWStages, (128 * 1024) / wsb));
  while (sw > 2 && static_cast<int>(smem_layout(wsb, x_stage, a_stages, sw, t.x_stages, ndb).total) > budget) --sw;
  t.w_stages = sw;
  t.smem = static_cast<int>(smem_layout(wsb, x_stage, a_stages, sw, t.x_stages, ndb).total);
  t.workspace = kCounterBytes + static_cast<size_t>(t.grid) * 2 * n_mma * 128 * sizeof(float);
  if (t.grid > kCounterBytes / 4 || t.smem > 227 * 1024) return t;
  t.ok = true;
  return t;
}

cudaError_t launch_tc(const TcParams& p, const TcPlan& plan, int fmt, int epi, bool xbf16, bool pdl, cudaStream_t s) {
  if (epi == kEpiSwiglu)
    return xbf16 ? launch_fmt<kEpiSwiglu, true>(p, plan, fmt, pdl, s) : launch_fmt<kEpiSwiglu, false>(p, plan, fmt, pdl, s);
  if (epi == kEpiTopk)   // selection over the logits of an lm_head: bf16 activations
    return xbf16 ? launch_fmt<kEpiTopk, true>(p, plan, fmt, pdl, s) : cudaErrorInvalidValue;
  return xbf16 ? launch_fmt<kEpiPlain, true>(p, plan, fmt, pdl, s) : launch_fmt<kEpiPlain, false>(p, plan, fmt, pdl, s);
}

}  // namespace kl
