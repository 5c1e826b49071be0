// C-ABI entry points (include/kl_b200.h): argument validation, path choice
// (tcgen05 GEMM vs CUDA-core GEMV), TMA descriptor encoding and launches.
// Nothing here allocates device memory or synchronises the stream, so every
// entry point can be captured into a CUDA graph.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "kl_common.cuh"
#include "kl_internal.h"

namespace kl {

// Device status word: bounded in-kernel waits record KL_ERR_TIMEOUT here.
__device__ int g_status_word = 0;

size_t head_topk_candidate_bytes(int n, int top_k);
cudaError_t launch_topk(const void* logits, bool xbf16, int n, int top_k, void* cand, float* values,
                        int64_t* ids, cudaStream_t s);

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  return fail(KL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceInfo {
  int sm_count = 0;
  int major = 0, minor = 0;
  int* status = nullptr;
  bool ready = false;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mutex;

int device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(KL_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    if ((e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute");
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_status_word)) != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress");
    d.status = static_cast<int*>(p);
    d.ready = true;
  }
  *out = d;
  return KL_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return fail(KL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return KL_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool is_w4(int f) { return f == KL_W4_SYM || f == KL_W4_ASYM; }
bool is_grouped(int f) { return f == KL_W8_GROUP || is_w4(f); }
size_t act_bytes(int dt) { return dt == KL_DT_F32 ? 4 : 2; }

// Whether the tcgen05 kernel takes this problem (device capability aside).
bool tc_shape_ok(int k, int w_format, int group) {
  if (w_format == KL_W8_ROW) return k % 16 == 0;
  if (is_w4(w_format)) return group == 128 && k % 128 == 0;
  return false;
}

// Whether the CTA-pair prefill kernel takes an (already tcgen05-eligible) problem.
bool prefill_applies(int m, int k, int w_format, int sm_count) {
  return w_format == KL_W8_ROW && m >= kPrefillMinM && k % prefill_k_block() == 0 && sm_count >= 2;
}

// Fill one tcgen05 problem (tensor maps + fields); the caller sets unit_begin.
int build_problem(TcProblem& pr, const void* x, int x_dtype, int m, int k, const void* w, int w_format, int n,
                  const void* scales, const void* zeros, int swiglu, void* y, bool transposed, long long ldy,
                  int n_mma, int kblk) {
  std::memset(&pr, 0, sizeof(pr));
  int rc;
  if (is_w4(w_format) && kblk == 128)
    rc = encode_2d(&pr.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, k / 2, n, k / 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_64B);
  else if (is_w4(w_format))
    rc = encode_2d(&pr.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, k / 2, n, k / 2, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    rc = encode_2d(&pr.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, k, n, k, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != KL_OK) return rc;
  rc = encode_2d(&pr.tmap_x, x_dtype == KL_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                 x, k, m, static_cast<uint64_t>(k) * act_bytes(x_dtype), 64, n_mma, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != KL_OK) return rc;
  if (w_format == KL_W4_ASYM && kblk == 256) {   // zeros ride with the weight stages (box 8 groups x 64 rows)
    rc = encode_2d(&pr.tmap_z, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, zeros, k / 128, n, static_cast<uint64_t>(k / 128) * 2,
                   8, 64, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != KL_OK) return rc;
  }
  pr.scales = scales;
  pr.zeros = zeros;
  pr.y = y;
  pr.ldy = ldy;
  pr.m = m;
  pr.n = n;
  pr.k = k;
  pr.n_out = swiglu ? n / 2 : n;
  pr.y_transposed = transposed ? 1 : 0;
  pr.vec_store = (aligned16(y) && ldy % 8 == 0) ? (transposed ? 2 : 1) : 0;
  tc_problem_tiles(pr, n_mma, kblk, swiglu != 0);
  return KL_OK;
}

// Units of one problem without building its tensor maps (host planning only).
long long problem_units(int m, int n, int k, int n_mma, int kblk, bool swiglu) {
  TcProblem pr;
  std::memset(&pr, 0, sizeof(pr));
  pr.m = m;
  pr.n = n;
  pr.k = k;
  pr.n_out = swiglu ? n / 2 : n;
  return tc_problem_tiles(pr, n_mma, kblk, swiglu);
}

// Whether the two-group 4-bit stages (K block 256) can take this problem: the
// asymmetric format copies a box of zeros per stage by TMA, which needs 16-byte
// rows of zeros (K % 1024 == 0) and a 16-byte-aligned zeros pointer.
bool two_group_ok(int fmt, int k, const void* zeros) {
  if (k % 256) return false;
  if (fmt == KL_W4_ASYM) return k % 1024 == 0 && aligned16(zeros);
  return true;
}

// K block for one GEMM on this device.
int choose_kblk_single(int m, int n, int k, int fmt, int n_mma, bool swiglu, int sm_count, const void* zeros) {
  if (is_w4(fmt) && !two_group_ok(fmt, k, zeros)) return 128;
  return tc_choose_kblk(fmt, n_mma, problem_units(m, n, k, n_mma, 256, swiglu), sm_count);
}

int validate_linear(const void* x, int x_dtype, int m, int k, const void* w, int w_format, int n, int group,
                    const void* scales, const void* zeros, const float* inverse, int swiglu, const void* y,
                    int flags) {
  if (!x || !w || !y) return fail(KL_ERR_INVALID, "x, w and y must be non-null");
  if (m <= 0 || k <= 0 || n <= 0) return fail(KL_ERR_INVALID, "dimensions must be positive (m=%d k=%d n=%d)", m, k, n);
  if (x_dtype != KL_DT_BF16 && x_dtype != KL_DT_F16) return fail(KL_ERR_INVALID, "activations must be bf16 or f16");
  if (w_format < KL_W8_ROW || w_format > KL_BF16_DENSE) return fail(KL_ERR_INVALID, "unknown weight format %d", w_format);
  if (swiglu && (n % 2)) return fail(KL_ERR_INVALID, "gate/up requires two equal row sets");
  if (is_grouped(w_format) && (group <= 0 || k % group)) return fail(KL_ERR_INVALID, "group must divide K");
  if (is_w4(w_format) && (k % 2 || group % 2)) return fail(KL_ERR_INVALID, "4-bit weights need an even K and group");
  if (w_format != KL_BF16_DENSE && !scales) return fail(KL_ERR_INVALID, "scales required");
  if (w_format == KL_W8_GROUP && !inverse) return fail(KL_ERR_INVALID, "inverse channel vector required");
  if (w_format == KL_W4_ASYM && !zeros) return fail(KL_ERR_INVALID, "zero points required");
  if ((flags & KL_FLAG_FORCE_SIMT) && (flags & KL_FLAG_FORCE_TC)) return fail(KL_ERR_INVALID, "conflicting path flags");
  return KL_OK;
}

}  // namespace

int report_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

}  // namespace kl

using namespace kl;

extern "C" {

size_t kl_linear_topk_workspace_bytes(int m, int n, int k, int w_format, int top_k);

const char* kl_status_string(int status) {
  switch (status) {
    case KL_OK: return "ok";
    case KL_ERR_INVALID: return "invalid argument";
    case KL_ERR_UNSUPPORTED: return "unsupported";
    case KL_ERR_CUDA: return "CUDA error";
    case KL_ERR_WORKSPACE: return "workspace missing or too small";
    case KL_ERR_TIMEOUT: return "in-kernel wait timed out";
    default: return "unknown status";
  }
}

const char* kl_last_error(void) { return g_last_error; }

int kl_version(void) { return 100; }

size_t kl_linear_workspace_bytes(int m, int n, int k, int w_format, int swiglu, int flags) {
  if (m <= 0 || n <= 0 || k <= 0 || (flags & KL_FLAG_FORCE_SIMT)) return 0;
  if (!(w_format == KL_W8_ROW || is_w4(w_format))) return 0;
  int sm = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sm = v;
  } else {
    cudaGetLastError();
  }
  const int mm = is_w4(w_format) ? std::min(m, 64) : m;
  const int n_mma = tc_choose_nmma(mm, w_format);
  // the zeros pointer is not known here: size for whichever K block the call picks
  const int kblk = choose_kblk_single(mm, n, k, w_format, n_mma, swiglu != 0, sm, nullptr);
  const TcPlan plan = plan_tc(n_mma, kblk, problem_units(mm, n, k, n_mma, kblk, swiglu != 0), w_format, sm);
  if (!plan.ok) return 0;
  const TcPlan p128 = plan_tc(n_mma, 128, problem_units(mm, n, k, n_mma, 128, swiglu != 0), w_format, sm);
  return (p128.ok && p128.workspace > plan.workspace) ? p128.workspace : plan.workspace;
}

int kl_linear(const void* x, int x_dtype, int m, int k, const void* w, int w_format, int n, int group,
              const void* scales, const void* zeros, const float* inverse, int swiglu, void* y, void* workspace,
              size_t workspace_bytes, int flags, void* stream) {
  int rc = validate_linear(x, x_dtype, m, k, w, w_format, n, group, scales, zeros, inverse, swiglu, y, flags);
  if (rc != KL_OK) return rc;
  DeviceInfo di;
  if ((rc = device_info(&di)) != KL_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n_out = swiglu ? n / 2 : n;
  const bool xbf16 = x_dtype == KL_DT_BF16;
  const bool transposed = (flags & KL_FLAG_Y_TRANSPOSED) != 0;
  const bool sm100 = di.major == 10 && di.minor == 0;
  const bool tc = sm100 && !(flags & KL_FLAG_FORCE_SIMT) && tc_shape_ok(k, w_format, group) && aligned16(x) &&
                  aligned16(w);
  if ((flags & KL_FLAG_FORCE_TC) && !tc)
    return fail(KL_ERR_UNSUPPORTED, "tcgen05 path not applicable (format %d, K %d, group %d, sm%d%d)", w_format, k,
                group, di.major, di.minor);
  if (!sm100) return fail(KL_ERR_UNSUPPORTED, "this library is built for sm_100a (device is sm%d%d)", di.major, di.minor);
  const size_t eb = act_bytes(x_dtype);

  if (tc && prefill_applies(m, k, w_format, di.sm_count)) {
    PfParams p;
    std::memset(&p, 0, sizeof(p));
    p.scales = scales;
    p.y = y;
    p.ldy = transposed ? m : n_out;
    p.m = m;
    p.n = n;
    p.k = k;
    p.n_out = n_out;
    p.y_transposed = transposed ? 1 : 0;
    p.vec_store = (aligned16(y) && p.ldy % 8 == 0) ? (transposed ? 2 : 1) : 0;
    p.status = di.status;
    prefill_tiles(p, swiglu != 0, di.sm_count);
    rc = encode_2d(&p.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, k, n, k, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != KL_OK) return rc;
    // each CTA of a pair loads half of the tile's tokens
    rc = encode_2d(&p.tmap_x, xbf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, k, m,
                   static_cast<uint64_t>(k) * eb, 64, static_cast<uint32_t>(p.tok / 2), CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != KL_OK) return rc;
    const cudaError_t e = launch_prefill(p, prefill_grid(p, di.sm_count), swiglu != 0, xbf16, (flags & KL_FLAG_PDL) != 0, s);
    if (e != cudaSuccess) return cuda_fail(e, "tcgen05 pair GEMM launch");
    return KL_OK;
  }

  if (sm100 && !(flags & (KL_FLAG_FORCE_SIMT | KL_FLAG_PERSISTENT | KL_FLAG_FORCE_TC)) && aligned16(x) &&
      aligned16(w) && (w_format == KL_W8_ROW || is_w4(w_format))) {
    // One or two tokens: full rows per CTA on CUDA cores, nothing exchanged
    // between CTAs (the shortest path after the dependency wait)
    const GemvChainPlan gp = plan_gemv_chain(m, n, k, w_format, group, swiglu != 0, di.sm_count);
    if (gp.ok) {
      GemvChainParams c;
      std::memset(&c, 0, sizeof(c));
      c.w = w;
      c.scales = scales;
      c.zeros = zeros;
      c.group = group;
      c.x = x;
      c.y = y;
      c.ldy = transposed ? m : n_out;
      c.m = m;
      c.k = k;
      c.n = n;
      c.n_out = n_out;
      c.rows = gp.rows;
      c.y_transposed = transposed ? 1 : 0;
      c.status = di.status;
      const cudaError_t e = launch_gemv_chain(c, gp, w_format, swiglu != 0, xbf16, (flags & KL_FLAG_PDL) != 0, s);
      if (e != cudaSuccess) return cuda_fail(e, "chain GEMV launch");
      return KL_OK;
    }
  }

  if (tc && w_format == KL_W8_ROW && !(flags & KL_FLAG_PERSISTENT)) {
    // One decode-size linear: the single-tile cluster kernel, whose fixed cost
    // after the previous kernel in the stream is a fraction of the persistent one's.
    const ChainPlan cp = plan_chain(m, n, k, swiglu != 0, di.sm_count);
    if (cp.ok) {
      ChainParams c;
      std::memset(&c, 0, sizeof(c));
      rc = encode_2d(&c.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, k, n, k, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc != KL_OK) return rc;
      rc = encode_2d(&c.tmap_x, xbf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, k, m,
                     static_cast<uint64_t>(k) * eb, 64, cp.n_mma, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc != KL_OK) return rc;
      c.scales = scales;
      c.y = y;
      c.ldy = transposed ? m : n_out;
      c.m = m;
      c.n = n;
      c.k = k;
      c.n_out = n_out;
      c.kb_total = (k + 127) / 128;
      c.bpc = cp.bpc;
      c.csize = cp.csize;
      c.y_transposed = transposed ? 1 : 0;
      c.status = di.status;
      const cudaError_t e = launch_chain(c, cp, swiglu != 0, xbf16, (flags & KL_FLAG_PDL) != 0, s);
      if (e == cudaSuccess) return KL_OK;
      // cudaErrorNotSupported: this device cannot hold a cluster of that size: persistent kernel
      if (e != cudaErrorNotSupported) return cuda_fail(e, "tcgen05 chain GEMM launch");
    }
  }

  if (tc) {
    const int mchunk = is_w4(w_format) ? 64 : m;
    for (int m0 = 0; m0 < m; m0 += mchunk) {
      const int mm = std::min(mchunk, m - m0);
      const int n_mma = tc_choose_nmma(mm, w_format);
      const int kblk = choose_kblk_single(mm, n, k, w_format, n_mma, swiglu != 0, di.sm_count, zeros);
      TcParams p;
      std::memset(&p, 0, sizeof(p));
      const char* xb = static_cast<const char*>(x) + static_cast<size_t>(m0) * k * eb;
      char* yb = static_cast<char*>(y) + (transposed ? static_cast<size_t>(m0) : static_cast<size_t>(m0) * n_out) * eb;
      rc = build_problem(p.single, xb, x_dtype, mm, k, w, w_format, n, scales, zeros, swiglu, yb, transposed,
                         transposed ? m : n_out, n_mma, kblk);
      if (rc != KL_OK) return rc;
      p.single.unit_begin = 0;
      const long long units = static_cast<long long>(p.single.m_tiles) * p.single.n_tiles * p.single.kb_total;
      const TcPlan plan = plan_tc(n_mma, kblk, units, w_format, di.sm_count);
      if (!plan.ok) return fail(KL_ERR_UNSUPPORTED, "no tcgen05 plan for m=%d n=%d k=%d", mm, n, k);
      if (!workspace || workspace_bytes < plan.workspace)
        return fail(KL_ERR_WORKSPACE, "workspace of %zu bytes required, %zu given", plan.workspace,
                    workspace ? workspace_bytes : 0);
      p.table = nullptr;
      p.count = 1;
      p.w_stages = plan.w_stages;
      p.x_stages = plan.x_stages;
      p.units = units;
      p.counters = static_cast<int*>(workspace);
      p.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
      p.status = di.status;
      const cudaError_t e = launch_tc(p, plan, w_format, swiglu ? kEpiSwiglu : kEpiPlain, xbf16,
                                      (flags & KL_FLAG_PDL) != 0, s);
      if (e != cudaSuccess) return cuda_fail(e, "tcgen05 GEMM launch");
    }
    return KL_OK;
  }

  const GemvPlan gp = plan_gemv(m, n_out, k, w_format, group, swiglu != 0, aligned16(w), di.sm_count);
  GemvArgs a;
  a.x = x;
  a.w = w;
  a.scales = scales;
  a.zeros = zeros;
  a.inverse = inverse;
  a.y = y;
  a.m = m;
  a.k = k;
  a.n_out = n_out;
  a.group = group;
  a.kpad = gp.kpad;
  a.y_transposed = transposed ? 1 : 0;
  a.ldy = transposed ? m : n_out;
  const cudaError_t e = launch_gemv(a, gp, w_format, swiglu != 0, xbf16, s);
  if (e != cudaSuccess) return cuda_fail(e, "GEMV launch");
  return KL_OK;
}

namespace {
struct GroupHeader {
  uint32_t magic, count;
  int n_mma, w_format, swiglu, x_dtype;
  long long units;
  int kblk;
  int int8_mma;                     // 1: KL_GROUPED_INT8_MMA (digits pass + kind::i8 GEMM)
  int rows_max;                     // int8 mode: largest m_tiles * T of the problems
  int pair;                         // 1: every problem runs on the CTA-pair prefill kernel (table of PfParams)
  uint8_t pad[256 - 48];
};
static_assert(sizeof(PfParams) <= sizeof(TcProblem), "a pair-mode table fits the table size");
static_assert(sizeof(GroupHeader) == 256, "group header");
constexpr uint32_t kGroupMagic = 0x4B4C4752u;   // "KLGR"
}  // namespace

size_t kl_grouped_table_bytes(int count) {
  if (count <= 0 || count > kMaxGroup) return 0;
  return sizeof(GroupHeader) + static_cast<size_t>(count) * sizeof(TcProblem);
}

// Digits area of one problem in the int8 mode: [m_tiles][i8_tile_rows(T)][K]
// int8, then m_tiles * T f32 token scales, each piece 256-byte aligned.
static size_t digits_plane_bytes(int m, int k, int tok) {
  const size_t tiles = static_cast<size_t>((m + tok - 1) / tok);
  return (tiles * i8_tile_rows(tok) * static_cast<size_t>(k) + 255) & ~static_cast<size_t>(255);
}
static size_t digits_scale_bytes(int m, int tok) {
  const size_t tiles = static_cast<size_t>((m + tok - 1) / tok);
  return (tiles * tok * sizeof(float) + 255) & ~static_cast<size_t>(255);
}

size_t kl_grouped_digits_bytes(const kl_problem* problems, int count, int flags) {
  if (!problems || count <= 0 || count > kMaxGroup || !(flags & KL_GROUPED_INT8_MMA)) return 0;
  int max_m = 0;
  for (int i = 0; i < count; ++i) max_m = std::max(max_m, problems[i].m);
  if (max_m <= 0) return 0;
  const int tok = tc_choose_tokens_i8(max_m);
  size_t total = 0;
  for (int i = 0; i < count; ++i) {
    if (problems[i].m <= 0 || problems[i].k <= 0) return 0;
    total += digits_plane_bytes(problems[i].m, problems[i].k, tok) + digits_scale_bytes(problems[i].m, tok);
  }
  return total;
}

int kl_grouped_encode(const kl_problem* problems, int count, int x_dtype, int w_format, int swiglu, void* host_table,
                      size_t table_bytes) {
  return kl_grouped_encode_ex(problems, count, x_dtype, w_format, swiglu, 0, nullptr, 0, host_table, table_bytes);
}

int kl_grouped_encode_ex(const kl_problem* problems, int count, int x_dtype, int w_format, int swiglu, int flags,
                         void* digits, size_t digits_bytes, void* host_table, size_t table_bytes) {
  if (!problems || !host_table) return fail(KL_ERR_INVALID, "problems and host_table must be non-null");
  if (flags & ~KL_GROUPED_INT8_MMA) return fail(KL_ERR_INVALID, "unknown grouped flags 0x%x", flags);
  const bool i8 = (flags & KL_GROUPED_INT8_MMA) != 0;
  if (i8) {
    if (!(w_format == KL_W8_ROW || w_format == KL_W4_ASYM) || x_dtype != KL_DT_BF16)
      return fail(KL_ERR_UNSUPPORTED, "the int8-MMA mode takes KL_W8_ROW or KL_W4_ASYM weights and bf16 activations");
    if (w_format == KL_W4_ASYM) {
      int mm = 0;
      for (int i = 0; i < count; ++i) {
        mm = std::max(mm, problems[i].m);
        if (problems[i].group != 128) return fail(KL_ERR_UNSUPPORTED, "the int8-MMA 4-bit mode takes group 128");
      }
      if (mm > 16) return fail(KL_ERR_UNSUPPORTED, "the int8-MMA 4-bit mode takes m <= 16");
    }
    if (!digits || (reinterpret_cast<uintptr_t>(digits) & 255u))
      return fail(KL_ERR_INVALID, "the int8-MMA mode needs a 256-byte-aligned digits buffer");
    const size_t need = kl_grouped_digits_bytes(problems, count, flags);
    if (need == 0 || digits_bytes < need)
      return fail(KL_ERR_WORKSPACE, "digits buffer of %zu bytes required, %zu given", need, digits_bytes);
  }
  if (count <= 0 || count > kMaxGroup) return fail(KL_ERR_INVALID, "count must be in [1, %d]", kMaxGroup);
  if (table_bytes < kl_grouped_table_bytes(count)) return fail(KL_ERR_INVALID, "host table too small");
  if (!(w_format == KL_W8_ROW || is_w4(w_format)))
    return fail(KL_ERR_UNSUPPORTED, "grouped launches take KL_W8_ROW or the 4-bit formats");
  int max_m = 0;
  for (int i = 0; i < count; ++i) {
    const kl_problem& q = problems[i];
    const int grp = is_w4(w_format) ? q.group : q.k;
    int rc = validate_linear(q.x, x_dtype, q.m, q.k, q.w, w_format, q.n, grp, q.scales, q.zeros, nullptr, swiglu,
                             q.y, 0);
    if (rc != KL_OK) return fail(rc, "problem %d: %s", i, g_last_error);
    if (!tc_shape_ok(q.k, w_format, grp) || !aligned16(q.x) || !aligned16(q.w))
      return fail(KL_ERR_UNSUPPORTED, "problem %d is not tcgen05-compatible (K %d, group %d, alignment)", i, q.k, grp);
    max_m = std::max(max_m, q.m);
  }
  if (is_w4(w_format) && max_m > 64) return fail(KL_ERR_UNSUPPORTED, "grouped 4-bit launches take m <= 64");
  GroupHeader* hd = static_cast<GroupHeader*>(host_table);
  std::memset(hd, 0, sizeof(*hd));
  hd->magic = kGroupMagic;
  hd->count = static_cast<uint32_t>(count);
  int sm_pair = 148, dev_pair = 0, v_pair = 0;
  if (cudaGetDevice(&dev_pair) == cudaSuccess &&
      cudaDeviceGetAttribute(&v_pair, cudaDevAttrMultiProcessorCount, dev_pair) == cudaSuccess && v_pair > 0)
    sm_pair = v_pair;
  else
    cudaGetLastError();
  // many-token groups: every problem on the CTA-pair kernel, the tiles of all
  // problems dealt round-robin to the pairs of one launch
  bool pair = !i8;
  for (int i = 0; i < count && pair; ++i)
    pair = prefill_applies(problems[i].m, problems[i].k, w_format, sm_pair);
  if (pair) {
    hd->pair = 1;
    hd->w_format = w_format;
    hd->swiglu = swiglu ? 1 : 0;
    hd->x_dtype = x_dtype;
    PfParams* tab = reinterpret_cast<PfParams*>(hd + 1);
    for (int i = 0; i < count; ++i) {
      const kl_problem& q = problems[i];
      PfParams& p = tab[i];
      std::memset(&p, 0, sizeof(p));
      p.scales = q.scales;
      p.y = q.y;
      p.m = q.m;
      p.n = q.n;
      p.k = q.k;
      p.n_out = swiglu ? q.n / 2 : q.n;
      p.ldy = p.n_out;
      p.vec_store = (aligned16(q.y) && p.ldy % 8 == 0) ? 1 : 0;
    }
    const int tiles = prefill_group_tiles(tab, count, swiglu != 0, sm_pair);
    for (int i = 0; i < count; ++i) {
      const kl_problem& q = problems[i];
      PfParams& p = tab[i];
      int rc = encode_2d(&p.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, q.w, q.k, q.n, q.k, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc != KL_OK) return rc;
      rc = encode_2d(&p.tmap_x, x_dtype == KL_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                     q.x, q.k, q.m, static_cast<uint64_t>(q.k) * act_bytes(x_dtype), 64,
                     static_cast<uint32_t>(p.tok / 2), CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc != KL_OK) return rc;
    }
    hd->n_mma = tab[0].tok;
    hd->units = tiles;
    return KL_OK;
  }
  hd->n_mma = i8 ? tc_choose_tokens_i8(max_m) : tc_choose_nmma(max_m, w_format);
  hd->int8_mma = i8 ? (w_format == KL_W4_ASYM ? 2 : 1) : 0;
  hd->w_format = w_format;
  hd->swiglu = swiglu ? 1 : 0;
  hd->x_dtype = x_dtype;
  TcProblem* tab = reinterpret_cast<TcProblem*>(hd + 1);
  int sm = 148, dev = 0, v = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
    sm = v;
  else
    cudaGetLastError();
  long long units256 = 0;
  for (int i = 0; i < count; ++i)
    units256 += problem_units(problems[i].m, problems[i].n, problems[i].k, hd->n_mma, 256, swiglu != 0);
  hd->kblk = hd->int8_mma == 2 ? 128 : tc_choose_kblk(i8 ? kFmtI8 : w_format, hd->n_mma, units256, sm);
  if (hd->kblk == 256 && is_w4(w_format)) {   // two 128-groups per stage: every problem must qualify
    for (int i = 0; i < count; ++i)
      if (!two_group_ok(w_format, problems[i].k, problems[i].zeros)) hd->kblk = 128;
  }
  long long units = 0;
  for (int i = 0; i < count; ++i) {
    const kl_problem& q = problems[i];
    const int n_out = swiglu ? q.n / 2 : q.n;
    int rc = build_problem(tab[i], q.x, x_dtype, q.m, q.k, q.w, w_format, q.n, q.scales, q.zeros, swiglu, q.y, false,
                           n_out, i8 ? 64 : hd->n_mma, hd->kblk);
    if (rc != KL_OK) return rc;
    if (i8) {
      // the MMA's B operand is the digit planes of the tile: i8_tile_rows(T) rows of K int8
      TcProblem& pr = tab[i];
      const int tok = hd->n_mma;
      pr.tok = tok;
      pr.x_src = q.x;
      pr.digits = static_cast<int8_t*>(digits);
      pr.digits_ld = q.k;
      tc_problem_tiles(pr, tok, hd->kblk, swiglu != 0);
      const size_t planes = digits_plane_bytes(q.m, q.k, tok);
      pr.tscale = reinterpret_cast<float*>(static_cast<char*>(digits) + planes);
      rc = encode_2d(&pr.tmap_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, pr.digits, q.k,
                     static_cast<uint64_t>(pr.m_tiles) * i8_tile_rows(tok), q.k, 128, i8_tile_rows(tok),
                     CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc != KL_OK) return rc;
      digits = static_cast<char*>(digits) + planes + digits_scale_bytes(q.m, tok);
      hd->rows_max = std::max(hd->rows_max, pr.m_tiles * tok);
    }
    tab[i].unit_begin = units;
    units += static_cast<long long>(tab[i].m_tiles) * tab[i].n_tiles * tab[i].kb_total;
  }
  hd->units = units;
  return KL_OK;
}

size_t kl_grouped_workspace_bytes(const void* host_table) {
  const GroupHeader* hd = static_cast<const GroupHeader*>(host_table);
  if (!hd || hd->magic != kGroupMagic) return 0;
  if (hd->pair) return 0;                       // whole-K tiles: no split-tile scratch
  int sm = 148, dev = 0, v = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
    sm = v;
  else
    cudaGetLastError();
  const int fmt = hd->int8_mma == 2 ? kFmtI8W4 : hd->int8_mma ? kFmtI8 : hd->w_format;
  const TcPlan plan = plan_tc(hd->n_mma, hd->kblk, hd->units, fmt, sm);
  return plan.ok ? plan.workspace : 0;
}

int kl_linear_grouped(const void* host_table, const void* device_table, void* workspace, size_t workspace_bytes,
                      int flags, void* stream) {
  const GroupHeader* hd = static_cast<const GroupHeader*>(host_table);
  if (!hd || hd->magic != kGroupMagic) return fail(KL_ERR_INVALID, "host_table was not built by kl_grouped_encode");
  if (hd->count > 1 && (!device_table || (reinterpret_cast<uintptr_t>(device_table) & 63u)))
    return fail(KL_ERR_INVALID, "device_table must be a 64-byte-aligned device copy of the table");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc != KL_OK) return rc;
  if (!(di.major == 10 && di.minor == 0))
    return fail(KL_ERR_UNSUPPORTED, "this library is built for sm_100a (device is sm%d%d)", di.major, di.minor);
  if (hd->pair) {
    const PfParams* host_pf = reinterpret_cast<const PfParams*>(hd + 1);
    PfLaunch l;
    std::memset(&l, 0, sizeof(l));
    l.single = host_pf[0];
    l.single.status = di.status;
    l.count = static_cast<int>(hd->count);
    l.table = l.count > 1 ? reinterpret_cast<const PfParams*>(static_cast<const char*>(device_table) + sizeof(GroupHeader))
                          : nullptr;
    l.tiles = static_cast<int>(hd->units);
    l.status = di.status;
    const int grid = 2 * std::max(1, std::min(l.tiles, di.sm_count / 2));
    const cudaError_t e = launch_prefill_group(l, grid, hd->swiglu != 0, hd->x_dtype == KL_DT_BF16,
                                               (flags & KL_FLAG_PDL) != 0, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "grouped tcgen05 pair GEMM launch");
    return KL_OK;
  }
  const int fmt = hd->int8_mma == 2 ? kFmtI8W4 : hd->int8_mma ? kFmtI8 : hd->w_format;
  const TcPlan plan = plan_tc(hd->n_mma, hd->kblk, hd->units, fmt, di.sm_count);
  if (!plan.ok) return fail(KL_ERR_UNSUPPORTED, "no tcgen05 plan for the group");
  if (!workspace || workspace_bytes < plan.workspace)
    return fail(KL_ERR_WORKSPACE, "workspace of %zu bytes required, %zu given", plan.workspace,
                workspace ? workspace_bytes : 0);
  const TcProblem* host_tab = reinterpret_cast<const TcProblem*>(hd + 1);
  TcParams p;
  std::memset(&p, 0, sizeof(p));
  p.count = static_cast<int>(hd->count);
  if (p.count == 1) {
    p.single = host_tab[0];
    p.table = nullptr;
  } else {
    p.table = reinterpret_cast<const TcProblem*>(static_cast<const char*>(device_table) + sizeof(GroupHeader));
  }
  p.w_stages = plan.w_stages;
  p.x_stages = plan.x_stages;
  p.units = hd->units;
  p.counters = static_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  p.status = di.status;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (hd->int8_mma) {
    // digits pass, then the GEMM chained to it with programmatic dependent
    // launch (its weight stream starts while the digits are written)
    cudaError_t e = launch_act_digits(p.table, host_tab[0], p.count, hd->rows_max, (flags & KL_FLAG_PDL) != 0, st);
    if (e != cudaSuccess) return cuda_fail(e, "activation digits launch");
    e = launch_tc_i8(p, plan, fmt, hd->swiglu ? kEpiSwiglu : kEpiPlain, true, st);
    if (e != cudaSuccess) return cuda_fail(e, "grouped int8 tcgen05 GEMM launch");
    return KL_OK;
  }
  const cudaError_t e = launch_tc(p, plan, hd->w_format, hd->swiglu ? kEpiSwiglu : kEpiPlain, hd->x_dtype == KL_DT_BF16,
                                  (flags & KL_FLAG_PDL) != 0, st);
  if (e != cudaSuccess) return cuda_fail(e, "grouped tcgen05 GEMM launch");
  return KL_OK;
}

int kl_project(const void* x, int k, const void* w, int w_is_int8, const float* scales, const float* inverse, int n,
               int group, int warps, int persistent, int swiglu, void* y, void* workspace, size_t workspace_bytes,
               void* stream) {
  (void)persistent;
  if (!x || !w || !y) return fail(KL_ERR_INVALID, "same CUDA device required");
  if (k <= 0 || n <= 0) return fail(KL_ERR_INVALID, "w: contiguous nonempty [N,K]");
  if (!(warps == 1 || warps == 4 || warps == 8)) return fail(KL_ERR_INVALID, "warps must be 1,4,8");
  if (swiglu && n % 2) return fail(KL_ERR_INVALID, "gate/up requires two equal row sets");
  if (w_is_int8) {
    if (group <= 0 || k % group) return fail(KL_ERR_INVALID, "group must divide K");
    if (!scales || !inverse) return fail(KL_ERR_INVALID, "FP32 contiguous scaling buffers required");
  }
  return kl_linear(x, KL_DT_BF16, 1, k, w, w_is_int8 ? KL_W8_GROUP : KL_BF16_DENSE, n, group, scales, nullptr,
                   inverse, swiglu, y, workspace, workspace_bytes, 0, stream);
}

int kl_int4_gemv(const void* x, int x_dtype, int k, const uint8_t* w, const float* scales, int n, int group,
                 int block_n, void* y, void* stream) {
  if (!(group == 32 || group == 64 || group == 128)) return fail(KL_ERR_INVALID, "group_size must be 32, 64, or 128");
  if (!(block_n == 8 || block_n == 16 || block_n == 32 || block_n == 64))
    return fail(KL_ERR_INVALID, "block_n must be 8,16,32,64");
  // The M = 1 W4 GEMV runs on the CUDA-core kernel (no workspace).
  return kl_linear(x, x_dtype, 1, k, w, KL_W4_SYM, n, group, scales, nullptr, nullptr, 0, y, nullptr, 0,
                   KL_FLAG_FORCE_SIMT, stream);
}

// Workspace of kl_int4_lm_head_topk: the fused path's (stream-K counters, which
// must stay zero between calls, partials and candidates), or for the other
// shapes the logits and candidates placed after the counter area.
size_t kl_int4_lm_head_topk_workspace_bytes(int n, int top_k, int block_n) {
  (void)block_n;
  if (n <= 0 || top_k <= 0) return 0;
  const size_t logits = (static_cast<size_t>(n) * 2 + 255) & ~size_t(255);
  return kCounterBytes + logits + head_topk_candidate_bytes(n, top_k);
}
namespace {
size_t int4_head_fused_bytes(int n, int k, int group, int top_k) {
  if (group != 128 || k % 128 != 0) return 0;
  return kl_linear_topk_workspace_bytes(1, n, k, KL_W4_SYM, top_k);
}
}  // namespace

int kl_int4_lm_head_topk(const void* x, int x_dtype, int k, const uint8_t* w, const float* scales, int n, int group,
                         int top_k, int block_n, float* values, int64_t* ids, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (!values || !ids) return fail(KL_ERR_INVALID, "values and ids must be non-null");
  if (top_k < 1 || top_k > 8 || top_k > block_n || top_k > n)
    return fail(KL_ERR_INVALID, "top_k must be between 1 and min(8,block_n,vocabulary)");
  // bf16, groups of 128: the tcgen05 GEMM selects candidates in its epilogue and
  // the logits are never written (the reference's _head_candidates,
  // learning/09_int4/kernels.py:37-50)
  const size_t fused = x_dtype == KL_DT_BF16 ? int4_head_fused_bytes(n, k, group, top_k) : 0;
  if (fused && workspace && workspace_bytes >= fused && aligned16(x) && aligned16(w))
    return kl_linear_topk(x, x_dtype, 1, k, w, KL_W4_SYM, n, group, scales, nullptr, top_k, 0, values, ids,
                          workspace, workspace_bytes, 0, stream);
  const size_t need = kl_int4_lm_head_topk_workspace_bytes(n, top_k, block_n);
  if (!workspace || workspace_bytes < need) return fail(KL_ERR_WORKSPACE, "workspace of %zu bytes required", need);
  char* logits = static_cast<char*>(workspace) + kCounterBytes;
  char* cand = logits + ((static_cast<size_t>(n) * 2 + 255) & ~size_t(255));
  int rc = kl_int4_gemv(x, x_dtype, k, w, scales, n, group, block_n, logits, stream);
  if (rc != KL_OK) return rc;
  const cudaError_t e = launch_topk(logits, x_dtype == KL_DT_BF16, n, top_k, cand, values, ids,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "top-k launch");
  return KL_OK;
}

size_t kl_topk_rows_workspace_bytes(int rows, int n, int top_k) {
  if (rows <= 0 || n <= 0 || top_k <= 0) return 0;
  return topk_rows_candidate_bytes(rows, n, top_k);
}

int kl_topk_rows(const void* logits, int dtype, int rows, int n, long long ld, long long index_offset, int top_k,
                 float* values, int64_t* ids, void* workspace, size_t workspace_bytes, void* stream) {
  if (!logits || !ids) return fail(KL_ERR_INVALID, "logits and ids must be non-null");
  if (dtype != KL_DT_BF16 && dtype != KL_DT_F16) return fail(KL_ERR_INVALID, "logits must be bf16 or f16");
  if (rows <= 0 || n <= 0 || ld < n) return fail(KL_ERR_INVALID, "need rows > 0, n > 0 and ld >= n");
  if (top_k < 1 || top_k > 8 || top_k > n) return fail(KL_ERR_INVALID, "top_k must be in [1, min(8, n)]");
  if (index_offset < 0) return fail(KL_ERR_INVALID, "index_offset must be non-negative");
  const size_t need = topk_rows_candidate_bytes(rows, n, top_k);
  if (!workspace || workspace_bytes < need) return fail(KL_ERR_WORKSPACE, "workspace of %zu bytes required", need);
  const cudaError_t e = launch_topk_rows(logits, dtype == KL_DT_BF16, rows, n, ld, index_offset, top_k, workspace,
                                         values, ids, static_cast<cudaStream_t>(stream), values == nullptr);
  return e == cudaSuccess ? KL_OK : cuda_fail(e, "top-k launch");
}

namespace {
// Plan of the fused lm_head top-k: the persistent tcgen05 kernel with the top-k
// epilogue (4-bit formats: at most 64 tokens per launch).
struct TopkPlan {
  bool ok;
  int n_mma, kblk;
  TcPlan tc;
  long long units;
  int n_tiles;
  size_t cand_offset, bytes;
};
TopkPlan plan_topk(int m, int n, int k, int w_format, int top_k, int sm_count, const void* zeros) {
  TopkPlan t{};
  t.ok = false;
  if (m <= 0 || n <= 0 || k <= 0 || top_k < 1 || top_k > 8) return t;
  if (!(w_format == KL_W8_ROW || (is_w4(w_format) && m <= 64))) return t;
  if (!tc_shape_ok(k, w_format, is_w4(w_format) ? 128 : k)) return t;
  t.n_mma = tc_choose_nmma(m, w_format);
  t.kblk = choose_kblk_single(m, n, k, w_format, t.n_mma, false, sm_count, zeros);
  t.units = problem_units(m, n, k, t.n_mma, t.kblk, false);
  t.tc = plan_tc(t.n_mma, t.kblk, t.units, w_format, sm_count);
  if (!t.tc.ok) return t;
  t.n_tiles = (n + 127) / 128;
  t.cand_offset = (t.tc.workspace + 255) & ~size_t(255);
  t.bytes = t.cand_offset + static_cast<size_t>(m) * t.n_tiles * top_k * sizeof(long long);
  t.ok = true;
  return t;
}
int sm_count_or_default() {
  int sm = 148, dev = 0, v = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
    sm = v;
  else
    cudaGetLastError();
  return sm;
}
}  // namespace

size_t kl_linear_topk_workspace_bytes(int m, int n, int k, int w_format, int top_k) {
  // the zeros pointer is not known here: size for whichever K block the call picks
  const int sm = sm_count_or_default();
  const TopkPlan a = plan_topk(m, n, k, w_format, top_k, sm, nullptr);
  if (!a.ok) return 0;
  size_t need = a.bytes;
  if (w_format == KL_W4_ASYM) {     // a 16-byte-aligned zeros pointer may take the two-group stages
    alignas(16) static const char probe[16] = {};
    const TopkPlan b = plan_topk(m, n, k, w_format, top_k, sm, probe);
    if (b.ok && b.bytes > need) need = b.bytes;
  }
  return need;
}

int kl_linear_topk(const void* x, int x_dtype, int m, int k, const void* w, int w_format, int n, int group,
                   const void* scales, const void* zeros, int top_k, long long index_offset, float* values,
                   int64_t* ids, void* workspace, size_t workspace_bytes, int flags, void* stream) {
  int rc = validate_linear(x, x_dtype, m, k, w, w_format, n, is_grouped(w_format) ? group : k, scales, zeros,
                           nullptr, 0, ids, 0);
  if (rc != KL_OK) return rc;
  if (top_k < 1 || top_k > 8 || top_k > n) return fail(KL_ERR_INVALID, "top_k must be in [1, min(8, N)]");
  if (index_offset < 0 || index_offset + n > 0x7FFFFFFFll) return fail(KL_ERR_INVALID, "row ids must stay below 2^31");
  DeviceInfo di;
  if ((rc = device_info(&di)) != KL_OK) return rc;
  if (!(di.major == 10 && di.minor == 0))
    return fail(KL_ERR_UNSUPPORTED, "this library is built for sm_100a (device is sm%d%d)", di.major, di.minor);
  if (x_dtype != KL_DT_BF16 || !aligned16(x) || !aligned16(w) || (is_w4(w_format) && group != 128))
    return fail(KL_ERR_UNSUPPORTED, "the fused top-k takes bf16 activations, 16-byte-aligned operands and, for "
                                    "4-bit weights, groups of 128");
  const TopkPlan tp = plan_topk(m, n, k, w_format, top_k, di.sm_count, zeros);
  if (!tp.ok) return fail(KL_ERR_UNSUPPORTED, "no fused top-k plan for m=%d n=%d k=%d format %d", m, n, k, w_format);
  if (!workspace || workspace_bytes < tp.bytes)
    return fail(KL_ERR_WORKSPACE, "workspace of %zu bytes required, %zu given", tp.bytes,
                workspace ? workspace_bytes : 0);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(ws + tp.cand_offset);
  TcParams p;
  std::memset(&p, 0, sizeof(p));
  // y is never written in this epilogue; the candidate buffer stands in for it
  rc = build_problem(p.single, x, x_dtype, m, k, w, w_format, n, scales, zeros, 0, cand, false, n, tp.n_mma, tp.kblk);
  if (rc != KL_OK) return rc;
  p.single.unit_begin = 0;
  p.single.cand = cand;
  p.single.topk = top_k;
  p.single.cand_ld = tp.n_tiles * top_k;
  p.single.index_offset = index_offset;
  p.single.vec_store = 0;
  p.count = 1;
  p.w_stages = tp.tc.w_stages;
  p.x_stages = tp.tc.x_stages;
  p.units = tp.units;
  p.counters = reinterpret_cast<int*>(ws);
  p.partials = reinterpret_cast<float*>(ws + kCounterBytes);
  p.status = di.status;
  cudaError_t e = launch_tc(p, tp.tc, w_format, kEpiTopk, true, (flags & KL_FLAG_PDL) != 0, s);
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 GEMM launch (top-k epilogue)");
  e = launch_topk_merge_rows(reinterpret_cast<const int64_t*>(cand), m, tp.n_tiles * top_k, top_k, values, ids, s);
  if (e != cudaSuccess) return cuda_fail(e, "top-k merge launch");
  return KL_OK;
}

int kl_topk_merge_rows(const int64_t* packed, int rows, int count, int top_k, float* values, int64_t* ids,
                       void* stream) {
  if (!packed || !values || !ids) return fail(KL_ERR_INVALID, "pointers must be non-null");
  if (rows <= 0 || count <= 0) return fail(KL_ERR_INVALID, "need rows > 0 and count > 0");
  if (top_k < 1 || top_k > 8 || top_k > count) return fail(KL_ERR_INVALID, "top_k must be in [1, min(8, count)]");
  const cudaError_t e = launch_topk_merge_rows(packed, rows, count, top_k, values, ids,
                                               static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KL_OK : cuda_fail(e, "top-k merge launch");
}

int kl_rmsnorm(const void* x, const void* residual, const void* weight, int dtype, int rows, int n, float eps,
               int precise, void* y, void* residual_out, void* stream) {
  if (!x || !weight || !y) return fail(KL_ERR_INVALID, "x, weight and y must be non-null");
  if ((residual == nullptr) != (residual_out == nullptr))
    return fail(KL_ERR_INVALID, "residual and residual_out must be given together");
  if (dtype != KL_DT_BF16 && dtype != KL_DT_F16 && dtype != KL_DT_F32) return fail(KL_ERR_INVALID, "unknown dtype %d", dtype);
  if (rows < 0 || n <= 0 || n > KL_RMSNORM_MAX_N)
    return fail(KL_ERR_INVALID, "need rows >= 0 and 0 < n <= %d (n=%d)", KL_RMSNORM_MAX_N, n);
  if (!(eps > 0.0f) || !(eps < 3.0e38f)) return fail(KL_ERR_INVALID, "epsilon must be finite and positive");
  if (rows == 0) return KL_OK;
  const cudaError_t e = launch_rmsnorm(x, residual, weight, dtype, rows, n, eps, precise ? 1 : 0, y, residual_out,
                                       static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KL_OK : cuda_fail(e, "rmsnorm launch");
}

int kl_quantize_w8_row(const void* w, int w_dtype, int n, int k, int8_t* q, void* scale_bf16, void* stream) {
  if (!w || !q || !scale_bf16) return fail(KL_ERR_INVALID, "null pointer");
  if (n <= 0 || k <= 0) return fail(KL_ERR_INVALID, "weight must be a nonempty [N,K] matrix");
  if (w_dtype < KL_DT_BF16 || w_dtype > KL_DT_F32) return fail(KL_ERR_INVALID, "weight dtype");
  const cudaError_t e = launch_quantize_w8_row(w, w_dtype, n, k, q, scale_bf16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KL_OK : cuda_fail(e, "quantize_w8_row");
}

int kl_quantize_w4(const void* w, int w_dtype, int n, int k, int group, int w_format, uint8_t* q, void* scales,
                   void* zeros, void* stream) {
  if (!w || !q || !scales) return fail(KL_ERR_INVALID, "null pointer");
  if (!is_w4(w_format)) return fail(KL_ERR_INVALID, "w_format must be KL_W4_SYM or KL_W4_ASYM");
  if (w_format == KL_W4_ASYM && !zeros) return fail(KL_ERR_INVALID, "zero points required");
  if (n <= 0 || k <= 0 || group <= 0 || group % 2 || k % group)
    return fail(KL_ERR_INVALID, "positive dimensions; an even group must divide K");
  if (w_dtype < KL_DT_BF16 || w_dtype > KL_DT_F32) return fail(KL_ERR_INVALID, "weight dtype");
  const cudaError_t e = launch_quantize_w4(w, w_dtype, n, k, group, w_format, q, scales, zeros,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KL_OK : cuda_fail(e, "quantize_w4");
}

int kl_dequantize(const void* w, int w_format, int n, int k, int group, const void* scales, const void* zeros,
                  const float* inverse, float* out, void* stream) {
  if (!w || !out) return fail(KL_ERR_INVALID, "null pointer");
  if (n <= 0 || k <= 0) return fail(KL_ERR_INVALID, "dimensions must be positive");
  if (w_format < KL_W8_ROW || w_format > KL_BF16_DENSE) return fail(KL_ERR_INVALID, "unknown weight format");
  if (is_grouped(w_format) && (group <= 0 || k % group)) return fail(KL_ERR_INVALID, "group must divide K");
  if (w_format != KL_BF16_DENSE && !scales) return fail(KL_ERR_INVALID, "scales required");
  if (w_format == KL_W8_GROUP && !inverse) return fail(KL_ERR_INVALID, "inverse required");
  if (w_format == KL_W4_ASYM && !zeros) return fail(KL_ERR_INVALID, "zeros required");
  const cudaError_t e = launch_dequantize(w, w_format, n, k, group, scales, zeros, inverse, out,
                                          static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? KL_OK : cuda_fail(e, "dequantize");
}

int kl_device_status(int device, int reset) {
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  int v = 0;
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_status_word, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_status_word, &zero, sizeof(int));
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "device status");
  return v;
}

int kl_describe_plan(int m, int n, int k, int w_format, int swiglu, int flags, int sm_count, int* out) {
  if (!out || sm_count <= 0) return fail(KL_ERR_INVALID, "out and sm_count required");
  std::memset(out, 0, 8 * sizeof(int));
  const int group = is_grouped(w_format) ? 128 : 0;
  const bool tc = !(flags & KL_FLAG_FORCE_SIMT) && tc_shape_ok(k, w_format, 128) && m > 0 && n > 0;
  if (!tc) {
    const GemvPlan gp = plan_gemv(m, swiglu ? n / 2 : n, k, w_format, group > 0 ? group : 1, swiglu != 0, true,
                                  sm_count);
    out[0] = 1;
    out[1] = gp.grid_x * gp.grid_y;
    out[2] = gp.threads;
    out[3] = gp.smem;
    return KL_OK;
  }
  if (prefill_applies(m, k, w_format, sm_count)) {
    PfParams pf;
    std::memset(&pf, 0, sizeof(pf));
    pf.m = m;
    pf.n = n;
    pf.k = k;
    pf.n_out = swiglu ? n / 2 : n;
    prefill_tiles(pf, swiglu != 0, sm_count);
    out[0] = 3;
    out[1] = prefill_grid(pf, sm_count);
    out[2] = prefill_threads();
    out[3] = prefill_smem_bytes(pf.tok);
    out[4] = pf.tok;                    // tokens per tile (pair MMA N)
    out[5] = prefill_w_stages();        // weight stages
    out[6] = pf.n_tiles * pf.m_tiles;
    out[7] = pf.n_tiles * pf.m_tiles * pf.kb_total;
    if (out[1] % 2 || out[1] > (sm_count & ~1) || out[3] > 227 * 1024)
      return fail(KL_ERR_INVALID, "pair plan out of range");
    return KL_OK;
  }
  if ((w_format == KL_W8_ROW || is_w4(w_format)) && !(flags & (KL_FLAG_PERSISTENT | KL_FLAG_FORCE_TC))) {
    const GemvChainPlan gp = plan_gemv_chain(m, n, k, w_format, group, swiglu != 0, sm_count);
    if (gp.ok) {
      out[0] = 5;
      out[1] = gp.grid;
      out[2] = 256;
      out[3] = gp.smem;
      out[4] = gp.mt;
      out[5] = gp.rpw;
      out[6] = gp.rows;
      out[7] = gp.grid;
      const int n_out = swiglu ? n / 2 : n;
      if (gp.grid * gp.rows < n_out || (gp.grid - 1) * gp.rows >= n_out || gp.rows > 8 * gp.rpw ||
          gp.smem > 227 * 1024)
        return fail(KL_ERR_INVALID, "chain GEMV plan out of range");
      return KL_OK;
    }
  }
  if (w_format == KL_W8_ROW && !(flags & KL_FLAG_PERSISTENT)) {
    const ChainPlan cp = plan_chain(m, n, k, swiglu != 0, sm_count);
    if (cp.ok) {
      out[0] = 4;
      out[1] = cp.n_tiles * cp.csize;
      out[2] = 256;
      out[3] = cp.smem;
      out[4] = cp.n_mma;
      out[5] = cp.bpc;
      out[6] = cp.n_tiles;
      out[7] = cp.csize;
      // every K block owned by exactly one CTA of the cluster, none empty
      const int kb = (k + 127) / 128;
      if (cp.csize > kChainMaxCluster || cp.bpc > kChainMaxBlocks || (cp.csize - 1) * cp.bpc >= kb ||
          cp.csize * cp.bpc < kb || cp.smem > 227 * 1024 || out[1] > 2 * sm_count)
        return fail(KL_ERR_INVALID, "chain plan out of range");
      return KL_OK;
    }
  }
  const int mm = is_w4(w_format) ? std::min(m, 64) : m;
  const int n_mma = tc_choose_nmma(mm, w_format);
  TcProblem pr;
  std::memset(&pr, 0, sizeof(pr));
  pr.m = mm;
  pr.n = n;
  pr.k = k;
  pr.n_out = swiglu ? n / 2 : n;
  const int kblk = choose_kblk_single(mm, n, k, w_format, n_mma, swiglu != 0, sm_count, nullptr);
  const long long units = tc_problem_tiles(pr, n_mma, kblk, swiglu != 0);
  const TcPlan plan = plan_tc(n_mma, kblk, units, w_format, sm_count);
  if (!plan.ok) return fail(KL_ERR_UNSUPPORTED, "no tcgen05 plan");
  out[0] = 2;
  out[1] = plan.grid;
  out[2] = tc_threads(w_format, plan.n_mma, plan.kblk);
  out[3] = plan.smem;
  out[4] = plan.n_mma;
  out[5] = plan.w_stages;
  out[6] = pr.m_tiles * pr.n_tiles;
  out[7] = static_cast<int>(plan.units);
  const long long KB = pr.kb_total;
  // Self-check of the stream-K partition used by the kernel.
  const long long G = plan.grid, U = plan.units;
  long long prev_hi = 0;
  for (long long c = 0; c < G; ++c) {
    const long long lo = unit_lo(c, U, G), hi = unit_lo(c + 1, U, G);
    if (lo != prev_hi || hi <= lo) return fail(KL_ERR_INVALID, "partition gap or empty range at CTA %lld", c);
    if (unit_owner(lo, U, G) != c || unit_owner(hi - 1, U, G) != c)
      return fail(KL_ERR_INVALID, "owner mismatch at CTA %lld", c);
    // partial segments of this CTA: at most the first and the last
    int partial = 0;
    for (long long t = lo / KB; t <= (hi - 1) / KB; ++t) {
      const long long s0 = std::max(lo, t * KB), s1 = std::min(hi, (t + 1) * KB);
      if (!(s0 == t * KB && s1 == (t + 1) * KB)) ++partial;
    }
    if (partial > 2) return fail(KL_ERR_INVALID, "CTA %lld has %d partial tiles", c, partial);
    prev_hi = hi;
  }
  if (prev_hi != U) return fail(KL_ERR_INVALID, "partition does not cover all units");
  const size_t ws_need = kCounterBytes + static_cast<size_t>(G) * 2 * plan.n_mma * 128 * sizeof(float);
  if (plan.workspace < ws_need) return fail(KL_ERR_INVALID, "workspace too small for the partition");
  return KL_OK;
}

}  // extern "C"
