// kl_linear_noalloc: the int8 row-scale linear for callers that cannot
// allocate device memory and so have no workspace to hand to kl_linear.
// Examples are an FFI binding that only receives the model's tensors from its
// host runtime and owns no device allocator, or code that runs while another
// library's CUDA-graph capture is in progress, where cudaMalloc is not allowed.
//
// The stream-K tcgen05 kernel needs scratch: per-CTA arrival counters that
// must be zero when a launch starts, and per-CTA f32 partial sums.  Here that
// scratch is one file-scope device array of KL_NOALLOC_SCRATCH_BYTES, enough
// for M <= KL_NOALLOC_MAX_M on devices with up to 160 SMs; every GPU that
// loads the library holds it until the process exits.  In host code the
// array's name is only a host-side stand-in, not a device address, so the
// device address is looked up with cudaGetSymbolAddress once per device, with
// that device current, and that address is what the kernel receives.
#include <algorithm>
#include <mutex>

#include "kl_common.cuh"
#include "kl_internal.h"

namespace kl {
namespace {

static_assert(KL_NOALLOC_SCRATCH_BYTES > kCounterBytes, "scratch holds the counters and the partials");
static_assert(KL_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size");

static __device__ __align__(256) unsigned char g_noalloc_scratch[KL_NOALLOC_SCRATCH_BYTES];

void* g_scratch_addr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// Device address of this device's scratch array (and its SM count), looked up
// on the first call made with the device current.  The address stays valid for
// the life of the device's primary context.
int scratch_address(void** out, int* sm_count) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return report_error(KL_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return report_error(KL_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return report_error(KL_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    int sm = 0;
    e = cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess || sm <= 0)
      return report_error(KL_ERR_CUDA, "cudaDeviceGetAttribute(SM count): %s", cudaGetErrorString(e));
    g_sm_count[dev] = sm;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  *sm_count = g_sm_count[dev];
  return KL_OK;
}

}  // namespace
}  // namespace kl

extern "C" int kl_linear_noalloc(const void* x, int x_dtype, int m, int k, const void* w, int n, const void* scales,
                                 int swiglu, void* y, void* stream) {
  using namespace kl;
  if (m < 1 || m > KL_NOALLOC_MAX_M)
    return report_error(KL_ERR_INVALID, "kl_linear_noalloc takes 1 <= m <= %d tokens (got m=%d); "
                        "larger batches need kl_linear with a caller-owned workspace", KL_NOALLOC_MAX_M, m);
  if (!x || !w || !y || !scales || k <= 0 || n <= 0)
    return report_error(KL_ERR_INVALID, "kl_linear_noalloc: x, w, scales and y must be non-null and k, n positive");
  const size_t need = kl_linear_workspace_bytes(m, n, k, KL_W8_ROW, swiglu, 0);
  if (need > KL_NOALLOC_SCRATCH_BYTES)
    return report_error(KL_ERR_WORKSPACE, "kl_linear_noalloc: this problem needs %zu bytes of scratch, the static "
                        "scratch holds %d bytes (device has too many SMs)", need, KL_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  int sm_count = 0;
  int rc = scratch_address(&scratch, &sm_count);
  if (rc != KL_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (need > 0) {
    // The arrival counters at the start of the scratch must be zero at launch.
    // A finished launch leaves them zero, but one that gave up on a timed-out
    // wait may not, so clear them on the caller's stream every time: one per
    // CTA of a stream-K grid, which has at most one CTA per SM.
    const size_t used = std::min<size_t>(kCounterBytes, (static_cast<size_t>(sm_count) * sizeof(int) + 255) & ~size_t(255));
    const cudaError_t e = cudaMemsetAsync(scratch, 0, used, s);
    if (e != cudaSuccess) return report_error(KL_ERR_CUDA, "cudaMemsetAsync(scratch counters): %s", cudaGetErrorString(e));
  }
  return kl_linear(x, x_dtype, m, k, w, KL_W8_ROW, n, k, scales, nullptr, nullptr, swiglu, y,
                   need > 0 ? scratch : nullptr, need > 0 ? static_cast<size_t>(KL_NOALLOC_SCRATCH_BYTES) : 0, 0,
                   stream);
}
