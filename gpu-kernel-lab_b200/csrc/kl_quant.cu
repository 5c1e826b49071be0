// Quantisers, the exact dequantiser, and the lm_head top-k selection kernels.
//
// Quantisers (offline weight packing, run once per weight on the GPU):
//   * per-row int8 with a bf16 scale -- reference
//     learning/10_cuda_decode/activation_int8.py:47-52 with group = K and
//     channel 1, the scale rounded to bf16 and used for q;
//   * symmetric int4 -- reference learning/09_int4/quantization.py:51-61;
//   * asymmetric int4 with bf16 scale and zero point.
// All use IEEE division and round-half-to-even (torch's round), so the codes
// match the reference's CPU quantisers bit for bit.
//
// Dequantiser: the exact f32 weights the GEMM kernels multiply, in the
// reference's operation order (q*s*inverse; signed*s; (q-z)*s).
//
// Top-k: per-block candidates then a one-block merge, ordered by (value
// descending, index ascending) -- for top-1 that is the reference's
// lowest-index tie rule (learning/09_int4/kernels.py:47-50,97).
#include "kl_common.cuh"
#include "kl_internal.h"

namespace kl {

namespace {

KL_DEVICE float load_w(const void* w, int dt, long long i) {
  if (dt == KL_DT_F32) return reinterpret_cast<const float*>(w)[i];
  if (dt == KL_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[i]);
  return __half2float(reinterpret_cast<const __half*>(w)[i]);
}

KL_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
KL_DEVICE float warp_min(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One CTA (256 threads) per weight row.
__global__ void __launch_bounds__(256) quant_w8_row_kernel(const void* w, int dt, int k, int8_t* q,
                                                           __nv_bfloat16* scale) {
  __shared__ float red[8];
  const long long base = static_cast<long long>(blockIdx.x) * k;
  float amax = 0.f;
  for (int i = threadIdx.x; i < k; i += blockDim.x) amax = fmaxf(amax, fabsf(load_w(w, dt, base + i)));
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  float s = __fdiv_rn(red[0], 127.0f);
  if (s == 0.f) s = 1.0f;
  const __nv_bfloat16 sb = __float2bfloat16_rn(s);
  const float sf = __bfloat162float(sb);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const float v = rintf(__fdiv_rn(load_w(w, dt, base + i), sf));
    q[base + i] = static_cast<int8_t>(fminf(fmaxf(v, -127.f), 127.f));
  }
  if (threadIdx.x == 0) scale[blockIdx.x] = sb;
}

// grid (N, ceil(groups / 8)); each warp owns one (row, group).
__global__ void __launch_bounds__(256) quant_w4_kernel(const void* w, int dt, int k, int group, int fmt,
                                                       uint8_t* q, void* scales, void* zeros) {
  const int row = blockIdx.x;
  const int g = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int groups = k / group;
  if (g >= groups) return;
  const long long base = static_cast<long long>(row) * k + static_cast<long long>(g) * group;
  float lo = INFINITY, hi = -INFINITY, amax = 0.f;
  for (int i = lane; i < group; i += 32) {
    const float v = load_w(w, dt, base + i);
    lo = fminf(lo, v);
    hi = fmaxf(hi, v);
    amax = fmaxf(amax, fabsf(v));
  }
  lo = warp_min(lo);
  hi = warp_max(hi);
  amax = warp_max(amax);
  const long long si = static_cast<long long>(row) * groups + g;
  uint8_t* qrow = q + static_cast<long long>(row) * (k / 2) + static_cast<long long>(g) * (group / 2);
  if (fmt == KL_W4_SYM) {
    float s = __fdiv_rn(amax, 7.0f);
    if (s == 0.f) s = 1.0f;
    for (int i = lane; i < group / 2; i += 32) {
      const float a = fminf(fmaxf(rintf(__fdiv_rn(load_w(w, dt, base + 2 * i), s)), -7.f), 7.f);
      const float b = fminf(fmaxf(rintf(__fdiv_rn(load_w(w, dt, base + 2 * i + 1), s)), -7.f), 7.f);
      const int ca = static_cast<int>(a) & 15, cb = static_cast<int>(b) & 15;
      qrow[i] = static_cast<uint8_t>(ca | (cb << 4));
    }
    if (lane == 0) reinterpret_cast<float*>(scales)[si] = s;
  } else {
    float s = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
    if (s == 0.f) s = 1.0f;
    const __nv_bfloat16 sb = __float2bfloat16_rn(s);
    const float sf = __bfloat162float(sb);
    const float z = fminf(fmaxf(rintf(__fdiv_rn(-lo, sf)), 0.f), 15.f);
    for (int i = lane; i < group / 2; i += 32) {
      const float a = fminf(fmaxf(__fadd_rn(rintf(__fdiv_rn(load_w(w, dt, base + 2 * i), sf)), z), 0.f), 15.f);
      const float b = fminf(fmaxf(__fadd_rn(rintf(__fdiv_rn(load_w(w, dt, base + 2 * i + 1), sf)), z), 0.f), 15.f);
      qrow[i] = static_cast<uint8_t>(static_cast<int>(a) | (static_cast<int>(b) << 4));
    }
    if (lane == 0) {
      reinterpret_cast<__nv_bfloat16*>(scales)[si] = sb;
      reinterpret_cast<__nv_bfloat16*>(zeros)[si] = __float2bfloat16_rn(z);
    }
  }
}

__global__ void dequant_kernel(const void* w, int fmt, int n, int k, int group, const void* scales,
                               const void* zeros, const float* inverse, float* out) {
  const long long total = static_cast<long long>(n) * k;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / k;
    const int col = static_cast<int>(i % k);
    float v;
    switch (fmt) {
      case KL_W8_ROW:
        v = __fmul_rn(static_cast<float>(static_cast<const int8_t*>(w)[i]),
                      __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(scales)[row]));
        break;
      case KL_W8_GROUP: {
        const float s = reinterpret_cast<const float*>(scales)[row * (k / group) + col / group];
        v = __fmul_rn(__fmul_rn(static_cast<float>(static_cast<const int8_t*>(w)[i]), s), inverse[col]);
        break;
      }
      case KL_W4_SYM: case KL_W4_ASYM: {
        const uint8_t b = static_cast<const uint8_t*>(w)[row * (k / 2) + col / 2];
        const int code = (col & 1) ? (b >> 4) : (b & 15);
        const long long si = row * (k / group) + col / group;
        if (fmt == KL_W4_SYM) {
          v = __fmul_rn(static_cast<float>(code >= 8 ? code - 16 : code), reinterpret_cast<const float*>(scales)[si]);
        } else {
          const float z = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(zeros)[si]);
          v = __fmul_rn(__fsub_rn(static_cast<float>(code), z),
                        __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(scales)[si]));
        }
        break;
      }
      default:
        v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[i]);
    }
    out[i] = v;
  }
}

// (value desc, index asc) total order.
KL_DEVICE bool better(float va, long long ia, float vb, long long ib) {
  return va > vb || (va == vb && ia < ib);
}

constexpr int kTopkPerThread = 4;
constexpr int kTopkThreads = 256;
constexpr int kTopkBlockItems = kTopkPerThread * kTopkThreads;

// Block-wide arg-best of one candidate per thread.
KL_DEVICE void block_best(float& v, long long& idx, float* sv, long long* si) {
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const long long oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (better(ov, oi, v, idx)) { v = ov; idx = oi; }
  }
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) { sv[w] = v; si[w] = idx; }
  __syncthreads();
  v = sv[0];
  idx = si[0];
  for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i)
    if (better(sv[i], si[i], v, idx)) { v = sv[i]; idx = si[i]; }
}

// Stage 1: logits (activation dtype) -> per-block top-k candidates, one row of
// logits per blockIdx.y (row stride `ld` elements); candidate ids are the
// element index plus `index_offset` (a vocabulary shard's first row).
template <bool XBF16>
__global__ void __launch_bounds__(kTopkThreads) topk_candidates_kernel(const void* logits, int n, long long ld,
                                                                       long long index_offset, int top_k,
                                                                       float* cand_v, long long* cand_i) {
  __shared__ float sv[32];
  __shared__ long long si[32];
  float v[kTopkPerThread];
  long long id[kTopkPerThread];
  const long long row = blockIdx.y;
  const long long base = static_cast<long long>(blockIdx.x) * kTopkBlockItems;
  const long long row0 = row * ld;
#pragma unroll
  for (int j = 0; j < kTopkPerThread; ++j) {
    const long long i = base + j * kTopkThreads + threadIdx.x;
    id[j] = i + index_offset;
    v[j] = i < n ? load_act<XBF16>(logits, row0 + i) : -INFINITY;
    if (i >= n) id[j] = 0x7fffffffffffffffll;
  }
  cand_v += (row * gridDim.x) * top_k;
  cand_i += (row * gridDim.x) * top_k;
  for (int r = 0; r < top_k; ++r) {
    float bv = -INFINITY;
    long long bi = 0x7fffffffffffffffll;
#pragma unroll
    for (int j = 0; j < kTopkPerThread; ++j)
      if (better(v[j], id[j], bv, bi)) { bv = v[j]; bi = id[j]; }
    block_best(bv, bi, sv, si);
#pragma unroll
    for (int j = 0; j < kTopkPerThread; ++j)
      if (id[j] == bi) { v[j] = -INFINITY; id[j] = 0x7fffffffffffffffll; }
    if (threadIdx.x == 0) {
      cand_v[blockIdx.x * top_k + r] = bv;
      cand_i[blockIdx.x * top_k + r] = bi;
    }
  }
}

// A (value, id) candidate packed in 64 bits: id in the high word, the f32
// value's bits in the low word (ids < 2^31).
KL_DEVICE long long pack_cand(float v, long long id) {
  return static_cast<long long>(static_cast<unsigned long long>(id) << 32 |
                                static_cast<unsigned long long>(__float_as_uint(v)));
}
KL_DEVICE float cand_value(long long p) { return __uint_as_float(static_cast<unsigned>(p & 0xFFFFFFFFll)); }
KL_DEVICE long long cand_id(long long p) { return static_cast<long long>(static_cast<unsigned long long>(p) >> 32); }

// Stage 2: one block per row merges that row's `count` candidates, given as
// separate arrays or packed (PACKED_IN), and writes the row's top-k as values +
// ids, or packed (PACKED_OUT, for an all-gather across ranks).
template <bool PACKED_IN, bool PACKED_OUT>
__global__ void __launch_bounds__(kTopkThreads) topk_merge_kernel(const float* cand_v, const long long* cand_i,
                                                                  int count, int top_k, float* values, int64_t* ids) {
  __shared__ float sv[32];
  __shared__ long long si[32];
  __shared__ long long chosen[8];
  const long long row = blockIdx.x;
  if constexpr (!PACKED_IN) cand_v += row * count;
  cand_i += row * count;
  if constexpr (!PACKED_OUT) values += row * top_k;
  ids += row * top_k;
  for (int r = 0; r < top_k; ++r) {
    float bv = -INFINITY;
    long long bi = 0x7fffffffffffffffll;
    for (int i = threadIdx.x; i < count; i += blockDim.x) {
      const float cv = PACKED_IN ? cand_value(cand_i[i]) : cand_v[i];
      const long long ci = PACKED_IN ? cand_id(cand_i[i]) : cand_i[i];
      bool taken = false;
      for (int q = 0; q < r; ++q) taken |= (ci == chosen[q]);
      if (!taken && better(cv, ci, bv, bi)) { bv = cv; bi = ci; }
    }
    block_best(bv, bi, sv, si);
    if (threadIdx.x == 0) {
      chosen[r] = bi;
      if constexpr (PACKED_OUT) {
        ids[r] = pack_cand(bv, bi);
      } else {
        values[r] = bv;
        ids[r] = bi;
      }
    }
    __syncthreads();
  }
}

// Merge of packed candidates in one pass.  A candidate's sort key is the
// order-preserving bits of its value (zero of either sign as +0) above the
// inverted id, so a larger key is the better candidate and ties go to the
// lower id.  Each thread keeps its best kMergeK keys sorted in registers; then
// top_k rounds pick the block's best head and its owner pops it.
constexpr int kMergeK = 8;
KL_DEVICE unsigned long long merge_key(long long packed) {
  uint32_t u = static_cast<uint32_t>(packed & 0xFFFFFFFFll);
  if ((u & 0x7FFFFFFFu) == 0u) u = 0u;
  const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  const uint32_t id = static_cast<uint32_t>(static_cast<unsigned long long>(packed) >> 32);
  return (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFu - id);
}
KL_DEVICE float merge_key_value(unsigned long long key) {
  const uint32_t ord = static_cast<uint32_t>(key >> 32);
  return __uint_as_float((ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord);
}
KL_DEVICE long long merge_key_id(unsigned long long key) {
  return static_cast<long long>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull));
}

template <bool PACKED_OUT, int NT>
__global__ void __launch_bounds__(NT) topk_merge_packed_kernel(const long long* cand, int count, int top_k,
                                                               float* values, int64_t* ids) {
  __shared__ unsigned long long wbest[2][NT / 32];
  const long long row = blockIdx.x;
  cand += row * count;
  unsigned long long best[kMergeK];
#pragma unroll
  for (int j = 0; j < kMergeK; ++j) best[j] = 0ull;
  constexpr int kBatch = 8;                // loads in flight per thread
  for (int base = threadIdx.x; base < count; base += NT * kBatch) {
    long long c[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = base + u * NT;
      c[u] = i < count ? __ldg(cand + i) : 0ll;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const unsigned long long key = base + u * NT < count ? merge_key(c[u]) : 0ull;
      if (key > best[kMergeK - 1]) {
        best[kMergeK - 1] = key;
#pragma unroll
        for (int j = kMergeK - 1; j > 0; --j) {
          if (best[j] > best[j - 1]) {
            const unsigned long long t = best[j];
            best[j] = best[j - 1];
            best[j - 1] = t;
          }
        }
      }
    }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int r = 0; r < top_k; ++r) {
    unsigned long long m = best[0];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, m, o);
      m = other > m ? other : m;
    }
    if (lane == 0) wbest[r & 1][w] = m;
    __syncthreads();                     // the other buffer is rewritten only after the next barrier
    m = wbest[r & 1][0];
#pragma unroll
    for (int i = 1; i < NT / 32; ++i) m = wbest[r & 1][i] > m ? wbest[r & 1][i] : m;
    if (best[0] == m && m != 0ull) {     // keys are unique: one owner pops its head
#pragma unroll
      for (int j = 0; j < kMergeK - 1; ++j) best[j] = best[j + 1];
      best[kMergeK - 1] = 0ull;
    }
    if (threadIdx.x == 0) {
      const float v = merge_key_value(m);
      const long long id = merge_key_id(m);
      if constexpr (PACKED_OUT) {
        ids[row * top_k + r] = pack_cand(v, id);
      } else {
        values[row * top_k + r] = v;
        ids[row * top_k + r] = id;
      }
    }
  }
}

}  // namespace

cudaError_t launch_quantize_w8_row(const void* w, int w_dtype, int n, int k, int8_t* q, void* scale, cudaStream_t s) {
  quant_w8_row_kernel<<<n, 256, 0, s>>>(w, w_dtype, k, q, reinterpret_cast<__nv_bfloat16*>(scale));
  return cudaGetLastError();
}

cudaError_t launch_quantize_w4(const void* w, int w_dtype, int n, int k, int group, int fmt,
                               uint8_t* q, void* scales, void* zeros, cudaStream_t s) {
  const int groups = k / group;
  quant_w4_kernel<<<dim3(n, (groups + 7) / 8), 256, 0, s>>>(w, w_dtype, k, group, fmt, q, scales, zeros);
  return cudaGetLastError();
}

cudaError_t launch_dequantize(const void* w, int fmt, int n, int k, int group, const void* scales,
                              const void* zeros, const float* inverse, float* out, cudaStream_t s) {
  const long long total = static_cast<long long>(n) * k;
  const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148ll * 16));
  dequant_kernel<<<blocks, 256, 0, s>>>(w, fmt, n, k, group, scales, zeros, inverse, out);
  return cudaGetLastError();
}

size_t head_topk_candidate_bytes(int n, int top_k) {
  const long long blocks = (static_cast<long long>(n) + kTopkBlockItems - 1) / kTopkBlockItems;
  return static_cast<size_t>(blocks) * top_k * (sizeof(float) + sizeof(long long)) + 256;
}

cudaError_t launch_topk(const void* logits, bool xbf16, int n, int top_k, void* cand, float* values,
                        int64_t* ids, cudaStream_t s) {
  return launch_topk_rows(logits, xbf16, 1, n, n, 0, top_k, cand, values, ids, s, false);
}

size_t topk_rows_candidate_bytes(int rows, int n, int top_k) {
  return static_cast<size_t>(rows) * (head_topk_candidate_bytes(n, top_k) - 256) + 256;
}

cudaError_t launch_topk_rows(const void* logits, bool xbf16, int rows, int n, long long ld, long long index_offset,
                             int top_k, void* cand, float* values, int64_t* ids, cudaStream_t s, bool packed_out) {
  const int blocks = (n + kTopkBlockItems - 1) / kTopkBlockItems;
  float* cv = reinterpret_cast<float*>(cand);
  long long* ci = reinterpret_cast<long long*>(
      (reinterpret_cast<uintptr_t>(cv + static_cast<size_t>(rows) * blocks * top_k) + 15) & ~uintptr_t(15));
  const dim3 grid(blocks, rows);
  if (xbf16) topk_candidates_kernel<true><<<grid, kTopkThreads, 0, s>>>(logits, n, ld, index_offset, top_k, cv, ci);
  else topk_candidates_kernel<false><<<grid, kTopkThreads, 0, s>>>(logits, n, ld, index_offset, top_k, cv, ci);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (packed_out) topk_merge_kernel<false, true><<<rows, kTopkThreads, 0, s>>>(cv, ci, blocks * top_k, top_k, values, ids);
  else topk_merge_kernel<false, false><<<rows, kTopkThreads, 0, s>>>(cv, ci, blocks * top_k, top_k, values, ids);
  return cudaGetLastError();
}

cudaError_t launch_topk_merge_rows(const int64_t* packed, int rows, int count, int top_k, float* values, int64_t* ids,
                                   cudaStream_t s) {
  const long long* in = reinterpret_cast<const long long*>(packed);
  // (1024-thread blocks measured slower for a single row: the rounds' block reductions cost more)
  if (values) topk_merge_packed_kernel<false, kTopkThreads><<<rows, kTopkThreads, 0, s>>>(in, count, top_k, values, ids);
  else topk_merge_packed_kernel<true, kTopkThreads><<<rows, kTopkThreads, 0, s>>>(in, count, top_k, nullptr, ids);
  return cudaGetLastError();
}

}  // namespace kl
