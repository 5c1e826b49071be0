/*
 * kl_b200.h -- C ABI of the B200 (sm_100a) weight-only quantized linear layer.
 *
 * Plain C: pointers, sizes and integer flags only; no framework types.  All
 * tensor pointers are DEVICE pointers (the caller owns every buffer), except
 * where a comment says otherwise.  `stream` is a cudaStream_t passed as void*
 * (NULL = the legacy default stream).  Every entry point returns a KL_* status
 * and never aborts the process; nothing here allocates device memory, so the
 * calls are safe inside CUDA-graph stream capture.
 *
 * Reference interfaces replaced (paths inside yashlabs-trying/gpu-kernel-lab):
 *   kl_project            <- learning/10_cuda_decode/warp_gemv.cu:56-90  project(x, w, scales,
 *                            inverse, group, warps, persistent, swiglu) (the pybind op, :91)
 *   kl_linear             <- the F.linear call sites the W8A16 op replaces:
 *                            serving/qwen_executor.py:173,227,231-232,238 and the
 *                            nn.Linear patches of profiling/decode_stage2_ablation.py:78-84
 *                            (same math as kl_project, generalised to x[M,K] and all formats)
 *   kl_int4_gemv          <- learning/09_int4/kernels.py:67-74      int4_gemv(x, packed, block_n)
 *   kl_int4_lm_head_topk  <- learning/09_int4/kernels.py:77-99      int4_lm_head_topk(...)
 *   kl_quantize_w8_row    <- learning/10_cuda_decode/activation_int8.py:47-52 with group = K,
 *                            alpha 0, bf16 scale (the BASELINE.json config 0 format)
 *   kl_quantize_w4        <- learning/09_int4/quantization.py:35-62 quantize_int4 (KL_W4_SYM),
 *                            and its asymmetric bf16 scale/zero sibling (KL_W4_ASYM)
 *   kl_dequantize         <- learning/10_cuda_decode/activation_int8.py:63-64 dequantize_int8,
 *                            learning/09_int4/quantization.py:65-71 dequantize_int4
 */
#ifndef KL_B200_H
#define KL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define KL_OK              0
#define KL_ERR_INVALID     1  /* bad argument: shape, dtype, alignment, flag      */
#define KL_ERR_UNSUPPORTED 2  /* valid request this device/build cannot run       */
#define KL_ERR_CUDA        3  /* a CUDA runtime / driver call failed              */
#define KL_ERR_WORKSPACE   4  /* workspace missing or smaller than required       */
#define KL_ERR_TIMEOUT     5  /* a bounded in-kernel wait gave up (device status) */

/* ---- element types --------------------------------------------------- */
#define KL_DT_BF16 0
#define KL_DT_F16  1
#define KL_DT_F32  2

/* ---- weight formats (all row-major [N, K] along K) ------------------- */
#define KL_W8_ROW     0 /* int8 q[N,K]; bf16 scale[N]:               w = q * s[n]           */
#define KL_W8_GROUP   1 /* int8 q[N,K]; f32 scales[N,K/g], f32 inverse[K]:
                           w = q * s[n,k/g] * inverse[k]  (reference CalibratedInt8)       */
#define KL_W4_SYM     2 /* uint8 [N,K/2] two's-complement nibbles, low nibble = even k;
                           f32 scales[N,K/g]: w = c * s  (reference PackedInt4)            */
#define KL_W4_ASYM    3 /* uint8 [N,K/2] unsigned nibbles, low = even k; bf16 scales and
                           bf16 zeros [N,K/g]:  w = (q - z) * s                            */
#define KL_BF16_DENSE 4 /* bf16 w[N,K] (reference project() with a BF16 weight)          */

/* ---- kl_linear flags ------------------------------------------------- */
#define KL_FLAG_FORCE_SIMT    1 /* use the CUDA-core kernel even where tcgen05 applies    */
#define KL_FLAG_FORCE_TC      2 /* require the tcgen05 kernel (KL_ERR_UNSUPPORTED if not)  */
#define KL_FLAG_PDL           4 /* launch with programmatic dependent launch (overlaps the
                                   weight prefetch with the previous kernel on the stream) */
#define KL_FLAG_Y_TRANSPOSED  8 /* write y as [N_out, M] (m contiguous) instead of [M, N_out] */
#define KL_FLAG_PERSISTENT   16 /* int8 decode (M <= 64): use the persistent stream-K kernel even
                                   where the single-tile cluster kernel for dependent chains applies */

/*
 * y = x @ dequant(w)^T   (optionally SwiGLU-fused), fp32 accumulation,
 * output rounded to the activation dtype.
 *   x      [M, K] contiguous, KL_DT_BF16 or KL_DT_F16
 *   w      per w_format; n = weight rows; group = K-group of the scales
 *          (ignored for KL_W8_ROW / KL_BF16_DENSE)
 *   swiglu 0: y is [M, N];  1: gate rows [0, N/2) precede up rows [N/2, N) and
 *          y = bf16(bf16(silu(bf16(gate))) * bf16(up)) is [M, N/2]
 *   workspace  device scratch of kl_linear_workspace_bytes(...) bytes; its first
 *          64 KiB must be zero before the first call on that buffer (the kernels
 *          leave it zero again).  May be NULL when that size is 0.  Calls that
 *          share a workspace must not run concurrently.
 */
int kl_linear(const void* x, int x_dtype, int m, int k,
              const void* w, int w_format, int n, int group,
              const void* scales, const void* zeros, const float* inverse,
              int swiglu, void* y, void* workspace, size_t workspace_bytes,
              int flags, void* stream);

/* Bytes of workspace kl_linear needs for this problem (0 if none). */
size_t kl_linear_workspace_bytes(int m, int n, int k, int w_format, int swiglu, int flags);

/*
 * kl_linear for KL_W8_ROW weights without a workspace argument.  No counterpart
 * in the reference: it serves callers that cannot allocate device memory, such
 * as an FFI binding handed only the model's tensors by a host runtime that owns
 * all device allocation, or code running while another library captures a
 * CUDA graph (cudaMalloc is not allowed then).
 *   Arguments mean what they mean for kl_linear (w_format KL_W8_ROW, no flags).
 *   Scratch: a file-scope device array of KL_NOALLOC_SCRATCH_BYTES inside this
 *     library, held on every GPU that loads it until the process exits.  Enough
 *     for m <= KL_NOALLOC_MAX_M on devices with up to 160 SMs; larger m returns
 *     KL_ERR_INVALID, a device whose plan needs more returns KL_ERR_WORKSPACE.
 *   The first call on each device looks up that device's scratch address (valid
 *     for the life of the device's primary context; a cudaDeviceReset ends it);
 *     make that first call before any stream capture.
 *   Every call clears the scratch's arrival counters on `stream` before the
 *     kernel.  All calls share the one array, so calls that overlap on the GPU
 *     (two streams, two host threads) race; keep them ordered on one stream.
 *   Allocates nothing: no cudaMalloc, no cudaFree, no allocating library call.
 */
#define KL_NOALLOC_MAX_M         64
#define KL_NOALLOC_SCRATCH_BYTES (10 * 1024 * 1024 + 64 * 1024)
int kl_linear_noalloc(const void* x, int x_dtype, int m, int k,
                      const void* w, int n, const void* scales,
                      int swiglu, void* y, void* stream);

/*
 * Grouped launch: many independent GEMMs (same weight format, activation dtype
 * and SwiGLU mode; any shapes) streamed by ONE persistent tcgen05 kernel --
 * no launch gaps, one stream-K partition over the weights of every problem.
 * No reference counterpart: it runs the BASELINE.json config 1 projection
 * set (independent activations per GEMM) as a single unit of work.
 *   1. kl_grouped_encode() builds the problem table in HOST memory
 *      (kl_grouped_table_bytes(count) bytes; TMA descriptors included);
 *   2. the caller copies it to a 64-byte-aligned DEVICE buffer;
 *   3. kl_linear_grouped() launches (both copies are passed: the host copy
 *      for the launch geometry, the device copy for the kernel).
 * Every x / y / w pointer stays fixed for the life of the table.
 */
typedef struct kl_problem {
  const void* x;        /* [m, k] activations                       */
  const void* w;        /* weights in the group's w_format          */
  const void* scales;
  const void* zeros;    /* KL_W4_ASYM only                          */
  void* y;              /* [m, n] or [m, n/2] with swiglu           */
  int m, n, k, group;   /* group: 128 for the 4-bit formats         */
} kl_problem;
size_t kl_grouped_table_bytes(int count);
int kl_grouped_encode(const kl_problem* problems, int count, int x_dtype, int w_format, int swiglu,
                      void* host_table, size_t table_bytes);
size_t kl_grouped_workspace_bytes(const void* host_table);
int kl_linear_grouped(const void* host_table, const void* device_table, void* workspace,
                      size_t workspace_bytes, int flags, void* stream);

/*
 * Int8 tensor-core mode of the grouped launch (bf16 activations; KL_W8_ROW
 * weights, or KL_W4_ASYM weights with group 128 and m <= 16).  No reference
 * counterpart: the same computation as the default mode, with int8 weights fed
 * to tcgen05.mma.kind::i8 unconverted (4-bit codes become the exact int8
 * q - z).
 * kl_linear_grouped then runs two kernels on the stream: a digits pass that
 * writes every token row as a power-of-two scale s_t = 2^(floor(log2 max|x|) - 21)
 * and three int8 planes h, m, l with x = s_t * (65536 h + 256 m + l) (exact
 * for every activation within a factor 2^14 of its token's largest, else
 * within s_t / 2), then the GEMM.  `digits` is a caller-owned, 256-byte-aligned
 * DEVICE buffer of kl_grouped_digits_bytes(...) bytes that stays fixed for
 * the life of the table (its address is in the table's tensor maps); calls
 * that share it must not overlap.  A token whose largest |x| is not finite
 * gets NaN outputs.
 *   flags: KL_GROUPED_INT8_MMA, or 0 for kl_grouped_encode's default mode
 *   (digits ignored).
 */
#define KL_GROUPED_INT8_MMA 1
size_t kl_grouped_digits_bytes(const kl_problem* problems, int count, int flags);
int kl_grouped_encode_ex(const kl_problem* problems, int count, int x_dtype, int w_format, int swiglu, int flags,
                         void* digits, size_t digits_bytes, void* host_table, size_t table_bytes);

/*
 * The reference's op, same arguments and checks (warp_gemv.cu:56-72):
 *   x bf16 [K]; w int8 [N,K] (w_is_int8 = 1, with f32 scales [N,K/group] and
 *   f32 inverse [K]) or bf16 [N,K] (w_is_int8 = 0, scales/inverse ignored);
 *   warps must be 1, 4 or 8; swiglu requires an even N.  y bf16 [N] or [N/2].
 * `warps` / `persistent` are accepted for interface compatibility; the launch
 * geometry is chosen for the B200.
 */
int kl_project(const void* x, int k, const void* w, int w_is_int8,
               const float* scales, const float* inverse, int n, int group,
               int warps, int persistent, int swiglu, void* y,
               void* workspace, size_t workspace_bytes, void* stream);

/* int4_gemv(x, packed, block_n): x bf16/f16 [K]; w KL_W4_SYM; y [N] in x's dtype. */
int kl_int4_gemv(const void* x, int x_dtype, int k, const uint8_t* w, const float* scales,
                 int n, int group, int block_n, void* y, void* stream);

/*
 * int4_lm_head_topk(x, packed, top_k, block_n): fused lm_head projection with
 * tile-local top-k and a global merge.  values f32 [top_k], ids int64 [top_k]
 * (descending; top-1 ties resolve to the lowest vocabulary index).
 * With bf16 x and groups of 128 it runs kl_linear_topk (the logits are never
 * written); other shapes write the logits into the workspace and select.
 * workspace: the larger of kl_int4_lm_head_topk_workspace_bytes(n, top_k,
 * block_n) and, for the fused path, kl_linear_topk_workspace_bytes(1, n, k,
 * KL_W4_SYM, top_k) bytes, under kl_linear's workspace rule (its first 64 KiB
 * zero before the first use; the calls leave it zero).
 */
int kl_int4_lm_head_topk(const void* x, int x_dtype, int k, const uint8_t* w,
                         const float* scales, int n, int group, int top_k, int block_n,
                         float* values, int64_t* ids, void* workspace,
                         size_t workspace_bytes, void* stream);
size_t kl_int4_lm_head_topk_workspace_bytes(int n, int top_k, int block_n);

/* Per-row W8 quantiser: w [N,K] (KL_DT_F32/BF16/F16) -> q int8 [N,K], scale bf16 [N]. */
int kl_quantize_w8_row(const void* w, int w_dtype, int n, int k,
                       int8_t* q, void* scale_bf16, void* stream);

/* 4-bit quantiser, w_format KL_W4_SYM (scales f32, zeros unused) or KL_W4_ASYM
 * (scales and zeros bf16).  q uint8 [N, K/2]. */
int kl_quantize_w4(const void* w, int w_dtype, int n, int k, int group, int w_format,
                   uint8_t* q, void* scales, void* zeros, void* stream);

/* Dequantise any format to f32 out[N,K] with the exact arithmetic the GEMM
 * kernels use (bit-exact against the reference dequantisers). */
int kl_dequantize(const void* w, int w_format, int n, int k, int group,
                  const void* scales, const void* zeros, const float* inverse,
                  float* out, void* stream);

/*
 * Fused lm_head top-k (learning/09_int4/kernels.py:37-50 _head_candidates and
 * :77-99 int4_lm_head_topk, generalised to M tokens, the int8 row format and
 * a vocabulary shard): the logits x @ dequant(w)^T are never written.  Each
 * 128-row tile of the tcgen05 GEMM selects, per token, its top_k rows in the
 * epilogue (values rounded to bf16 as the logits would be, value descending,
 * the lower row first on ties) and a merge kernel reduces the tiles'
 * candidates.
 *   x bf16 [M, K]; w KL_W8_ROW, or KL_W4_SYM / KL_W4_ASYM with group 128 and
 *   M <= 64; 1 <= top_k <= min(8, N); ids are row + index_offset (a shard's
 *   first vocabulary row).
 *   values f32 [M, top_k] and ids int64 [M, top_k]; with values == NULL, ids
 *   receives packed candidates (row << 32 | f32 value bits), the form
 *   kl_topk_merge_rows takes after a gather across ranks.
 *   workspace: kl_linear_topk_workspace_bytes(...) bytes; its first 64 KiB
 *   follow kl_linear's workspace rule (zero before the first use).
 * Returns KL_ERR_UNSUPPORTED for shapes the tcgen05 kernel does not take.
 */
size_t kl_linear_topk_workspace_bytes(int m, int n, int k, int w_format, int top_k);
int kl_linear_topk(const void* x, int x_dtype, int m, int k, const void* w, int w_format, int n, int group,
                   const void* scales, const void* zeros, int top_k, long long index_offset, float* values,
                   int64_t* ids, void* workspace, size_t workspace_bytes, int flags, void* stream);

/* ---- diagnostics -------------------------------------------------------- */
const char* kl_status_string(int status);
/* Message describing the last non-OK status returned on the calling thread. */
const char* kl_last_error(void);
/* Reads the device status word set by bounded in-kernel waits (synchronises
 * the device); reset != 0 clears it.  Returns a KL_* code. */
int kl_device_status(int device, int reset);
/* Version of this library: major*10000 + minor*100 + patch. */
int kl_version(void);

/*
 * Top-k over rows of logits, for lm_heads whose logits are split across GPUs:
 * the candidate and merge stages of learning/09_int4/kernels.py:37-50 and
 * :77-99 (tile-local top-k, then a merge; value descending, the lower index
 * first on ties), generalised to `rows` rows and to an index offset.
 *   kl_topk_rows: logits [rows, ld] (bf16/f16, first n of each row used) ->
 *     values f32 [rows, top_k], ids int64 [rows, top_k] = column + index_offset
 *     (a vocabulary shard passes its first row).  1 <= top_k <= 8.  With
 *     values == NULL, ids receives packed candidates instead: (id << 32) | the
 *     f32 value's bits, one int64 per candidate (ids < 2^31), ready to gather.
 *   kl_topk_merge_rows: packed candidates int64 [rows, count] (every rank's
 *     packed kl_topk_rows output, gathered) -> values f32 / ids int64
 *     [rows, top_k], the rows' global top_k.
 */
size_t kl_topk_rows_workspace_bytes(int rows, int n, int top_k);
int kl_topk_rows(const void* logits, int dtype, int rows, int n, long long ld,
                 long long index_offset, int top_k, float* values, int64_t* ids,
                 void* workspace, size_t workspace_bytes, void* stream);
int kl_topk_merge_rows(const int64_t* packed, int rows, int count, int top_k,
                       float* values, int64_t* ids, void* stream);

/*
 * Qwen RMSNorm of each row of x [rows, n] (bf16, f16 or f32; weight [n] of the
 * same type), optionally fused with the residual add that precedes it.
 *
 * Replaces triton_qwen_rmsnorm and triton_qwen_residual_rmsnorm
 * (learning/03_rmsnorm/qwen_rmsnorm.py:66-131), with the operation order of
 * their kernels (:13-51):
 *   c = T(x + residual), written to residual_out
 *   y = T(T(c * rsqrt(mean(c^2) + eps)) * weight)
 * residual and residual_out are both NULL for the plain norm. With precise != 0
 * the scale is 1/sqrt instead of rsqrt. rows may be 0 (nothing to do). All
 * buffers are contiguous; y and residual_out must not overlap the inputs.
 */
#define KL_RMSNORM_MAX_N 16384
int kl_rmsnorm(const void* x, const void* residual, const void* weight, int dtype,
               int rows, int n, float eps, int precise, void* y, void* residual_out,
               void* stream);

/*
 * Host-only description of the launch plan kl_linear would use on a device
 * with `sm_count` SMs, and a self-check of its work partition (every
 * (tile, k-block) unit covered exactly once, workspace slots in bounds).
 * Needs no GPU.  Returns KL_OK and fills `out` (array of 8 ints:
 * kernel, grid, threads, smem bytes,
 * n_mma (tcgen05 token tile), stages, tiles, units); kernel 1 = CUDA-core GEMV,
 * 2 = tcgen05 stream-K GEMM, 3 = tcgen05 CTA-pair prefill GEMM (int8 row scale, M >= 256),
 * 4 = tcgen05 single-tile cluster GEMM for dependent chains (int8 row scale, M <= 64;
 * there stages = K blocks of 128 per CTA and units = CTAs per cluster),
 * 5 = CUDA-core GEMV for dependent chains (int8 row scale or 4-bit groups of 128
 * as described here, M <= 2; there n_mma = tokens per pass, stages = output rows
 * per warp, tiles = output rows per CTA, units = CTAs).
 * KL_FLAG_FORCE_TC keeps kernels 2-4 (tcgen05) for problems kernel 5 would take.
 */
int kl_describe_plan(int m, int n, int k, int w_format, int swiglu, int flags,
                     int sm_count, int* out);

#ifdef __cplusplus
}
#endif
#endif /* KL_B200_H */
