// Host/device structures shared by the kernels and the C-ABI dispatch layer.
#pragma once
#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace kl {

// ---------------------------------------------------------------- SIMT GEMV
struct GemvArgs {
  const void* x;          // [M, K] activations (bf16 / f16)
  const void* w;          // weights, per format
  const void* scales;
  const void* zeros;
  const float* inverse;
  void* y;                // [M, n_out] or [n_out, M]
  int m, k, n_out, group, kpad, y_transposed;
  long long ldy;          // y row stride (n_out, or the full M when transposed)
};
struct GemvPlan {
  bool vec;               // 16-byte vector kernel (else scalar)
  int mt, grid_x, grid_y, threads, smem, kpad;
};
int chunk_elems(int fmt);
GemvPlan plan_gemv(int m, int n_out, int k, int fmt, int group, bool swiglu, bool aligned, int sm_count);
cudaError_t launch_gemv(const GemvArgs& a, const GemvPlan& p, int fmt, bool swiglu, bool xbf16, cudaStream_t s);

// ------------------------------------------------------------ tcgen05 GEMM
// Swap-AB weight-only GEMM: D[n, m] = W[n, :] . X[m, :] with W (128 rows per
// tile) converted to bf16/f16 into tensor memory as the MMA's A operand and X
// (n_mma tokens per tile) TMA-staged in shared memory as the B operand.
constexpr int kTcRows = 128;          // weight rows per tile (MMA M)
// Block composition is per kernel instantiation (TcRoles in kl_tc_gemm.cu).
constexpr int kCounterBytes = 64 * 1024;
constexpr int kMaxDevices = 64;

// Records a formatted message for kl_last_error() and returns `code`.
int report_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
constexpr int kMaxGroup = 512;        // problems per grouped launch
constexpr int kMaxWStages = 16;

// Internal format id of the int8-MMA mode of KL_W8_ROW weights (kl_tc_i8.cu):
// the activations are split into three int8 digit planes per token and the
// weights feed tcgen05.mma.kind::i8 without conversion.
constexpr int kFmtI8 = 16;
// Internal format id of the int8-MMA mode of asymmetric 4-bit weights
// (KL_W4_ASYM, group 128): nibbles become int8 (q - z) in TMEM, one 128-group
// per stage and accumulator, the same digit planes as kFmtI8.
constexpr int kFmtI8W4 = 17;
// Digit rows of one token tile of T tokens: the h, m and l planes (T rows
// each), padded to a legal MMA N (a multiple of 16).
__host__ __device__ constexpr int i8_tile_rows(int t) { return (3 * t + 15) / 16 * 16; }

// One GEMM of a launch (256-byte aligned so it can live in a device table).
struct alignas(64) TcProblem {
  CUtensorMap tmap_w;                 // int8 [N, K] (box 128 B x 64 rows) or u8 [N, K/2] (64 B x 64 rows)
  CUtensorMap tmap_x;                 // bf16/f16 [M, K] (box 64 elems x n_mma rows), 128B swizzle
  CUtensorMap tmap_z;                 // KL_W4_ASYM two-group stages: bf16 zeros [N, K/128] (box 8 x 64 rows)
  const void* scales;                 // KL_W8_ROW: bf16 [N]; KL_W4_*: per group of 128
  const void* zeros;                  // KL_W4_ASYM: bf16 [N, K/128]
  void* y;
  long long ldy;                      // y row stride: n_out ([M, n_out]) or M ([n_out, M])
  long long unit_begin;               // first global work unit of this problem
  int m, n, k, n_out;                 // n = weight rows, n_out = output columns
  int m_tiles, n_tiles, kb_total;     // kb_total = k blocks per tile
  int y_transposed;
  int vec_store;                      // y 16-byte aligned, ldy % 8 == 0: 16-byte stores (1 row-major, 2 transposed)
  // top-k epilogue (kl_linear_topk): instead of y, each (tile, token) writes its
  // topk best (value, row + index_offset) candidates, packed, at
  // cand[token * cand_ld + n_tile * topk + slot]
  unsigned long long* cand;
  long long index_offset;
  int topk, cand_ld;
  // int8-MMA mode: the bf16 activations x_src [m, k] are split by the digits
  // pass into digits [m_tiles][i8_tile_rows(T)][digits_ld] (h, m, l planes of
  // T rows, zero padding rows) and one power-of-two scale per token,
  // tscale [m_tiles * T]; tmap_x covers digits
  const void* x_src;
  int8_t* digits;
  float* tscale;
  long long digits_ld;
  int tok;                            // token tile T (the MMA's N is i8_tile_rows(T))
};

struct TcParams {
  TcProblem single;                   // the problem when count == 1
  const TcProblem* table;             // device table when count > 1
  int count;
  int w_stages, x_stages;
  long long units;                    // total (tile, k-block) units over all problems
  float* partials;                    // [grid][2][n_mma][128] f32
  int* counters;                      // [grid] split-tile arrival counters (zero between calls)
  int* status;                        // device status word (bounded-wait failures)
};

struct TcPlan {
  bool ok;
  int n_mma, kblk, w_stages, x_stages, grid, smem;
  long long units;
  size_t workspace;                   // counters + partials
};
int tc_choose_nmma(int m, int fmt);
int tc_threads(int fmt, int n_mma, int kblk);  // block size of the tcgen05 kernel
// Fill the tiling fields of a problem (m_tiles, n_tiles, kb_total) for K blocks
// of kblk elements; returns its unit count.
long long tc_problem_tiles(TcProblem& pr, int n_mma, int kblk, bool swiglu);
// K elements per pipeline stage: 256 for the int8 decode path when the work
// keeps every SM busy (fewer hand-offs per byte), else 128.
int tc_choose_kblk(int fmt, int n_mma, long long units_at_256, int sm_count);
TcPlan plan_tc(int n_mma, int kblk, long long units, int fmt, int sm_count);
// epilogue: 0 outputs, 1 SwiGLU outputs, 2 top-k candidates (TcProblem::cand)
constexpr int kEpiPlain = 0, kEpiSwiglu = 1, kEpiTopk = 2;
cudaError_t launch_tc(const TcParams& p, const TcPlan& plan, int fmt, int epi, bool xbf16, bool pdl, cudaStream_t s);
// int8-MMA mode (kl_tc_i8.cu): token tile T in {8, 16, 32, 64}.
int tc_choose_tokens_i8(int m);
int tc_threads_i8();
// The digits pass over every problem of a launch (host_tab: the problems, for
// the grid; dev_tab: the same table in device memory, or null for one problem
// passed by value), then the GEMM.
cudaError_t launch_act_digits(const TcProblem* dev_tab, const TcProblem& single, int count, int rows_max,
                              bool pdl, cudaStream_t s);
cudaError_t launch_tc_i8(const TcParams& p, const TcPlan& plan, int fmt, int epi, bool pdl, cudaStream_t s);

// ---- dependent-chain decode GEMM: one 128-row tile per cluster (kl_tc_chain.cu)
// For one int8 row-scale linear with M <= 64 launched after the op that
// produces its input: the CTAs of a cluster split the tile's K range, stream
// their weights and convert them into tensor memory before the programmatic
// dependent-launch wait, and reduce the K-split partial sums through
// distributed shared memory after it.
constexpr int kChainMaxM = 64;
constexpr int kChainMaxCluster = 8;   // portable cluster sizes only
constexpr int kChainMaxBlocks = 8;    // 128-wide K blocks per CTA
struct ChainParams {
  CUtensorMap tmap_w;                 // int8 [N, K], box 128 B x 64 rows, 128B swizzle
  CUtensorMap tmap_x;                 // bf16/f16 [M, K], box 64 elems x n_mma rows, 128B swizzle
  const void* scales;                 // bf16 [N]
  void* y;
  long long ldy;
  int m, n, k, n_out;
  int kb_total;                       // 128-wide K blocks of the problem
  int bpc;                            // K blocks per CTA (the last CTA of a cluster may have fewer)
  int csize;                          // CTAs per cluster = K splits of a tile
  int y_transposed;
  int* status;
};
struct ChainPlan {
  bool ok;
  int n_mma, bpc, csize, n_tiles, smem;
};
ChainPlan plan_chain(int m, int n, int k, bool swiglu, int sm_count);
cudaError_t launch_chain(const ChainParams& p, const ChainPlan& plan, bool swiglu, bool xbf16, bool pdl,
                         cudaStream_t s);

// ---- dependent-chain decode GEMV on CUDA cores for one or two tokens (kl_gemv_chain.cu)
constexpr int kGemvChainMaxM = 2;
constexpr int kGemvChainMinSmem = 80 * 1024;   // at most two CTAs per SM
constexpr int kGemvChainMaxSmem = 227 * 1024;
struct GemvChainParams {
  const void* w;                      // int8 [N, K] or packed 4-bit [N, K/2]
  const void* scales;                 // bf16 [N] (int8 rows); bf16 / f32 [N, K/group] (4-bit)
  const void* zeros;                  // bf16 [N, K/group] (asymmetric 4-bit), else unused
  const void* x;                      // [M, K] bf16/f16
  void* y;
  long long ldy;
  int m, k, n, n_out, group;
  int rows;                           // output rows per CTA
  int y_transposed;
  int* status;
};
struct GemvChainPlan {
  bool ok;
  int mt, rows, grid, smem;
  int rpw;                            // output rows per warp (4, or 8 above 32 rows per CTA)
};
// Formats: KL_W8_ROW, KL_W4_ASYM, KL_W4_SYM (group a multiple of 16 dividing K).
GemvChainPlan plan_gemv_chain(int m, int n, int k, int w_format, int group, bool swiglu, int sm_count);
cudaError_t launch_gemv_chain(const GemvChainParams& p, const GemvChainPlan& plan, int w_format, bool swiglu,
                              bool xbf16, bool pdl, cudaStream_t s);

// ---- prefill: int8 row-scale GEMM on CTA pairs (kl_tc_prefill.cu)
constexpr int kPrefillMinM = 256;     // token count from which kl_linear uses the pair kernel
struct PfParams {
  CUtensorMap tmap_w;                 // int8 [N, K], box 128 x 64 rows, 128B swizzle
  CUtensorMap tmap_x;                 // bf16/f16 [M, K], box 64 x (tok / 2) rows, 128B swizzle
  const void* scales;                 // bf16 [N]
  void* y;
  long long ldy;
  int m, n, k, n_out;
  int n_tiles, m_tiles, kb_total;
  int tok;                            // tokens per tile: 192, 128 or 64 (the x tensor map's box is tok / 2 rows)
  int y_transposed;
  int vec_store;                      // y 16-byte aligned, ldy % 8 == 0: 16-byte stores (1 row-major, 2 transposed)
  int* status;
  int tile_begin;                     // grouped launches: first global tile of this problem
};
// One launch of the pair kernel: one problem, or a device table of problems
// (same SwiGLU mode, activation type and token tile) whose tiles are dealt out
// round-robin to the CTA pairs as one sequence.
struct PfLaunch {
  PfParams single;                    // the problem when count == 1
  const PfParams* table;              // device table when count > 1 (64-byte-aligned entries)
  int count;
  int tiles;                          // tiles of all problems
  int* status;
};
int prefill_threads();
int prefill_w_stages();               // weight-ring depth of the pair kernel
int prefill_smem_bytes(int tok);
int prefill_k_block();
int prefill_choose_tokens(int m, int n_tiles, int sm_count);
void prefill_tiles(PfParams& p, bool swiglu, int sm_count);
int prefill_grid(const PfParams& p, int sm_count);
cudaError_t launch_prefill(const PfParams& p, int grid, bool swiglu, bool xbf16, bool pdl, cudaStream_t s);
// Token tile for a group of problems (fills each problem's n_tiles / m_tiles /
// kb_total / tok / tile_begin; returns the total tiles).
int prefill_group_tiles(PfParams* probs, int count, bool swiglu, int sm_count);
cudaError_t launch_prefill_group(const PfLaunch& l, int grid, bool swiglu, bool xbf16, bool pdl, cudaStream_t s);

// Work partition shared by the kernel and the host-side self-check:
// CTA c owns units [lo(c), lo(c+1)) with lo(c) = floor(c * units / grid).
__host__ __device__ inline long long unit_lo(long long c, long long units, long long grid) {
  return (c * units) / grid;
}
// Owner CTA of unit u: the largest c with lo(c) <= u.
__host__ __device__ inline long long unit_owner(long long u, long long units, long long grid) {
  return ((u + 1) * grid + units - 1) / units - 1;
}

// ------------------------------------------------------------------ top-k
// Per-row top-k over logits rows (value descending, lower index first on ties).
size_t head_topk_candidate_bytes(int n, int top_k);
size_t topk_rows_candidate_bytes(int rows, int n, int top_k);
// packed_out: ids receives (id << 32 | f32 value bits) pairs and values is unused
cudaError_t launch_topk_rows(const void* logits, bool xbf16, int rows, int n, long long ld, long long index_offset,
                             int top_k, void* cand, float* values, int64_t* ids, cudaStream_t s, bool packed_out);
// Qwen RMSNorm (kl_rmsnorm.cu); residual/residual_out both null for the plain norm
cudaError_t launch_rmsnorm(const void* x, const void* residual, const void* weight, int dtype, int rows, int n,
                           float eps, int precise, void* y, void* residual_out, cudaStream_t s);
// values == nullptr: ids receives the merged candidates packed (for a gather across ranks)
cudaError_t launch_topk_merge_rows(const int64_t* packed, int rows, int count, int top_k, float* values, int64_t* ids,
                                   cudaStream_t s);

// ---------------------------------------------------------- quantisation
cudaError_t launch_quantize_w8_row(const void* w, int w_dtype, int n, int k, int8_t* q, void* scale, cudaStream_t s);
cudaError_t launch_quantize_w4(const void* w, int w_dtype, int n, int k, int group, int fmt,
                               uint8_t* q, void* scales, void* zeros, cudaStream_t s);
cudaError_t launch_dequantize(const void* w, int fmt, int n, int k, int group, const void* scales,
                              const void* zeros, const float* inverse, float* out, cudaStream_t s);

}  // namespace kl
