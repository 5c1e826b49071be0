// Shared device helpers for the B200 (sm_100a) quantized-linear kernels:
// status codes, bf16 bit tricks, and thin inline-PTX wrappers for mbarriers,
// TMA (cp.async.bulk.tensor), tcgen05 (TMEM alloc / ld / st / mma / commit)
// and programmatic dependent launch.  Every spin-wait here is bounded: it
// gives up after a wall-clock limit, records an error code in a device status
// word and returns false, so no kernel in this library can hang a GPU.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kl_b200.h"

#define KL_DEVICE __device__ __forceinline__

namespace kl {

// Wall-clock limit for any single wait inside a kernel (nanoseconds).  Normal
// waits last nanoseconds to microseconds; this only fires if a producer never
// arrives (a logic error), turning a would-be hang into an error status.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;   // 2 s

KL_DEVICE unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Record a KL_ERR_* code in the device status word (first error wins).
KL_DEVICE void record_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

KL_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
KL_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}
KL_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
KL_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}
KL_DEVICE void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
KL_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Wait, bounded by time only, for the phase with the given parity to complete
// (used on teardown paths).  Returns false if the limit passed first.
KL_DEVICE bool mbar_wait_time(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 255u) == 0 && globaltimer() - t0 > kWaitLimitNs) return false;
  }
}

// ----------------------------------------------------------------------- TMA
KL_DEVICE void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];"
      :: "r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar) : "memory");
}
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from
// global memory into this CTA's shared memory, counted on an mbarrier.
KL_DEVICE void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
// Prefetch a tile of a tensor into L2 (no shared memory, no completion signal).
KL_DEVICE void tma_prefetch_l2_2d(const CUtensorMap* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" :: "l"(map), "r"(x), "r"(y) : "memory");
}
KL_DEVICE void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" :: "l"(map) : "memory");
}

// -------------------------------------------------- programmatic dependent launch
KL_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
KL_DEVICE void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------- tcgen05
KL_DEVICE void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(dst_smem), "r"(ncols) : "memory");
}
KL_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
KL_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
KL_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KL_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
KL_DEVICE void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
KL_DEVICE void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc]; kind::f16 (bf16/f16 inputs, f32 accumulate).
KL_DEVICE void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
      :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// High word of a SW128 K-major shared-memory descriptor (SBO 1024 B, version 1,
// SWIZZLE_128B); smem_desc_sw128_lo below builds the low word.
constexpr uint32_t kSmemDescSw128Hi = (1024u >> 4) | (1u << 14) | (2u << 29);
// tc_mma_ts with the B descriptor given as (low word, constant high word).
KL_DEVICE void tc_mma_ts_lo(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_desc_lo, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n .reg .b64 bd;\n setp.ne.b32 p, %5, 0;\n mov.b64 bd, {%2, %3};\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %4, p;\n}"
      :: "r"(d_tmem), "r"(a_tmem), "r"(b_desc_lo), "n"(kSmemDescSw128Hi), "r"(idesc), "r"(accumulate) : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]; kind::i8 (signed 8-bit A and B,
// s32 accumulate).  Both descriptors are SW128 K-major, given by their low
// words (the high word is kSmemDescSw128Hi).
KL_DEVICE void tc_mma_ss_i8(uint32_t d_tmem, uint32_t a_desc_lo, uint32_t b_desc_lo, uint32_t idesc,
                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n .reg .b64 ad, bd;\n setp.ne.b32 p, %4, 0;\n mov.b64 ad, {%1, %5};\n"
      " mov.b64 bd, {%2, %5};\n tcgen05.mma.cta_group::1.kind::i8 [%0], ad, bd, %3, p;\n}"
      :: "r"(d_tmem), "r"(a_desc_lo), "r"(b_desc_lo), "r"(idesc), "r"(accumulate), "n"(kSmemDescSw128Hi)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]; kind::i8 (A: four signed 8-bit values
// per TMEM column along K; B: SW128 K-major, low descriptor word given).
KL_DEVICE void tc_mma_ts_i8_lo(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_desc_lo, uint32_t idesc,
                               uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n .reg .b64 bd;\n setp.ne.b32 p, %5, 0;\n mov.b64 bd, {%2, %3};\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], bd, %4, p;\n}"
      :: "r"(d_tmem), "r"(a_tmem), "r"(b_desc_lo), "n"(kSmemDescSw128Hi), "r"(idesc), "r"(accumulate) : "memory");
}
// ------------------------------------------------ CTA pairs (cta_group::2)
// A 2-CTA cluster whose tensor cores run one MMA over both CTAs' operands.
KL_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared-memory address of the same variable in CTA `rank` of the cluster.
KL_DEVICE uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(addr), "r"(rank));
  return d;
}
// Arrive on an mbarrier that may live in another CTA of the cluster.  The
// default (.release at CTA scope) form: TMEM writes are ordered by the
// tcgen05 fences around the signal, and a cluster-scope release would also
// wait for every outstanding memory operation of the thread (~1300 cycles
// per arrive measured here).
KL_DEVICE void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}
KL_DEVICE bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// All threads of all CTAs of the cluster (start-up / teardown only).
KL_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of a cluster barrier phase, executed per thread (not warp-aligned):
// every thread of the cluster arrives once per phase, and waits before arriving again.
KL_DEVICE void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
KL_DEVICE void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
// Arrive without ordering this thread's earlier memory operations (a release at
// cluster scope waits for all of them).
KL_DEVICE void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads of them (a bulk copy issued after a barrier).
KL_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from
// this CTA's shared memory into another CTA's (cluster address), counted on an
// mbarrier of the destination CTA (cluster address).
KL_DEVICE void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes, uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(dst_cluster), "r"(src_cta), "r"(bytes), "r"(bar_cluster) : "memory");
}
// 16-byte store into another CTA's shared memory (cluster address) that counts
// its bytes on an mbarrier of that CTA (also a cluster address).
KL_DEVICE void st_async_v4(uint32_t remote_addr, float a, float b, float c, float d, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];"
               :: "r"(remote_addr), "r"(__float_as_uint(a)), "r"(__float_as_uint(b)), "r"(__float_as_uint(c)),
                  "r"(__float_as_uint(d)), "r"(remote_bar)
               : "memory");
}
KL_DEVICE void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(dst_smem), "r"(ncols) : "memory");
}
KL_DEVICE void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
KL_DEVICE void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc] over the CTA pair (M = 256: 128 rows of
// A and D in each CTA; B split along N between the two CTAs' shared memory).
KL_DEVICE void tc_mma_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_desc_lo, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n .reg .b64 bd;\n setp.ne.b32 p, %5, 0;\n mov.b64 bd, {%2, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], bd, %4, {%6, %6, %6, %6, %6, %6, %6, %6}, p;\n}"
      :: "r"(d_tmem), "r"(a_tmem), "r"(b_desc_lo), "n"(kSmemDescSw128Hi), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}
// Arrive once on the mbarrier at the same offset in every CTA of `mask` when the
// pair's previously issued MMAs complete.
KL_DEVICE void tc_commit_pair_mc(uint32_t bar, uint16_t mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               :: "r"(bar), "h"(mask) : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of the pair's leader CTA (`bar` is a cluster address).
KL_DEVICE void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];"
      :: "r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar) : "memory");
}

// True in exactly one active lane of the warp (all lanes must call it).
KL_DEVICE bool elect_one() {
  uint32_t pred;
  asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}" : "=r"(pred));
  return pred != 0;
}
// Arrive (once) on an mbarrier when all previously issued tcgen05 ops of this thread complete.
KL_DEVICE void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar) : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
KL_DEVICE void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
KL_DEVICE void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
         "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Shared-memory matrix descriptor for tcgen05 (K-major operand, 128-byte
// swizzle, 8-row x 128-byte atoms stacked at 1024-byte stride).
//   bits  0-13 start address >> 4     bits 16-29 leading byte offset >> 4
//   bits 32-45 stride byte offset >> 4  bits 46-47 version (1 on sm_100)
//   bits 49-51 base offset (0: atoms are 1024-byte aligned)
//   bits 61-63 layout (2 = SWIZZLE_128B)
KL_DEVICE uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;                    // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;            // SBO = 1024 B
  d |= static_cast<uint64_t>(1u) << 46;                    // version
  d |= static_cast<uint64_t>(2u) << 61;                    // SWIZZLE_128B
  return d;
}

// The same descriptor split into its two 32-bit words, for issue loops that
// only advance the start address: the address field (bits 0-13) never carries
// into bit 14 because shared-memory addresses are below 256 KB.
KL_DEVICE uint32_t smem_desc_sw128_lo(uint32_t saddr) { return ((saddr >> 4) & 0x3FFFu) | (1u << 16); }

// Instruction descriptor, kind::f16: f32 accumulator, A and B both bf16 (or both
// f16), both K-major, shape M x N.
//   bits 4-5 D format (1 = f32)   bits 7-9 A format   bits 10-12 B format
//   (0 = f16, 1 = bf16)  bit 15/16 A/B major (0 = K)  bits 17-22 N >> 3
//   bits 24-28 M >> 4
__host__ __device__ constexpr uint32_t make_idesc_f16(int m, int n, bool bf16) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// Instruction descriptor, kind::i8: s32 accumulator (bits 4-5 = 2), A and B
// signed 8-bit (format 1 at bits 7-9 and 10-12), both K-major, shape M x N.
__host__ __device__ constexpr uint32_t make_idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// ---------------------------------------------------------- int -> bf16 bits
KL_DEVICE uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
template <int LUT>
KL_DEVICE uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
  return d;
}
KL_DEVICE uint32_t fma_bf16x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
KL_DEVICE uint32_t fma_f16x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Four signed int8 values (one 32-bit word, byte i = element i) -> two packed
// bf16x2 words holding the same integers exactly: {e0,e1} and {e2,e3}.
// With v = q & 0x7F and s = q & 0x80, the bf16 bit patterns 0x4300|v and
// 0x4300|s are the numbers 128+v and 128+2s/... (128 or 256), so
// (0x4300|v) - (0x4300|s) = v - 128*[s != 0] = q, computed exactly by one
// bf16x2 fma with multiplier -1.
KL_DEVICE void s8x4_to_bf16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t t0 = prmt(w, 0x43434343u, 0x4140u);   // [e0, 43, e1, 43]
  const uint32_t t1 = prmt(w, 0x43434343u, 0x4342u);   // [e2, 43, e3, 43]
  // a = t & 0xFF7FFF7F ; b = (t & 0x00800080) | 0x43004300
  const uint32_t a0 = t0 & 0xFF7FFF7Fu, a1 = t1 & 0xFF7FFF7Fu;
  const uint32_t b0 = lop3<0xEA>(t0, 0x00800080u, 0x43004300u);
  const uint32_t b1 = lop3<0xEA>(t1, 0x00800080u, 0x43004300u);
  lo = fma_bf16x2(b0, 0xBF80BF80u, a0);                 // a - b
  hi = fma_bf16x2(b1, 0xBF80BF80u, a1);
}
// Exact int8 -> bf16 with half of the integer-pipe work moved to the FMA pipe.
// With u = q ^ 0x80 = q + 128, the halfword 0x43uu is the bf16 value v = 128 + u
// when u < 128 (q < 0) and v = 2u when u >= 128 (q >= 0: bit 7 of u lands in the
// exponent), so r = v - 256 is q for q < 0 and 2q for q >= 0, and
// q = r - relu(r) / 2.  Every intermediate is an integer with at most 8
// significant bits, so each bf16 operation is exact.
KL_DEVICE uint32_t fma_relu_bf16x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.relu.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
KL_DEVICE void s8x4_to_bf16x4_fma(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t v0 = prmt(u, 0x43434343u, 0x4140u);    // [u0, 43, u1, 43]
  const uint32_t v1 = prmt(u, 0x43434343u, 0x4342u);    // [u2, 43, u3, 43]
  constexpr uint32_t kOne = 0x3F803F80u, kM256 = 0xC380C380u, kMHalf = 0xBF00BF00u;   // 1, -256, -0.5
  const uint32_t r0 = fma_bf16x2(v0, kOne, kM256), r1 = fma_bf16x2(v1, kOne, kM256);
  const uint32_t p0 = fma_relu_bf16x2(v0, kOne, kM256), p1 = fma_relu_bf16x2(v1, kOne, kM256);
  lo = fma_bf16x2(p0, kMHalf, r0);
  hi = fma_bf16x2(p1, kMHalf, r1);
}
// Same for f16: 0x6400|u is 1024+u for u < 1024; u = q ^ 0x80 = q + 128.
KL_DEVICE void s8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t t0 = prmt(u, 0x64646464u, 0x4140u);
  const uint32_t t1 = prmt(u, 0x64646464u, 0x4342u);
  // t - 1152 (0x6480 = 1152 in f16)
  lo = fma_f16x2(t0, 0x3C003C00u, 0xE480E480u);
  hi = fma_f16x2(t1, 0x3C003C00u, 0xE480E480u);
}

// Byte i of a word of 4-bit codes (low nibble = even k) -> {lo - z, hi - z}.
// With s = w >> 4, prmt(w, s, sel_i) puts byte i of w in the low half and
// byte i of s (whose low nibble is the high nibble of byte i of w) in the high
// half.  Masking to the low nibble of each half and XOR-ing in the magic 0x43
// (bf16: 0x43.0n = 128 + n) gives {128+lo, 128+hi}; one fma adds -(128 + z).
// `magic_xor` = 0x43004300 for unsigned codes; 0x43084308 also flips nibble
// bit 3, mapping two's-complement codes c to c + 8, so the symmetric format is
// the same conversion with z = 8.  All results are small integers: exact.
KL_DEVICE constexpr uint32_t nib_sel(int i) {
  return static_cast<uint32_t>(i | (i << 4) | ((4 + i) << 8) | ((4 + i) << 12));
}
KL_DEVICE uint32_t u4x2_to_bf16x2(uint32_t w, uint32_t s, uint32_t sel, uint32_t magic_xor, uint32_t bias) {
  const uint32_t t = prmt(w, s, sel);
  const uint32_t m = lop3<0x6A>(t, 0x000F000Fu, magic_xor);   // (t & 0x000F000F) ^ magic
  return fma_bf16x2(m, 0x3F803F80u, bias);                    // m * 1 + bias
}
// f16 variant: 0x64.0n = 1024 + n; magic_xor 0x64006400 / 0x64086408.
KL_DEVICE uint32_t u4x2_to_f16x2(uint32_t w, uint32_t s, uint32_t sel, uint32_t magic_xor, uint32_t bias) {
  const uint32_t t = prmt(w, s, sel);
  const uint32_t m = lop3<0x6A>(t, 0x000F000Fu, magic_xor);
  return fma_f16x2(m, 0x3C003C00u, bias);
}

// Transposing warp reduction of V (power of two <= 32) values.  Afterwards the
// lane `l` holds the full sum of value index ((l >> (5 - log2 V)) restricted) --
// see value_index_of_lane.
template <int V>
KL_DEVICE float warp_reduce_multi(float (&v)[V]) {
  const int lane = threadIdx.x & 31;
  int cnt = V;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (cnt > 1) {
      const bool upper = (lane & off) != 0;
      const int half = cnt >> 1;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (i < half) {
          const float send = upper ? v[i] : v[i + half];
          const float keep = upper ? v[i + half] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      cnt = half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
  return v[0];
}
template <int V>
KL_DEVICE int value_index_of_lane(int lane) {
  // index bits are taken from lane bits 4, 3, ... (most significant first)
  int idx = 0, cnt = V, bit = 16;
  while (cnt > 1) {
    idx += (lane & bit) ? (cnt >> 1) : 0;
    cnt >>= 1;
    bit >>= 1;
  }
  return idx;
}

KL_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
KL_DEVICE uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Round f32 to the activation dtype and back (bf16 when BF16, else f16).
template <bool BF16>
KL_DEVICE float round_act(float v) {
  if constexpr (BF16) return __bfloat162float(__float2bfloat16_rn(v));
  else return __half2float(__float2half_rn(v));
}
template <bool BF16>
KL_DEVICE void store_act(void* base, long long idx, float v) {
  if constexpr (BF16) reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
  else reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v);
}
template <bool BF16>
KL_DEVICE float load_act(const void* base, long long idx) {
  if constexpr (BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
  else return __half2float(reinterpret_cast<const __half*>(base)[idx]);
}

// Model-ordered SwiGLU epilogue (bf16 boundaries after each projection and
// after SiLU), the contract of the reference's fused gate/up kernels.
template <bool BF16>
KL_DEVICE float swiglu_model_ordered(float gate, float up) {
  gate = round_act<BF16>(gate);
  up = round_act<BF16>(up);
  const float act = round_act<BF16>(gate / (1.0f + expf(-gate)));
  return act * up;
}

// The same epilogue with the SFU exponential and division (a few ulp before the
// bf16 rounding of the activation): for epilogues that evaluate SiLU on every
// element of a large tile.
template <bool BF16>
KL_DEVICE float swiglu_model_ordered_fast(float gate, float up) {
  gate = round_act<BF16>(gate);
  up = round_act<BF16>(up);
  const float act = round_act<BF16>(__fdividef(gate, 1.0f + __expf(-gate)));
  return act * up;
}

}  // namespace kl
