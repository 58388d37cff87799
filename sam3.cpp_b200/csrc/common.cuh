// Device-side primitives shared by the sm_100a kernels of the encoder engine:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM alloc, MMA,
// commit, loads) and the shared-memory / instruction descriptors they take.
//
// Every wait in this engine is bounded: a wait that does not complete within
// kWaitNs nanoseconds (globaltimer) records an error code in the kernel's
// error word, raises the CTA-local abort flag and returns false, so that the
// kernel can unwind (free TMEM, return) instead of spinning forever.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace s3b {

// Error codes written to the device error word (first writer wins).
enum DevErr : int {
  kErrNone = 0,
  kErrWaitFull = 1,     // MMA warp timed out waiting for a TMA stage
  kErrWaitEmpty = 2,    // producer timed out waiting for a free stage
  kErrWaitTmemFull = 3, // epilogue timed out waiting for an accumulator
  kErrWaitTmemEmpty = 4,// MMA warp timed out waiting for the epilogue
  kErrWaitDrain = 5,    // producer timed out draining in-flight copies
  kErrWaitMisc = 6,
};

static constexpr unsigned long long kWaitNs = 2000ull * 1000ull * 1000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of the phase of `parity` (mbarrier.test_wait never suspends the thread).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but the thread may be suspended until the phase completes
// or `hint_ns` nanoseconds pass, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of `parity` to complete. Returns false (after
// recording `code`) on timeout or when another role of the CTA aborted.
// Between checks of the abort flag and of the time limit the waiting thread
// sleeps in the barrier (up to 1 ms per try).
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                              int code, unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      if (err) atomicCAS(err, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int code) {
  return mbar_wait_for(bar, parity, abort_flag, err, code, kWaitNs);
}

// As mbar_wait, with cluster-scope acquire: for phases completed by release
// arrives from the other CTA of a pair (shared-memory data written by that
// CTA's threads, read after the wait by this CTA's pair MMAs).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  int* err, int code) {
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity, 1000000u)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitNs) {
      if (err) atomicCAS(err, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
__device__ __forceinline__ void tma_load_2d(const void* map, uint64_t* bar, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(const void* map, uint64_t* bar, void* dst, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(const void* map, uint64_t* bar, void* dst, int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (f16/bf16 in, f32 acc).
// A operand read from TMEM (K-major: lane = row, each 32-bit column holds two consecutive K
// elements, 8 columns per K = 16 step), B from shared memory
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- CTA pairs (cluster of 2, cta_group::2)
// A pair of CTAs on two SMs computes one 256-row tile: each CTA holds 128
// rows of A and half of B in its own shared memory and 128 accumulator rows
// in its own TMEM; the even CTA (the leader) issues the MMAs for both. Every
// tcgen05 instruction of a kernel that uses pairs is the cta_group::2 form.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the variable at `saddr` (shared::cta) in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// all threads of both CTAs; orders each CTA's earlier memory operations before the other's later ones
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// TMA 2-D load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (`cluster_bar` from cluster_addr).
__device__ __forceinline__ void tma_load_2d_pair(const void* map, uint32_t cluster_bar, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(cluster_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_pair(const void* map, uint32_t cluster_bar, void* dst, int x, int y,
                                                 int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(cluster_bar), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (+)= A * B^T over the pair: M = 256 (128 rows per CTA), A / B descriptors
// are this CTA's addresses, the same offsets are used in the peer.
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at this shared offset in every CTA of `cta_mask`
// when all previously issued pair MMAs of this thread complete.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns: thread t of the warp receives
// row (lane base + t), columns [col, col+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 64 f16 = 128 B, 8-row atoms of 1024 B):
// start address and strides in 16-byte units, LBO unused (1), SBO = 1024 B,
// descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: D f32, A/B f16 (fmt 0) or bf16 (fmt 1),
// both K-major, N>>3 at bits [17,23), M>>4 at bits [24,29).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int ab_fmt) {
  return (1u << 4) | ((uint32_t)ab_fmt << 7) | ((uint32_t)ab_fmt << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------- math
// GELU with the erf form (ggml_gelu_erf, sam3.cpp:3794 / 3882): x Phi(x) with
// Phi(x) = 1 - h for x >= 0 and h for x < 0, h = erfc(|x| / sqrt(2)) / 2, and
// erfc by Abramowitz & Stegun eq. 7.1.28: erfc(z) = (1 + a1 z + ... + a6 z^6)^-16,
// |error| <= 3e-7. The argument scale 1/sqrt(2) and the factor 1/2 (as 2^(1/16))
// are folded into the coefficients, so h = 1 / q(|x|)^16 with q of degree 6:
// six FMAs, four squarings and one reciprocal (the MLP epilogue evaluates it
// for every hidden element). Max abs error of the GELU 8e-7 on [-12, 12].
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gelu_erf(float x) {
  const float ax = fabsf(x);
  float q = fmaf(5.6212996640e-06f, ax, 5.1055209009e-05f);
  q = fmaf(q, ax, 3.9686137011e-05f);
  q = fmaf(q, ax, 3.4227392389e-03f);
  q = fmaf(q, ax, 2.2076998457e-02f);
  q = fmaf(q, ax, 5.2075163037e-02f);
  q = fmaf(q, ax, 1.0442737824e+00f);
  q *= q;
  q *= q;
  q *= q;
  q *= q;
  const float h = rcp_approx(q);  // 0 once q^16 overflows (|x| > ~60): Phi = 1 or 0
  return x * (x >= 0.0f ? 1.0f - h : h);
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed two-wide f32 arithmetic (sm_100: one instruction for two lanes of a 64-bit register pair).
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// GELU with the tanh form (ggml_gelu, sam3.cpp:4449) on a pair of values, as x * sigmoid(2u) = x / (1 + 2^t) with u = k0 (x + k1 x^3) and
// t = -2 u / ln 2 = x (c1 + c3 x^2): 5 two-wide FMA-pipe operations and 2 MUFU operations per value
// (ex2, rcp). Large positive t gives 2^t = inf and x * 0; large negative t gives x * 1.
__device__ __forceinline__ void gelu_tanh2(float& a, float& b) {
  const float c1 = -2.3022082f, c3 = -0.10294324f;  // -2 k0 / ln 2, times k1 = 0.044715 (k0 = sqrt(2/pi))
  const unsigned long long x = f2_pack(a, b);
  const unsigned long long t = f2_mul(f2_fma(f2_mul(x, x), f2_pack(c3, c3), f2_pack(c1, c1)), x);
  float ta, tb;
  f2_unpack(t, ta, tb);
  const unsigned long long d = f2_add(f2_pack(ex2_approx(ta), ex2_approx(tb)), f2_pack(1.0f, 1.0f));
  float da, db;
  f2_unpack(d, da, db);
  f2_unpack(f2_mul(x, f2_pack(rcp_approx(da), rcp_approx(db))), a, b);
}

// gelu_erf on a pair of values: the degree-6 polynomial and the four squarings run two-wide.
__device__ __forceinline__ void gelu_erf2(float& a, float& b) {
  const unsigned long long ax = f2_pack(fabsf(a), fabsf(b));
  unsigned long long q = f2_fma(f2_pack(5.6212996640e-06f, 5.6212996640e-06f), ax,
                                f2_pack(5.1055209009e-05f, 5.1055209009e-05f));
  q = f2_fma(q, ax, f2_pack(3.9686137011e-05f, 3.9686137011e-05f));
  q = f2_fma(q, ax, f2_pack(3.4227392389e-03f, 3.4227392389e-03f));
  q = f2_fma(q, ax, f2_pack(2.2076998457e-02f, 2.2076998457e-02f));
  q = f2_fma(q, ax, f2_pack(5.2075163037e-02f, 5.2075163037e-02f));
  q = f2_fma(q, ax, f2_pack(1.0442737824e+00f, 1.0442737824e+00f));
  q = f2_mul(q, q);
  q = f2_mul(q, q);
  q = f2_mul(q, q);
  q = f2_mul(q, q);
  float qa, qb;
  f2_unpack(q, qa, qb);
  const float ha = rcp_approx(qa), hb = rcp_approx(qb);
  a *= a >= 0.0f ? 1.0f - ha : ha;
  b *= b >= 0.0f ? 1.0f - hb : hb;
}

}  // namespace s3b
