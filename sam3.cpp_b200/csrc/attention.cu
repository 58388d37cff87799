// Flash attention for the encoder hot path (no mask, softmax(q.k * scale) v).
//
// Replaces ggml_flash_attn_ext at sam3.cpp:3774 (ViT windowed / global),
// sam3.cpp:4395 (Hiera, q-pooled Nq < Nk) and sam3.cpp:9267, 9312 (memory
// attention, one 256-d head, Nk up to 7*H*W + 4*P keys). The semantics of
// the reference have no mask; the only masking here is of the padding of our
// own key tiling (keys >= nk).
//
// Design: one CTA = 4 warps = 64 queries of one (batch, head); each warp owns
// 16 query rows. K/V tiles of 64 keys are double-buffered in shared memory with
// cp.async; S = Q K^T and O += P V run on mma.m16n8k16 (f16 in, f32 acc), the
// online softmax keeps P in registers (the S accumulator fragments are the A
// fragments of P V). Rows are padded by 16 bytes so ldmatrix is conflict-free.
#include "common.cuh"
#include "kernels.h"

namespace s3b {
namespace {

constexpr int kBQ = 64;
constexpr int kBKV = 64;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const unsigned sz = valid ? 16u : 0u;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Loads `rows` x D halves (row stride `ld` elements in global) into a padded
// shared tile; rows at or beyond `valid_rows` are zero-filled.
template <int D, int DR>
__device__ __forceinline__ void load_tile(__half* s, const __half* g, long long ld, int valid_rows, int tid) {
  constexpr int LD = D + 8;
  constexpr int CH = DR / 8;  // only the DR real columns come from global memory
  for (int i = tid; i < kBKV * CH; i += 128) {
    const int r = i / CH, c = i - r * CH;
    const bool ok = r < valid_rows;
    cp_async16(s + r * LD + c * 8, ok ? (const void*)(g + (long long)r * ld + c * 8) : (const void*)g, ok);
  }
}

// D: compute head dim (multiple of 16); DR: real head dim (multiple of 8). For
// DR < D (Hiera-L's 72 -> 80) the pad columns stay zero in shared memory, which
// leaves q.k unchanged and gives zero output columns that are not stored.
// ONE: nk <= 64, a single key tile: K and V take one buffer each (40 KB instead of 66 KB of shared memory
// at d = 96), so five CTAs fit on an SM instead of three (Hiera-T's stage-0 windows, 64 x 64).
template <int D, int DR, bool ONE = false>
__global__ void __launch_bounds__(128) attn_fwd_kernel(AttnParams p) {
  constexpr int LD = D + 8;
  constexpr int NT = D / 8;  // n-tiles of the output
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half* sQ = reinterpret_cast<__half*>(smem_raw);
  __half* sK = sQ + kBQ * LD;
  __half* sV = sK + (ONE ? 1 : 2) * kBKV * LD;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // 1-D grid, query tile fastest: the tiles of one (batch, head) run together and share K/V in L2
  const int n_qt = (p.nq + kBQ - 1) / kBQ;
  const int bh = (int)(blockIdx.x / n_qt);
  const int b = bh / p.heads, h = bh - (bh / p.heads) * p.heads;
  const int q0 = (int)(blockIdx.x - (unsigned)bh * n_qt) * kBQ;
  const __half* Qg = p.q + (long long)b * p.q_b + (long long)h * p.q_h + (long long)q0 * p.q_n;
  const __half* Kg = p.k + (long long)b * p.k_b + (long long)h * p.k_h;
  const __half* Vg = p.v + (long long)b * p.v_b + (long long)h * p.v_h;

  if constexpr (DR < D) {
    constexpr int PADC = (DR < D) ? D - DR : 1;
    for (int i = tid; i < (kBQ + (ONE ? 2 : 4) * kBKV) * PADC; i += 128) {
      const int r = i / PADC, c = DR + i % PADC;
      sQ[r * LD + c] = __float2half_rn(0.f);
    }
  }
  load_tile<D, DR>(sQ, Qg, p.q_n, p.nq - q0, tid);
  load_tile<D, DR>(sK, Kg, p.k_n, p.nk, tid);
  load_tile<D, DR>(sV, Vg, p.v_n, p.nk, tid);
  cp_async_commit();

  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = p.scale * 1.4426950408889634f;

  const int nkt = (p.nk + kBKV - 1) / kBKV;
  const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
  const int g = lane >> 2, t4 = lane & 3;

  for (int j = 0; j < nkt; ++j) {
    const int buf = ONE ? 0 : (j & 1);
    if (!ONE && j + 1 < nkt) {
      const int nb = buf ^ 1;
      load_tile<D, DR>(sK + nb * kBKV * LD, Kg + (long long)(j + 1) * kBKV * p.k_n, p.k_n, p.nk - (j + 1) * kBKV, tid);
      load_tile<D, DR>(sV + nb * kBKV * LD, Vg + (long long)(j + 1) * kBKV * p.v_n, p.v_n, p.nk - (j + 1) * kBKV, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    // S = Q K^T for this warp's 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
    const uint32_t kb = sKa + (uint32_t)(buf * kBKV * LD * 2);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      {
        const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int c = kk * 16 + 8 * (lane >> 4);
        ldsm_x4(sQa + (uint32_t)((r * LD + c) * 2), a0, a1, a2, a3);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + 8 * (lane >> 4);
        const int c = kk * 16 + 8 * ((lane >> 3) & 1);
        ldsm_x4(kb + (uint32_t)((r * LD + c) * 2), b0, b1, b2, b3);
        mma16816(s[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816(s[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }

    // mask the padding keys of the last tile
    const int kbase = j * kBKV;
    if (kbase + kBKV > p.nk) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int key = kbase + n * 8 + 2 * t4;
        if (key >= p.nk) { s[n][0] = -INFINITY; s[n][2] = -INFINITY; }
        if (key + 1 >= p.nk) { s[n][1] = -INFINITY; s[n][3] = -INFINITY; }
      }
    }

    // online softmax (rows g and g+8 of the warp's 16)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
      mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0 * sl2), mn1 = fmaxf(m1, mx1 * sl2);
    const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    l0 *= al0;
    l1 *= al1;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= al0; o[n][1] *= al0;
      o[n][2] *= al1; o[n][3] *= al1;
    }
    uint32_t pa[8][2];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = exp2f(s[n][0] * sl2 - mn0), p1 = exp2f(s[n][1] * sl2 - mn0);
      const float p2 = exp2f(s[n][2] * sl2 - mn1), p3 = exp2f(s[n][3] * sl2 - mn1);
      l0 += p0 + p1;
      l1 += p2 + p3;
      pa[n][0] = pack_h2(p0, p1);
      pa[n][1] = pack_h2(p2, p3);
    }

    // O += P V
    const uint32_t vb = sVa + (uint32_t)(buf * kBKV * LD * 2);
#pragma unroll
    for (int kk = 0; kk < kBKV / 16; ++kk) {
      const uint32_t a0 = pa[2 * kk][0], a1 = pa[2 * kk][1], a2 = pa[2 * kk + 1][0], a3 = pa[2 * kk + 1][1];
#pragma unroll
      for (int dp = 0; dp < NT / 2; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int c = dp * 16 + 8 * (lane >> 4);
        ldsm_x4_t(vb + (uint32_t)((r * LD + c) * 2), b0, b1, b2, b3);
        mma16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;
  const long long orow0 = r0 < p.nq ? map_row(p.omap, (long long)b * p.nq + r0) : -1;
  const long long orow1 = r1 < p.nq ? map_row(p.omap, (long long)b * p.nq + r1) : -1;
  __half* ob = p.o + (long long)h * DR;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int c = n * 8 + 2 * t4;
    if (c >= DR) continue;
    if (orow0 >= 0)
      *reinterpret_cast<__half2*>(ob + orow0 * p.o_n + c) = __floats2half2_rn(o[n][0] * inv0, o[n][1] * inv0);
    if (orow1 >= 0)
      *reinterpret_cast<__half2*>(ob + orow1 * p.o_n + c) = __floats2half2_rn(o[n][2] * inv1, o[n][3] * inv1);
  }
}

// Small windows (nq <= 16, nk <= NKP <= 64; Hiera's pooled and stage-1/2
// windows, e.g. 16 queries x 16 keys): one warp per (batch, head), four per
// CTA, each with its own Q (16 rows), K and V (NKP rows) in shared memory; S,
// the softmax and P V of the single key tile stay in registers.
// Warps per CTA of attn_small_kernel: 4, or for 64-key windows (30 KB of shared memory per warp, so one
// 4-warp CTA per SM) as many as one CTA's shared memory holds, up to 8: each warp waits for its loads before
// computing, so the warps in flight per SM set the throughput.
template <int D, int NKP>
constexpr int small_warps() {
  return NKP < 64 ? 4 : (232448 / ((16 + 2 * NKP) * (D + 8) * 2) < 8 ? 232448 / ((16 + 2 * NKP) * (D + 8) * 2) : 8);
}

template <int D, int DR, int NKP>
__global__ void __launch_bounds__(32 * small_warps<D, NKP>()) attn_small_kernel(AttnParams p, int batch_heads) {
  constexpr int LD = D + 8;
  constexpr int NT = D / 8;
  constexpr int WROWS = 16 + 2 * NKP;  // Q, K, V rows of one warp
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x * small_warps<D, NKP>() + warp;
  if (bh >= batch_heads) return;  // whole warp; no CTA-wide barrier below
  __half* sQ = reinterpret_cast<__half*>(smem_raw) + warp * WROWS * LD;
  __half* sK = sQ + 16 * LD;
  __half* sV = sK + NKP * LD;
  const int b = bh / p.heads, h = bh - (bh / p.heads) * p.heads;
  const __half* Qg = p.q + (long long)b * p.q_b + (long long)h * p.q_h;
  const __half* Kg = p.k + (long long)b * p.k_b + (long long)h * p.k_h;
  const __half* Vg = p.v + (long long)b * p.v_b + (long long)h * p.v_h;
  if constexpr (DR < D) {
    constexpr int PADC = (DR < D) ? D - DR : 1;
    for (int i = lane; i < WROWS * PADC; i += 32) sQ[(i / PADC) * LD + DR + i % PADC] = __float2half_rn(0.f);
  }
  constexpr int CH = DR / 8;  // 16-byte chunks per row
  for (int i = lane; i < 16 * CH; i += 32) {
    const int r = i / CH, c = i - r * CH;
    const bool ok = r < p.nq;
    cp_async16(sQ + r * LD + c * 8, ok ? (const void*)(Qg + (long long)r * p.q_n + c * 8) : (const void*)Qg, ok);
  }
  for (int i = lane; i < NKP * CH; i += 32) {
    const int r = i / CH, c = i - r * CH;
    const bool ok = r < p.nk;
    cp_async16(sK + r * LD + c * 8, ok ? (const void*)(Kg + (long long)r * p.k_n + c * 8) : (const void*)Kg, ok);
    cp_async16(sV + r * LD + c * 8, ok ? (const void*)(Vg + (long long)r * p.v_n + c * 8) : (const void*)Vg, ok);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncwarp();

  const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
  const int g = lane >> 2, t4 = lane & 3;
  float s[NKP / 8][4];
#pragma unroll
  for (int n = 0; n < NKP / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t a0, a1, a2, a3;
    {
      const int r = (lane & 7) + 8 * ((lane >> 3) & 1);
      const int c = kk * 16 + 8 * (lane >> 4);
      ldsm_x4(sQa + (uint32_t)((r * LD + c) * 2), a0, a1, a2, a3);
    }
#pragma unroll
    for (int np = 0; np < NKP / 16; ++np) {
      uint32_t b0, b1, b2, b3;
      const int r = np * 16 + (lane & 7) + 8 * (lane >> 4);
      const int c = kk * 16 + 8 * ((lane >> 3) & 1);
      ldsm_x4(sKa + (uint32_t)((r * LD + c) * 2), b0, b1, b2, b3);
      mma16816(s[2 * np], a0, a1, a2, a3, b0, b1);
      mma16816(s[2 * np + 1], a0, a1, a2, a3, b2, b3);
    }
  }
  // softmax over the nk real keys (rows g and g+8)
  const float sl2 = p.scale * 1.4426950408889634f;
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int n = 0; n < NKP / 8; ++n) {
    const int key = n * 8 + 2 * t4;
    if (key >= p.nk) { s[n][0] = -INFINITY; s[n][2] = -INFINITY; }
    if (key + 1 >= p.nk) { s[n][1] = -INFINITY; s[n][3] = -INFINITY; }
    mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
    mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float mn0 = mx0 * sl2, mn1 = mx1 * sl2;
  float l0 = 0.f, l1 = 0.f;
  uint32_t pa[NKP / 8][2];
#pragma unroll
  for (int n = 0; n < NKP / 8; ++n) {
    const float p0 = exp2f(s[n][0] * sl2 - mn0), p1 = exp2f(s[n][1] * sl2 - mn0);
    const float p2 = exp2f(s[n][2] * sl2 - mn1), p3 = exp2f(s[n][3] * sl2 - mn1);
    l0 += p0 + p1;
    l1 += p2 + p3;
    pa[n][0] = pack_h2(p0, p1);
    pa[n][1] = pack_h2(p2, p3);
  }
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < NKP / 16; ++kk) {
    const uint32_t a0 = pa[2 * kk][0], a1 = pa[2 * kk][1], a2 = pa[2 * kk + 1][0], a3 = pa[2 * kk + 1][1];
#pragma unroll
    for (int dp = 0; dp < NT / 2; ++dp) {
      uint32_t b0, b1, b2, b3;
      const int r = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
      const int c = dp * 16 + 8 * (lane >> 4);
      ldsm_x4_t(sVa + (uint32_t)((r * LD + c) * 2), b0, b1, b2, b3);
      mma16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
      mma16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  const int r0 = g, r1 = g + 8;
  const long long orow0 = r0 < p.nq ? map_row(p.omap, (long long)b * p.nq + r0) : -1;
  const long long orow1 = r1 < p.nq ? map_row(p.omap, (long long)b * p.nq + r1) : -1;
  __half* ob = p.o + (long long)h * DR;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int c = n * 8 + 2 * t4;
    if (c >= DR) continue;
    if (orow0 >= 0)
      *reinterpret_cast<__half2*>(ob + orow0 * p.o_n + c) = __floats2half2_rn(o[n][0] * inv0, o[n][1] * inv0);
    if (orow1 >= 0)
      *reinterpret_cast<__half2*>(ob + orow1 * p.o_n + c) = __floats2half2_rn(o[n][2] * inv1, o[n][3] * inv1);
  }
}

template <int D, int DR, int NKP>
int launch_small(const AttnParams& p, int batch_heads, cudaStream_t st) {
  constexpr int W = small_warps<D, NKP>();
  constexpr size_t smem = (size_t)W * (16 + 2 * NKP) * (D + 8) * 2;
  static_assert(W >= 4 && smem <= 232448, "shared memory per CTA");
  if (kernel_setup(attn_small_kernel<D, DR, NKP>, smem) <= 0) return -13;
  const long long n_cta = ((long long)batch_heads + W - 1) / W;
  if (n_cta > 0x7fffffffLL) return -2;
  attn_small_kernel<D, DR, NKP><<<(unsigned)n_cta, 32 * W, smem, st>>>(p, batch_heads);
  return launch_status("attention (small windows)");
}

template <int D, int DR>
int launch_small_nk(const AttnParams& p, int batch_heads, cudaStream_t st) {
  if (p.nk <= 16) return launch_small<D, DR, 16>(p, batch_heads, st);
  if (p.nk <= 32) return launch_small<D, DR, 32>(p, batch_heads, st);
  if (p.nk <= 48) return launch_small<D, DR, 48>(p, batch_heads, st);
  return launch_small<D, DR, 64>(p, batch_heads, st);
}

template <int D, int DR>
int launch_attn(const AttnParams& p, int batch_heads, cudaStream_t st) {
  if constexpr (D <= 128) {
    if (p.nq <= 16 && p.nk <= 64) return launch_small_nk<D, DR>(p, batch_heads, st);
  }
  const long long n_cta = (long long)((p.nq + kBQ - 1) / kBQ) * batch_heads;
  if (n_cta > 0x7fffffffLL) return -2;
  if (p.nk <= kBKV) {
    constexpr size_t smem1 = (size_t)(kBQ + 2 * kBKV) * (D + 8) * 2;
    if (kernel_setup(attn_fwd_kernel<D, DR, true>, smem1) <= 0) return -13;
    attn_fwd_kernel<D, DR, true><<<(unsigned)n_cta, 128, smem1, st>>>(p);
    return launch_status("attention");
  }
  constexpr size_t smem = (size_t)(kBQ + 4 * kBKV) * (D + 8) * 2;
  if (kernel_setup(attn_fwd_kernel<D, DR>, smem) <= 0) return -13;
  attn_fwd_kernel<D, DR><<<(unsigned)n_cta, 128, smem, st>>>(p);
  return launch_status("attention");
}

}  // namespace

int attention(const AttnParams& p, int D, int batch_heads, cudaStream_t st) {
  if (p.nq <= 0 || p.nk <= 0 || batch_heads <= 0 || p.heads <= 0) return -1;
  if ((p.q_n % 8) || (p.k_n % 8) || (p.v_n % 8) || (p.q_b % 8) || (p.k_b % 8) || (p.v_b % 8) || (p.q_h % 8) ||
      (p.k_h % 8) || (p.v_h % 8) || (p.o_n % 2))
    return -2;
  switch (D) {
    case 64: return launch_attn<64, 64>(p, batch_heads, st);
    case 72: return launch_attn<80, 72>(p, batch_heads, st);
    case 80: return launch_attn<80, 80>(p, batch_heads, st);
    case 96: return launch_attn<96, 96>(p, batch_heads, st);
    case 128: return launch_attn<128, 128>(p, batch_heads, st);
    case 256: return launch_attn<256, 256>(p, batch_heads, st);
    default: return -3;
  }
}

}  // namespace s3b
