// Persistent warp-specialised tensor-core GEMM for sm_100a.
//
//   C[M,N] = A[M,K] * B[N,K]^T, A/B f16 K-major, f32 accumulation in TMEM.
//
// This kernel replaces ggml_mul_mat + ggml_add(bias) (+ activation, RoPE,
// residual add, and the permute/cont copies around them) on the encoder hot
// path: ViT blocks sam3.cpp:3738-3798, Hiera blocks sam3.cpp:4317-4454,
// memory attention sam3.cpp:9250-9325, and the convolutions lowered to
// GEMMs (patch embed 3815/4470, neck 3880-3918, FPN 4547).
//
// Roles (320 threads, one CTA per SM, persistent over output tiles):
//   warp 0     TMA producer: 128x64 A tile + BNx64 B tile per stage (SW128)
//   warp 1     MMA issuer: 4 x tcgen05.mma (K=16) per stage into TMEM;
//              owns the TMEM allocation (2 accumulators of BN columns)
//   warps 2-9  epilogue: warps w and w+4 share TMEM lane quarter (w % 4) and
//              split the tile's columns in halves.
// The accumulator is double-buffered so the epilogue of tile i overlaps the
// main loop of tile i+1.
//
// Epilogue, TMA path (plain row-major outputs): each 128-row column chunk of
// 128 bytes is moved TMEM -> registers (bias, activation, RoPE) -> a 128B-
// swizzled shared staging buffer (double-buffered per half) -> global by one
// TMA tensor store. When the residual is the output itself (x += f(x)) the
// chunk of x is first TMA-loaded into the same staging buffer and added in
// registers. Other layouts (deconvolution pixel scatter, row remaps,
// broadcast residuals) use direct per-row stores.
#include "common.cuh"
#include "kernels.h"

#include <stdio.h>

#include <map>
#include <mutex>
#include <utility>

namespace s3b {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
// threads of a CTA with `ew` epilogue warps (plus the TMA and MMA warps)
constexpr int gemm_threads(int ew, int dw = 0) { return 64 + 32 * (ew + dw); }
// QB (quantised B operand): warps that dequantise each stage's weight tile (4 beside 16 epilogue
// warps, 8 beside 8)
constexpr int dequant_warps(int ew) { return ew >= 16 ? 4 : 8; }
constexpr uint32_t kStageBufBytes = 16384;  // 128 rows x 128 B

int g_gemm_pairs = 2;         // 256-row tiles on SM pairs: 0 never, 1 long-K GEMMs, 2 every wide GEMM
int g_gemm_wide_epi = 1;      // 16 epilogue warps for short-K GEMMs: 0 never, 1 always

// kernel_setup callbacks: co-resident work units of a persistent GEMM on the current device, one CTA
// per SM, or one cluster of 2 CTAs per SM pair (the cluster occupancy query)
int sm_units(const void*, size_t, int) { return num_sms(); }
int pair_units(const void* kernel, size_t smem, int threads) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * (num_sms() / 2));
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return -13;
  }
  return n;
}


// Two f32 -> one packed f16x2 register (lo in the low half), round to nearest even.
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// ---- quantised B operand (QB 1: q4_0, QB 2: q8_0), dequantised in shared memory
// A value v = q * d (q8_0) or (q - 8) * d (q4_0) with d the f16 block scale: the
// integer becomes an exact f16 through the 0x6400 exponent trick (0x6400 | u is
// 1024 + u for u < 1024), the offset is subtracted exactly, and one rounded f16
// multiply by d gives round_f16(q * d), the value the load-time dequantisation
// (f32 product, then f16 rounding) produces: the product of two f16 values is
// exact in f32, so both round the same real number once.
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t byte_perm(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
// q4_0 plane word (8 values of one row): nibble p (bits 4p) holds value 2p and
// nibble p + 4 (bits 16 + 4p) value 2p + 1, so pair p is (w >> 4p) & 0x000F000F.
__device__ __forceinline__ uint4 dequant8_q4(uint32_t w, uint32_t d2) {
  const uint32_t off = 0x64086408u;  // 1032 = 1024 + 8
  uint4 o;
  o.x = h2_mul(h2_sub((w & 0x000F000Fu) | 0x64006400u, off), d2);
  o.y = h2_mul(h2_sub(((w >> 4) & 0x000F000Fu) | 0x64006400u, off), d2);
  o.z = h2_mul(h2_sub(((w >> 8) & 0x000F000Fu) | 0x64006400u, off), d2);
  o.w = h2_mul(h2_sub(((w >> 12) & 0x000F000Fu) | 0x64006400u, off), d2);
  return o;
}
// q8_0: 8 int8 values in two words; q ^ 0x80 = q + 128 in [0, 255].
__device__ __forceinline__ uint4 dequant8_q8(uint2 w, uint32_t d2) {
  const uint32_t off = 0x64806480u;  // 1152 = 1024 + 128
  const uint32_t u0 = w.x ^ 0x80808080u, u1 = w.y ^ 0x80808080u;
  uint4 o;
  o.x = h2_mul(h2_sub(byte_perm(u0, 0x64u, 0x4140u), off), d2);
  o.y = h2_mul(h2_sub(byte_perm(u0, 0x64u, 0x4342u), off), d2);
  o.z = h2_mul(h2_sub(byte_perm(u1, 0x64u, 0x4140u), off), d2);
  o.w = h2_mul(h2_sub(byte_perm(u1, 0x64u, 0x4342u), off), d2);
  return o;
}

// Block-form planes -> f16 rows [N][ldo] (the staged path of weights_quantised = 1): one thread
// per 32-value block; consecutive threads take consecutive blocks of a row, so the value loads (16
// or 32 bytes each) and the 64-byte f16 stores are contiguous across a warp. The values are the
// same round_f16(q * d) the in-GEMM dequantisation and the load-time conversion produce.
template <int QB>
__global__ void __launch_bounds__(256) dequant_planes_kernel(const uint8_t* __restrict__ values,
                                                             const uint16_t* __restrict__ scales, int N, int K,
                                                             __half* __restrict__ out, long long ldo) {
  const int nb = K / 32;
  const long long total = (long long)N * nb;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / nb), kb = (int)(i - (long long)n * nb);
    const uint32_t d = scales[(long long)kb * N + n];
    const uint32_t d2 = d | (d << 16);
    uint4* o = reinterpret_cast<uint4*>(out + (long long)n * ldo + (long long)kb * 32);
    if (QB == 1) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(values + (long long)n * (K / 2) + (long long)kb * 16));
      o[0] = dequant8_q4(w.x, d2);
      o[1] = dequant8_q4(w.y, d2);
      o[2] = dequant8_q4(w.z, d2);
      o[3] = dequant8_q4(w.w, d2);
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(values + (long long)n * K + (long long)kb * 32);
      const uint4 a = __ldg(src), b = __ldg(src + 1);
      o[0] = dequant8_q8(make_uint2(a.x, a.y), d2);
      o[1] = dequant8_q8(make_uint2(a.z, a.w), d2);
      o[2] = dequant8_q8(make_uint2(b.x, b.y), d2);
      o[3] = dequant8_q8(make_uint2(b.z, b.w), d2);
    }
  }
}

struct StageJobs {
  const uint8_t* values[kMaxStageJobs];
  const uint16_t* scales[kMaxStageJobs];
  __half* out[kMaxStageJobs];
  int N[kMaxStageJobs], K[kMaxStageJobs], q4[kMaxStageJobs];
  long long start[kMaxStageJobs + 1];  // first block index of each job (prefix sums of N * K / 32)
  int n;
};

// The weights of one block / layer in one launch: a grid-stride loop over the concatenated 32-value
// blocks of all jobs, each block done as in dequant_planes_kernel.
__global__ void __launch_bounds__(256) dequant_planes_multi_kernel(const StageJobs J) {
  const long long total = J.start[J.n];
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    int j = 0;
    while (j + 1 < J.n && i >= J.start[j + 1]) ++j;
    const long long b = i - J.start[j];
    const int K = J.K[j], N = J.N[j], nb = K / 32;
    const int n = (int)(b / nb), kb = (int)(b - (long long)n * nb);
    const uint32_t d = J.scales[j][(long long)kb * N + n];
    const uint32_t d2 = d | (d << 16);
    uint4* o = reinterpret_cast<uint4*>(J.out[j] + (long long)n * K + (long long)kb * 32);
    if (J.q4[j]) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(J.values[j] + (long long)n * (K / 2) + (long long)kb * 16));
      o[0] = dequant8_q4(w.x, d2);
      o[1] = dequant8_q4(w.y, d2);
      o[2] = dequant8_q4(w.z, d2);
      o[3] = dequant8_q4(w.w, d2);
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(J.values[j] + (long long)n * K + (long long)kb * 32);
      const uint4 a = __ldg(src), c = __ldg(src + 1);
      o[0] = dequant8_q8(make_uint2(a.x, a.y), d2);
      o[1] = dequant8_q8(make_uint2(a.z, a.w), d2);
      o[2] = dequant8_q8(make_uint2(c.x, c.y), d2);
      o[3] = dequant8_q8(make_uint2(c.z, c.w), d2);
    }
  }
}

// All loops over the 16 values below are fully unrolled with compile-time
// indices (tails are predicated), so v[] stays in registers.
__device__ __forceinline__ void store16(void* base, long long idx, int is_f32, const float (&v)[16], int n_valid,
                                        bool vec_ok) {
  if (is_f32) {
    float* p = reinterpret_cast<float*>(base) + idx;
    if (vec_ok && n_valid == 16) {
#pragma unroll
      for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < n_valid) p[i] = v[i];
    }
  } else {
    __half* p = reinterpret_cast<__half*>(base) + idx;
    if (vec_ok && n_valid == 16) {
      *reinterpret_cast<uint4*>(p) = make_uint4(pack_h2(v[0], v[1]), pack_h2(v[2], v[3]), pack_h2(v[4], v[5]),
                                                pack_h2(v[6], v[7]));
      *reinterpret_cast<uint4*>(p + 8) = make_uint4(pack_h2(v[8], v[9]), pack_h2(v[10], v[11]),
                                                    pack_h2(v[12], v[13]), pack_h2(v[14], v[15]));
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < n_valid) p[i] = __float2half_rn(v[i]);
    }
  }
}

// bias + activation + RoPE + scale on 16 consecutive columns [gc, gc+16) of
// row gr; rope_pos = RoPE position of the row (gr % rope_mod), or -1 for none.
// SB: the bias of these 16 columns is staged in shared memory at sbias (16-byte aligned) instead of read
// from global memory.
template <bool SB = false>
__device__ __forceinline__ void epi_math16(const EpiParams& ep, int rope_pos, int gc, int N, float (&v)[16],
                                           const float* sbias = nullptr) {
  const int n_valid = min(16, N - gc);
  if (SB) {
    if (ep.bias) {
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 b = *reinterpret_cast<const float4*>(sbias + i);  // one address for the warp: broadcast
        f2_unpack(f2_add(f2_pack(v[i], v[i + 1]), f2_pack(b.x, b.y)), v[i], v[i + 1]);
        f2_unpack(f2_add(f2_pack(v[i + 2], v[i + 3]), f2_pack(b.z, b.w)), v[i + 2], v[i + 3]);
      }
    }
  } else if (ep.bias) {
    if (ep.mode == EPI_DECONV2) {
      const int c0 = gc % ep.cout;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < n_valid) v[i] += __ldg(ep.bias + (c0 + i) % ep.cout);
    } else if (n_valid == 16 && ((reinterpret_cast<uintptr_t>(ep.bias + gc) & 15) == 0)) {
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(ep.bias + gc + i));
        f2_unpack(f2_add(f2_pack(v[i], v[i + 1]), f2_pack(b.x, b.y)), v[i], v[i + 1]);
        f2_unpack(f2_add(f2_pack(v[i + 2], v[i + 3]), f2_pack(b.z, b.w)), v[i + 2], v[i + 3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < n_valid) v[i] += __ldg(ep.bias + gc + i);
    }
  }
  // one uniform branch per activation, so the 16 independent evaluations interleave
  if (ep.act == ACT_GELU_ERF) {
#pragma unroll
    for (int i = 0; i < 16; i += 2) gelu_erf2(v[i], v[i + 1]);
  } else if (ep.act == ACT_GELU_TANH) {
#pragma unroll
    for (int i = 0; i < 16; i += 2) gelu_tanh2(v[i], v[i + 1]);
  } else if (ep.act == ACT_RELU) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = fmaxf(v[i], 0.0f);
  }
  if (rope_pos >= 0 && gc < ep.rope_cols) {
    // position-major table: the (cos, sin) pairs of one frequency for consecutive positions are
    // adjacent, so the 32 rows (positions) of a warp read one contiguous 256-byte run per pair
    const float2* tb = reinterpret_cast<const float2*>(ep.rope) + rope_pos;
    const long long pstride = ep.rope_mod;
    const int d0 = gc % ep.rope_D;  // even: gc and rope_D are even
    if ((ep.rope_D & 15) == 0 && (ep.rope_cols & 15) == 0 && n_valid == 16) {
      // the 16 columns lie inside one head: 8 consecutive frequencies
      const float2* t2 = tb + (long long)(d0 >> 1) * pstride;
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const float2 cs = __ldg(t2 + (long long)(i >> 1) * pstride);
        const float a = v[i], b = v[i + 1];
        v[i] = a * cs.x - b * cs.y;
        v[i + 1] = a * cs.y + b * cs.x;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        if (i + 1 < n_valid && gc + i < ep.rope_cols) {
          const int d = (d0 + i) % ep.rope_D;
          const float2 cs = __ldg(tb + (long long)(d >> 1) * pstride);
          const float a = v[i], b = v[i + 1];
          v[i] = a * cs.x - b * cs.y;
          v[i + 1] = a * cs.y + b * cs.x;
        }
      }
    }
  }
  if (ep.out_scale != 1.0f) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] *= ep.out_scale;
  }
}

// Direct-store epilogue for 16 columns (row remaps, broadcast residuals, deconvolution scatter).
__device__ __forceinline__ void epi_store_direct16(const EpiParams& ep, long long gr, int gc, int N, float (&v)[16]) {
  const int n_valid = min(16, N - gc);
  if (ep.mode == EPI_STORE) {
    const long long orow = map_row(ep.map, gr);
    if (orow < 0) return;
    if (ep.resid) {
      long long rrow;
      if (ep.resid_up) {
        const long long HW = (long long)ep.map.H * ep.map.W;
        const long long f = orow / HW;
        const int rem = (int)(orow - f * HW);
        const int y = rem / ep.map.W, x = rem - (rem / ep.map.W) * ep.map.W;
        const int W2 = ep.map.W / 2, H2 = ep.map.H / 2;
        rrow = (f * H2 + y / 2) * W2 + x / 2;
      } else {
        rrow = ep.resid_mod ? orow % ep.resid_mod : orow;
      }
      const float* rp = ep.resid + rrow * ep.ldr + gc;
      if (n_valid == 16 && (ep.ldr % 4) == 0) {
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const float4 t = *reinterpret_cast<const float4*>(rp + i);
          v[i] += t.x; v[i + 1] += t.y; v[i + 2] += t.z; v[i + 3] += t.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i < n_valid) v[i] += rp[i];
      }
    }
    store16(ep.out, orow * ep.ldo + gc, ep.out_f32, v, n_valid, (ep.ldo % 16) == 0);
    return;
  }
  if (ep.mode == EPI_DECONV2) {
    const long long HW = (long long)ep.map.H * ep.map.W;
    const long long f = gr / HW;
    const int rem = (int)(gr - f * HW);
    const int y = rem / ep.map.W, x = rem - y * ep.map.W;
    const int kpos = gc / ep.cout;
    const int co = gc - kpos * ep.cout;
    const int ky = kpos >> 1, kx = kpos & 1;
    const long long opix = (f * 2 * ep.map.H + 2 * y + ky) * (2LL * ep.map.W) + 2 * x + kx;
    const bool vec_ok = (ep.cout % 16) == 0 && (ep.ldo % 16) == 0;
    store16(ep.out, opix * ep.ldo + co, ep.out_f32, v, n_valid, vec_ok);
  }
}

// 16 TMEM columns into R[o..o+15] (o a compile-time constant keeps R in registers).
#define TMEM_LD16(taddr, R, o)                                                                              \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "                                                    \
               "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"                            \
               : "=r"(R[o + 0]), "=r"(R[o + 1]), "=r"(R[o + 2]), "=r"(R[o + 3]), "=r"(R[o + 4]),           \
                 "=r"(R[o + 5]), "=r"(R[o + 6]), "=r"(R[o + 7]), "=r"(R[o + 8]), "=r"(R[o + 9]),           \
                 "=r"(R[o + 10]), "=r"(R[o + 11]), "=r"(R[o + 12]), "=r"(R[o + 13]), "=r"(R[o + 14]),      \
                 "=r"(R[o + 15])                                                                            \
               : "r"(taddr))

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

// Waits for a phase without looking at the abort flag (used only to drain).
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity, int* err) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitNs) {
      if (err) atomicCAS(err, 0, kErrWaitDrain);
      return;
    }
  }
}

__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void tma_store_2d(const void* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_store_4d(const void* map, const void* src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ void tma_store_5d(const void* map, const void* src, int x, int y, int z, int w, int v) {
  asm volatile("cp.async.bulk.tensor.5d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5, %6}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// PAIR: clusters of 2 CTAs on two SMs share one 256 x BN tile (cta_group::2):
// each CTA loads its 128 rows of A and BN/2 rows of B per stage (so a stage
// is 32 KB instead of 48 KB at BN = 256 and more stages fit), the even CTA
// issues M = 256 MMAs over both CTAs' shared memory into both TMEMs, and
// each CTA runs the epilogue of its own 128 rows. Stage completion is counted
// on the leader's `full` barrier; the leader's commits arrive on `empty` /
// `tfull` of both CTAs; both epilogues release accumulators on the leader's
// `tempty`.
// EW: epilogue warps, 8 (2 column groups) or 16 (4 column groups, for epilogues
// that would otherwise outlast the main loop).
// BLK (pixel-block tiling of a channel-last f16 input map [conv_F][conv_H][conv_W][conv_C]):
// a tile's 128 rows are an 8 x 16 pixel block (the pair's two CTAs take vertically adjacent
// blocks), loaded by 4-D TMA.
//   BLK 1, implicit 3x3 / pad 1 convolution (A never materialised): k-block kb = (tap, 64-channel
//     block) is the block shifted by the tap; TMA zero-fills the taps outside the map, which is
//     the padding. The output tile goes out through a 4-D TMA store that clips at the map's edges.
//   BLK 2, 2x2 / stride 2 deconvolution (EPI_DECONV2 columns (ky*2 + kx)*cout + co): for one ky,
//     the columns (kx, co) of the block's pixels are a regular box of the [F][2H][2W][cout]
//     output, (kx*cout + co, x, ky, y, f) with strides (1, 2 cout, 2W cout, 4W cout, 4HW cout):
//     one 5-D TMA store per chunk instead of scattered 16-value stores.
template <int CONV_TY_BLOCKS>
__device__ __forceinline__ void conv_tile_origin(int mt, const EpiParams& ep, uint32_t rank, int* x0, int* y0,
                                                 int* f) {
  const int txn = (ep.conv_W + 15) / 16;
  const int tyn = (ep.conv_H + 8 * CONV_TY_BLOCKS - 1) / (8 * CONV_TY_BLOCKS);
  const int tx = mt % txn, r = mt / txn;
  const int ty = r % tyn;
  *f = r / tyn;
  *x0 = tx * 16;
  *y0 = ty * 8 * CONV_TY_BLOCKS + (int)rank * 8;
}

// QB (quantised weights; 0: f16 B via TMA): the weight tile of a k-step arrives as
// block values (QB 1, q4_0: 32 bytes of nibbles per row; QB 2, q8_0: 64 int8 per
// row; tmB over the value plane) plus the two f16 block scales of each row (tmS
// over the [K/32][N] scale plane) in one of QS landing buffers (a ring of its own,
// `qfull` / `qempty`, filled by lane 1 of the producer warp up to QS k-steps ahead,
// so that the load latency stays off the stage ring). The dequant_warps(EW) warps
// after the epilogue warps wait for the stage's B buffer to be free (`empty`) and
// for the landing buffer, write the f16 tile into the B buffer in the SW128 layout
// the TMA would have produced, fence it for the async proxy, release the landing
// buffer and arrive on `full` (with pairs: on the leader's `full`, whose count then
// includes both CTAs' dequantising warps).
// Column tile of linear tile t (row tile t / tiles_n): the column order is rotated by the row tile, so that
// a persistent CTA whose tile stride is a multiple of tiles_n still meets every column tile. Without the
// rotation such a CTA would meet one column tile only, and when N is not a multiple of BN the CTAs holding
// the narrow last column tile idle while the others work (Hiera-T stage-0 qkv, N = 288 on 74 SM pairs).
__device__ __forceinline__ int tile_col(int t, int tiles_n) { return (t % tiles_n + t / tiles_n) % tiles_n; }

template <int BN, int STAGES, bool TMA_EPI, bool PAIR, int EW, int BLK = 0, int QB = 0, int QS = 0>
__global__ void __launch_bounds__(gemm_threads(EW, QB ? dequant_warps(EW) : 0), 1)
    gemm_f16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR,
                       const __grid_constant__ CUtensorMap tmS, int M, int N, int K, EpiParams ep,
                       int resid_in_place, int* err) {
  constexpr int BN_CTA = PAIR ? BN / 2 : BN;  // rows of B this CTA loads per stage
  constexpr int TM = PAIR ? 2 * kBM : kBM;    // output rows per tile
  constexpr uint32_t A_BYTES = kBM * kBK * 2;
  constexpr uint32_t B_BYTES = BN_CTA * kBK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t STAGING = TMA_EPI ? 4 * kStageBufBytes : 0;
  constexpr uint32_t BIAS_BYTES = TMA_EPI ? BN * 4 : 0;
  constexpr int DW = QB ? dequant_warps(EW) : 0;
  constexpr uint32_t QROW = QB == 1 ? 32 : 64;              // value bytes per weight row per stage
  constexpr uint32_t QV_BYTES = QB ? BN_CTA * QROW : 0;     // block values of the stage
  constexpr uint32_t Q_BYTES = QB ? QV_BYTES + 4 * BN_CTA : 0;  // + 2 f16 scales per row
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(BLK == 0 || TMA_EPI, "pixel-block tiles store through TMA");
  static_assert(QB == 0 || BLK == 0, "quantised weights: plain GEMMs only");
  static_assert((QB == 0) == (QS == 0), "landing buffers exactly for quantised weights");
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512 || TMEM_COLS == 128, "TMEM columns must be a power of 2");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sC = sB + STAGES * B_BYTES;  // staging (TMA epilogue only), 1024-aligned
  float* sBias = reinterpret_cast<float*>(sC + STAGING);  // TMA epilogue: the tile's bias, BN floats
  uint8_t* sQ = sC + STAGING + BIAS_BYTES;  // QB landing buffers, 512-byte multiples
  uint64_t* full = reinterpret_cast<uint64_t*>(sQ + QS * Q_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint64_t* rfull = mma_done + 1;  // [half*2 + buf]: residual chunk landed in its staging buffer
  uint64_t* qfull = rfull + 4;     // [QS] (QB): a k-step's block values and scales landed
  uint64_t* qempty = qfull + QS;   // [QS] (QB): the dequantising warps have read the landing buffer
  uint64_t* dq = qempty + QS;      // [STAGES] (QB pairs, peer CTA): its half of the B tile is written
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(dq + (QS ? STAGES : 0));
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;  // CTA within the pair; 0 issues the MMAs
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int n_units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int tiles_m = (M + TM - 1) / TM;
  const int tiles_n = (N + BN - 1) / BN;
  const int n_tiles = tiles_m * tiles_n;
  const int nk = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // QB: the producer's arrive (A bytes) + one arrive per dequantising warp of this CTA (+ with
      // pairs, one relayed arrive for all of the peer's)
      mbar_init(&full[s], QB ? 1 + DW + (PAIR ? 1 : 0) : 1);
      mbar_init(&empty[s], 1);
      if (QB) mbar_init(&dq[s], DW);
    }
    for (int s = 0; s < QS; ++s) {
      mbar_init(&qfull[s], 1);
      mbar_init(&qempty[s], DW);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      // pairs: the leader's epilogue warps + one arrive relayed for all of the peer's (quantised
      // weights: every warp of both CTAs arrives on the leader's barrier)
      mbar_init(&tempty[a], PAIR ? (QB ? 2 * EW : (rank == 0 ? EW + 1 : EW)) : EW);
    }
    mbar_init(mma_done, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&rfull[i], 1);
    *s_abort = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (QB) tma_prefetch_desc(&tmS);
    if (TMA_EPI) tma_prefetch_desc(&tmC);
    if (TMA_EPI && resid_in_place) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(s_tmem, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(s_tmem, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;        // bit s: stage s has been armed at least once
      uint32_t armed_phase = 0;  // bit s: parity of the last arming of stage s
      bool ok = true;
      const int cbn = BLK == 1 ? ep.conv_C / kBK : 1;  // 64-channel blocks per tap
      for (int t = unit; t < n_tiles && ok; t += n_units) {
        const int m0 = (t / tiles_n) * TM + (int)rank * kBM;
        const int n0 = tile_col(t, tiles_n) * BN + (int)rank * BN_CTA;
        int cx = 0, cy = 0, cf = 0;
        if (BLK) conv_tile_origin<PAIR ? 2 : 1>(t / tiles_n, ep, rank, &cx, &cy, &cf);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, s_abort, err, kErrWaitEmpty)) { ok = false; break; }
          // BLK 1: k-block kb = tap (ky, kx) x channel block cb, the block shifted by (kx - 1, ky - 1);
          // BLK 2: channel block kb of the block itself
          const int tap = BLK == 1 ? kb / cbn : 4;
          const int cb = BLK == 1 ? kb - tap * cbn : kb;
          const int ky = tap / 3, kx = tap - 3 * (tap / 3);
          if (QB) {
            // A as usual (the weight tile comes through the landing ring, lane 1)
            if (PAIR) {
              const uint32_t fb = cluster_addr(smem_u32(&full[stage]), 0);
              if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * A_BYTES);
              tma_load_2d_pair(&tmA, fb, sA + stage * A_BYTES, kb * kBK, m0);
            } else {
              mbar_arrive_expect_tx(&full[stage], A_BYTES);
              tma_load_2d(&tmA, &full[stage], sA + stage * A_BYTES, kb * kBK, m0);
            }
          } else if (PAIR) {
            // both CTAs' bytes complete the leader's barrier; only the leader arms it
            const uint32_t fb = cluster_addr(smem_u32(&full[stage]), 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
            if (BLK)
              tma_load_4d_pair(&tmA, fb, sA + stage * A_BYTES, cb * kBK, cx + kx - 1, cy + ky - 1, cf);
            else
              tma_load_2d_pair(&tmA, fb, sA + stage * A_BYTES, kb * kBK, m0);
            tma_load_2d_pair(&tmB, fb, sB + stage * B_BYTES, kb * kBK, n0);
          } else {
            mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
            if (BLK)
              tma_load_4d(&tmA, &full[stage], sA + stage * A_BYTES, cb * kBK, cx + kx - 1, cy + ky - 1, cf);
            else
              tma_load_2d(&tmA, &full[stage], sA + stage * A_BYTES, kb * kBK, m0);
            tma_load_2d(&tmB, &full[stage], sB + stage * B_BYTES, kb * kBK, n0);
          }
          armed |= 1u << stage;
          armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Every issued copy lands before the CTA may exit. With pairs the copies
      // are counted on the leader, so wait instead for the MMA's release of
      // each stage's last use (which also makes every commit that targets this
      // CTA's `empty` barriers land before exit).
      for (int s = 0; s < STAGES; ++s)
        if (armed & (1u << s)) mbar_wait_drain(PAIR ? &empty[s] : &full[s], (armed_phase >> s) & 1u, err);
    } else if (QB && lane == 1) {
      // landing ring: the block values and scales of every k-step of this CTA's half of the weight
      // tile, up to QS k-steps ahead of the dequantising warps
      int qi = 0;
      uint32_t qph = 0;
      uint32_t armed = 0, armed_phase = 0;
      bool ok = true;
      for (int t = unit; t < n_tiles && ok; t += n_units) {
        const int n0 = tile_col(t, tiles_n) * BN + (int)rank * BN_CTA;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&qempty[qi], qph ^ 1, s_abort, err, kErrWaitEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&qfull[qi], Q_BYTES);
          tma_load_2d(&tmB, &qfull[qi], sQ + qi * Q_BYTES, kb * (int)QROW, n0);
          tma_load_2d(&tmS, &qfull[qi], sQ + qi * Q_BYTES + QV_BYTES, n0, kb * 2);
          armed |= 1u << qi;
          armed_phase = (armed_phase & ~(1u << qi)) | (qph << qi);
          if (++qi == QS) { qi = 0; qph ^= 1; }
        }
      }
      for (int s = 0; s < QS; ++s)
        if (armed & (1u << s)) mbar_wait_drain(&qfull[s], (armed_phase >> s) & 1u, err);
    }
  } else if (warp == 1) {
    if (!QB && PAIR && lane == 0 && rank == 1) {
      // the peer's MMA warp is otherwise idle: it relays "this CTA's epilogue warps have read the
      // accumulator" to the leader's `tempty`, one cluster-scope arrive per tile instead of one per
      // warp (per-warp cluster releases stalled the short-K GEMMs' epilogues on membar)
      const uint32_t tempty_leader = cluster_addr(smem_u32(&tempty[0]), 0);
      int acc = 0;
      uint32_t aphase = 0;
      for (int t = unit; t < n_tiles; t += n_units) {
        if (!mbar_wait(&tempty[acc], aphase, s_abort, err, kErrWaitMisc)) break;
        mbar_arrive_cluster(tempty_leader + (uint32_t)(acc * 8));
        if (++acc == 2) { acc = 0; aphase ^= 1; }
      }
    }
    if (QB && PAIR && lane == 0 && rank == 1) {
      // the peer's MMA warp is otherwise idle: it relays "this CTA's half of the B tile is written"
      // to the leader's `full` barrier, one cluster-scope arrive per k-step instead of one per warp
      const uint32_t full_leader = cluster_addr(smem_u32(&full[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = unit; t < n_tiles && ok; t += n_units) {
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&dq[stage], phase, s_abort, err, kErrWaitMisc)) { ok = false; break; }
          mbar_arrive_cluster(full_leader + (uint32_t)(stage * 8));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_f16(TM, BN, 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      bool ok = true;
      bool issued = false;
      for (int t = unit; t < n_tiles && ok; t += n_units) {
        if (!mbar_wait(&tempty[acc], aphase ^ 1, s_abort, err, kErrWaitTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!((QB && PAIR) ? mbar_wait_cluster(&full[stage], phase, s_abort, err, kErrWaitFull)
                             : mbar_wait(&full[stage], phase, s_abort, err, kErrWaitFull))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sdesc_k_sw128(smem_u32(sA + stage * A_BYTES));
          const uint64_t db = sdesc_k_sw128(smem_u32(sB + stage * B_BYTES));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            if (PAIR)
              tc_mma_f16_pair(d_tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (kb | kk) != 0 ? 1u : 0u);
            else
              tc_mma_f16(d_tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          issued = true;
          if (PAIR) tc_commit_pair(&empty[stage], 3); else tc_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (PAIR) tc_commit_pair(&tfull[acc], 3); else tc_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; aphase ^= 1; }
      }
      // All MMAs complete before TMEM is released.
      if (issued) {
        if (PAIR) tc_commit_pair(mma_done, 1); else tc_commit(mma_done);
        mbar_wait_drain(mma_done, 0, err);
      }
    }
  } else if (QB && warp >= 2 + EW) {
    // Dequantising warps. Unit u = (row u >> 1, block u & 1) of the stage: one 32-value block of a
    // weight row (16 nibble bytes or 32 int8, one scale) -> four 16-byte chunks of the SW128 row.
    // A warp's 32 units are 16 consecutive rows: its block loads cover 512 contiguous bytes and its
    // chunk stores 4 distinct 16-byte positions per bank group, both conflict-free.
    constexpr int UNITS = 2 * BN_CTA;
    constexpr int DT = (DW > 0 ? DW : 1) * 32;
    static_assert(UNITS % DT == 0, "units per dequantising thread");
    const int dt = (int)threadIdx.x - 32 * (2 + EW);
    int stage = 0, qi = 0;
    uint32_t phase = 0, qph = 0;
    bool ok = true;
    for (int t = unit; t < n_tiles && ok; t += n_units) {
      for (int kb = 0; kb < nk; ++kb) {
        // the stage's B buffer is free (its last MMAs completed) and the k-step's blocks landed
        if (!mbar_wait(&empty[stage], phase ^ 1, s_abort, err, kErrWaitEmpty) ||
            !mbar_wait(&qfull[qi], qph, s_abort, err, kErrWaitMisc)) {
          ok = false;
          break;
        }
        const uint8_t* qv = sQ + qi * Q_BYTES;
        const uint16_t* qs = reinterpret_cast<const uint16_t*>(qv + QV_BYTES);
        uint8_t* sb = sB + stage * B_BYTES;
#pragma unroll
        for (int u = dt; u < UNITS; u += DT) {
          const int r = u >> 1, b = u & 1;
          const uint32_t d = qs[b * BN_CTA + r];
          const uint32_t d2 = d | (d << 16);
          uint4 o[4];
          if (QB == 1) {
            const uint4 w = *reinterpret_cast<const uint4*>(qv + r * 32 + b * 16);
            o[0] = dequant8_q4(w.x, d2);
            o[1] = dequant8_q4(w.y, d2);
            o[2] = dequant8_q4(w.z, d2);
            o[3] = dequant8_q4(w.w, d2);
          } else {
            const uint4 w0 = *reinterpret_cast<const uint4*>(qv + r * 64 + b * 32);
            const uint4 w1 = *reinterpret_cast<const uint4*>(qv + r * 64 + b * 32 + 16);
            o[0] = dequant8_q8(make_uint2(w0.x, w0.y), d2);
            o[1] = dequant8_q8(make_uint2(w0.z, w0.w), d2);
            o[2] = dequant8_q8(make_uint2(w1.x, w1.y), d2);
            o[3] = dequant8_q8(make_uint2(w1.z, w1.w), d2);
          }
          uint8_t* row = sb + r * 128;
#pragma unroll
          for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(row + (((4 * b + j) ^ (r & 7)) << 4)) = o[j];
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&qempty[qi]);
          mbar_arrive(PAIR && rank == 1 ? &dq[stage] : &full[stage]);
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
        if (++qi == QS) { qi = 0; qph ^= 1; }
      }
    }
  } else {
    // Epilogue: EW warps in G = EW/4 column groups; the 4 warps of a group cover
    // the 4 TMEM lane quarters (the tile's 128 rows) of the group's CG columns.
    // The 4 staging buffers (16 KB) are split NBUF per group.
    constexpr int G = EW / 4;
    constexpr int CG = BN / G;
    constexpr int NBUF = 4 / G;
    const int q = warp & 3;
    const int grp = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const bool leader = ((warp - 2) & 3) == 0 && lane == 0;  // issues this group's TMA copies
    int acc = 0;
    uint32_t aphase = 0;
    uint32_t chunk_ctr = 0;
    uint32_t r_issued0 = 0, r_issued1 = 0, r_used0 = 0, r_used1 = 0;  // residual loads per staging buffer
    // residual chunks are TMA-loaded into the staging buffers (two per group with 8 warps, one
    // with 16: the second chunk of a group then waits for the first chunk's store to read it)
    const bool out_f32 = ep.out_f32 != 0;
    const int rip = resid_in_place;
    const int cw = out_f32 ? 32 : 64;                   // chunk = 128 B of columns: 32 f32 or 64 f16
    // staging buffer of chunk `ctr`, and how many chunks used that buffer before it
    auto buf_of = [&](uint32_t ctr) -> int { return grp * NBUF + (NBUF == 1 ? 0 : (int)(ctr & 1)); };
    auto buf_uses = [&](uint32_t ctr) -> uint32_t { return NBUF == 1 ? ctr : (ctr >> 1); };
    // the TMA store that last used the buffer has read it
    auto wait_buf_read = [&]() {
      if (NBUF == 1) bulk_wait_read0(); else bulk_wait_read1();
    };
    // Residual chunk `ctr` (columns gcb.., rows m0..) -> its staging buffer, once
    // the TMA store that last used that buffer has finished reading it.
    // all_read: wait for every earlier TMA store to have read its buffer (the chunk two ahead reuses the
    // buffer of the store just issued)
    auto issue_resid = [&](uint32_t ctr, int gcb, int m0, bool all_read = false) {
      const int bsel = buf_of(ctr);
      if (all_read) bulk_wait_read0(); else wait_buf_read();
      if (gcb < N) {
        mbar_arrive_expect_tx(&rfull[bsel], kStageBufBytes);
        // the residual's row: the output row itself, or (resid_mod: a table repeated every
        // resid_mod rows, a multiple of the 128-row tile or wrap-padded) its row inside the table
        const int rrow = ep.resid_mod ? (int)((long long)m0 % ep.resid_mod) : m0;
        tma_load_2d(&tmR, &rfull[bsel], sC + bsel * kStageBufBytes, gcb, rrow);
      } else {
        mbar_arrive(&rfull[bsel]);
      }
      if (NBUF == 1 || !(ctr & 1)) ++r_issued0; else ++r_issued1;
    };
    // this CTA's epilogue warps release an accumulator on the MMA-issuing CTA's barrier
    auto release_acc = [&](int a) {
      if (PAIR && QB)
        mbar_arrive_cluster(cluster_addr(smem_u32(&tempty[a]), 0));
      else
        mbar_arrive(&tempty[a]);  // pairs: the peer's warps arrive on its own barrier, relayed below
    };
    for (int t = unit; t < n_tiles; t += n_units) {
      const int m0 = (t / tiles_n) * TM + (int)rank * kBM;
      const int n0 = tile_col(t, tiles_n) * BN;
      int cx = 0, cy = 0, cf = 0;
      if (BLK) conv_tile_origin<PAIR ? 2 : 1>(t / tiles_n, ep, rank, &cx, &cy, &cf);
      // a column group wholly past N (the last column tile of an N that is not a multiple of BN) has
      // nothing to store: it only takes part in the accumulator hand-over
      const bool grp_live = n0 + grp * CG < N;
      const bool sb_on = TMA_EPI && ep.bias != nullptr && grp_live;
      // the first residual chunks do not depend on the accumulator: fetch them during the main loop, one per
      // staging buffer of the group (two with 8 epilogue warps), so a short-K GEMM waits for one residual
      // load per tile instead of one per chunk
      const int pre = (NBUF == 2 && CG >= 2 * cw) ? 2 : 1;
      if (TMA_EPI && rip && leader && grp_live) {
        issue_resid(chunk_ctr, n0 + grp * CG, m0);
        if (pre == 2) issue_resid(chunk_ctr + 1, n0 + grp * CG + cw, m0, true);
      }
      // the bias of the group's columns goes to shared memory once per tile, before the accumulator wait,
      // instead of sitting in every chunk's critical path as an L2 load. The previous tile's reads of the
      // slice finished before its last group barrier; without a residual the first chunk's group barrier
      // orders these stores before the reads.
      if (sb_on) {
        const int gt = ((warp - 2) & 3) * 32 + lane;  // thread within the group
        if (gt < CG) {
          const int col = n0 + grp * CG + gt;
          sBias[grp * CG + gt] = col < N ? __ldg(ep.bias + (ep.mode == EPI_DECONV2 ? col % ep.cout : col)) : 0.0f;
        }
        if (rip) named_bar(1 + grp, 128);
      }
      if (!mbar_wait(&tfull[acc], aphase, s_abort, err, kErrWaitTmemFull)) break;
      tc_fence_after();
      if (!grp_live) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(acc);
        if (++acc == 2) { acc = 0; aphase ^= 1; }
        continue;
      }
      const long long gr = (long long)m0 + row;
      const int rope_pos = (ep.rope && gr < ep.rope_rows) ? (int)(gr % ep.rope_mod) : -1;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + grp * CG);
      if (TMA_EPI) {
        bool ok = true;
        for (int c0 = 0; c0 < CG; c0 += cw) {
          const int gcb = n0 + grp * CG + c0;
          const int bsel = buf_of(chunk_ctr);
          uint8_t* buf = sC + bsel * kStageBufBytes;
          // the chunk goes through registers 32 columns at a time; the first 32 are
          // loaded from TMEM while the staging buffer is awaited
          uint32_t r[32];
          TMEM_LD16(tbase + (uint32_t)c0, r, 0);
          TMEM_LD16(tbase + (uint32_t)(c0 + 16), r, 16);
          if (rip) {
            // parity of this buffer's residual barrier = number of its earlier uses & 1
            if (!mbar_wait(&rfull[bsel], buf_uses(chunk_ctr) & 1u, s_abort, err, kErrWaitMisc)) {
              tc_wait_ld();
              ok = false;
              break;
            }
            if (NBUF == 1 || !(chunk_ctr & 1)) ++r_used0; else ++r_used1;
          } else {
            if (leader) wait_buf_read();
            named_bar(1 + grp, 128);
          }
          uint8_t* rowp = buf + row * 128;
#pragma unroll
          for (int s0 = 0; s0 < 64; s0 += 32) {
            if (s0 < cw) {
              if (s0 > 0) {
                TMEM_LD16(tbase + (uint32_t)(c0 + s0), r, 0);
                TMEM_LD16(tbase + (uint32_t)(c0 + s0 + 16), r, 16);
              }
              tc_wait_ld();
              if (c0 + cw >= CG && s0 + 32 >= cw) {
                // accumulator fully read: hand TMEM back to the MMA warp early
                tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(acc);
              }
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                float v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[j * 16 + i]);
                const int gc = gcb + s0 + j * 16;
                if (gc < N) epi_math16<true>(ep, rope_pos, gc, N, v, sBias + (gc - n0));
                if (out_f32) {
#pragma unroll
                  for (int u = 0; u < 4; ++u) {
                    const int unit = (s0 + j * 16) / 4 + u;  // 16-byte unit within the 128-byte row
                    float4* sp = reinterpret_cast<float4*>(rowp + ((unit ^ (row & 7)) << 4));
                    if (rip) {
                      const float4 rv = *sp;
                      f2_unpack(f2_add(f2_pack(v[4 * u], v[4 * u + 1]), f2_pack(rv.x, rv.y)), v[4 * u], v[4 * u + 1]);
                      f2_unpack(f2_add(f2_pack(v[4 * u + 2], v[4 * u + 3]), f2_pack(rv.z, rv.w)), v[4 * u + 2],
                                v[4 * u + 3]);
                    }
                    *sp = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                  }
                } else {
#pragma unroll
                  for (int u = 0; u < 2; ++u) {
                    const int unit = (s0 + j * 16) / 8 + u;
                    *reinterpret_cast<uint4*>(rowp + ((unit ^ (row & 7)) << 4)) =
                        make_uint4(pack_h2(v[8 * u], v[8 * u + 1]), pack_h2(v[8 * u + 2], v[8 * u + 3]),
                                   pack_h2(v[8 * u + 4], v[8 * u + 5]), pack_h2(v[8 * u + 6], v[8 * u + 7]));
                  }
                }
              }
            }
          }
          fence_proxy_async_smem();
          named_bar(1 + grp, 128);
          if (leader && gcb < N) {
            if (BLK == 1) {
              tma_store_4d(&tmC, buf, gcb, cx, cy, cf);
            } else if (BLK == 2) {
              const int ky = gcb / (2 * ep.cout);  // a chunk never straddles a ky (2 cout is a multiple of 64)
              tma_store_5d(&tmC, buf, gcb - ky * 2 * ep.cout, cx, ky, cy, cf);
            } else {
              tma_store_2d(&tmC, buf, gcb, m0);
            }
            bulk_commit();
          }
          if (rip && leader && c0 + pre * cw < CG) issue_resid(chunk_ctr + pre, gcb + pre * cw, m0, pre == 2);
          ++chunk_ctr;
        }
        if (!ok) break;
      } else {
#pragma unroll 1
        for (int c = 0; c < CG; c += 16) {
          uint32_t r[16];
          TMEM_LD16(tbase + (uint32_t)c, r, 0);
          tc_wait_ld();
          if (c + 16 >= CG) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(acc);
          }
          const int gc = n0 + grp * CG + c;
          if (gr < M && gc < N) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
            epi_math16(ep, rope_pos, gc, N, v);
            epi_store_direct16(ep, gr, gc, N, v);
          }
        }
      }
      if (++acc == 2) { acc = 0; aphase ^= 1; }
    }
    if (TMA_EPI && leader) {
      bulk_wait_all();
      // a residual load issued but never consumed (only after an abort) lands before exit
      if (r_issued0 > r_used0) mbar_wait_drain(&rfull[grp * NBUF + 0], (r_issued0 - 1) & 1u, err);
      if (NBUF == 2 && r_issued1 > r_used1) mbar_wait_drain(&rfull[grp * NBUF + 1], (r_issued1 - 1) & 1u, err);
    }
  }

  tc_fence_before();
  __syncthreads();
  // pairs: the leader's MMAs (which read the peer's shared memory and write its
  // TMEM) and all remote arrives are complete before either CTA frees or exits
  if (PAIR) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2D tensor map over a row-major [rows][ld] matrix, box = box_rows x (128 B), SW128.
int make_map_2d(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld, int box_rows,
                int elem_bytes) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return -10;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * elem_bytes) % 16 != 0) return -11;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * elem_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / elem_bytes), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -12;
}

// 4-D tensor map over a channel-last [F][H][W][C] map, box = (128 B of channels) x 16 x 8 x 1
// (an 8 x 16 pixel block, 128 rows of 128 B in the SW128 layout of a 2-D tile), SW128;
// coordinates outside the map read as zero (loads) or are not written (stores).
int make_map_conv(CUtensorMap* map, const void* base, int F, int H, int W, int C, int elem_bytes) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return -10;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || ((long long)C * elem_bytes) % 16 != 0) return -11;
  cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)F};
  cuuint64_t strides[3] = {(cuuint64_t)C * elem_bytes, (cuuint64_t)W * C * elem_bytes,
                           (cuuint64_t)H * W * C * elem_bytes};
  cuuint32_t box[4] = {(cuuint32_t)(128 / elem_bytes), 16, 8, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -12;
}

// 5-D tensor map over the [F][2H][2W][cout] output of a 2x2 / stride 2 deconvolution seen as
// (kx*cout + co, x, ky, y, f), box = (128 B) x 16 x 1 x 8 x 1 (the 8 x 16 input-pixel block's
// outputs for one ky and 128 B of (kx, co)), SW128.
int make_map_deconv_out(CUtensorMap* map, const void* base, int F, int H, int W, int cout, int elem_bytes) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return -10;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || ((long long)cout * elem_bytes) % 16 != 0) return -11;
  const cuuint64_t c = (cuuint64_t)cout, eb = (cuuint64_t)elem_bytes;
  cuuint64_t dims[5] = {2 * c, (cuuint64_t)W, 2, (cuuint64_t)H, (cuuint64_t)F};
  cuuint64_t strides[4] = {2 * c * eb, 2 * (cuuint64_t)W * c * eb, 4 * (cuuint64_t)W * c * eb,
                           4 * (cuuint64_t)H * W * c * eb};
  cuuint32_t box[5] = {(cuuint32_t)(128 / elem_bytes), 16, 1, 8, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -12;
}

// Unswizzled 2-D tensor map over a row-major [rows][cols] matrix of `dtype` (row stride ld elements),
// box = box_cols x box_rows: the quantised weight planes of QB GEMMs.
int make_map_plain_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, long long rows,
                      long long cols, long long ld, int box_cols, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return -10;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * elem_bytes) % 16 != 0 ||
      (box_cols * elem_bytes) % 16 != 0)
    return -11;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * elem_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -12;
}

// BLK 1 / 2: A is the channel-last input map (geometry in ep.conv_*) of gemm_conv3x3 /
// gemm_deconv2x2 and M the number of pixel-block tiles x the tile rows.
// QB 1 / 2: B is the q4_0 nibble plane [N][K/2] / q8_0 value plane [N][K] (ldb unused) and
// scales the f16 block-scale plane [K/32][N].
template <int BN, int STAGES, bool TMA_EPI, bool PAIR, int EW = 8, int BLK = 0, int QB = 0, int QS = 0>
int launch_gemm(const __half* A, long long lda, const void* B, long long ldb, int M, int N, int K,
                const EpiParams& ep, int resid_in_place, int* err, cudaStream_t st,
                const __half* scales = nullptr) {
  constexpr int BN_CTA = PAIR ? BN / 2 : BN;
  constexpr int DW = QB ? dequant_warps(EW) : 0;
  constexpr int QROW = QB == 1 ? 32 : 64;
  CUtensorMap ma, mb, mc, mr, ms;
  int rc = BLK ? make_map_conv(&ma, A, ep.conv_F, ep.conv_H, ep.conv_W, ep.conv_C, 2)
               : make_map_2d(&ma, A, M, K, lda, kBM, 2);
  if (rc) return rc;
  if (QB) {
    const long long row_bytes = QB == 1 ? K / 2 : K;
    rc = make_map_plain_2d(&mb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, row_bytes, row_bytes, QROW, BN_CTA);
    if (rc) return rc;
    rc = make_map_plain_2d(&ms, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K / 32, N, N, BN_CTA, 2);
  } else {
    rc = make_map_2d(&mb, B, N, K, ldb, BN_CTA, 2);
    ms = mb;  // unused
  }
  if (rc) return rc;
  if (TMA_EPI) {
    const int eb = ep.out_f32 ? 4 : 2;
    if (BLK == 1) rc = make_map_conv(&mc, ep.out, ep.conv_F, ep.conv_H, ep.conv_W, N, eb);
    else if (BLK == 2) rc = make_map_deconv_out(&mc, ep.out, ep.conv_F, ep.conv_H, ep.conv_W, ep.cout, eb);
    else rc = make_map_2d(&mc, ep.out, M, N, ep.ldo, kBM, eb);
    if (rc) return rc;
  } else {
    mc = ma;  // unused
  }
  if (TMA_EPI && resid_in_place && static_cast<const void*>(ep.resid) != ep.out) {
    // a separate f32 residual (resid_mod rows repeated, or M rows)
    rc = make_map_2d(&mr, ep.resid, ep.resid_mod ? ep.resid_mod + (ep.resid_wrap_pad ? kBM : 0) : M, N, ep.ldr, kBM, 4);
    if (rc) return rc;
  } else {
    mr = mc;
  }
  constexpr size_t q_bytes = QB ? (size_t)BN_CTA * QROW + 4 * BN_CTA : 0;
  constexpr size_t smem = 1024 + (size_t)STAGES * (kBM + BN_CTA) * kBK * 2 + (size_t)QS * q_bytes +
                          (TMA_EPI ? 4 * kStageBufBytes + BN * 4 : 0) +
                          (2 * STAGES + 2 * QS + (QS ? STAGES : 0) + 9) * 8 + 16;
  static_assert(smem <= 232448, "shared memory per CTA");
  auto kernel = gemm_f16_tc_kernel<BN, STAGES, TMA_EPI, PAIR, EW, BLK, QB, QS>;
  constexpr int kThreads = gemm_threads(EW, DW);
  // co-resident CTAs (or SM pairs), set up once per device
  const int max_units = kernel_setup(reinterpret_cast<const void*>(kernel), smem,
                                     PAIR ? pair_units : sm_units, kThreads);
  if (max_units <= 0) return -13;
  const int tm = PAIR ? 2 * kBM : kBM;
  const int tiles = ((M + tm - 1) / tm) * ((N + BN - 1) / BN);
  const int units = tiles < max_units ? tiles : max_units;
  if (!PAIR) {
    kernel<<<units, kThreads, smem, st>>>(ma, mb, mc, mr, ms, M, N, K, ep, resid_in_place, err);
    return launch_status("gemm");
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * units);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ma, mb, mc, mr, ms, M, N, K, ep, resid_in_place, err);
  if (e != cudaSuccess) {
    fprintf(stderr, "s3b: CUDA error at gemm (pair) launch: %s (%d)\n", cudaGetErrorString(e), (int)e);
    cudaGetLastError();
    return -14;
  }
  return launch_status("gemm (pair)");
}

}  // namespace

void* tensor_map_encoder() { return reinterpret_cast<void*>(get_encode_fn()); }

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return 0;
  fprintf(stderr, "s3b: CUDA error at %s launch: %s (%d)\n", what, cudaGetErrorString(e), (int)e);
  return -14;
}

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_sms_mu;    // guards g_sms
std::mutex g_setup_mu;  // guards g_setup (num_sms may be called while it is held)
int g_sms[kMaxDevices] = {0};
// (device, kernel) -> the value kernel_setup computed there
std::map<std::pair<int, const void*>, int> g_setup;
}  // namespace

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lock(g_sms_mu);
  if (g_sms[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sms[dev] = n > 0 ? n : 148;
  }
  return g_sms[dev];
}

int kernel_setup(const void* kernel, size_t smem, int (*units)(const void*, size_t, int), int threads) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -13;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  const auto key = std::make_pair(dev, kernel);
  const auto it = g_setup.find(key);
  if (it != g_setup.end()) return it->second;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    cudaGetLastError();
    return -13;
  }
  const int v = units ? units(kernel, smem, threads) : 1;
  if (v <= 0) return -13;
  g_setup[key] = v;
  return v;
}

// Checks the epilogue parameters of a plain GEMM and decides whether its output leaves through the
// TMA epilogue (and whether that epilogue adds the residual in place). Returns 0 or a negative code.
static int route_epilogue(const EpiParams& ep, int N, bool* tma_epi_out, int* rip_out) {
  if (ep.mode == EPI_DECONV2 && (ep.cout <= 0 || N != 4 * ep.cout)) return -3;
  if (ep.mode != EPI_STORE && ep.mode != EPI_DECONV2) return -3;
  if (ep.rope && (ep.rope_D <= 0 || (ep.rope_D & 1) || ep.rope_mod <= 0)) return -3;
  const int eb = ep.out_f32 ? 4 : 2;
  // TMA epilogue: plain row-major output; the residual (f32 outputs) absent, the output itself, or a
  // separate f32 matrix, possibly a table repeated every resid_mod rows (a multiple of the 128-row tile,
  // so no tile straddles a repeat, or wrap-padded by 128 rows), loaded by TMA into the staging buffer
  const bool resid_sep = ep.resid != nullptr && static_cast<const void*>(ep.resid) != ep.out;
  const bool resid_ok =
      ep.resid == nullptr ||
      (ep.out_f32 && !ep.resid_up &&
       (resid_sep ? ((ep.resid_mod == 0 || ep.resid_mod % kBM == 0 || ep.resid_wrap_pad) && (ep.ldr * 4) % 16 == 0 &&
                     ep.ldr >= N &&
                     (reinterpret_cast<uintptr_t>(ep.resid) & 15) == 0)
                  : (ep.resid_mod == 0 && ep.ldr == ep.ldo)));
  const bool tma_epi = ep.mode == EPI_STORE && ep.map.kind == 0 && resid_ok &&
                       (reinterpret_cast<uintptr_t>(ep.out) & 15) == 0 && (ep.ldo * eb) % 16 == 0 && ep.ldo >= N;
  *tma_epi_out = tma_epi;
  *rip_out = (tma_epi && ep.resid) ? 1 : 0;
  return 0;
}

int gemm_f16(const __half* A, long long lda, const __half* B, long long ldb, int M, int N, int K,
             const EpiParams& ep, int* err, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0) return -1;
  if (lda < K || ldb < K) return -2;
  bool tma_epi = false;
  int resid_in_place = 0;
  const int rc = route_epilogue(ep, N, &tma_epi, &resid_in_place);
  if (rc) return rc;
  if (tma_epi) {
    if (N <= 128) return launch_gemm<128, 4, true, false>(A, lda, B, ldb, M, N, K, ep, resid_in_place, err, st);
    // short-K GEMMs (QKV + RoPE, MLP fc1 + GELU, attention proj + residual): their epilogue outlasts
    // the main loop with 8 epilogue warps, so they run 16 (measured 4-12% faster on the f32
    // in-place-residual proj, 2-20% on the f16 ones)
    if (K < 2048 && g_gemm_wide_epi) {
      // with 16 epilogue warps the pair main loop pays off (measured 3-4% on QKV + RoPE, 15% on the
      // f32 in-place-residual attention proj: 788 -> 905 TF/s at 8 ViT frames)
      if (M > 2 * kBM && (g_gemm_pairs == 2 || (g_gemm_pairs == 1 && !ep.out_f32)))
        return launch_gemm<256, 5, true, true, 16>(A, lda, B, ldb, M, N, K, ep, resid_in_place, err, st);
      return launch_gemm<256, 3, true, false, 16>(A, lda, B, ldb, M, N, K, ep, resid_in_place, err, st);
    }
    // 256-row tiles on SM pairs where the main loop dominates (long K): measured faster for
    // K = 4736 (ViT fc2), slower for K = 1024 GEMMs whose epilogue (GELU, RoPE, residual)
    // already takes longer than their main loop
    if (g_gemm_pairs && M > 2 * kBM && (K >= 2048 || g_gemm_pairs == 2))
      return launch_gemm<256, 5, true, true>(A, lda, B, ldb, M, N, K, ep, resid_in_place, err, st);
    return launch_gemm<256, 3, true, false>(A, lda, B, ldb, M, N, K, ep, resid_in_place, err, st);
  }
  if (N <= 128) return launch_gemm<128, 6, false, false>(A, lda, B, ldb, M, N, K, ep, 0, err, st);
  return launch_gemm<256, 4, false, false>(A, lda, B, ldb, M, N, K, ep, 0, err, st);
}

template <int QB>
static int gemm_q_launch(const __half* A, long long lda, const QWeight& w, int M, int N, int K, const EpiParams& ep,
                         bool tma_epi, int rip, int* err, cudaStream_t st) {
  // 4 stages of A / f16 B and as many landing buffers as fit beside them (6 for q4_0, 3 for q8_0);
  // the direct-store variant (no staging buffers, 256 B rows per CTA) 3 stages and 6 / 4 buffers
  constexpr int QSP = QB == 1 ? 6 : 3;
  constexpr int QSD = QB == 1 ? 6 : 4;
  if (tma_epi) {
    // 256-row tiles on SM pairs (each CTA dequantises half of the weight tile); 16 epilogue warps for
    // the short-K GEMMs, as for f16 weights
    if (K < 2048 && g_gemm_wide_epi)
      return launch_gemm<256, 4, true, true, 16, 0, QB, QSP>(A, lda, w.values, 0, M, N, K, ep, rip, err, st,
                                                            w.scales);
    return launch_gemm<256, 4, true, true, 8, 0, QB, QSP>(A, lda, w.values, 0, M, N, K, ep, rip, err, st, w.scales);
  }
  return launch_gemm<256, 3, false, false, 8, 0, QB, QSD>(A, lda, w.values, 0, M, N, K, ep, 0, err, st, w.scales);
}

int dequant_planes_f16(const QWeight& w, int N, int K, __half* out, long long ldo, cudaStream_t st) {
  if (N <= 0 || K <= 0 || K % 32 || ldo < K || ldo % 8 || !w.values || !w.scales || !out) return -2;
  if ((reinterpret_cast<uintptr_t>(w.values) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return -11;
  const long long total = (long long)N * (K / 32);
  const long long cap = (long long)num_sms() * 8;
  const long long want = (total + 255) / 256;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(w.scales);
  const uint8_t* v = reinterpret_cast<const uint8_t*>(w.values);
  if (w.type == QT_Q4_0) dequant_planes_kernel<1><<<grid, 256, 0, st>>>(v, sc, N, K, out, ldo);
  else if (w.type == QT_Q8_0) dequant_planes_kernel<2><<<grid, 256, 0, st>>>(v, sc, N, K, out, ldo);
  else return -2;
  return launch_status("dequant_planes");
}

int dequant_planes_multi(const StageJob* jobs, int n, cudaStream_t st) {
  if (n <= 0 || n > kMaxStageJobs) return -2;
  StageJobs J;
  J.n = n;
  J.start[0] = 0;
  for (int j = 0; j < n; ++j) {
    const StageJob& a = jobs[j];
    if (a.N <= 0 || a.K <= 0 || a.K % 32 || !a.w.values || !a.w.scales || !a.out) return -2;
    if (a.w.type != QT_Q4_0 && a.w.type != QT_Q8_0) return -2;
    if ((reinterpret_cast<uintptr_t>(a.w.values) & 15) || (reinterpret_cast<uintptr_t>(a.out) & 15)) return -11;
    J.values[j] = reinterpret_cast<const uint8_t*>(a.w.values);
    J.scales[j] = reinterpret_cast<const uint16_t*>(a.w.scales);
    J.out[j] = a.out;
    J.N[j] = a.N;
    J.K[j] = a.K;
    J.q4[j] = a.w.type == QT_Q4_0;
    J.start[j + 1] = J.start[j] + (long long)a.N * (a.K / 32);
  }
  const long long cap = (long long)num_sms() * 8;
  const long long want = (J.start[n] + 255) / 256;
  dequant_planes_multi_kernel<<<(unsigned)(want < cap ? want : cap), 256, 0, st>>>(J);
  return launch_status("dequant_planes_multi");
}

int gemm_q(const __half* A, long long lda, const QWeight& w, int M, int N, int K, const EpiParams& ep, int* err,
           cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0) return -1;
  if (lda < K || K % 32 || N % 8 || !w.values || !w.scales) return -2;
  if ((reinterpret_cast<uintptr_t>(w.values) & 15) || (reinterpret_cast<uintptr_t>(w.scales) & 15)) return -2;
  bool tma_epi = false;
  int rip = 0;
  const int rc = route_epilogue(ep, N, &tma_epi, &rip);
  if (rc) return rc;
  if (w.type == QT_Q4_0) return gemm_q_launch<1>(A, lda, w, M, N, K, ep, tma_epi, rip, err, st);
  if (w.type == QT_Q8_0) return gemm_q_launch<2>(A, lda, w, M, N, K, ep, tma_epi, rip, err, st);
  return -2;
}

int gemm_conv3x3(const __half* x, int F, int H, int W, int C, const __half* Bw, long long ldb, int N,
                 const EpiParams& ep_in, int* err, cudaStream_t st) {
  if (F <= 0 || H <= 0 || W <= 0 || C <= 0 || N <= 0 || C % kBK) return -2;
  // plain stores of the whole [F][H][W][N] output: no residual, RoPE, row map or strided rows
  if (ep_in.mode != EPI_STORE || ep_in.map.kind != 0 || ep_in.resid || ep_in.rope || ep_in.ldo != N) return -2;
  if ((reinterpret_cast<uintptr_t>(ep_in.out) & 15) || ((long long)N * (ep_in.out_f32 ? 4 : 2)) % 16) return -2;
  EpiParams ep = ep_in;
  ep.conv_F = F;
  ep.conv_H = H;
  ep.conv_W = W;
  ep.conv_C = C;
  const int K = 9 * C;
  const bool pair = g_gemm_pairs != 0;
  const long long tiles = (long long)F * ((W + 15) / 16) * ((H + (pair ? 15 : 7)) / (pair ? 16 : 8));
  const long long m_virtual = tiles * (pair ? 2 * kBM : kBM);
  if (m_virtual > 0x7fffffffLL) return -2;
  if (pair) return launch_gemm<256, 5, true, true, 8, 1>(x, C, Bw, ldb, (int)m_virtual, N, K, ep, 0, err, st);
  return launch_gemm<256, 3, true, false, 8, 1>(x, C, Bw, ldb, (int)m_virtual, N, K, ep, 0, err, st);
}

int gemm_deconv2x2(const __half* x, int F, int H, int W, int Cin, const __half* Bw, long long ldb, int cout,
                   const EpiParams& ep_in, int* err, cudaStream_t st) {
  if (F <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cin % 8 || cout <= 0 || cout % 32) return -2;
  if (ep_in.resid || ep_in.rope || ep_in.map.kind != 0) return -2;
  if ((reinterpret_cast<uintptr_t>(ep_in.out) & 15) || (reinterpret_cast<uintptr_t>(x) & 15)) return -2;
  EpiParams ep = ep_in;
  ep.mode = EPI_DECONV2;
  ep.cout = cout;
  ep.conv_F = F;
  ep.conv_H = H;
  ep.conv_W = W;
  ep.conv_C = Cin;
  const int N = 4 * cout, K = Cin;
  const bool pair = g_gemm_pairs != 0;
  const long long tiles = (long long)F * ((W + 15) / 16) * ((H + (pair ? 15 : 7)) / (pair ? 16 : 8));
  const long long m_virtual = tiles * (pair ? 2 * kBM : kBM);
  if (m_virtual > 0x7fffffffLL) return -2;
  if (pair) return launch_gemm<256, 5, true, true, 16, 2>(x, Cin, Bw, ldb, (int)m_virtual, N, K, ep, 0, err, st);
  return launch_gemm<256, 3, true, false, 16, 2>(x, Cin, Bw, ldb, (int)m_virtual, N, K, ep, 0, err, st);
}

void set_gemm_pairs(int mode) { g_gemm_pairs = mode; }
void set_gemm_wide_epilogue(int mode) { g_gemm_wide_epi = mode; }
int gemm_config_id() { return g_gemm_pairs * 2 + g_gemm_wide_epi; }

}  // namespace s3b
