// Tensor-core (tcgen05 / TMEM / TMA) flash attention for head dim 64: the
// ViT windowed and global attention of sam3_vit_block_forward
// (ggml_flash_attn_ext at sam3.cpp:3774; softmax(q k^T / 8) v, no mask).
//
// One CTA = one 128-query tile of one (window, head); 10 warps, 2 CTAs / SM.
// TMEM (256 columns): S [0,128), O [128,192), P [192,256).
//   warp 0     TMA: Q tile once, then K_j, V_j through a 5-slot ring (two key
//              tiles of look-ahead). The tensor map is 3-D (channels, token,
//              window) over the fused [tokens][3E] qkv buffer, so a tile never
//              reads another window (rows past the window are zero-filled).
//   warp 1     MMA: S = Q K_j^T (M=128, N=128, K=64) into TMEM; after the
//              softmax wrote P_j: O += P_j V_j (M=128, N=64, K=128; A = P read
//              from TMEM, B = V as an MN-major shared-memory operand) into one
//              TMEM accumulator kept across tiles.
//   warps 2-9  softmax. Each query row (TMEM lane) is shared by two threads,
//              one per 64-key half of the tile: row max over its half (two
//              32-column TMEM reads), one exchange of the partial maxima
//              through shared memory, then p = 2^(s*scale*log2e - m) written
//              to TMEM as f16 pairs (the A operand of the P V product).
//              TMEMP = false (a tuning option) keeps the earlier layout: P in
//              a 128B-swizzled shared-memory operand and a 3-slot ring.
//              The reference max m only moves when the row max grows by more
//              than 2^8 (so P <= 256, exact enough in f16); only then are the
//              row's running sum and its O row in TMEM rescaled, which after
//              the first tiles is rare. Each thread keeps its half's sum; the
//              two are added once at the end, when O is read, divided by the
//              sum and stored (32 columns per thread).
// Every wait is bounded; a timeout records an error code and the CTA unwinds
// without skipping any named barrier.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace s3b {
namespace {

constexpr int kD = 64;
constexpr int kBQ = 128;
constexpr int kBK = 128;
constexpr int kSlots = 3;
constexpr uint32_t kTileBytes = kBK * kD * 2;  // 16 KB: 128 rows x 128 B
constexpr uint32_t kPBytes = kBQ * kBK * 2;    // 32 KB: two 128 x 64 swizzled halves
constexpr int kSoftmaxWarps = 8;
constexpr int kThreads = 64 + 32 * kSoftmaxWarps;
constexpr float kLazyMax = 8.0f;  // log2 of the largest P value before the reference max moves
constexpr int kXchgBytes = (2 * 2 * kBQ + 2 * kBQ) * 4;  // partial maxima (2 slots x 2 halves) + final sums

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

// MN-major, 128B-swizzled operand (rows of 64 f16 along N, consecutive rows
// along K): SBO = 1024 B between 8-row groups, LBO = stride between 64-wide N
// atoms (a single atom here).
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(kTileBytes >> 4) << 16;  // LBO (unused: N == 64)
  d |= (uint64_t)(1024u >> 4) << 32;       // SBO
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, for x <= 8 (the softmax exponent), to take part of the
// exponentials off the MUFU unit. Cody-Waite range reduction x = n + f,
// n = rint(x) taken from the low mantissa bits of x + 1.5*2^23, f in
// [-0.5, 0.5]; 2^f by a degree-3 polynomial fitted here for minimum maximum
// relative error on that interval (7.5e-5, below the f16 half ulp of P); 2^n
// added to the exponent field. x is clamped at -126 so the exponent stays in
// range (P rounds to 0 in f16 there anyway).
__device__ __forceinline__ float exp2_poly3(float x) {
  x = fmaxf(x, -126.f);
  const float j = x + 12582912.f;
  const float f = x - (j - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.0551716685f, f, 0.2426111251f), f, 0.6932609677f), f, 0.9999280572f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(j) << 23));
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100)
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

#define TMEM_LD32(taddr, R)                                                                                  \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "                                                     \
               "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"                                     \
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                    \
               : "=r"(R[0]), "=r"(R[1]), "=r"(R[2]), "=r"(R[3]), "=r"(R[4]), "=r"(R[5]), "=r"(R[6]),         \
                 "=r"(R[7]), "=r"(R[8]), "=r"(R[9]), "=r"(R[10]), "=r"(R[11]), "=r"(R[12]), "=r"(R[13]),     \
                 "=r"(R[14]), "=r"(R[15]), "=r"(R[16]), "=r"(R[17]), "=r"(R[18]), "=r"(R[19]), "=r"(R[20]),  \
                 "=r"(R[21]), "=r"(R[22]), "=r"(R[23]), "=r"(R[24]), "=r"(R[25]), "=r"(R[26]), "=r"(R[27]),  \
                 "=r"(R[28]), "=r"(R[29]), "=r"(R[30]), "=r"(R[31])                                          \
               : "r"(taddr))

#define TMEM_ST16(taddr, R)                                                                                  \
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "                                               \
               "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),                     \
               "r"(R[0]), "r"(R[1]), "r"(R[2]), "r"(R[3]), "r"(R[4]), "r"(R[5]), "r"(R[6]), "r"(R[7]),       \
               "r"(R[8]), "r"(R[9]), "r"(R[10]), "r"(R[11]), "r"(R[12]), "r"(R[13]), "r"(R[14]), "r"(R[15])  \
               : "memory")

#define TMEM_ST8(taddr, R)                                                                                   \
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(R[0]), \
               "r"(R[1]), "r"(R[2]), "r"(R[3]), "r"(R[4]), "r"(R[5]), "r"(R[6]), "r"(R[7])                    \
               : "memory")

#define TMEM_ST32(taddr, R)                                                                                  \
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "                                               \
               "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"                                    \
               "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),             \
               "r"(R[0]), "r"(R[1]), "r"(R[2]), "r"(R[3]), "r"(R[4]), "r"(R[5]), "r"(R[6]), "r"(R[7]),       \
               "r"(R[8]), "r"(R[9]), "r"(R[10]), "r"(R[11]), "r"(R[12]), "r"(R[13]), "r"(R[14]), "r"(R[15]), \
               "r"(R[16]), "r"(R[17]), "r"(R[18]), "r"(R[19]), "r"(R[20]), "r"(R[21]), "r"(R[22]),           \
               "r"(R[23]), "r"(R[24]), "r"(R[25]), "r"(R[26]), "r"(R[27]), "r"(R[28]), "r"(R[29]),           \
               "r"(R[30]), "r"(R[31])                                                                        \
               : "memory")

__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity, int* err) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitNs) {
      if (err) atomicCAS(err, 0, kErrWaitDrain);
      return;
    }
  }
}

// Max over this thread's 64 keys of the tile (TMEM columns [cbase, cbase+64) of
// its lane), in log2 units; MASKED: keys at or past kvalid are tiling padding.
template <bool MASKED>
__device__ __forceinline__ float half_row_max(uint32_t taddr, int cbase, int kvalid, float sl2) {
  float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
  for (int c = 0; c < kBK / 2; c += 32) {
    if (MASKED && cbase + c >= kvalid) break;
    uint32_t r[32];
    TMEM_LD32(taddr + (uint32_t)c, r);
    tc_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[e] = __uint_as_float(r[i + e]);
        if (MASKED) v[e] = cbase + c + i + e < kvalid ? v[e] : -INFINITY;
      }
      mx0 = fmax3f(mx0, v[0], v[1]);
      mx1 = fmax3f(mx1, v[2], v[3]);
      mx2 = fmax3f(mx2, v[4], v[5]);
      mx3 = fmax3f(mx3, v[6], v[7]);
    }
  }
  return fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
}

// p = 2^(s*sl2 - m) over this thread's 64 keys, written as f16 into its row of
// the 128B-swizzled P half (`prow`), returns the row sum; MASKED: padding keys
// inside the last 32-key chunk get p = 0 (the P V product reads to its end).
// The warp arrives on s_empty right after its last read of S (as half_row_p_tmem).
template <bool MASKED, int NPOLY>
__device__ __forceinline__ float half_row_p(uint32_t taddr, int cbase, int kvalid, float sl2, float m, uint8_t* prow,
                                            int row, uint64_t* s_empty) {
  const unsigned long long sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(-m, -m);
  unsigned long long acc0 = f2_pack(0.f, 0.f), acc1 = acc0;
  bool released = false;
#pragma unroll
  for (int c = 0; c < kBK / 2; c += 32) {
    if (MASKED && cbase + c >= kvalid) break;
    uint32_t r[32];
    TMEM_LD32(taddr + (uint32_t)c, r);
    tc_wait_ld();
    if (c + 32 >= kBK / 2 || (MASKED && cbase + c + 32 >= kvalid)) {  // this warp's last read of S
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(s_empty);
      released = true;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float p[8];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const int i = 8 * u + e;
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), sl2x2, negm2), x0, x1);
        p[e] = e < NPOLY ? exp2_poly3(x0) : ex2(x0);
        p[e + 1] = e + 1 < NPOLY ? exp2_poly3(x1) : ex2(x1);
        if (MASKED) {
          p[e] = cbase + c + i < kvalid ? p[e] : 0.f;
          p[e + 1] = cbase + c + i + 1 < kvalid ? p[e + 1] : 0.f;
        }
      }
      acc0 = f2_add(acc0, f2_add(f2_pack(p[0], p[1]), f2_pack(p[4], p[5])));
      acc1 = f2_add(acc1, f2_add(f2_pack(p[2], p[3]), f2_pack(p[6], p[7])));
      const int unit = (c >> 3) + u;  // 16-byte unit (8 keys) inside the 128-byte row
      *reinterpret_cast<uint4*>(prow + ((unit ^ (row & 7)) << 4)) =
          make_uint4(pack_h2(p[0], p[1]), pack_h2(p[2], p[3]), pack_h2(p[4], p[5]), pack_h2(p[6], p[7]));
    }
  }
  if (!released) {  // no key of this half is real: S was not read
    tc_fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(s_empty);
  }
  float a0, a1, b0, b1;
  f2_unpack(acc0, a0, a1);
  f2_unpack(acc1, b0, b1);
  return (a0 + a1) + (b0 + b1);
}

// As half_row_p, but P goes to TMEM (the A operand of the P V product): this thread's 64 keys as
// 32 columns of f16 pairs of its lane, starting at p_taddr. The warp arrives on s_empty right after
// its last read of S, so the MMA warp computes the next S while the exponentials run.
template <bool MASKED, int NPOLY>
__device__ __forceinline__ float half_row_p_tmem(uint32_t taddr, int cbase, int kvalid, float sl2, float m,
                                                 uint32_t p_taddr, uint64_t* s_empty) {
  // the scale-and-shift and the row sum run two-wide (packed f32x2); the exponentials one by one
  const unsigned long long sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(-m, -m);
  unsigned long long acc0 = f2_pack(0.f, 0.f), acc1 = acc0;
  bool released = false;
#pragma unroll
  for (int c = 0; c < kBK / 2; c += 32) {
    if (MASKED && cbase + c >= kvalid) break;
    uint32_t r[32];
    TMEM_LD32(taddr + (uint32_t)c, r);
    tc_wait_ld();
    if (c + 32 >= kBK / 2 || (MASKED && cbase + c + 32 >= kvalid)) {  // this warp's last read of S
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(s_empty);
      released = true;
    }
    uint32_t pk[16];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float p[8];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const int i = 8 * u + e;
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), sl2x2, negm2), x0, x1);
        p[e] = e < NPOLY ? exp2_poly3(x0) : ex2(x0);
        p[e + 1] = e + 1 < NPOLY ? exp2_poly3(x1) : ex2(x1);
        if (MASKED) {
          p[e] = cbase + c + i < kvalid ? p[e] : 0.f;
          p[e + 1] = cbase + c + i + 1 < kvalid ? p[e + 1] : 0.f;
        }
      }
      acc0 = f2_add(acc0, f2_add(f2_pack(p[0], p[1]), f2_pack(p[4], p[5])));
      acc1 = f2_add(acc1, f2_add(f2_pack(p[2], p[3]), f2_pack(p[6], p[7])));
#pragma unroll
      for (int e = 0; e < 4; ++e) pk[4 * u + e] = pack_h2(p[2 * e], p[2 * e + 1]);
    }
    TMEM_ST16(p_taddr + (uint32_t)(c / 2), pk);
  }
  if (!released) {  // no key of this half is real: S was not read
    tc_fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(s_empty);
  }
  float a0, a1, b0, b1;
  f2_unpack(acc0, a0, a1);
  f2_unpack(acc1, b0, b1);
  return (a0 + a1) + (b0 + b1);
}

struct TcAttnArgs {
  int heads, ntok, nwin;
  int q_col, k_col, v_col;  // column offsets (elements) of q / k / v of head 0 in a row
  __half* o;
  long long o_n;
  RowMap omap;
  float sl2;  // softmax scale * log2(e)
};

// NPOLY of every 8 softmax exponentials use exp2_poly3, the rest MUFU ex2.
// PMODE (where P, the A operand of the P V product, lives): 1 TMEM (columns [192,256); its shared
// memory goes to two more K/V slots); 0 a 128B-swizzled shared-memory operand. (Alternating the two
// per tile, to double-buffer P, measured slower: the smaller K/V ring and the register spills cost
// more than the wait for the previous P V that it removes.)
template <int NPOLY, int PMODE>
__global__ void __launch_bounds__(kThreads, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm, TcAttnArgs a, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem;                          // 16 KB
  constexpr int kSl = PMODE == 1 ? 5 : kSlots;
  uint8_t* sKV = sQ + kTileBytes;              // kSl x 16 KB
  uint8_t* sP = sKV + kSl * kTileBytes;        // 32 KB (shared-memory P only)
  float* xmax = reinterpret_cast<float*>(sP + (PMODE == 1 ? 0 : kPBytes));  // [2 slots][2 halves][128 rows]
  float* xsum = xmax + 4 * kBQ;                          // [2 halves][128 rows]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xsum + 2 * kBQ);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                // [kSl]
  uint64_t* kv_empty = kv_full + kSl;          // [kSl]
  uint64_t* s_full = kv_empty + kSl;
  uint64_t* s_empty = s_full + 1;
  uint64_t* p_full = s_empty + 1;
  uint64_t* p_empty = p_full + 1;              // P buffer free (the previous P V has completed)
  uint64_t* o_done = p_empty + 1;
  uint64_t* mma_done = o_done + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid, query tile fastest: the tiles of one (window, head) run together and share K/V in L2.
  // Blocks take the units from the end: the qkv rows the projection GEMM wrote last are still in L2,
  // and the output rows written last (the first windows) are the first the next GEMM reads.
  const unsigned unit = gridDim.x - 1 - blockIdx.x;
  const int n_qt = (a.ntok + kBQ - 1) / kBQ;
  const int bh = (int)(unit / n_qt);
  const int qb = (int)(unit - (unsigned)bh * n_qt);
  const int w = bh / a.heads, h = bh - w * a.heads;
  const int nkb = (a.ntok + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kSl; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, kSoftmaxWarps);
    mbar_init(p_full, kSoftmaxWarps);
    mbar_init(p_empty, 1);
    mbar_init(o_done, 1);
    mbar_init(mma_done, 1);
    *s_abort = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, 256);  // S: columns [0,128), O: [128,192)
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      // Q once, then K_0, V_0, K_1, V_1, ... through the ring
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_3d(&tm, q_full, sQ, a.q_col + h * kD, qb * kBQ, w);
      uint32_t armed = 0, armed_phase = 0;
      bool ok = true;
      for (int t = 0; t < 2 * nkb && ok; ++t) {
        const int s = t % kSl;
        const uint32_t use = (uint32_t)(t / kSl);
        if (!mbar_wait(&kv_empty[s], (use & 1) ^ 1, s_abort, err, kErrWaitEmpty)) { ok = false; break; }
        mbar_arrive_expect_tx(&kv_full[s], kTileBytes);
        const int j = t >> 1;
        const int col = ((t & 1) ? a.v_col : a.k_col) + h * kD;
        tma_load_3d(&tm, &kv_full[s], sKV + s * kTileBytes, col, j * kBK, w);
        armed |= 1u << s;
        armed_phase = (armed_phase & ~(1u << s)) | ((use & 1) << s);
      }
      mbar_wait_drain(q_full, 0, err);
      for (int s = 0; s < kSl; ++s)
        if (armed & (1u << s)) mbar_wait_drain(&kv_full[s], (armed_phase >> s) & 1u, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(kBQ, kBK, 0);                    // both K-major
      constexpr uint32_t idesc_s64 = idesc_f16(kBQ, kBK / 2, 0);              // ragged last key tile
      constexpr uint32_t idesc_o = idesc_f16(kBQ, kD, 0) | (1u << 16);        // B (V) MN-major
      bool ok = mbar_wait(q_full, 0, s_abort, err, kErrWaitFull);
      tc_fence_after();
      const uint64_t dq = sdesc_k_sw128(smem_u32(sQ));
      bool issued = false;
      // S_j = Q K_j^T; only the first 64 key columns when at most 64 keys of the tile are real
      auto issue_s = [&](int j) -> bool {
        const int t = 2 * j, s = t % kSl;
        if (!mbar_wait(&kv_full[s], (uint32_t)(t / kSl) & 1, s_abort, err, kErrWaitFull)) return false;
        if (j > 0 && !mbar_wait(s_empty, (uint32_t)(j - 1) & 1, s_abort, err, kErrWaitMisc)) return false;
        tc_fence_after();
        const uint64_t dk = sdesc_k_sw128(smem_u32(sKV + s * kTileBytes));
        const uint32_t ids = (a.ntok - j * kBK <= kBK / 2) ? idesc_s64 : idesc_s;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) tc_mma_f16(tmem, dq + (uint64_t)(kk * 2), dk + (uint64_t)(kk * 2), ids, kk != 0);
        tc_commit(s_full);
        tc_commit(&kv_empty[s]);
        issued = true;
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nkb && ok; ++j) {
        if (j + 1 < nkb && !issue_s(j + 1)) { ok = false; break; }
        // O += P_j V_j (after the softmax wrote P_j and, where needed, rescaled O)
        const int t = 2 * j + 1, s = t % kSl;
        if (!mbar_wait(p_full, (uint32_t)j & 1, s_abort, err, kErrWaitMisc)) { ok = false; break; }
        if (!mbar_wait(&kv_full[s], (uint32_t)(t / kSl) & 1, s_abort, err, kErrWaitFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t pa = smem_u32(sP), va = smem_u32(sKV + s * kTileBytes);
        // K steps that hold a real key (the softmax writes P only up to the chunk holding the last key)
        const int nk16 = min(kBK / 16, (a.ntok - j * kBK + 15) / 16);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          if (kk >= nk16) break;
          // P: two 128 x 64 K-major halves (32 B per K step inside a half); V: 16 key rows = 2048 B per K step
          const uint64_t dv = sdesc_mn_sw128(va + (uint32_t)(kk * 2048));
          if (PMODE == 1) {
            // P from TMEM: 8 columns (16 keys as f16 pairs) per K step
            tc_mma_f16_ts(tmem + 128, tmem + 192 + (uint32_t)(kk * 8), dv, idesc_o, (j > 0 || kk != 0) ? 1u : 0u);
          } else {
            const uint64_t dp = sdesc_k_sw128(pa + (uint32_t)((kk >> 2) * (kBQ * 128) + (kk & 3) * 32));
            tc_mma_f16(tmem + 128, dp, dv, idesc_o, (j > 0 || kk != 0) ? 1u : 0u);
          }
        }
        tc_commit(&kv_empty[s]);
        tc_commit(p_empty);
      }
      if (ok) tc_commit(o_done);
      if (issued) {
        tc_commit(mma_done);
        mbar_wait_drain(mma_done, 0, err);
      }
    }
  } else {
    // softmax: warp w owns TMEM lanes 32*(w%4) .. +31 (query rows) and key half hsel of every tile
    const int q4 = warp & 3;
    const int hsel = (warp - 2) >> 2;
    const int row = q4 * 32 + lane;
    const int cbase = hsel * (kBK / 2);
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t o_addr = tmem + lane_off + 128 + (uint32_t)(hsel * (kD / 2));
    // a warp whose 32 query rows are all tiling padding only keeps the barrier protocol
    const bool rows_live = qb * kBQ + q4 * 32 < a.ntok;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {  // every softmax warp runs every iteration (named barriers)
      if (ok) ok = mbar_wait(s_full, (uint32_t)j & 1, s_abort, err, kErrWaitTmemFull);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const int kvalid = a.ntok - j * kBK;  // keys at or past this count are tiling padding
      // partial row max over this thread's key half (4 independent chains)
      const bool full_tile = kvalid >= kBK;  // every tile but a ragged last one
      const uint32_t s_addr = tmem + lane_off + (uint32_t)cbase;
      float pm = -INFINITY;
      if (ok && rows_live)
        pm = full_tile ? half_row_max<false>(s_addr, cbase, kvalid, a.sl2)
                       : half_row_max<true>(s_addr, cbase, kvalid, a.sl2);
      // exchange the partial maxima of the two halves of each row (slot j & 1 is rewritten
      // two tiles later, after the partner has passed the next barrier)
      xmax[((j & 1) * 2 + hsel) * kBQ + row] = pm;
      named_bar(1, 32 * kSoftmaxWarps);
      const float m_tile = fmaxf(pm, xmax[((j & 1) * 2 + (hsel ^ 1)) * kBQ + row]);
      // lazy reference max: move it only when the row max grows by more than 2^kLazyMax
      // (always at the first tile); both threads of a row take the same decision
      float alpha = 1.f;
      bool resc = false;
      if (m_tile > m_ref + kLazyMax) {
        alpha = ex2(m_ref - m_tile);  // 0 at the first tile
        resc = j > 0;
        m_ref = m_tile;
        l *= alpha;
      }
      // P buffer free and O final for tile j-1 (the previous P V has completed)
      if (ok && j > 0) ok = mbar_wait(p_empty, (uint32_t)(j - 1) & 1, s_abort, err, kErrWaitMisc);
      ok = __all_sync(0xffffffffu, ok);
      const bool p_pass = ok && rows_live;  // the P pass releases S itself
      constexpr bool p_tmem = PMODE == 1;
      if (p_pass) {
        tc_fence_after();
        // p = 2^(s*sl2 - m_ref), row sum, f16 P into the A operand (half hsel)
        if (p_tmem) {
          const uint32_t p_addr = tmem + lane_off + 192 + (uint32_t)(hsel * (kBK / 4));
          l += full_tile ? half_row_p_tmem<false, NPOLY>(s_addr, cbase, kvalid, a.sl2, m_ref, p_addr, s_empty)
                         : half_row_p_tmem<true, NPOLY>(s_addr, cbase, kvalid, a.sl2, m_ref, p_addr, s_empty);
        } else {
          uint8_t* prow = sP + hsel * (kBQ * 128) + row * 128;
          l += full_tile ? half_row_p<false, NPOLY>(s_addr, cbase, kvalid, a.sl2, m_ref, prow, row, s_empty)
                         : half_row_p<true, NPOLY>(s_addr, cbase, kvalid, a.sl2, m_ref, prow, row, s_empty);
        }
        // the reference max moved: rescale this thread's 32 columns of the row's running O
        if (__any_sync(0xffffffffu, resc)) {
          uint32_t o[32];
          TMEM_LD32(o_addr, o);
          tc_wait_ld();
          const float f = resc ? alpha : 1.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          TMEM_ST32(o_addr, o);
          tc_wait_st();
        }
      }
      // S read (unless already released by the P pass), P written, O rescaled: hand them to the MMA warp
      tc_wait_st();
      tc_fence_before();
      if (!p_tmem) fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (!p_pass) mbar_arrive(s_empty);
        mbar_arrive(p_full);
      }
    }
    // all P V products complete
    if (ok) ok = mbar_wait(o_done, 0, s_abort, err, kErrWaitMisc);
    ok = __all_sync(0xffffffffu, ok);
    xsum[hsel * kBQ + row] = l;
    named_bar(1, 32 * kSoftmaxWarps);
    const float lt = l + xsum[(hsel ^ 1) * kBQ + row];
    if (ok && rows_live) {
      tc_fence_after();
      uint32_t o[32];
      TMEM_LD32(o_addr, o);
      tc_wait_ld();
      const int qi = qb * kBQ + row;
      if (qi < a.ntok) {
        const long long orow = map_row(a.omap, (long long)w * a.ntok + qi);
        if (orow >= 0) {
          const float inv = 1.0f / lt;
          uint4* op = reinterpret_cast<uint4*>(a.o + orow * a.o_n + h * kD + hsel * (kD / 2));
#pragma unroll
          for (int u = 0; u < 4; ++u)
            op[u] = make_uint4(pack_h2(__uint_as_float(o[8 * u]) * inv, __uint_as_float(o[8 * u + 1]) * inv),
                               pack_h2(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv),
                               pack_h2(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv),
                               pack_h2(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------- two query tiles per CTA (FA kernel)
// One persistent CTA per SM walks work units = (window, head, pair of 128-query tiles), with 96-key
// tiles (576 = 6 x 96 and 5184 = 54 x 96: the ViT windows and the global grid have no ragged tile).
// 10 warps:
//   warp 0     TMA: a unit's Q tiles into one of two Q buffers (the next unit's Q loads while the
//              current one computes), then K_j, V_j (96 rows) through an 8-slot ring, across units.
//   warp 1+t   MMA issue for tile t (t = 0, 1), one thread each, in order: S_t(n) = Q_t K_j^T
//              (128 x 96 x 64) into TMEM region n & 1 of the tile, then O_t += P_t(n - 1) V_{j-1} with P
//              read from the region S_t(n - 1) was written to. The two issuers wait (bounded, suspended)
//              only on their own tile's barriers, so a tile whose softmax lags never holds up the other.
//              Every K / V ring entry and Q buffer is released by both issuers (barrier count 2).
//   warps 4-7  softmax of tile 0, warps 8-11 of tile 1 (warp 3 idle): one query row per thread (TMEM lane), the 96
//              scores of the row in registers; row max, lazy reference max (moved only when the row max
//              grows by more than 2^8, then the sum and the O row are rescaled), p = 2^(s * scale *
//              log2 e - m) written as f16 pairs over the scores it came from (the region's first 48
//              columns), and at the end of the unit O / sum stored through the output row map.
// TMEM (512 columns): tile t region r at 192 t + 96 r, O_t at 384 + 64 t. A region is rewritten by the
// next-but-one S of its tile only after the P V product that read it: the MMAs of the issuing thread
// execute in order, and S_t(n + 2) is issued after P V(n).
// No named barriers: the roles meet only on mbarriers, every wait is bounded, and a timeout unwinds
// every role to the final __syncthreads.
constexpr int kFaWarps = 12;
constexpr int kFaThreads = 32 * kFaWarps;
constexpr int kFaBK = 96;
constexpr int kFaSlots = 8;
constexpr uint32_t kFaKVBytes = kFaBK * kD * 2;  // 12 KB
constexpr uint32_t kFaTmemCols = 512;

// One key tile of one query row (this thread's TMEM lane) in the FA kernel: the row's 96 scores from the TMEM
// region at r_addr, their maximum (three-input max), the lazy reference max, p = 2^(s * sl2 - m_ref) written back
// as f16 pairs over the region's first 48 columns, and the row sum added to l. MASKED: keys at or past kvalid are
// tiling padding (p = 0); full tiles compile without any per-key select. Returns true when the reference max moved
// after the first key tile, i.e. when the row of O must be rescaled by alpha.
template <bool MASKED, int NPOLY>
__device__ __forceinline__ bool fa_row_tile(uint32_t r_addr, int kvalid, float sl2, bool first, float& m_ref,
                                            float& l, float& alpha) {
  uint32_t r[kFaBK];
  TMEM_LD32(r_addr, r);
  TMEM_LD32(r_addr + 32, (r + 32));
  TMEM_LD32(r_addr + 64, (r + 64));
  tc_wait_ld();
  if (MASKED) {
#pragma unroll
    for (int i = 0; i < kFaBK; ++i)
      if (i >= kvalid) r[i] = __float_as_uint(-INFINITY);
  }
  float mx0 = fmax3f(__uint_as_float(r[0]), __uint_as_float(r[1]), __uint_as_float(r[2]));
  float mx1 = fmax3f(__uint_as_float(r[3]), __uint_as_float(r[4]), __uint_as_float(r[5]));
  float mx2 = fmax3f(__uint_as_float(r[6]), __uint_as_float(r[7]), __uint_as_float(r[8]));
  float mx3 = fmax3f(__uint_as_float(r[9]), __uint_as_float(r[10]), __uint_as_float(r[11]));
#pragma unroll
  for (int i = 12; i < kFaBK; i += 8) {
    mx0 = fmax3f(mx0, __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
    mx1 = fmax3f(mx1, __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
    mx2 = fmax3f(mx2, __uint_as_float(r[i + 4]), __uint_as_float(r[i + 5]));
    mx3 = fmax3f(mx3, __uint_as_float(r[i + 6]), __uint_as_float(r[i + 7]));
  }
  const float m_tile = fmax3f(mx0, mx1, fmaxf(mx2, mx3)) * sl2;
  bool resc = false;
  alpha = 1.f;
  if (m_tile > m_ref + kLazyMax) {  // always at the first key tile
    alpha = ex2(m_ref - m_tile);
    resc = !first;
    m_ref = m_tile;
    l *= alpha;
  }
  // the region's previous reader, P V(n - 2), completed before S(n) was written
  const unsigned long long sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(-m_ref, -m_ref);
  unsigned long long acc0 = f2_pack(0.f, 0.f), acc1 = acc0;
#pragma unroll
  for (int c = 0; c < kFaBK / 16; ++c) {  // 16 keys (8 packed columns) per store
    uint32_t pk[8];
#pragma unroll
    for (int u8 = 0; u8 < 2; ++u8) {
      float pv[8];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const int i = 16 * c + 8 * u8 + e;
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), sl2x2, negm2), x0, x1);
        pv[e] = e < NPOLY ? exp2_poly3(x0) : ex2(x0);
        pv[e + 1] = e + 1 < NPOLY ? exp2_poly3(x1) : ex2(x1);
        if (MASKED) {
          pv[e] = i < kvalid ? pv[e] : 0.f;
          pv[e + 1] = i + 1 < kvalid ? pv[e + 1] : 0.f;
        }
      }
      acc0 = f2_add(acc0, f2_add(f2_pack(pv[0], pv[1]), f2_pack(pv[4], pv[5])));
      acc1 = f2_add(acc1, f2_add(f2_pack(pv[2], pv[3]), f2_pack(pv[6], pv[7])));
#pragma unroll
      for (int e = 0; e < 4; ++e) pk[4 * u8 + e] = pack_h2(pv[2 * e], pv[2 * e + 1]);
    }
    TMEM_ST8(r_addr + 8 * c, pk);
  }
  float a0, a1, b0, b1;
  f2_unpack(acc0, a0, a1);
  f2_unpack(acc1, b0, b1);
  l += (a0 + a1) + (b0 + b1);
  return resc;
}

struct FaArgs {
  int heads, ntok, nwin;
  int q_col, k_col, v_col;
  __half* o;
  long long o_n;
  RowMap omap;
  float sl2;
  int n_qp;     // query-tile pairs per (window, head)
  int n_units;  // nwin * heads * n_qp
};

template <int NPOLY>
__global__ void __launch_bounds__(kFaThreads, 1)
    attn_fa_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv, FaArgs a,
                   int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem;                        // [2 buffers][2 tiles] x 16 KB
  uint8_t* sKV = sQ + 4 * kTileBytes;        // kFaSlots x 12 KB (1024-byte multiples)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kFaSlots * kFaKVBytes);
  uint64_t* q_full = bars;                   // [2]
  uint64_t* q_empty = q_full + 2;            // [2]
  uint64_t* kv_full = q_empty + 2;           // [kFaSlots]
  uint64_t* kv_empty = kv_full + kFaSlots;   // [kFaSlots]
  uint64_t* s_full = kv_empty + kFaSlots;    // [2 tiles][2 regions]: one barrier per region, so the two
                                             // S products in flight for a tile never share a phase count
  uint64_t* p_full = s_full + 4;             // [2 tiles]
  uint64_t* pv_done = p_full + 2;            // [2 tiles]
  uint64_t* mma_done = pv_done + 2;          // [2 tiles]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(mma_done + 2);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (a.ntok + kFaBK - 1) / kFaBK;
  const int stride = gridDim.x;
  const int n_it = a.n_units > (int)blockIdx.x ? (a.n_units - 1 - (int)blockIdx.x) / stride + 1 : 0;
  // tile 1 of a unit exists when the unit's second query tile holds a real query
  auto has_tile1 = [&](int it) -> bool {
    const int u = (int)blockIdx.x + it * stride;
    return (2 * (u % a.n_qp) + 1) * kBQ < a.ntok;
  };

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 2);  // released by both issuers
      mbar_init(&s_full[2 * b], 1);
      mbar_init(&s_full[2 * b + 1], 1);
      mbar_init(&p_full[b], 4);
      mbar_init(&pv_done[b], 1);
      mbar_init(&mma_done[b], 1);
    }
    for (int s = 0; s < kFaSlots; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 2);  // released by both issuers
    }
    *s_abort = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tkv);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, kFaTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t armed = 0, armed_phase = 0, q_armed = 0, q_phase = 0;
      long long g = 0;  // ring loads so far
      bool ok = true;
      for (int it = 0; it < n_it && ok; ++it) {
        const int u = (int)blockIdx.x + it * stride;
        const int bh = u / a.n_qp, qp = u - bh * a.n_qp;
        const int w = bh / a.heads, h = bh - w * a.heads;
        const bool two = has_tile1(it);
        const int qb = it & 1;
        if (!mbar_wait(&q_empty[qb], ((uint32_t)(it >> 1) & 1) ^ 1, s_abort, err, kErrWaitEmpty)) { ok = false; break; }
        mbar_arrive_expect_tx(&q_full[qb], (two ? 2 : 1) * kTileBytes);
        tma_load_3d(&tq, &q_full[qb], sQ + (2 * qb) * kTileBytes, a.q_col + h * kD, 2 * qp * kBQ, w);
        if (two) tma_load_3d(&tq, &q_full[qb], sQ + (2 * qb + 1) * kTileBytes, a.q_col + h * kD, (2 * qp + 1) * kBQ, w);
        q_armed |= 1u << qb;
        q_phase = (q_phase & ~(1u << qb)) | ((uint32_t)((it >> 1) & 1) << qb);
        for (int t = 0; t < 2 * nkb; ++t, ++g) {  // K_0, V_0, K_1, V_1, ...
          const int s = (int)(g % kFaSlots);
          const uint32_t use = (uint32_t)(g / kFaSlots);
          if (!mbar_wait(&kv_empty[s], (use & 1) ^ 1, s_abort, err, kErrWaitEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[s], kFaKVBytes);
          const int col = ((t & 1) ? a.v_col : a.k_col) + h * kD;
          tma_load_3d(&tkv, &kv_full[s], sKV + s * kFaKVBytes, col, (t >> 1) * kFaBK, w);
          armed |= 1u << s;
          armed_phase = (armed_phase & ~(1u << s)) | ((use & 1) << s);
        }
      }
      // no copy may still be landing when the CTA exits
      for (int b = 0; b < 2; ++b)
        if (q_armed & (1u << b)) mbar_wait_drain(&q_full[b], (q_phase >> b) & 1u, err);
      for (int s = 0; s < kFaSlots; ++s)
        if (armed & (1u << s)) mbar_wait_drain(&kv_full[s], (armed_phase >> s) & 1u, err);
    }
  } else if (warp == 1 || warp == 2) {
    if (lane == 0) {
      const int t = warp - 1;
      constexpr uint32_t idesc_s = idesc_f16(kBQ, kFaBK, 0);            // Q, K both K-major
      constexpr uint32_t idesc_o = idesc_f16(kBQ, kD, 0) | (1u << 16);  // B (V) MN-major
      const uint32_t q_base = smem_u32(sQ), kv_base = smem_u32(sKV);
      uint32_t ns = 0, npv = 0;
      bool ok = true, issued = false;
      // ring entry of K_j (v = 0) or V_j (v = 1) of unit iteration it
      auto slot = [&](int it, int j, int v, uint32_t* par) -> int {
        const long long g = 2LL * nkb * it + 2 * j + v;
        *par = (uint32_t)(g / kFaSlots) & 1;
        return (int)(g % kFaSlots);
      };
      for (int it = 0; it < n_it && ok; ++it) {
        const int qb = it & 1;
        uint32_t par;
        if (t == 1 && !has_tile1(it)) {
          // no second query tile in this unit: release its Q buffer and ring entries as they fill, so
          // the counts of both issuers stay in step
          if (!mbar_wait(&q_full[qb], (uint32_t)(it >> 1) & 1, s_abort, err, kErrWaitFull)) { ok = false; break; }
          mbar_arrive(&q_empty[qb]);
          for (int e = 0; e < 2 * nkb && ok; ++e) {
            const int sl = slot(it, e >> 1, e & 1, &par);
            if (!mbar_wait(&kv_full[sl], par, s_abort, err, kErrWaitFull)) { ok = false; break; }
            mbar_arrive(&kv_empty[sl]);
          }
          continue;
        }
        if (!mbar_wait(&q_full[qb], (uint32_t)(it >> 1) & 1, s_abort, err, kErrWaitFull)) { ok = false; break; }
        tc_fence_after();
        const uint64_t dq = sdesc_k_sw128(q_base + (uint32_t)((2 * qb + t) * kTileBytes));
        // S(n) = Q K_j^T into region n & 1 (its last reader, P V(n - 2), was issued before by this thread)
        auto issue_s = [&](int j) -> bool {
          uint32_t pk;
          const int sk = slot(it, j, 0, &pk);
          if (!mbar_wait(&kv_full[sk], pk, s_abort, err, kErrWaitFull)) return false;
          tc_fence_after();
          const uint64_t dk = sdesc_k_sw128(kv_base + (uint32_t)(sk * kFaKVBytes));
          const uint32_t sa = tmem + (uint32_t)(192 * t + 96 * (ns & 1));
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            tc_mma_f16(sa, dq + (uint64_t)(kk * 2), dk + (uint64_t)(kk * 2), idesc_s, kk != 0);
          tc_commit(&s_full[2 * t + (ns & 1)]);
          tc_commit(&kv_empty[sk]);
          if (j == nkb - 1) tc_commit(&q_empty[qb]);
          ++ns;
          issued = true;
          return true;
        };
        // O += P(npv) V_j, P read from the region of S(npv)
        auto issue_pv = [&](int j) -> bool {
          uint32_t pv_par;
          const int sv = slot(it, j, 1, &pv_par);
          if (!mbar_wait(&p_full[t], npv & 1, s_abort, err, kErrWaitMisc)) return false;
          if (!mbar_wait(&kv_full[sv], pv_par, s_abort, err, kErrWaitFull)) return false;
          tc_fence_after();
          const uint32_t va = kv_base + (uint32_t)(sv * kFaKVBytes);
          const uint32_t pa = tmem + (uint32_t)(192 * t + 96 * (npv & 1));
          const int nk16 = min(kFaBK / 16, (a.ntok - j * kFaBK + 15) / 16);  // K steps holding a real key
#pragma unroll
          for (int kk = 0; kk < kFaBK / 16; ++kk) {
            if (kk >= nk16) break;
            tc_mma_f16_ts(tmem + 384 + 64 * t, pa + (uint32_t)(kk * 8), sdesc_mn_sw128(va + (uint32_t)(kk * 2048)),
                          idesc_o, (j > 0 || kk != 0) ? 1u : 0u);
          }
          tc_commit(&pv_done[t]);
          tc_commit(&kv_empty[sv]);
          ++npv;
          issued = true;
          return true;
        };
        if (!issue_s(0)) { ok = false; break; }
        for (int j = 0; j < nkb && ok; ++j) {
          if (j + 1 < nkb && !issue_s(j + 1)) { ok = false; break; }
          if (!issue_pv(j)) { ok = false; break; }
        }
      }
      if (issued) {
        tc_commit(&mma_done[t]);
        mbar_wait_drain(&mma_done[t], 0, err);
      }
    }
  } else if (warp >= 4) {
    // softmax: warps 4-7 tile 0, warps 8-11 tile 1; TMEM lanes 32*(warp % 4) .. +31
    const int t = (warp - 4) >> 2;
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t o_addr = tmem + lane_off + 384 + 64 * t;
    uint32_t n = 0;  // S / P count of this tile (its TMEM region is n & 1)
    bool ok = true;
    for (int it = 0; it < n_it && ok; ++it) {
      if (t == 1 && !has_tile1(it)) continue;
      const int u = (int)blockIdx.x + it * stride;
      const int bh = u / a.n_qp, qp = u - bh * a.n_qp;
      const int w = bh / a.heads, h = bh - w * a.heads;
      const int qt = 2 * qp + t;
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < nkb; ++j, ++n) {
        // S(n) of this tile: region n & 1, its barrier's use (n >> 1)
        if (!mbar_wait(&s_full[2 * t + (n & 1)], (n >> 1) & 1, s_abort, err, kErrWaitTmemFull)) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const uint32_t r_addr = tmem + lane_off + (uint32_t)(192 * t + 96 * (n & 1));
        const int kvalid = a.ntok - j * kFaBK;  // keys at or past this count are padding
        float alpha;
        const bool resc = kvalid >= kFaBK ? fa_row_tile<false, NPOLY>(r_addr, kvalid, a.sl2, j == 0, m_ref, l, alpha)
                                          : fa_row_tile<true, NPOLY>(r_addr, kvalid, a.sl2, j == 0, m_ref, l, alpha);
        // O_t current: the previous P V product of this tile has completed (also keeps this thread's walk
        // over the pv_done phases in order)
        if (j > 0 && !mbar_wait(&pv_done[t], (n - 1) & 1, s_abort, err, kErrWaitMisc)) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        // the reference max moved (rare after the first key tile): rescale this row of O_t
        if (__any_sync(0xffffffffu, resc)) {
          uint32_t o[32];
          const float f = resc ? alpha : 1.f;
#pragma unroll
          for (int cc = 0; cc < kD; cc += 32) {
            TMEM_LD32(o_addr + cc, o);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            TMEM_ST32(o_addr + cc, o);
          }
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok) break;
      // the unit's last P V product has completed: O_t / l to the output rows
      if (!mbar_wait(&pv_done[t], (n - 1) & 1, s_abort, err, kErrWaitMisc)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t o[kD];
      TMEM_LD32(o_addr, o);
      TMEM_LD32(o_addr + 32, (o + 32));
      tc_wait_ld();
      const int qi = qt * kBQ + row;
      if (qi < a.ntok) {
        const long long orow = map_row(a.omap, (long long)w * a.ntok + qi);
        if (orow >= 0) {
          const float inv = 1.0f / l;
          uint4* op = reinterpret_cast<uint4*>(a.o + orow * a.o_n + h * kD);
#pragma unroll
          for (int u8 = 0; u8 < 8; ++u8)
            op[u8] = make_uint4(pack_h2(__uint_as_float(o[8 * u8]) * inv, __uint_as_float(o[8 * u8 + 1]) * inv),
                                pack_h2(__uint_as_float(o[8 * u8 + 2]) * inv, __uint_as_float(o[8 * u8 + 3]) * inv),
                                pack_h2(__uint_as_float(o[8 * u8 + 4]) * inv, __uint_as_float(o[8 * u8 + 5]) * inv),
                                pack_h2(__uint_as_float(o[8 * u8 + 6]) * inv, __uint_as_float(o[8 * u8 + 7]) * inv));
        }
      }
      // these TMEM loads completed (wait::ld) before this thread's next p_full arrive, and the next unit's
      // first P V product (accumulate = 0) is issued only after that arrive
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kFaTmemCols);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

void* tensor_map_encoder();  // gemm.cu

// q, k, v of head h of window w: base[w*ntok + n][col + h*64], one row stride for all three.
int attention_tc64(const __half* base, long long ld, int q_col, int k_col, int v_col, int heads, int ntok, int nwin,
                   __half* o, long long o_n, const RowMap& omap, float scale, int exp_poly, int p_mode,
                   int* err, cudaStream_t st) {
  typedef void (*KernelFn)(const CUtensorMap, TcAttnArgs, int*);
  static const KernelFn kernels[2][5] = {
      {attn_tc_kernel<0, 0>, attn_tc_kernel<1, 0>, attn_tc_kernel<2, 0>, attn_tc_kernel<3, 0>, attn_tc_kernel<4, 0>},
      {attn_tc_kernel<0, 1>, attn_tc_kernel<1, 1>, attn_tc_kernel<2, 1>, attn_tc_kernel<3, 1>, attn_tc_kernel<4, 1>}};
  if (exp_poly < 0 || exp_poly > 4 || p_mode < 0 || p_mode > 1) return -2;
  EncodeTiledFn enc = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!enc) return -10;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16 || (q_col % 8) || (k_col % 8) || (v_col % 8) ||
      (o_n % 8) || (reinterpret_cast<uintptr_t>(o) & 15))
    return -2;
  CUtensorMap tm;
  cuuint64_t dims[3] = {(cuuint64_t)ld, (cuuint64_t)ntok, (cuuint64_t)nwin};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(ld * 2 * ntok)};
  cuuint32_t box[3] = {(cuuint32_t)kD, (cuuint32_t)kBK, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return -12;
  TcAttnArgs a;
  a.heads = heads;
  a.ntok = ntok;
  a.nwin = nwin;
  a.q_col = q_col;
  a.k_col = k_col;
  a.v_col = v_col;
  a.o = o;
  a.o_n = o_n;
  a.omap = omap;
  a.sl2 = scale * 1.4426950408889634f;
  const size_t smem = p_mode == 1 ? 1024 + kTileBytes * (1 + 5) + kXchgBytes + 24 * 8 + 16
                                  : 1024 + kTileBytes * (1 + kSlots) + kPBytes + kXchgBytes + 24 * 8 + 16;
  const KernelFn kfn = kernels[p_mode][exp_poly];
  if (kernel_setup(kfn, smem) <= 0) return -13;
  const long long n_cta = (long long)((ntok + kBQ - 1) / kBQ) * nwin * heads;
  if (n_cta > 0x7fffffffLL) return -2;
  kfn<<<(unsigned)n_cta, kThreads, smem, st>>>(tm, a, err);
  return launch_status("attention_tc64");
}

int attention_fa64(const __half* base, long long ld, int q_col, int k_col, int v_col, int heads, int ntok, int nwin,
                   __half* o, long long o_n, const RowMap& omap, float scale, int exp_poly, int* err,
                   cudaStream_t st) {
  typedef void (*KernelFn)(const CUtensorMap, const CUtensorMap, FaArgs, int*);
  static const KernelFn kernels[5] = {attn_fa_kernel<0>, attn_fa_kernel<1>, attn_fa_kernel<2>, attn_fa_kernel<3>,
                                      attn_fa_kernel<4>};
  if (exp_poly < 0 || exp_poly > 4 || ntok <= 0 || nwin <= 0 || heads <= 0) return -2;
  EncodeTiledFn enc = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!enc) return -10;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16 || (q_col % 8) || (k_col % 8) || (v_col % 8) ||
      (o_n % 8) || (reinterpret_cast<uintptr_t>(o) & 15))
    return -2;
  // 3-D maps (channels, token, window) over the fused qkv buffer: 128-row Q boxes, 96-row K / V boxes;
  // rows past the window's last token read zeros
  CUtensorMap tq, tkv;
  cuuint64_t dims[3] = {(cuuint64_t)ld, (cuuint64_t)ntok, (cuuint64_t)nwin};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(ld * 2 * ntok)};
  cuuint32_t box_q[3] = {(cuuint32_t)kD, (cuuint32_t)kBQ, 1};
  cuuint32_t box_kv[3] = {(cuuint32_t)kD, (cuuint32_t)kFaBK, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  if (enc(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box_q, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
      enc(&tkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box_kv, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return -12;
  FaArgs a;
  a.heads = heads;
  a.ntok = ntok;
  a.nwin = nwin;
  a.q_col = q_col;
  a.k_col = k_col;
  a.v_col = v_col;
  a.o = o;
  a.o_n = o_n;
  a.omap = omap;
  a.sl2 = scale * 1.4426950408889634f;
  const int n_qt = (ntok + kBQ - 1) / kBQ;
  a.n_qp = (n_qt + 1) / 2;
  const long long units = (long long)a.n_qp * nwin * heads;
  if (units > 0x7fffffffLL) return -2;
  a.n_units = (int)units;
  constexpr size_t smem = 1024 + 4 * kTileBytes + kFaSlots * kFaKVBytes + (14 + 2 * kFaSlots) * 8 + 16;
  static_assert(smem <= 232448, "shared memory per CTA");
  static_assert(kFaKVBytes % 1024 == 0, "K / V slots keep the 1024-byte alignment of the 128B swizzle");
  const KernelFn kfn = kernels[exp_poly];
  if (kernel_setup(kfn, smem) <= 0) return -13;
  const int grid = (int)std::min<long long>(units, (long long)num_sms());
  kfn<<<grid, kFaThreads, smem, st>>>(tq, tkv, a, err);
  return launch_status("attention_fa64");
}

}  // namespace s3b
