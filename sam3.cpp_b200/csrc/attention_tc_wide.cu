// Tensor-core (tcgen05 / TMEM / TMA) flash attention for head dims 72, 96 and
// 256 with separate q / k / v operands:
//   d = 256  memory attention of the video tracker (sam3_build_mem_attn_graph,
//            ggml_flash_attn_ext at sam3.cpp:9267 and 9312; one head, scale
//            1/16): self-attention over the 64x64 current tokens and
//            cross-attention to the memory bank (7 x 4096 + pointer tokens);
//   d = 96   SAM 2.1 Hiera-T blocks, d = 72 Hiera-L blocks
//            (sam2_hiera_block_forward, ggml_flash_attn_ext at sam3.cpp:4395),
//            windowed and global, heads as column offsets of the fused qkv
//            buffer, windows as the batch.
//
// One CTA = one 128-query tile of one (batch, head) and one range of key tiles
// (64 keys each); 6 warps:
//   warp 0     TMA: the Q tile once, then K_j, V_j through a 3-slot ring, in
//              64-column (128-byte, SW128) boxes; Q, K and V have their own 3-D
//              tensor maps (columns, rows, batch) whose column extent ends at the
//              tensor's last head, so padded boxes read zeros, never a
//              neighbour's or a row's end.
//   warp 1     MMA: S_j = Q K_j^T (M=128, N=64, K = d rounded up to 16) into S
//              buffer j&1; after the softmax wrote P_j: O += P_j V_j (M=128,
//              N = d rounded up to 16, K=64, V as an MN-major operand). S_{j+2}
//              is issued right after P_j V_j, so scores for the next tiles are
//              computed while the softmax threads work on the current one.
//   warps 2-5  softmax, one query row per thread (TMEM lane): row max over the
//              64 keys, p = 2^(s*scale*log2e - m) as f16 into the 128B-swizzled
//              A operand; the reference max m moves only when the row max grows
//              by more than 2^8, and only then are the sum and the row of O in
//              TMEM rescaled. At the end O is divided by the sum and stored, or,
//              when the keys are split over several CTAs, written unnormalised
//              with m and the sum for a combine kernel.
// d = 72: the S product runs K = 80, so the 8 padding columns of the Q tile are
// zeroed in shared memory before the first MMA (the matching K columns then
// contribute nothing). Every wait is bounded; a timeout records an error code
// and the CTA unwinds.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace s3b {
namespace {

constexpr int kBQ = 128;
constexpr int kBK = 64;
constexpr int kSlots = 3;
constexpr uint32_t kPBytes = kBQ * kBK * 2;  // 16 KB: one atom of 128 rows x 128 B
constexpr int kThreads = 192;
constexpr float kLazyMax = 8.0f;
constexpr uint32_t kOCol = 128;              // S buffers at TMEM columns [0,64), [64,128); O from 128

template <int D>
struct WideCfg {
  static constexpr int DK = (D + 15) / 16 * 16;              // K of Q K^T and N of P V
  static constexpr int NA = (DK + 63) / 64;                  // 64-column swizzle atoms loaded per row
  static constexpr uint32_t QBytes = kBQ * NA * 128;         // Q tile: NA atoms of 128 rows x 128 B
  static constexpr uint32_t KVAtom = kBK * 128;              // 8 KB: 64 rows x 128 B
  static constexpr uint32_t KVBytes = NA * KVAtom;
  static constexpr uint32_t TmemCols = kOCol + DK <= 256 ? 256 : 512;
  static constexpr int MinBlocks = TmemCols <= 256 ? 2 : 1;  // CTAs per SM (TMEM, shared memory)
  // P buffers: two for the one-CTA-per-SM d = 256 kernel, so the softmax of key tile j writes P_j while
  // the P V product of tile j - 1 still reads its buffer; one where two CTAs share the SM's shared memory
  static constexpr int NP = MinBlocks == 1 ? 2 : 1;
  static constexpr size_t Smem = 1024 + QBytes + kSlots * KVBytes + NP * kPBytes + 24 * 8 + 16;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

// MN-major SW128 operand (V: rows = keys along K, 64 values of d per 128-byte
// row): SBO = 1024 B between 8-key groups, LBO = 8 KB between 64-wide d atoms.
__device__ __forceinline__ uint64_t sdesc_mn_sw128_v(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((kBK * 128) >> 4) << 16;  // LBO
  d |= (uint64_t)(1024u >> 4) << 32;        // SBO
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
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

#define TMEM_LD16(taddr, R)                                                                                  \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "                                                     \
               "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"                             \
               : "=r"(R[0]), "=r"(R[1]), "=r"(R[2]), "=r"(R[3]), "=r"(R[4]), "=r"(R[5]), "=r"(R[6]),         \
                 "=r"(R[7]), "=r"(R[8]), "=r"(R[9]), "=r"(R[10]), "=r"(R[11]), "=r"(R[12]), "=r"(R[13]),     \
                 "=r"(R[14]), "=r"(R[15])                                                                    \
               : "r"(taddr))

#define TMEM_ST16(taddr, R)                                                                                  \
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "                                               \
               "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),                     \
               "r"(R[0]), "r"(R[1]), "r"(R[2]), "r"(R[3]), "r"(R[4]), "r"(R[5]), "r"(R[6]), "r"(R[7]),       \
               "r"(R[8]), "r"(R[9]), "r"(R[10]), "r"(R[11]), "r"(R[12]), "r"(R[13]), "r"(R[14]), "r"(R[15])  \
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

struct WideArgs {
  int heads, nq, nk;
  int head_rows;      // 1: head h of batch b is row block b*heads + h (layout [B][H][n][d]); 0: columns h*x_h
  int q_h, k_h, v_h;  // column offset (elements) of head h = h * x_h (head_rows == 0)
  __half* o;
  long long o_n;      // output row stride; row = map_row(omap, b*nq + i), head h at column h*d
  RowMap omap;
  float sl2;          // softmax scale * log2(e)
  // key split: CTA `split` of a query tile covers key tiles [split*tiles_per, +tiles_per); with
  // n_split > 1 it writes its unnormalised O, reference max and sum to ws_o / ws_ml for the combine
  int n_split, tiles_per;
  float* ws_o;   // [bh][split][nq][d]
  float* ws_ml;  // [bh][split][nq][2]
};

// Max over the 64 keys of the tile (TMEM columns [0, 64) of this lane's S
// buffer), in log2 units; MASKED: keys at or past kvalid are padding.
template <bool MASKED>
__device__ __forceinline__ float row_max64(uint32_t taddr, int kvalid, float sl2) {
  float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
  for (int c = 0; c < kBK; c += 32) {
    if (MASKED && c >= kvalid) break;
    uint32_t r[32];
    TMEM_LD32(taddr + (uint32_t)c, r);
    tc_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      float v0 = __uint_as_float(r[i]), v1 = __uint_as_float(r[i + 1]);
      float v2 = __uint_as_float(r[i + 2]), v3 = __uint_as_float(r[i + 3]);
      if (MASKED) {
        v0 = c + i < kvalid ? v0 : -INFINITY;
        v1 = c + i + 1 < kvalid ? v1 : -INFINITY;
        v2 = c + i + 2 < kvalid ? v2 : -INFINITY;
        v3 = c + i + 3 < kvalid ? v3 : -INFINITY;
      }
      mx0 = fmaxf(mx0, v0);
      mx1 = fmaxf(mx1, v1);
      mx2 = fmaxf(mx2, v2);
      mx3 = fmaxf(mx3, v3);
    }
  }
  return fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
}

// p = 2^(s*sl2 - m) over the 64 keys into this thread's row of the swizzled P
// atom; returns the row sum. MASKED: padding keys inside the last 32-key chunk
// get p = 0 (the P V product reads to the end of that chunk).
template <bool MASKED>
__device__ __forceinline__ float row_p64(uint32_t taddr, int kvalid, float sl2, float m, uint8_t* prow, int row) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
  for (int c = 0; c < kBK; c += 32) {
    if (MASKED && c >= kvalid) break;
    uint32_t r[32];
    TMEM_LD32(taddr + (uint32_t)c, r);
    tc_wait_ld();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float p[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int i = 8 * u + e;
        p[e] = ex2(fmaf(__uint_as_float(r[i]), sl2, -m));
        if (MASKED) p[e] = c + i < kvalid ? p[e] : 0.f;
      }
      s0 += p[0] + p[4];
      s1 += p[1] + p[5];
      s2 += p[2] + p[6];
      s3 += p[3] + p[7];
      const int unit = (c >> 3) + u;  // 16-byte unit (8 keys) inside the 128-byte row
      *reinterpret_cast<uint4*>(prow + ((unit ^ (row & 7)) << 4)) =
          make_uint4(pack_h2(p[0], p[1]), pack_h2(p[2], p[3]), pack_h2(p[4], p[5]), pack_h2(p[6], p[7]));
    }
  }
  return (s0 + s1) + (s2 + s3);
}

template <int D>
__global__ void __launch_bounds__(kThreads, WideCfg<D>::MinBlocks)
    attn_wide_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, WideArgs a, int* err) {
  using C = WideCfg<D>;
  constexpr int DK = C::DK, NA = C::NA;
  constexpr bool kPadQ = DK > D;  // Q columns [D, DK) must read as zero
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem;                           // NA atoms of 16 KB
  uint8_t* sKV = sQ + C::QBytes;                // kSlots x NA x 8 KB
  constexpr int NP = C::NP;
  uint8_t* sP = sKV + kSlots * C::KVBytes;      // NP x 16 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + NP * kPBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                 // [kSlots]
  uint64_t* kv_empty = kv_full + kSlots;        // [kSlots]
  uint64_t* s_full = kv_empty + kSlots;         // [2]
  uint64_t* s_empty = s_full + 2;               // [2]
  uint64_t* p_full = s_empty + 2;               // [NP]: P_j written (barrier j % NP)
  uint64_t* p_empty = p_full + 2;               // [NP]: the P V product that read buffer j % NP completed
  uint64_t* pv_done = p_empty + 2;              // [2] (NP = 2): P V_j completed (barrier j & 1), O current
  uint64_t* o_done = pv_done + 2;
  uint64_t* mma_done = o_done + 1;
  uint64_t* q_ready = mma_done + 1;             // Q padding zeroed (d = 72)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(q_ready + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid, query tile fastest: the tiles of one (batch, head) run together and share K/V in L2.
  // Blocks take the units from the end, for the same L2 reuse with the GEMMs before and after as in the
  // d = 64 kernel.
  const unsigned unit = gridDim.x - 1 - blockIdx.x;
  const int n_qt = (a.nq + kBQ - 1) / kBQ;
  const int qb = (int)(unit % (unsigned)n_qt);
  const int rest = (int)(unit / (unsigned)n_qt);
  const int split = rest % a.n_split;
  const int bh = rest / a.n_split;
  const int b = bh / a.heads, h = bh - b * a.heads;
  const int rb = a.head_rows ? bh : b;  // row block (batch coordinate of the maps)
  const int hc = a.head_rows ? 0 : h;   // head index used for the column offset
  // this CTA's key tiles: global tiles j0 .. j0 + nkb - 1 (local index j below); never empty
  const int j0 = split * a.tiles_per;
  const int nkb = min((a.nk + kBK - 1) / kBK - j0, a.tiles_per);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&p_full[b], 4);
      mbar_init(&p_empty[b], 1);
      mbar_init(&pv_done[b], 1);
    }
    mbar_init(o_done, 1);
    mbar_init(mma_done, 1);
    mbar_init(q_ready, 4);
    *s_abort = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, C::TmemCols);  // S buffers: [0,64), [64,128); O: [128, 128 + DK)
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, C::QBytes);
#pragma unroll
      for (int at = 0; at < NA; ++at)
        tma_load_3d(&tq, q_full, sQ + at * (kBQ * 128), hc * a.q_h + at * 64, qb * kBQ, rb);
      uint32_t armed = 0, armed_phase = 0;
      bool ok = true;
      for (int t = 0; t < 2 * nkb && ok; ++t) {  // K_0, V_0, K_1, V_1, ...
        const int s = t % kSlots;
        const uint32_t use = (uint32_t)(t / kSlots);
        if (!mbar_wait(&kv_empty[s], (use & 1) ^ 1, s_abort, err, kErrWaitEmpty)) { ok = false; break; }
        mbar_arrive_expect_tx(&kv_full[s], C::KVBytes);
        const int j = t >> 1;
        const CUtensorMap* map = (t & 1) ? &tv : &tk;
        const int col0 = hc * ((t & 1) ? a.v_h : a.k_h);
#pragma unroll
        for (int at = 0; at < NA; ++at)
          tma_load_3d(map, &kv_full[s], sKV + s * C::KVBytes + at * C::KVAtom, col0 + at * 64, (j0 + j) * kBK, rb);
        armed |= 1u << s;
        armed_phase = (armed_phase & ~(1u << s)) | ((use & 1) << s);
      }
      mbar_wait_drain(q_full, 0, err);
      for (int s = 0; s < kSlots; ++s)
        if (armed & (1u << s)) mbar_wait_drain(&kv_full[s], (armed_phase >> s) & 1u, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(kBQ, kBK, 0);                 // Q, K both K-major
      constexpr uint32_t idesc_o = idesc_f16(kBQ, DK, 0) | (1u << 16);     // B (V) MN-major
      bool ok = mbar_wait(kPadQ ? q_ready : q_full, 0, s_abort, err, kErrWaitFull);
      tc_fence_after();
      const uint32_t qa = smem_u32(sQ);
      bool issued = false;
      // S_j = Q K_j^T into S buffer j & 1 (free once the softmax released S_{j-2})
      auto issue_s = [&](int j) -> bool {
        const int t = 2 * j, s = t % kSlots, sb = j & 1;
        if (!mbar_wait(&kv_full[s], (uint32_t)(t / kSlots) & 1, s_abort, err, kErrWaitFull)) return false;
        if (j >= 2 && !mbar_wait(&s_empty[sb], (uint32_t)((j - 2) >> 1) & 1, s_abort, err, kErrWaitMisc))
          return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(sKV + s * C::KVBytes);
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk & 3) * 32);
          const uint64_t dq = sdesc_k_sw128(qa + (uint32_t)((kk >> 2) * (kBQ * 128)) + off);
          const uint64_t dk = sdesc_k_sw128(ka + (uint32_t)((kk >> 2) * C::KVAtom) + off);
          tc_mma_f16(tmem + (uint32_t)(sb * kBK), dq, dk, idesc_s, kk != 0);
        }
        tc_commit(&s_full[sb]);
        tc_commit(&kv_empty[s]);
        issued = true;
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nkb > 1) ok = issue_s(1);
      for (int j = 0; j < nkb && ok; ++j) {
        // O += P_j V_j (after the softmax wrote P_j and, where needed, rescaled O)
        const int t = 2 * j + 1, s = t % kSlots, pb = j % NP;
        if (!mbar_wait(&p_full[pb], (uint32_t)(j / NP) & 1, s_abort, err, kErrWaitMisc)) { ok = false; break; }
        if (!mbar_wait(&kv_full[s], (uint32_t)(t / kSlots) & 1, s_abort, err, kErrWaitFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t pa = smem_u32(sP + pb * kPBytes), va = smem_u32(sKV + s * C::KVBytes);
        const int nk16 = min(kBK / 16, (a.nk - (j0 + j) * kBK + 15) / 16);  // K steps holding a real key
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          if (kk >= nk16) break;
          const uint64_t dp = sdesc_k_sw128(pa + (uint32_t)(kk * 32));
          const uint64_t dv = sdesc_mn_sw128_v(va + (uint32_t)(kk * 2048));  // 16 key rows per K step
          tc_mma_f16(tmem + kOCol, dp, dv, idesc_o, (j > 0 || kk != 0) ? 1u : 0u);
        }
        tc_commit(&kv_empty[s]);
        tc_commit(&p_empty[pb]);
        if (NP == 2) tc_commit(&pv_done[j & 1]);
        if (j + 2 < nkb && !issue_s(j + 2)) { ok = false; break; }
      }
      if (ok) tc_commit(o_done);
      if (issued) {
        tc_commit(mma_done);
        mbar_wait_drain(mma_done, 0, err);
      }
    }
  } else {
    // softmax: warp w owns TMEM lanes 32*(w%4) .. +31 (query rows)
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const bool rows_live = qb * kBQ + q4 * 32 < a.nq;  // else only the barrier protocol
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    if constexpr (kPadQ) {
      // zero this row's Q columns [D, DK) (one 16-byte unit of the last atom)
      ok = mbar_wait(q_full, 0, s_abort, err, kErrWaitFull);
      if (ok) {
        constexpr int col = D % 64;  // first padding column inside its atom
        static_assert(DK - D == 8 && col % 8 == 0, "d = 72-like padding: one 16-byte unit");
        uint8_t* qrow = sQ + (D / 64) * (kBQ * 128) + row * 128;
        *reinterpret_cast<uint4*>(qrow + (((col >> 3) ^ (row & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
      ok = __all_sync(0xffffffffu, ok);
    }
    for (int j = 0; j < nkb && ok; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&s_full[sb], (uint32_t)(j >> 1) & 1, s_abort, err, kErrWaitTmemFull)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int kvalid = a.nk - (j0 + j) * kBK;
      const bool full_tile = kvalid >= kBK;
      const uint32_t s_addr = tmem + lane_off + (uint32_t)(sb * kBK);
      float alpha = 1.f;
      bool resc = false;
      if (rows_live) {
        const float m_tile = full_tile ? row_max64<false>(s_addr, kvalid, a.sl2) : row_max64<true>(s_addr, kvalid, a.sl2);
        if (m_tile > m_ref + kLazyMax) {  // always at the first tile
          alpha = ex2(m_ref - m_tile);
          resc = j > 0;
          m_ref = m_tile;
          l *= alpha;
        }
      }
      // P buffer j % NP free (its last reader, P V_{j-NP}, completed; with one buffer that also makes O
      // final for tile j - 1)
      const int pb = j % NP;
      if (j >= NP && !mbar_wait(&p_empty[pb], (uint32_t)(j / NP - 1) & 1, s_abort, err, kErrWaitMisc)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (rows_live) {
        tc_fence_after();
        uint8_t* prow = sP + pb * kPBytes + row * 128;
        l += full_tile ? row_p64<false>(s_addr, kvalid, a.sl2, m_ref, prow, row)
                       : row_p64<true>(s_addr, kvalid, a.sl2, m_ref, prow, row);
      }
      // with two P buffers, O is current only once P V_{j-1} completed: waited for only when a row of
      // this warp rescales (its barrier cannot run two phases ahead: P V_{j+1} needs this tile's P_{j+1})
      if (NP == 2 && __any_sync(0xffffffffu, resc) &&
          !mbar_wait(&pv_done[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1, s_abort, err, kErrWaitMisc))
        ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (rows_live) {
        tc_fence_after();
        if (__any_sync(0xffffffffu, resc)) {
          const float f = resc ? alpha : 1.f;
#pragma unroll 1
          for (int c = 0; c < DK; c += 16) {
            uint32_t o[16];
            TMEM_LD16(tmem + lane_off + kOCol + (uint32_t)c, o);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            TMEM_ST16(tmem + lane_off + kOCol + (uint32_t)c, o);
          }
          tc_wait_st();
        }
      }
      // S_j read, P_j written, O rescaled: hand them to the MMA warp
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_empty[sb]);
        mbar_arrive(&p_full[pb]);
      }
    }
    if (ok) ok = mbar_wait(o_done, 0, s_abort, err, kErrWaitMisc);
    ok = __all_sync(0xffffffffu, ok);
    if (ok && rows_live) {
      tc_fence_after();
      const int qi = qb * kBQ + row;
      if (a.n_split > 1) {
        // partial result of this key split: O relative to 2^m_ref, the reference max and the sum
        const size_t pidx = ((size_t)bh * a.n_split + split) * a.nq + qi;
#pragma unroll 1
        for (int c = 0; c < DK; c += 16) {
          uint32_t o[16];
          TMEM_LD16(tmem + lane_off + kOCol + (uint32_t)c, o);
          tc_wait_ld();
          if (qi < a.nq) {
            float4* op = reinterpret_cast<float4*>(a.ws_o + pidx * D + c);
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (c + 4 * u < D)
                op[u] = make_float4(__uint_as_float(o[4 * u]), __uint_as_float(o[4 * u + 1]),
                                    __uint_as_float(o[4 * u + 2]), __uint_as_float(o[4 * u + 3]));
          }
        }
        if (qi < a.nq) *reinterpret_cast<float2*>(a.ws_ml + pidx * 2) = make_float2(m_ref, l);
      } else {
        const long long orow = qi < a.nq ? map_row(a.omap, (long long)b * a.nq + qi) : -1;
        const float inv = 1.0f / l;
#pragma unroll 1
        for (int c = 0; c < DK; c += 16) {
          uint32_t o[16];
          TMEM_LD16(tmem + lane_off + kOCol + (uint32_t)c, o);
          tc_wait_ld();
          if (orow >= 0) {
            uint4* op = reinterpret_cast<uint4*>(a.o + orow * a.o_n + h * D + c);
#pragma unroll
            for (int u = 0; u < 2; ++u)
              if (c + 8 * u < D)
                op[u] = make_uint4(pack_h2(__uint_as_float(o[8 * u]) * inv, __uint_as_float(o[8 * u + 1]) * inv),
                                   pack_h2(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv),
                                   pack_h2(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv),
                                   pack_h2(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TmemCols);
  }
}

// ---------------------------------------------------------------- 128-key tiles (d = 256; d = 72 / 96 as an option)
// The d = 256 products on the kernel above issue 20 MMAs per 64 keys, 16 of them N = 64 (S = Q K^T over
// d = 256 in K = 16 steps); this kernel takes 128-key tiles, so S runs N = 128 and each 128 keys cost 24
// MMAs (16 for S, 8 for P V with N = 256) instead of 40. P goes back to TMEM over the scores it came from
// (the A operand of P V), which frees the shared memory for 128-key K and V tiles beside the Q tile: one
// slot each at d = 256 (64 KB tiles), two at d <= 128 (32 KB tiles), K_j / V_j in slot j % slots. TMEM (512
// columns): S / P regions r = 0, 1 at 128 r (S_j in region j & 1), O at 256. 7 warps:
//   warp 0     TMA: the Q tile, then K_j (64-column boxes of 128 rows) once S_{j-slots} has read its slot
//   warp 6     TMA: V_j once P V_{j-slots} has read its slot
//   warp 1     MMA: S_0, S_1, then per key tile j: O += P_j V_j (A = P_j from TMEM), S_{j+2}. S_{j+2}
//              rewrites the region P_j was read from; the MMAs of one thread execute in order.
//   warps 2-5  softmax, one query row per thread (TMEM lane): the row's 128 scores in registers, row max,
//              lazy reference max (moved only when the row max grows by more than 2^8, then the sum and
//              the O row are rescaled once P V_{j-1} has completed), p = 2^(s * scale * log2 e - m) as f16
//              pairs over the region's first 64 columns; at the end O / sum, or with key splits the
//              unnormalised O, m and sum for the combine kernel.
constexpr int kB2 = 128;                    // keys per tile
constexpr uint32_t kAtom2 = 128 * 128;      // 16 KB: 128 rows x 128 B
constexpr int kThreads2 = 224;
template <int D>
struct Cfg2 {
  static constexpr int DK = WideCfg<D>::DK;         // K of Q K^T and N of P V (d rounded up to 16)
  static constexpr int NA = WideCfg<D>::NA;         // 64-column atoms per row
  static constexpr uint32_t Tile = NA * kAtom2;     // Q, K or V tile of 128 rows
  // K / V slots each: two where they fit beside Q (d <= 128), so the copy of a key tile starts one MMA round
  // earlier; one for d = 256
  static constexpr int KVB = NA <= 2 ? 2 : 1;
  static constexpr size_t Smem = 1024 + (1 + 2 * KVB) * (size_t)Tile + 16 * 8 + 16;
};

__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// MN-major SW128 V operand of 128 key rows: SBO = 1024 B between 8-key groups, LBO = 16 KB between the
// 64-wide d atoms.
__device__ __forceinline__ uint64_t sdesc_mn_v128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(kAtom2 >> 4) << 16;  // LBO
  d |= (uint64_t)(1024u >> 4) << 32;   // SBO
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

#define TMEM_ST32W(taddr, R)                                                                                 \
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "                                               \
               "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"                                    \
               "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),             \
               "r"(R[0]), "r"(R[1]), "r"(R[2]), "r"(R[3]), "r"(R[4]), "r"(R[5]), "r"(R[6]), "r"(R[7]),       \
               "r"(R[8]), "r"(R[9]), "r"(R[10]), "r"(R[11]), "r"(R[12]), "r"(R[13]), "r"(R[14]), "r"(R[15]), \
               "r"(R[16]), "r"(R[17]), "r"(R[18]), "r"(R[19]), "r"(R[20]), "r"(R[21]), "r"(R[22]),           \
               "r"(R[23]), "r"(R[24]), "r"(R[25]), "r"(R[26]), "r"(R[27]), "r"(R[28]), "r"(R[29]),           \
               "r"(R[30]), "r"(R[31])                                                                        \
               : "memory")

// One 128-key tile of one query row: scores from the region at r_addr, row max, lazy reference max,
// P as f16 pairs over the region's first 64 columns, row sum added to l. MASKED: keys at or past kvalid
// are padding (p = 0). Returns true when the reference max moved after the first tile.
template <bool MASKED>
__device__ __forceinline__ bool row_tile128(uint32_t r_addr, int kvalid, float sl2, bool first, float& m_ref,
                                            float& l, float& alpha) {
  uint32_t r[kB2];
  TMEM_LD32(r_addr, r);
  TMEM_LD32(r_addr + 32, (r + 32));
  TMEM_LD32(r_addr + 64, (r + 64));
  TMEM_LD32(r_addr + 96, (r + 96));
  tc_wait_ld();
  if (MASKED) {
#pragma unroll
    for (int i = 0; i < kB2; ++i)
      if (i >= kvalid) r[i] = __float_as_uint(-INFINITY);
  }
  float mx0 = __uint_as_float(r[0]), mx1 = __uint_as_float(r[1]), mx2 = __uint_as_float(r[2]),
        mx3 = __uint_as_float(r[3]);
#pragma unroll
  for (int i = 4; i < kB2 - 4; i += 8) {
    mx0 = fmax3f(mx0, __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
    mx1 = fmax3f(mx1, __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
    mx2 = fmax3f(mx2, __uint_as_float(r[i + 4]), __uint_as_float(r[i + 5]));
    mx3 = fmax3f(mx3, __uint_as_float(r[i + 6]), __uint_as_float(r[i + 7]));
  }
  mx0 = fmax3f(mx0, __uint_as_float(r[kB2 - 4]), __uint_as_float(r[kB2 - 3]));
  mx1 = fmax3f(mx1, __uint_as_float(r[kB2 - 2]), __uint_as_float(r[kB2 - 1]));
  const float m_tile = fmax3f(mx0, mx1, fmaxf(mx2, mx3)) * sl2;
  bool resc = false;
  alpha = 1.f;
  if (m_tile > m_ref + kLazyMax) {  // always at the first key tile
    alpha = ex2(m_ref - m_tile);
    resc = !first;
    m_ref = m_tile;
    l *= alpha;
  }
  const unsigned long long sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(-m_ref, -m_ref);
  unsigned long long acc0 = f2_pack(0.f, 0.f), acc1 = acc0;
#pragma unroll
  for (int c = 0; c < kB2 / 64; ++c) {  // 64 keys (32 packed columns) per store
    uint32_t pk[32];
#pragma unroll
    for (int u8 = 0; u8 < 8; ++u8) {
      float pv[8];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const int i = 64 * c + 8 * u8 + e;
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), sl2x2, negm2), x0, x1);
        pv[e] = ex2(x0);
        pv[e + 1] = ex2(x1);
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
    TMEM_ST32W(r_addr + 32 * c, pk);
  }
  float a0, a1, b0, b1;
  f2_unpack(acc0, a0, a1);
  f2_unpack(acc1, b0, b1);
  l += (a0 + a1) + (b0 + b1);
  return resc;
}

template <int D>
__global__ void __launch_bounds__(kThreads2, 1)
    attn128k_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, WideArgs a, int* err) {
  using C = Cfg2<D>;
  constexpr int DK = C::DK, NA = C::NA, KVB = C::KVB;
  constexpr uint32_t kTile2 = C::Tile;
  constexpr bool kPadQ = DK > D;  // Q columns [D, DK) must read as zero (d = 72)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTile2;        // [KVB] slots: K_j in slot j % KVB
  uint8_t* sV = sK + KVB * kTile2;  // [KVB] slots: V_j in slot j % KVB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + KVB * kTile2);
  uint64_t* q_full = bars;
  uint64_t* s_full = bars + 1;    // [2]: S_j in region j & 1
  uint64_t* p_full = bars + 3;    // P_j written (4 softmax warps)
  uint64_t* pv_done = bars + 4;   // P V_j completed
  uint64_t* o_done = bars + 5;
  uint64_t* mma_done = bars + 6;
  uint64_t* q_ready = bars + 7;   // Q padding columns zeroed (d = 72)
  uint64_t* k_full = bars + 8;    // [KVB]
  uint64_t* k_empty = k_full + KVB;
  uint64_t* v_full = k_empty + KVB;
  uint64_t* v_empty = v_full + KVB;
  static_assert(8 + 4 * KVB <= 16, "barrier area");
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned unit = gridDim.x - 1 - blockIdx.x;
  const int n_qt = (a.nq + kBQ - 1) / kBQ;
  const int qb = (int)(unit % (unsigned)n_qt);
  const int rest = (int)(unit / (unsigned)n_qt);
  const int split = rest % a.n_split;
  const int bh = rest / a.n_split;
  const int b = bh / a.heads, h = bh - b * a.heads;
  const int rb = a.head_rows ? bh : b;
  const int hc = a.head_rows ? 0 : h;
  const int j0 = split * a.tiles_per;
  const int nkb = min((a.nk + kB2 - 1) / kB2 - j0, a.tiles_per);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KVB; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(o_done, 1);
    mbar_init(mma_done, 1);
    mbar_init(q_ready, 4);
    *s_abort = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0 || warp == 6) {
    if (lane == 0) {
      // warp 0: Q, then K_j; warp 6: V_j. A slot is refilled once the product that read it completed.
      const bool is_k = warp == 0;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      uint8_t* dst = is_k ? sK : sV;
      const CUtensorMap* map = is_k ? &tk : &tv;
      const int col0 = hc * (is_k ? a.k_h : a.v_h);
      if (is_k) {
        mbar_arrive_expect_tx(q_full, kTile2);
#pragma unroll
        for (int at = 0; at < NA; ++at) tma_load_3d(&tq, q_full, sQ + at * kAtom2, hc * a.q_h + at * 64, qb * kBQ, rb);
      }
      int armed = -1;
      for (int j = 0; j < nkb; ++j) {
        const int sl = j % KVB;
        const uint32_t use = (uint32_t)(j / KVB);
        if (!mbar_wait(&empty[sl], (use & 1) ^ 1, s_abort, err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&full[sl], kTile2);
#pragma unroll
        for (int at = 0; at < NA; ++at)
          tma_load_3d(map, &full[sl], dst + sl * kTile2 + at * kAtom2, col0 + at * 64, (j0 + j) * kB2, rb);
        armed = j;
      }
      // no copy may still be landing when the CTA exits: the last arming of each slot
      if (is_k) mbar_wait_drain(q_full, 0, err);
      for (int j = armed; j >= 0 && j > armed - KVB; --j)
        mbar_wait_drain(&full[j % KVB], (uint32_t)(j / KVB) & 1, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(kBQ, kB2, 0);              // Q, K both K-major
      constexpr uint32_t idesc_o = idesc_f16(kBQ, DK, 0) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(kPadQ ? q_ready : q_full, 0, s_abort, err, kErrWaitFull);
      tc_fence_after();
      const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK), va = smem_u32(sV);
      bool issued = false;
      auto issue_s = [&](int j) -> bool {
        const int sl = j % KVB;
        if (!mbar_wait(&k_full[sl], (uint32_t)(j / KVB) & 1, s_abort, err, kErrWaitFull)) return false;
        tc_fence_after();
        const uint32_t sa = tmem + (uint32_t)((j & 1) * kB2);
        const uint32_t kb = ka + (uint32_t)(sl * kTile2);
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * kAtom2 + (kk & 3) * 32);
          tc_mma_f16(sa, sdesc_k_sw128(qa + off), sdesc_k_sw128(kb + off), idesc_s, kk != 0);
        }
        tc_commit(&s_full[j & 1]);
        tc_commit(&k_empty[sl]);
        issued = true;
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nkb > 1) ok = issue_s(1);
      for (int j = 0; j < nkb && ok; ++j) {
        if (!mbar_wait(p_full, (uint32_t)j & 1, s_abort, err, kErrWaitMisc)) { ok = false; break; }
        const int vsl = j % KVB;
        if (!mbar_wait(&v_full[vsl], (uint32_t)(j / KVB) & 1, s_abort, err, kErrWaitFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t pa = tmem + (uint32_t)((j & 1) * kB2);
        const uint32_t vb = va + (uint32_t)(vsl * kTile2);
        const int nk16 = min(kB2 / 16, (a.nk - (j0 + j) * kB2 + 15) / 16);  // K steps holding a real key
#pragma unroll
        for (int kk = 0; kk < kB2 / 16; ++kk) {
          if (kk >= nk16) break;
          tc_mma_f16_ts(tmem + 256, pa + (uint32_t)(kk * 8), sdesc_mn_v128(vb + (uint32_t)(kk * 2048)), idesc_o,
                        (j > 0 || kk != 0) ? 1u : 0u);
        }
        tc_commit(pv_done);
        tc_commit(&v_empty[vsl]);
        if (j + 2 < nkb && !issue_s(j + 2)) { ok = false; break; }
      }
      if (ok) tc_commit(o_done);
      if (issued) {
        tc_commit(mma_done);
        mbar_wait_drain(mma_done, 0, err);
      }
    }
  } else {
    // softmax: warp w owns TMEM lanes 32*(w%4) .. +31 (query rows)
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const bool rows_live = qb * kBQ + q4 * 32 < a.nq;  // else only the barrier protocol
    const uint32_t o_addr = tmem + lane_off + 256;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    if constexpr (kPadQ) {
      // zero this row's Q columns [D, DK) (one 16-byte unit of the last atom)
      ok = mbar_wait(q_full, 0, s_abort, err, kErrWaitFull);
      if (ok) {
        constexpr int col = D % 64;  // first padding column inside its atom
        static_assert(DK - D == 8 && col % 8 == 0, "d = 72-like padding: one 16-byte unit");
        uint8_t* qrow = sQ + (D / 64) * kAtom2 + row * 128;
        *reinterpret_cast<uint4*>(qrow + (((col >> 3) ^ (row & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
      ok = __all_sync(0xffffffffu, ok);
    }
    for (int j = 0; j < nkb && ok; ++j) {
      if (!mbar_wait(&s_full[j & 1], (uint32_t)(j >> 1) & 1, s_abort, err, kErrWaitTmemFull)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int kvalid = a.nk - (j0 + j) * kB2;
      const uint32_t r_addr = tmem + lane_off + (uint32_t)((j & 1) * kB2);
      float alpha = 1.f;
      bool resc = false;
      if (rows_live)
        resc = kvalid >= kB2 ? row_tile128<false>(r_addr, kvalid, a.sl2, j == 0, m_ref, l, alpha)
                             : row_tile128<true>(r_addr, kvalid, a.sl2, j == 0, m_ref, l, alpha);
      // O current: P V_{j-1} has completed (also keeps this thread's walk over the pv_done phases in order;
      // P V_j needs this tile's P_j, so the barrier is never two phases ahead)
      if (j > 0 && !mbar_wait(pv_done, (uint32_t)(j - 1) & 1, s_abort, err, kErrWaitMisc)) ok = false;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      if (rows_live && __any_sync(0xffffffffu, resc)) {
        const float f = resc ? alpha : 1.f;
#pragma unroll 1
        for (int c = 0; c < DK; c += 16) {
          uint32_t o[16];
          TMEM_LD16(o_addr + (uint32_t)c, o);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          TMEM_ST16(o_addr + (uint32_t)c, o);
        }
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok) ok = mbar_wait(o_done, 0, s_abort, err, kErrWaitMisc);
    ok = __all_sync(0xffffffffu, ok);
    if (ok && rows_live) {
      tc_fence_after();
      const int qi = qb * kBQ + row;
      if (a.n_split > 1) {
        const size_t pidx = ((size_t)bh * a.n_split + split) * a.nq + qi;
#pragma unroll 1
        for (int c = 0; c < DK; c += 16) {
          uint32_t o[16];
          TMEM_LD16(o_addr + (uint32_t)c, o);
          tc_wait_ld();
          if (qi < a.nq) {
            float4* op = reinterpret_cast<float4*>(a.ws_o + pidx * D + c);
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (c + 4 * u < D)
                op[u] = make_float4(__uint_as_float(o[4 * u]), __uint_as_float(o[4 * u + 1]),
                                    __uint_as_float(o[4 * u + 2]), __uint_as_float(o[4 * u + 3]));
          }
        }
        if (qi < a.nq) *reinterpret_cast<float2*>(a.ws_ml + pidx * 2) = make_float2(m_ref, l);
      } else {
        const long long orow = qi < a.nq ? map_row(a.omap, (long long)b * a.nq + qi) : -1;
        const float inv = 1.0f / l;
#pragma unroll 1
        for (int c = 0; c < DK; c += 16) {
          uint32_t o[16];
          TMEM_LD16(o_addr + (uint32_t)c, o);
          tc_wait_ld();
          if (orow >= 0) {
            uint4* op = reinterpret_cast<uint4*>(a.o + orow * a.o_n + h * D + c);
#pragma unroll
            for (int u = 0; u < 2; ++u)
              if (c + 8 * u < D)
              op[u] = make_uint4(pack_h2(__uint_as_float(o[8 * u]) * inv, __uint_as_float(o[8 * u + 1]) * inv),
                                 pack_h2(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv),
                                 pack_h2(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv),
                                 pack_h2(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Merges the key splits of each query row: M = max of the splits' reference
// maxima, O = sum_s 2^(m_s - M) O_s, l = sum_s 2^(m_s - M) l_s, out = O / l
// (f16). One warp per row.
template <int D>
__global__ void __launch_bounds__(256) attn_wide_combine_kernel(WideArgs a, long long rows) {
  const long long r = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int bh = (int)(r / a.nq), qi = (int)(r - (long long)bh * a.nq);
  const int b = bh / a.heads, h = bh - b * a.heads;
  float mmax = -INFINITY;
  for (int s = 0; s < a.n_split; ++s)
    mmax = fmaxf(mmax, a.ws_ml[(((size_t)bh * a.n_split + s) * a.nq + qi) * 2]);
  constexpr int PER = (D + 31) / 32;  // columns lane + 32*i
  float acc[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) acc[i] = 0.f;
  float lsum = 0.f;
  for (int s = 0; s < a.n_split; ++s) {
    const size_t pr = ((size_t)bh * a.n_split + s) * a.nq + qi;
    const float2 ml = *reinterpret_cast<const float2*>(a.ws_ml + pr * 2);
    const float w = ml.x == -INFINITY ? 0.f : ex2(ml.x - mmax);
    lsum += w * ml.y;
    const float* op = a.ws_o + pr * D;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i < D) acc[i] += w * op[lane + 32 * i];
  }
  const long long orow = map_row(a.omap, (long long)b * a.nq + qi);
  if (orow < 0) return;
  const float inv = 1.0f / lsum;
  __half* o = a.o + orow * a.o_n + h * D;
#pragma unroll
  for (int i = 0; i < PER; ++i)
    if (lane + 32 * i < D) o[lane + 32 * i] = __float2half_rn(acc[i] * inv);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 3-D map (columns, rows, batch) over x[b*xb + n*xn + col] with `cols` columns
// (the tensor's own extent: reads past it return zeros), box = 64 columns x
// box_rows x 1, SW128.
int map3(EncodeTiledFn enc, CUtensorMap* m, const __half* x, long long cols, long long xn, long long xb, int rows,
         int batch, int box_rows) {
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (xn % 8) || (xb % 8) || cols <= 0 || cols > xn) return -2;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(xn * 2), (cuuint64_t)(xb * 2)};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(x), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? 0
             : -12;
}

template <int D>
int launch_wide(const AttnParams& p, int batch_heads, float* ws, size_t ws_bytes, int bk128, int* err,
                cudaStream_t st) {
  using C = WideCfg<D>;
  EncodeTiledFn enc = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!enc) return -10;
  if (p.heads <= 0 || batch_heads % p.heads || p.nq <= 0 || p.nk <= 0) return -2;
  if ((p.o_n % 8) || (reinterpret_cast<uintptr_t>(p.o) & 15) || ((long long)p.heads * D > p.o_n)) return -2;
  // heads either as column offsets inside a row (fused projections) or as
  // consecutive row blocks ([B][H][n][d]); anything else is not supported here
  const bool head_rows = p.heads > 1 && p.q_h >= (long long)p.nq * p.q_n;
  int blocks;
  long long qb, kb, vb, qc, kc, vc;  // batch strides and column extents
  if (head_rows) {
    if (p.k_h < (long long)p.nk * p.k_n || p.v_h < (long long)p.nk * p.v_n) return -2;
    if (batch_heads > p.heads &&
        (p.q_b != p.heads * p.q_h || p.k_b != p.heads * p.k_h || p.v_b != p.heads * p.v_h))
      return -2;
    blocks = batch_heads;
    qb = p.q_h;
    kb = p.k_h;
    vb = p.v_h;
    qc = kc = vc = D;
  } else {
    if ((p.q_h % 8) || (p.k_h % 8) || (p.v_h % 8)) return -2;
    blocks = batch_heads / p.heads;
    // a single batch may carry any batch stride; use one that satisfies the map's rules
    qb = blocks > 1 ? p.q_b : (long long)p.nq * p.q_n;
    kb = blocks > 1 ? p.k_b : (long long)p.nk * p.k_n;
    vb = blocks > 1 ? p.v_b : (long long)p.nk * p.v_n;
    qc = (long long)(p.heads - 1) * p.q_h + D;
    kc = (long long)(p.heads - 1) * p.k_h + D;
    vc = (long long)(p.heads - 1) * p.v_h + D;
  }
  // d = 256 runs the 128-key-tile kernel, d = 72 / 96 when `bk128` is set
  const bool k128 = D == 256 || (bk128 && (D == 72 || D == 96));
  const int BK = k128 ? kB2 : kBK;
  CUtensorMap tq, tk, tv;
  int rc = map3(enc, &tq, p.q, qc, p.q_n, qb, p.nq, blocks, kBQ);
  if (!rc) rc = map3(enc, &tk, p.k, kc, p.k_n, kb, p.nk, blocks, BK);
  if (!rc) rc = map3(enc, &tv, p.v, vc, p.v_n, vb, p.nk, blocks, BK);
  if (rc) return rc;
  WideArgs a;
  a.heads = p.heads;
  a.head_rows = head_rows ? 1 : 0;
  a.nq = p.nq;
  a.nk = p.nk;
  a.q_h = (int)p.q_h;
  a.k_h = (int)p.k_h;
  a.v_h = (int)p.v_h;
  a.o = p.o;
  a.o_n = p.o_n;
  a.omap = p.omap;
  a.sl2 = p.scale * 1.4426950408889634f;
  // split the keys over CTAs when the query tiles alone leave SMs idle (e.g. one head of 4096 queries:
  // 32 tiles on 148 SMs), keeping at least 4 key tiles per split and no split empty
  const int n_qt = (p.nq + kBQ - 1) / kBQ;
  const long long units = (long long)n_qt * batch_heads;
  const long long slots = (long long)num_sms() * (k128 ? 1 : C::MinBlocks);
  const int nkb = (p.nk + BK - 1) / BK;
  int n_split = 1;
  if (ws && units < slots) n_split = (int)std::max(1LL, std::min(slots / units, (long long)nkb / 4));
  int tiles_per = (nkb + n_split - 1) / n_split;
  n_split = (nkb + tiles_per - 1) / tiles_per;
  if (n_split > 1 && ws_bytes < attention_wide_ws_bytes(D, n_split, batch_heads, p.nq)) {
    n_split = 1;
    tiles_per = nkb;
  }
  a.n_split = n_split;
  a.tiles_per = tiles_per;
  a.ws_o = ws;
  a.ws_ml = ws ? ws + (size_t)n_split * batch_heads * p.nq * D : nullptr;
  static_assert(C::Smem <= 232448 && Cfg2<D>::Smem <= 232448, "shared memory per CTA");
  const long long n_cta = units * n_split;
  if (n_cta > 0x7fffffffLL) return -2;
  if (k128) {
    if (kernel_setup(attn128k_kernel<D>, Cfg2<D>::Smem) <= 0) return -13;
    attn128k_kernel<D><<<(unsigned)n_cta, kThreads2, Cfg2<D>::Smem, st>>>(tq, tk, tv, a, err);
  } else {
    if (kernel_setup(attn_wide_kernel<D>, (size_t)C::Smem) <= 0) return -13;
    attn_wide_kernel<D><<<(unsigned)n_cta, kThreads, C::Smem, st>>>(tq, tk, tv, a, err);
  }
  int rc2 = launch_status("attention_wide");
  if (rc2 || n_split == 1) return rc2;
  const long long rows = (long long)batch_heads * p.nq;
  attn_wide_combine_kernel<D><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(a, rows);
  return launch_status("attention_wide combine");
}

}  // namespace

size_t attention_wide_ws_bytes(int d, int n_split, int batch_heads, int nq) {
  return (size_t)n_split * batch_heads * nq * (d + 2) * sizeof(float);
}

int attention_wide_max_split(int d, long long units) {
  const long long slots = (long long)num_sms() * (d == 256 ? 1 : 2);
  return units < slots ? (int)(slots / units) : 1;
}

int attention_wide(const AttnParams& p, int d, int batch_heads, float* ws, size_t ws_bytes, int bk128, int* err,
                   cudaStream_t st) {
  switch (d) {
    case 64: return launch_wide<64>(p, batch_heads, ws, ws_bytes, bk128, err, st);
    case 72: return launch_wide<72>(p, batch_heads, ws, ws_bytes, bk128, err, st);
    case 96: return launch_wide<96>(p, batch_heads, ws, ws_bytes, bk128, err, st);
    case 256: return launch_wide<256>(p, batch_heads, ws, ws_bytes, bk128, err, st);
    default: return -2;
  }
}

}  // namespace s3b
