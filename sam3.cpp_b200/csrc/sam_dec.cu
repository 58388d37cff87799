// Kernels of the SAM mask decoder (sm_100a).
//
// Replaces the ggml graph of sam3_build_sam_dec_graph (sam3.cpp:10544-10757): the TwoWay
// transformer blocks (sam3_twoway_block_forward, 10436-10500) with their 8-head attentions
// (sam3_sam_attention, 10164-10262), the output upscaling (two 2x2 transposed convolutions, the
// 1x1 projections of the high-resolution features, LayerNorm2d, GELU-erf) and the hypernetwork /
// IoU / object-score MLPs (sam3_mlp_forward, 10503-10518).
//
// Work split: the image side (H x H tokens of 256 channels) runs its projections on the tcgen05
// GEMM (mask_decoder.cpp); these kernels cover what is left:
//   - the token side (6 output tokens + the prompt tokens, at most kTokMaxRows rows): linear layers
//     as warp-per-column dot products that stream each f16 weight row once, LayerNorm, attention;
//   - the two cross-attentions, whose head dim is 16 (internal dim 128 over 8 heads), too narrow for
//     a tensor-core tile: tokens -> image splits the H*H keys over CTAs (partial softmax + merge),
//     image -> tokens runs one thread per (image row, head) over the few token keys;
//   - the image keys' residual LayerNorm with the f16 operands of the next GEMMs in one pass;
//   - the two upscaling stages as tiled per-pixel kernels that keep their weights in shared memory
//     and never write the 4H x 4H x 32 upscaled map: the second stage ends in the four mask
//     products, so only the masks leave the SM.
#include "common.cuh"
#include "kernels.h"

namespace s3b {
namespace {

inline int dec_grid(long long n, int threads, int per_sm = 16) {
  long long g = (n + threads - 1) / threads;
  const long long cap = (long long)num_sms() * per_sm;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

inline int dec_launch_ok() { return launch_status("mask decoder kernel"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void unpack8(const uint4 w, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 r;
  __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
  return r;
}

// ---------------------------------------------------------------- token-side linear layers
struct TokJobs {
  TokJob j[kTokMaxJobs];
};

constexpr int kTokThreads = 256, kTokWarps = 8, kTokCols = 32;  // 32 output columns per CTA
constexpr int kTokSmemFloats = 8192;                                  // 32 KB of staged input rows

// CTA (blockIdx.x, blockIdx.y): columns [32 x, 32 x + 32) of job y, one per lane; the 8 warps split the
// reduction dimension into contiguous slices. The job's input rows are staged in shared memory in K
// chunks of kTokSmemFloats / RB columns; each lane streams its column's weight slice (16-byte loads)
// and accumulates it against all R rows; the 8 partial sums per (row, column) meet in shared memory.
template <int RB>
__global__ void __launch_bounds__(kTokThreads) tok_linear_kernel(const TokJobs jobs) {
  const TokJob& jb = jobs.j[blockIdx.y];
  const int n0 = blockIdx.x * kTokCols;
  if (n0 >= jb.N) return;  // uniform over the CTA
  extern __shared__ __align__(16) float tok_smem[];
  float* xs = tok_smem;                          // [RB][KC]
  float* red = tok_smem + kTokSmemFloats;        // [kTokWarps][RB][kTokCols]
  constexpr int KC = kTokSmemFloats / RB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = n0 + lane;
  const int R = jb.R;
  float acc[RB];
#pragma unroll
  for (int r = 0; r < RB; ++r) acc[r] = 0.f;
  for (int k0 = 0; k0 < jb.K; k0 += KC) {
    const int kc = min(KC, jb.K - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < R * kc; i += kTokThreads) {
      const int r = i / kc, c = i - r * kc;
      float v = jb.x[r * jb.ldx + k0 + c];
      if (jb.x2) v += jb.x2[r * jb.ldx + k0 + c];
      xs[r * KC + c] = v;
    }
    __syncthreads();
    // this warp's slice of the chunk, in whole 8-value vectors
    const int nvec = kc / 8, per = (nvec + kTokWarps - 1) / kTokWarps;
    const int v0 = warp * per, v1 = min(nvec, v0 + per);
    if (n < jb.N) {
      const __half* w = jb.W + (long long)n * jb.ldw + k0;
      for (int vv = v0; vv < v1; ++vv) {
        const int c = vv * 8;
        float wf[8];
        unpack8(*reinterpret_cast<const uint4*>(w + c), wf);
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          if (r < R) {
            const float4 a = *reinterpret_cast<const float4*>(&xs[r * KC + c]);
            const float4 b = *reinterpret_cast<const float4*>(&xs[r * KC + c + 4]);
            float s = acc[r];
            s = fmaf(a.x, wf[0], s);
            s = fmaf(a.y, wf[1], s);
            s = fmaf(a.z, wf[2], s);
            s = fmaf(a.w, wf[3], s);
            s = fmaf(b.x, wf[4], s);
            s = fmaf(b.y, wf[5], s);
            s = fmaf(b.z, wf[6], s);
            s = fmaf(b.w, wf[7], s);
            acc[r] = s;
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RB; ++r)
    if (r < R) red[(warp * RB + r) * kTokCols + lane] = acc[r];
  __syncthreads();
  for (int i = threadIdx.x; i < R * kTokCols; i += kTokThreads) {
    const int r = i / kTokCols, c = i - r * kTokCols;
    const int col = n0 + c;
    if (col >= jb.N) continue;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kTokWarps; ++w) v += red[(w * RB + r) * kTokCols + c];
    v += jb.b ? jb.b[col] : 0.f;
    if (jb.act == 1) v = fmaxf(v, 0.f);
    else if (jb.act == 2) v = 1.f / (1.f + expf(-v));
    if (jb.resid) v += jb.resid[r * jb.ldr + col];
    jb.y[r * jb.ldy + col] = v;
  }
}

template <int RB>
constexpr size_t tok_smem_bytes() {
  return (size_t)(kTokSmemFloats + kTokWarps * RB * kTokCols) * 4;
}

// ---------------------------------------------------------------- token LayerNorm
// One warp per row, C / 32 values per lane (C <= 1024); two-pass mean / variance in f32.
__global__ void __launch_bounds__(256) tok_ln_kernel(const float* a, const float* b, long long ld, int rows, int C,
                                                     const float* g, const float* beta, float eps, float* y) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[32];
  const int per = C / 32;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (i < per) {
      const int c = i * 32 + lane;
      v[i] = a[row * ld + c] + (b ? b[row * ld + c] : 0.f);
      s += v[i];
    }
  }
  const float mean = warp_sum(s) / (float)C;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (i < per) {
      const float d = v[i] - mean;
      q = fmaf(d, d, q);
    }
  const float rstd = rsqrtf(warp_sum(q) / (float)C + eps);
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (i < per) {
      const int c = i * 32 + lane;
      y[row * ld + c] = (v[i] - mean) * rstd * g[c] + beta[c];
    }
}

// ---------------------------------------------------------------- token self-attention
// One CTA; the nt rows of q, k and v (heads * hd <= 256 columns each) are staged in shared memory, then
// thread (token i, head h) computes its softmax row over the nt keys and its hd outputs.
__global__ void __launch_bounds__(256) tok_attn_kernel(const float* q, long long ldq, const float* k, long long ldk,
                                                       const float* v, long long ldv, int nt, int heads, int hd,
                                                       float scale, float* out, long long ldo) {
  extern __shared__ float tsm[];  // q, k, v rows [nt][cols + 1] each
  const int cols = heads * hd, ld = cols + 1;
  float* qs = tsm;
  float* ks = qs + nt * ld;
  float* vs = ks + nt * ld;
  for (int i = threadIdx.x; i < nt * cols; i += blockDim.x) {
    const int r = i / cols, c = i - r * cols;
    qs[r * ld + c] = q[r * ldq + c];
    ks[r * ld + c] = k[r * ldk + c];
    vs[r * ld + c] = v[r * ldv + c];
  }
  __syncthreads();
  const int t = threadIdx.x;
  if (t >= nt * heads) return;
  const int i = t / heads, h = t - i * heads;
  const float* qi = qs + i * ld + h * hd;
  float s[kTokMaxRows];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kTokMaxRows; ++j) {
    if (j < nt) {
      const float* kj = ks + j * ld + h * hd;
      float d = 0.f;
      for (int c = 0; c < hd; ++c) d = fmaf(qi[c], kj[c], d);
      s[j] = d * scale;
      m = fmaxf(m, s[j]);
    }
  }
  float l = 0.f;
#pragma unroll
  for (int j = 0; j < kTokMaxRows; ++j)
    if (j < nt) {
      s[j] = expf(s[j] - m);
      l += s[j];
    }
  const float inv = 1.f / l;
  for (int c = 0; c < hd; ++c) {
    float o = 0.f;
#pragma unroll
    for (int j = 0; j < kTokMaxRows; ++j)
      if (j < nt) o = fmaf(s[j], vs[j * ld + h * hd + c], o);
    out[i * ldo + h * hd + c] = o * inv;
  }
}

// ---------------------------------------------------------------- tokens -> image attention (hd 16)
// CTA c: keys [c*64, c*64 + 64). K / V rows of the chunk staged in shared memory (f16, 8 heads x 16);
// thread (token i, head h) computes the chunk's max, exp-sum and weighted value sum.
constexpr int kHd = 16;
__global__ void __launch_bounds__(256) t2i_partial_kernel(const float* q, long long ldq, const __half* k,
                                                          long long ldk, const __half* v, long long ldv, int nt,
                                                          int heads, long long nkv, float scale, float* ws) {
  __shared__ __align__(16) __half ks[kT2iChunk][8 * kHd];
  __shared__ __align__(16) __half vs[kT2iChunk][8 * kHd];
  const long long j0 = (long long)blockIdx.x * kT2iChunk;
  const int nj = (int)min((long long)kT2iChunk, nkv - j0);
  const int cols = heads * kHd;  // <= 128
  const int vec = cols / 8;
  for (int i = threadIdx.x; i < nj * vec; i += blockDim.x) {
    const int r = i / vec, c = (i - r * vec) * 8;
    *reinterpret_cast<uint4*>(&ks[r][c]) = *reinterpret_cast<const uint4*>(k + (j0 + r) * ldk + c);
    *reinterpret_cast<uint4*>(&vs[r][c]) = *reinterpret_cast<const uint4*>(v + (j0 + r) * ldv + c);
  }
  __syncthreads();
  const int t = threadIdx.x;
  if (t >= nt * heads) return;
  const int i = t / heads, h = t - i * heads;
  float qv[kHd];
#pragma unroll
  for (int d = 0; d < kHd; ++d) qv[d] = q[i * ldq + h * kHd + d] * scale;
  float m = -INFINITY;
  for (int j = 0; j < nj; ++j) {
    float kf[kHd];
    unpack8(*reinterpret_cast<const uint4*>(&ks[j][h * kHd]), *reinterpret_cast<float(*)[8]>(&kf[0]));
    unpack8(*reinterpret_cast<const uint4*>(&ks[j][h * kHd + 8]), *reinterpret_cast<float(*)[8]>(&kf[8]));
    float s = 0.f;
#pragma unroll
    for (int d = 0; d < kHd; ++d) s = fmaf(qv[d], kf[d], s);
    m = fmaxf(m, s);
  }
  float l = 0.f, o[kHd];
#pragma unroll
  for (int d = 0; d < kHd; ++d) o[d] = 0.f;
  for (int j = 0; j < nj; ++j) {
    float kf[kHd], vf[kHd];
    unpack8(*reinterpret_cast<const uint4*>(&ks[j][h * kHd]), *reinterpret_cast<float(*)[8]>(&kf[0]));
    unpack8(*reinterpret_cast<const uint4*>(&ks[j][h * kHd + 8]), *reinterpret_cast<float(*)[8]>(&kf[8]));
    unpack8(*reinterpret_cast<const uint4*>(&vs[j][h * kHd]), *reinterpret_cast<float(*)[8]>(&vf[0]));
    unpack8(*reinterpret_cast<const uint4*>(&vs[j][h * kHd + 8]), *reinterpret_cast<float(*)[8]>(&vf[8]));
    float s = 0.f;
#pragma unroll
    for (int d = 0; d < kHd; ++d) s = fmaf(qv[d], kf[d], s);
    const float p = expf(s - m);
    l += p;
#pragma unroll
    for (int d = 0; d < kHd; ++d) o[d] = fmaf(p, vf[d], o[d]);
  }
  float* w = ws + ((long long)blockIdx.x * nt * heads + t) * (kHd + 2);
  w[0] = m;
  w[1] = l;
#pragma unroll
  for (int d = 0; d < kHd; ++d) w[2 + d] = o[d];
}

// thread (token i, head h, d): merges the chunks' partial results.
__global__ void __launch_bounds__(256) t2i_combine_kernel(const float* ws, int nt, int heads, int n_chunks, float* out,
                                                          long long ldo) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= nt * heads * kHd) return;
  const int th = t / kHd, d = t - th * kHd;
  const int i = th / heads, h = th - i * heads;
  const long long stride = (long long)nt * heads * (kHd + 2);
  float M = -INFINITY;
  for (int c = 0; c < n_chunks; ++c) M = fmaxf(M, ws[c * stride + th * (kHd + 2)]);
  float L = 0.f, O = 0.f;
  for (int c = 0; c < n_chunks; ++c) {
    const float* w = ws + c * stride + th * (kHd + 2);
    const float e = expf(w[0] - M);
    L = fmaf(w[1], e, L);
    O = fmaf(w[2 + d], e, O);
  }
  out[i * ldo + h * kHd + d] = O / L;
}

// ---------------------------------------------------------------- image -> tokens attention (hd 16)
// Thread (row p, head h): online softmax over the nt token keys staged in shared memory.
__global__ void __launch_bounds__(256) i2t_kernel(const __half* q, long long ldq, const float* k, long long ldk,
                                                  const float* v, long long ldv, int nt, int heads, long long n,
                                                  float scale, __half* out, long long ldo) {
  __shared__ float ks[kTokMaxRows][8 * kHd];
  __shared__ float vs[kTokMaxRows][8 * kHd];
  const int cols = heads * kHd;
  for (int i = threadIdx.x; i < nt * cols; i += blockDim.x) {
    const int r = i / cols, c = i - r * cols;
    ks[r][c] = k[r * ldk + c];
    vs[r][c] = v[r * ldv + c];
  }
  __syncthreads();
  const long long total = n * heads;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (long long)gridDim.x * blockDim.x) {
    const long long p = t / heads;
    const int h = (int)(t - p * heads);
    float qv[kHd];
    unpack8(*reinterpret_cast<const uint4*>(q + p * ldq + h * kHd), *reinterpret_cast<float(*)[8]>(&qv[0]));
    unpack8(*reinterpret_cast<const uint4*>(q + p * ldq + h * kHd + 8), *reinterpret_cast<float(*)[8]>(&qv[8]));
#pragma unroll
    for (int d = 0; d < kHd; ++d) qv[d] *= scale;
    float m = -INFINITY, l = 0.f, o[kHd];
#pragma unroll
    for (int d = 0; d < kHd; ++d) o[d] = 0.f;
    for (int j = 0; j < nt; ++j) {
      float s = 0.f;
#pragma unroll
      for (int d = 0; d < kHd; ++d) s = fmaf(qv[d], ks[j][h * kHd + d], s);
      const float mn = fmaxf(m, s);
      const float corr = expf(m - mn), pj = expf(s - mn);
      l = fmaf(l, corr, pj);
#pragma unroll
      for (int d = 0; d < kHd; ++d) o[d] = fmaf(o[d], corr, pj * vs[j][h * kHd + d]);
      m = mn;
    }
    const float inv = 1.f / l;
    float r0[8], r1[8];
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      r0[d] = o[d] * inv;
      r1[d] = o[8 + d] * inv;
    }
    *reinterpret_cast<uint4*>(out + p * ldo + h * kHd) = pack8(r0);
    *reinterpret_cast<uint4*>(out + p * ldo + h * kHd + 8) = pack8(r1);
  }
}

// ---------------------------------------------------------------- image keys
// One warp per row of 256 channels, 8 consecutive channels per lane.
__global__ void __launch_bounds__(256) dec_keys_kernel(const float* x, long long rows, int mode, const float* add0,
                                                       const float* add1, const float* g, const float* beta,
                                                       float eps, const float* pe, float* keys, __half* k16,
                                                       __half* kpe16) {
  const int lane = threadIdx.x & 31;
  const int c = lane * 8;
  for (long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += (long long)gridDim.x * 8) {
    const float* xr = x + row * 256 + c;
    float v[8];
    *reinterpret_cast<float4*>(&v[0]) = *reinterpret_cast<const float4*>(xr);
    *reinterpret_cast<float4*>(&v[4]) = *reinterpret_cast<const float4*>(xr + 4);
    if (mode == 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (add1) v[i] += add1[c + i];
        v[i] += add0[c + i];
      }
    } else {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[i];
      const float mean = warp_sum(s) * (1.f / 256.f);
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[i] -= mean;
        q = fmaf(v[i], v[i], q);
      }
      const float rstd = rsqrtf(warp_sum(q) * (1.f / 256.f) + eps);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = v[i] * rstd * g[c + i] + beta[c + i];
    }
    float* kr = keys + row * 256 + c;
    *reinterpret_cast<float4*>(kr) = *reinterpret_cast<const float4*>(&v[0]);
    *reinterpret_cast<float4*>(kr + 4) = *reinterpret_cast<const float4*>(&v[4]);
    *reinterpret_cast<uint4*>(k16 + row * 256 + c) = pack8(v);
    const float* pr = pe + row * 256 + c;
    float w[8];
    *reinterpret_cast<float4*>(&w[0]) = *reinterpret_cast<const float4*>(pr);
    *reinterpret_cast<float4*>(&w[4]) = *reinterpret_cast<const float4*>(pr + 4);
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] += v[i];
    *reinterpret_cast<uint4*>(kpe16 + row * 256 + c) = pack8(w);
  }
}

// ---------------------------------------------------------------- upscaling stage 1
// Persistent CTAs over tiles of 64 consecutive pixels. Thread (pair pp, group cg): pixels 2 pp and
// 2 pp + 1 of the tile, output channels 8 cg .. 8 cg + 7. The tile's feat_s1 rows are staged as f16
// (the projection's input rounding) and the projection weight, transposed to [k][co], stays in
// shared memory for the CTA's lifetime. The LayerNorm2d statistics of a pixel are reduced over the
// 8 lanes that hold its 64 channels.
constexpr int kU1Tile = 64, kU1Pad = 264, kU1WPad = 72;
struct U1Smem {
  __half feat[kU1Tile][kU1Pad];
  __half w[256][kU1WPad];
};

__global__ void __launch_bounds__(256) dec_up1_kernel(const float* up1, const float* feat, const __half* wsrc,
                                                      const float* bs1, const float* g, const float* beta, float eps,
                                                      long long n, __half* out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  U1Smem& S = *reinterpret_cast<U1Smem*>(smem_raw);
  const int t = threadIdx.x;
  for (int i = t; i < 64 * 256; i += 256) {
    const int co = i >> 8, k = i & 255;
    S.w[k][co] = wsrc[co * 256 + k];
  }
  const int pp = t >> 3, cg = t & 7;
  float bias[8], gg[8], bb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    bias[i] = bs1[cg * 8 + i];
    gg[i] = g[cg * 8 + i];
    bb[i] = beta[cg * 8 + i];
  }
  const long long tiles = (n + kU1Tile - 1) / kU1Tile;
  for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const long long p0 = tile * kU1Tile;
    const int np = (int)min((long long)kU1Tile, n - p0);
    __syncthreads();
    for (int i = t; i < kU1Tile * 64; i += 256) {  // 64 float4 per row
      const int r = i >> 6, c = (i & 63) * 4;
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < np) f = *reinterpret_cast<const float4*>(feat + (p0 + r) * 256 + c);
      *reinterpret_cast<__half2*>(&S.feat[r][c]) = __floats2half2_rn(f.x, f.y);
      *reinterpret_cast<__half2*>(&S.feat[r][c + 2]) = __floats2half2_rn(f.z, f.w);
    }
    __syncthreads();
    float acc[2][8];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[a][i] = 0.f;
    const int ra = 2 * pp, rb = 2 * pp + 1;
    for (int k0 = 0; k0 < 256; k0 += 8) {
      float fa[8], fb[8];
      unpack8(*reinterpret_cast<const uint4*>(&S.feat[ra][k0]), fa);
      unpack8(*reinterpret_cast<const uint4*>(&S.feat[rb][k0]), fb);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        float w[8];
        unpack8(*reinterpret_cast<const uint4*>(&S.w[k0 + kk][cg * 8]), w);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          acc[0][i] = fmaf(fa[kk], w[i], acc[0][i]);
          acc[1][i] = fmaf(fb[kk], w[i], acc[1][i]);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      const int r = 2 * pp + a;
      const bool live = r < np;
      float v[8];
      if (live) {
        const float* u = up1 + (p0 + r) * 64 + cg * 8;
        *reinterpret_cast<float4*>(&v[0]) = *reinterpret_cast<const float4*>(u);
        *reinterpret_cast<float4*>(&v[4]) = *reinterpret_cast<const float4*>(u + 4);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[i] += acc[a][i] + bias[i];
        s += v[i];
      }
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      const float mean = s * (1.f / 64.f);
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[i] -= mean;
        q = fmaf(v[i], v[i], q);
      }
      q += __shfl_xor_sync(0xffffffffu, q, 1);
      q += __shfl_xor_sync(0xffffffffu, q, 2);
      q += __shfl_xor_sync(0xffffffffu, q, 4);
      const float rstd = rsqrtf(q * (1.f / 64.f) + eps);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = gelu_erf(v[i] * rstd * gg[i] + bb[i]);
      if (live) *reinterpret_cast<uint4*>(out + (p0 + r) * 64 + cg * 8) = pack8(v);
    }
  }
}

// ---------------------------------------------------------------- upscaling stage 2 + masks
// Persistent CTAs over tiles of 128 pixels of one output row y. Thread (pair pp, group cg): pixels
// x0 + 4 (pp / 2) + (pp % 2) and that + 2 (the same kernel position of the transposed convolution,
// so the two share its weights), channels 8 cg .. 8 cg + 7 of 32. The four mask products are reduced
// over the 4 lanes of a pixel; lane cg writes mask cg.
constexpr int kMTile = 128, kMPad = 264, kMWPad = 40;
struct MSmem {
  __half feat[kMTile][kMPad];
  __half w0[256][kMWPad];     // conv_s0 weight, [k][co]
  __half w2[4][64][kMWPad];   // deconv2 weight per kernel position, [ci][co]
};

__global__ void __launch_bounds__(256) dec_masks_kernel(const __half* u1, const __half* w2src, const float* b2,
                                                        const float* feat, const __half* w0src, const float* bs0,
                                                        const float* hyper, int S, float* masks) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  MSmem& Sm = *reinterpret_cast<MSmem*>(smem_raw);
  const int t = threadIdx.x;
  for (int i = t; i < 32 * 256; i += 256) {
    const int co = i >> 8, k = i & 255;
    Sm.w0[k][co] = w0src[co * 256 + k];
  }
  for (int i = t; i < 4 * 32 * 64; i += 256) {
    const int row = i >> 6, ci = i & 63;  // row = kpos*32 + co
    Sm.w2[row >> 5][ci][row & 31] = w2src[row * 64 + ci];
  }
  const int pp = t >> 2, cg = t & 3;
  float bd[8], bp[8], hy[4][8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    bd[i] = b2[cg * 8 + i];
    bp[i] = bs0[cg * 8 + i];
#pragma unroll
    for (int m = 0; m < 4; ++m) hy[m][i] = hyper[m * 32 + cg * 8 + i];
  }
  const int xoff = 4 * (pp >> 1) + (pp & 1);
  const int tiles_x = (S + kMTile - 1) / kMTile;
  const long long tiles = (long long)S * tiles_x;
  const int Sh = S / 2;
  const long long plane = (long long)S * S;
  for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int y = (int)(tile / tiles_x), x0 = (int)(tile - (long long)y * tiles_x) * kMTile;
    const int nx = min(kMTile, S - x0);
    __syncthreads();
    const float* frow = feat + ((long long)y * S + x0) * 256;
    for (int i = t; i < kMTile * 64; i += 256) {
      const int r = i >> 6, c = (i & 63) * 4;
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < nx) f = *reinterpret_cast<const float4*>(frow + (long long)r * 256 + c);
      *reinterpret_cast<__half2*>(&Sm.feat[r][c]) = __floats2half2_rn(f.x, f.y);
      *reinterpret_cast<__half2*>(&Sm.feat[r][c + 2]) = __floats2half2_rn(f.z, f.w);
    }
    __syncthreads();
    float acc[2][8];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[a][i] = 0.f;
    // 1x1 projection of feat_s0 (256 -> 32)
    for (int k0 = 0; k0 < 256; k0 += 8) {
      float fa[8], fb[8];
      unpack8(*reinterpret_cast<const uint4*>(&Sm.feat[xoff][k0]), fa);
      unpack8(*reinterpret_cast<const uint4*>(&Sm.feat[xoff + 2][k0]), fb);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        float w[8];
        unpack8(*reinterpret_cast<const uint4*>(&Sm.w0[k0 + kk][cg * 8]), w);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          acc[0][i] = fmaf(fa[kk], w[i], acc[0][i]);
          acc[1][i] = fmaf(fb[kk], w[i], acc[1][i]);
        }
      }
    }
    // 2x2 / stride 2 transposed convolution of u1 (64 -> 32): the kernel position is (y % 2, x % 2)
    const int xa = x0 + xoff, xb = xa + 2;
    const int kp = (y & 1) * 2 + (xa & 1);
    const __half* ua = u1 + ((long long)(y >> 1) * Sh + min(xa >> 1, Sh - 1)) * 64;
    const __half* ub = u1 + ((long long)(y >> 1) * Sh + min(xb >> 1, Sh - 1)) * 64;
    float dv[2][8];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int i = 0; i < 8; ++i) dv[a][i] = 0.f;
    for (int c0 = 0; c0 < 64; c0 += 8) {
      float fa[8], fb[8];
      unpack8(*reinterpret_cast<const uint4*>(ua + c0), fa);
      unpack8(*reinterpret_cast<const uint4*>(ub + c0), fb);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        float w[8];
        unpack8(*reinterpret_cast<const uint4*>(&Sm.w2[kp][c0 + kk][cg * 8]), w);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          dv[0][i] = fmaf(fa[kk], w[i], dv[0][i]);
          dv[1][i] = fmaf(fb[kk], w[i], dv[1][i]);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      float pm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // (deconv + its bias) + (projection + its bias), then GELU-erf (sam3.cpp:10675-10693)
        const float u = gelu_erf((dv[a][i] + bd[i]) + (acc[a][i] + bp[i]));
#pragma unroll
        for (int m = 0; m < 4; ++m) pm[m] = fmaf(hy[m][i], u, pm[m]);
      }
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        pm[m] += __shfl_xor_sync(0xffffffffu, pm[m], 1);
        pm[m] += __shfl_xor_sync(0xffffffffu, pm[m], 2);
      }
      const int xx = a ? xb : xa;
      if (xx - x0 < nx) {
        const float val = cg == 0 ? pm[0] : cg == 1 ? pm[1] : cg == 2 ? pm[2] : pm[3];
        masks[cg * plane + (long long)y * S + xx] = val;
      }
    }
  }
}

// The mask a tracking step keeps (sam3_propagate_single, sam3.cpp:11395-11430): token 0 without multimask
// output, else the best IoU among tokens 1 .. n-1 (first on ties); the object pointer's token is the
// chosen one when use_mm_token, else token 0. Every CTA takes the same decision from the n IoU values and
// copies its share of the plane; CTA 0 also writes the token and the scores.
__global__ void __launch_bounds__(256) pick_mask_kernel(const float* masks, long long plane, const float* iou,
                                                        const float* tokens, int n_masks, int multimask,
                                                        int use_mm_token, float* out_mask, float* out_token,
                                                        float* out_scores, const float* obj) {
  int best = 0;
  if (multimask && n_masks > 1) {
    best = 1;
    for (int m = 2; m < n_masks; ++m)
      if (iou[m] > iou[best]) best = m;
  }
  if (out_mask) {
    const float4* src = reinterpret_cast<const float4*>(masks + best * plane);
    float4* dst = reinterpret_cast<float4*>(out_mask);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < plane / 4; i += (long long)gridDim.x * blockDim.x)
      dst[i] = src[i];
  }
  if (blockIdx.x == 0) {
    if (out_token) {
      const int t = use_mm_token ? best : 0;
      for (int i = threadIdx.x; i < 256; i += blockDim.x) out_token[i] = tokens[t * 256 + i];
    }
    if (out_scores && threadIdx.x == 0) {
      out_scores[0] = iou[best];
      out_scores[1] = obj ? *obj : 0.f;
      out_scores[2] = (float)best;
    }
  }
}

}  // namespace

// ---------------------------------------------------------------- launchers
static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int pick_mask(const float* masks, long long plane, const float* iou, const float* tokens, int n_masks, int multimask,
              int use_mm_token, float* out_mask, float* out_token, float* out_scores, const float* obj,
              cudaStream_t st) {
  if (!masks || !iou || !tokens || n_masks <= 0 || plane <= 0 || plane % 4) return -2;
  if (!al16(masks) || (out_mask && !al16(out_mask))) return -11;
  pick_mask_kernel<<<dec_grid(plane / 4, 256, 2), 256, 0, st>>>(masks, plane, iou, tokens, n_masks, multimask,
                                                                 use_mm_token, out_mask, out_token, out_scores, obj);
  return dec_launch_ok();
}

int tok_linear(const TokJob* jobs, int n_jobs, cudaStream_t st) {
  if (n_jobs <= 0 || n_jobs > kTokMaxJobs) return -1;
  TokJobs J;
  int maxN = 0, maxR = 0;
  for (int i = 0; i < n_jobs; ++i) {
    const TokJob& j = jobs[i];
    if (!j.x || !j.W || !j.y || j.R <= 0 || j.R > kTokMaxRows || j.N <= 0 || j.K <= 0 || j.K % 8 || j.ldw % 8 ||
        j.ldw < j.K)
      return -2;
    if (!al16(j.W)) return -11;
    J.j[i] = j;
    maxN = max(maxN, j.N);
    maxR = max(maxR, j.R);
  }
  const dim3 grid((maxN + kTokCols - 1) / kTokCols, n_jobs);
  if (maxR <= 8) {
    if (kernel_setup(tok_linear_kernel<8>, tok_smem_bytes<8>()) < 0) return -13;
    tok_linear_kernel<8><<<grid, kTokThreads, tok_smem_bytes<8>(), st>>>(J);
  } else if (maxR <= 16) {
    if (kernel_setup(tok_linear_kernel<16>, tok_smem_bytes<16>()) < 0) return -13;
    tok_linear_kernel<16><<<grid, kTokThreads, tok_smem_bytes<16>(), st>>>(J);
  } else {
    if (kernel_setup(tok_linear_kernel<32>, tok_smem_bytes<32>()) < 0) return -13;
    tok_linear_kernel<32><<<grid, kTokThreads, tok_smem_bytes<32>(), st>>>(J);
  }
  return dec_launch_ok();
}

int tok_layernorm(const float* a, const float* b, long long ld, int rows, int C, const float* g, const float* beta,
                  float eps, float* y, cudaStream_t st) {
  if (!a || !y || !g || !beta || rows <= 0 || C <= 0 || C > 1024 || C % 32) return -2;
  tok_ln_kernel<<<(rows + 7) / 8, 256, 0, st>>>(a, b, ld, rows, C, g, beta, eps, y);
  return dec_launch_ok();
}

int tok_attention(const float* q, long long ldq, const float* k, long long ldk, const float* v, long long ldv,
                  int nt, int heads, int hd, float scale, float* out, long long ldo, cudaStream_t st) {
  if (!q || !k || !v || !out || nt <= 0 || nt > kTokMaxRows || heads <= 0 || nt * heads > 256 || hd <= 0 || hd > 32 ||
      heads * hd > 256)
    return -2;
  const size_t smem = (size_t)3 * nt * (heads * hd + 1) * 4;
  if (kernel_setup(tok_attn_kernel, (size_t)3 * kTokMaxRows * 257 * 4) < 0) return -13;
  tok_attn_kernel<<<1, 256, smem, st>>>(q, ldq, k, ldk, v, ldv, nt, heads, hd, scale, out, ldo);
  return dec_launch_ok();
}

long long t2i_ws_floats(int nt, int heads, long long nkv) {
  return ((nkv + kT2iChunk - 1) / kT2iChunk) * nt * heads * (kHd + 2);
}

int t2i_attention(const float* q, long long ldq, const __half* k, long long ldk, const __half* v, long long ldv,
                  int nt, int heads, long long nkv, float scale, float* ws, float* out, long long ldo,
                  cudaStream_t st) {
  if (!q || !k || !v || !ws || !out || nt <= 0 || nt > kTokMaxRows || heads <= 0 || heads > 8 || nt * heads > 256 ||
      nkv <= 0)
    return -2;
  if (!al16(k) || !al16(v) || ldk % 8 || ldv % 8) return -11;
  const long long chunks = (nkv + kT2iChunk - 1) / kT2iChunk;
  if (chunks > (1LL << 30)) return -2;
  t2i_partial_kernel<<<(unsigned)chunks, 256, 0, st>>>(q, ldq, k, ldk, v, ldv, nt, heads, nkv, scale, ws);
  int rc = dec_launch_ok();
  if (rc) return rc;
  const int n = nt * heads * kHd;
  t2i_combine_kernel<<<(n + 255) / 256, 256, 0, st>>>(ws, nt, heads, (int)chunks, out, ldo);
  return dec_launch_ok();
}

int i2t_attention(const __half* q, long long ldq, const float* k, long long ldk, const float* v, long long ldv,
                  int nt, int heads, long long n, float scale, __half* out, long long ldo, cudaStream_t st) {
  if (!q || !k || !v || !out || nt <= 0 || nt > kTokMaxRows || heads <= 0 || heads > 8 || n <= 0) return -2;
  if (!al16(q) || !al16(out) || ldq % 8 || ldo % 8) return -11;
  i2t_kernel<<<dec_grid(n * heads, 256, 8), 256, 0, st>>>(q, ldq, k, ldk, v, ldv, nt, heads, n, scale, out, ldo);
  return dec_launch_ok();
}

int dec_keys(const float* x, long long rows, int mode, const float* add0, const float* add1, const float* g,
             const float* beta, float eps, const float* pe, float* keys, __half* k16, __half* kpe16, cudaStream_t st) {
  if (!x || rows <= 0 || !pe || !keys || !k16 || !kpe16 || (mode == 0 && !add0) || (mode == 1 && (!g || !beta)) ||
      (mode != 0 && mode != 1))
    return -2;
  if (!al16(x) || !al16(pe) || !al16(keys) || !al16(k16) || !al16(kpe16)) return -11;
  dec_keys_kernel<<<dec_grid(rows * 32, 256), 256, 0, st>>>(x, rows, mode, add0, add1, g, beta, eps, pe, keys, k16,
                                                             kpe16);
  return dec_launch_ok();
}

int dec_upscale1(const float* up1, const float* feat_s1, const __half* ws1, const float* bs1, const float* g,
                 const float* beta, float eps, long long n, __half* out, cudaStream_t st) {
  if (!up1 || !feat_s1 || !ws1 || !bs1 || !g || !beta || !out || n <= 0) return -2;
  if (!al16(up1) || !al16(feat_s1) || !al16(out)) return -11;
  const size_t smem = sizeof(U1Smem);
  if (kernel_setup(dec_up1_kernel, smem) < 0) return -13;
  const long long tiles = (n + kU1Tile - 1) / kU1Tile;
  const int grid = (int)min(tiles, (long long)num_sms() * 3);
  dec_up1_kernel<<<grid, 256, smem, st>>>(up1, feat_s1, ws1, bs1, g, beta, eps, n, out);
  return dec_launch_ok();
}

int dec_masks(const __half* u1, const __half* w2, const float* b2, const float* feat_s0, const __half* ws0,
              const float* bs0, const float* hyper, int S, float* masks, cudaStream_t st) {
  if (!u1 || !w2 || !b2 || !feat_s0 || !ws0 || !bs0 || !hyper || !masks || S <= 0 || S % 2) return -2;
  if (!al16(u1) || !al16(feat_s0) || !al16(w2)) return -11;
  const size_t smem = sizeof(MSmem);
  if (kernel_setup(dec_masks_kernel, smem) < 0) return -13;
  const long long tiles = (long long)S * ((S + kMTile - 1) / kMTile);
  const int grid = (int)min(tiles, (long long)num_sms() * 2);
  dec_masks_kernel<<<grid, 256, smem, st>>>(u1, w2, b2, feat_s0, ws0, bs0, hyper, S, masks);
  return dec_launch_ok();
}

}  // namespace s3b
