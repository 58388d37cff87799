// Memory-bound kernels of the encoder hot path: LayerNorm (with the window
// partition folded into its row gather), im2col for the convolutions that
// run as tensor-core GEMMs, 2x2 max pools, q-pooling inside windows, image
// normalisation, casts, and ggml block dequantisation.
//
// Reference ops replaced: ggml_norm + mul + add (sam3.cpp:1036-1060, 3825,
// 4307, 4442), ggml_win_part / sam2_window_partition (3730, 4190-4228),
// ggml_pool_2d MAX (3914, 4283-4292), sam3_preprocess_image /
// sam2_preprocess_image normalisation (3486-3544), ggml type traits
// to_float for Q4_0 / Q4_1 / Q8_0 (1065-1081, 3167-3174).
#include "common.cuh"
#include "kernels.h"

namespace s3b {
namespace {

constexpr int kMaxVec = 16;  // float4 per lane -> C <= 2048

// The LayerNorms run between GEMMs that sweep their row tiles upwards: the rows a GEMM wrote last are the
// ones still in L2. Blocks, which start roughly in index order, therefore take rows from the end: the
// first reads hit the previous GEMM's most recent output, and the rows written last, the low ones, are
// the first the next GEMM reads. Rows are independent, so the order changes no value.
__device__ __forceinline__ unsigned layernorm_block_rev() { return gridDim.x - 1 - blockIdx.x; }

// One warp per R rows, NV = ceil(C / 128) float4 per lane and row held in
// registers (so the register footprint, and with it the number of rows in
// flight per SM, follows the row width; narrow rows are batched R to a warp so
// their loads overlap). The row is streamed (read once), the output is left in
// L2 for the GEMM that consumes it next.
template <int NV, int R>
__global__ void __launch_bounds__(256) layernorm_kernel(const float* __restrict__ x, long long ldx,
                                                        void* __restrict__ y, int y_f32, long long ldy, long long rows,
                                                        int C, const float* __restrict__ gamma,
                                                        const float* __restrict__ beta, float eps, RowMap map) {
  // blocks take rows from the end (see layernorm_block_rev)
  const long long row0 = ((long long)layernorm_block_rev() * (blockDim.x >> 5) + (threadIdx.x >> 5)) * R;
  const int lane = threadIdx.x & 31;
  const int nvec = C >> 2;
  float4 v[R][NV];
  long long src[R];  // input row; -1: padding row of a window partition; -2: past the last row
#pragma unroll
  for (int r = 0; r < R; ++r) {
    src[r] = row0 + r < rows ? map_row(map, row0 + r) : -2;
    const float* xr = x + (src[r] > 0 ? src[r] : 0) * ldx;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int vi = lane + 32 * i;
      v[r][i] = (src[r] >= 0 && vi < nvec) ? __ldcs(reinterpret_cast<const float4*>(xr + 4 * vi))
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  float mean[R], rstd[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) sum += (v[r][i].x + v[r][i].y) + (v[r][i].z + v[r][i].w);
    mean[r] = sum;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1)
#pragma unroll
    for (int r = 0; r < R; ++r) mean[r] += __shfl_xor_sync(0xffffffffu, mean[r], o);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    mean[r] /= (float)C;
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) {
        const float a = v[r][i].x - mean[r], b = v[r][i].y - mean[r], c = v[r][i].z - mean[r], d = v[r][i].w - mean[r];
        var += (a * a + b * b) + (c * c + d * d);
      }
    }
    rstd[r] = var;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1)
#pragma unroll
    for (int r = 0; r < R; ++r) rstd[r] += __shfl_xor_sync(0xffffffffu, rstd[r], o);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (src[r] == -2) continue;
    const long long row = row0 + r;
    if (src[r] < 0) {
      // padding row of a window partition: zeros (sam3.cpp:4199-4207 pads after the norm)
      if (y_f32) {
        float* yo = reinterpret_cast<float*>(y) + row * ldy;
        for (int c = lane; c < C; c += 32) yo[c] = 0.f;
      } else {
        __half* yo = reinterpret_cast<__half*>(y) + row * ldy;
        for (int c = lane; c < C; c += 32) yo[c] = __float2half_rn(0.f);
      }
      continue;
    }
    const float rs = rsqrtf(rstd[r] / (float)C + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) {
        const float4 g = *reinterpret_cast<const float4*>(gamma + 4 * vi);
        const float4 b = beta ? *reinterpret_cast<const float4*>(beta + 4 * vi) : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 o;
        o.x = (v[r][i].x - mean[r]) * rs * g.x + b.x;
        o.y = (v[r][i].y - mean[r]) * rs * g.y + b.y;
        o.z = (v[r][i].z - mean[r]) * rs * g.z + b.z;
        o.w = (v[r][i].w - mean[r]) * rs * g.w + b.w;
        if (y_f32) {
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + row * ldy + 4 * vi) = o;
        } else {
          __half2 h0 = __floats2half2_rn(o.x, o.y), h1 = __floats2half2_rn(o.z, o.w);
          uint2 u;
          u.x = *reinterpret_cast<uint32_t*>(&h0);
          u.y = *reinterpret_cast<uint32_t*>(&h1);
          *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(y) + row * ldy + 4 * vi) = u;
        }
      }
    }
  }
}

// Patch columns of the image convolutions (ViT 14x14 / s14, Hiera 7x7 / s4 / p3) staged through shared
// memory: one block per (frame, output row). The block first writes the k input rows its patches read (all
// channels, f16, zeros for the padding; from the f32 CHW planes, or with U8 straight from the uint8 HWC frame
// with the preprocessing's normalisation in f32, (p / 255 - mean) / std), then its OW x Kpad
// slab of the column matrix, which is contiguous, in consecutive 16-byte stores. Column = (ci*k + ky)*k + kx.
template <bool U8>
__global__ void __launch_bounds__(256) patch_cols_kernel(const void* __restrict__ src, int Cin, int H, int W, int k,
                                                         int stride, int pad, int OH, int OW, __half* __restrict__ out,
                                                         int Kpad, float m0, float m1, float m2, float s0, float s1,
                                                         float s2) {
  extern __shared__ uint8_t pc_smem[];
  const int Wp = (OW - 1) * stride + k;  // input columns the row's patches span, from ix = -pad
  __half* rows = reinterpret_cast<__half*>(pc_smem);            // [Cin][k][Wp]
  int* coff = reinterpret_cast<int*>(pc_smem + (((size_t)Cin * k * Wp * 2 + 15) & ~(size_t)15));  // [Kpad]
  const int b = blockIdx.x / OH, oy = blockIdx.x - b * OH;
  const int K = Cin * k * k;
  for (int c = threadIdx.x; c < Kpad; c += blockDim.x) {
    if (c < K) {
      const int ci = c / (k * k), r = c - ci * k * k, ky = r / k, kx = r - ky * k;
      coff[c] = (ci * k + ky) * Wp + kx;
    } else {
      coff[c] = -1;
    }
  }
  for (int r = 0; r < Cin * k; ++r) {
    const int ci = r / k, ky = r - ci * k;
    const int iy = oy * stride - pad + ky;
    __half* dst = rows + (size_t)r * Wp;
    for (int xx = threadIdx.x; xx < Wp; xx += blockDim.x) {
      const int ix = xx - pad;
      float v = 0.f;
      if (iy >= 0 && iy < H && ix >= 0 && ix < W) {
        if (U8) {
          const float p = (float)reinterpret_cast<const uint8_t*>(src)[(((size_t)b * H + iy) * W + ix) * 3 + ci];
          v = ci == 0 ? (p / 255.0f - m0) / s0 : ci == 1 ? (p / 255.0f - m1) / s1 : (p / 255.0f - m2) / s2;
        } else {
          v = reinterpret_cast<const float*>(src)[(((size_t)b * Cin + ci) * H + iy) * W + ix];
        }
      }
      dst[xx] = __float2half_rn(v);
    }
  }
  __syncthreads();
  const int vpr = Kpad >> 3;
  uint4* o = reinterpret_cast<uint4*>(out + ((size_t)b * OH + oy) * OW * Kpad);
  const __half zero = __float2half_rn(0.f);
  for (int t = threadIdx.x; t < OW * vpr; t += blockDim.x) {
    const int ox = t / vpr, v = t - ox * vpr;
    const int base = ox * stride;
    __half h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int off = coff[8 * v + e];
      h[e] = off >= 0 ? rows[off + base] : zero;
    }
    o[t] = *reinterpret_cast<const uint4*>(h);
  }
}

__global__ void im2col_3x3_cl_kernel(const __half* __restrict__ x, int B, int H, int W, int C,
                                     __half* __restrict__ out) {
  const int c8n = C / 8;
  const long long total = (long long)B * H * W * 9 * c8n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c8 = (int)(i % c8n);
    const long long t = i / c8n;
    const int tap = (int)(t % 9);
    const long long pix = t / 9;
    const long long b = pix / ((long long)H * W);
    const int rem = (int)(pix - b * H * W);
    const int y = rem / W, xx = rem - (rem / W) * W;
    const int iy = y + tap / 3 - 1, ix = xx + tap % 3 - 1;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (iy >= 0 && iy < H && ix >= 0 && ix < W)
      val = *reinterpret_cast<const uint4*>(x + ((b * H + iy) * W + ix) * C + c8 * 8);
    *reinterpret_cast<uint4*>(out + pix * 9 * C + (long long)tap * C + c8 * 8) = val;
  }
}

template <typename T>
__device__ __forceinline__ T tmax(T a, T b);
template <>
__device__ __forceinline__ float tmax<float>(float a, float b) { return fmaxf(a, b); }
template <>
__device__ __forceinline__ __half tmax<__half>(__half a, __half b) { return __hmax(a, b); }

template <typename T>
__global__ void maxpool2_cl_kernel(const T* __restrict__ x, int B, int H, int W, int C, T* __restrict__ y) {
  // 16 bytes (4 f32 or 8 f16 channels) per thread; 32-bit index math (the
  // launcher checks the element count)
  constexpr int V = 16 / sizeof(T);
  const int OH = H / 2, OW = W / 2, cv = C / V, ohw = OH * OW;
  const int total = B * ohw * cv;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int c = i % cv, pix = i / cv;
    const int b = pix / ohw, rem = pix - b * ohw;
    const int oy = rem / OW, ox = rem - oy * OW;
    const uint4* p = reinterpret_cast<const uint4*>(x + (((long long)b * H + 2 * oy) * W + 2 * ox) * C) + c;
    const long long wr = (long long)W * cv;  // one input row, in 16-byte units
    uint4 q[4] = {__ldcs(p), __ldcs(p + cv), __ldcs(p + wr), __ldcs(p + wr + cv)};
    uint4 r;
    const T* a0 = reinterpret_cast<const T*>(&q[0]);
    const T* a1 = reinterpret_cast<const T*>(&q[1]);
    const T* a2 = reinterpret_cast<const T*>(&q[2]);
    const T* a3 = reinterpret_cast<const T*>(&q[3]);
    T* o = reinterpret_cast<T*>(&r);
#pragma unroll
    for (int e = 0; e < V; ++e) o[e] = tmax(tmax(a0[e], a1[e]), tmax(a2[e], a3[e]));
    reinterpret_cast<uint4*>(y)[i] = r;
  }
}

// 2x2 max pool of the (ws x ws) token grid of each window; 8 channels per thread.
__global__ void qpool_kernel(const __half* __restrict__ q, long long ld, long long nwin, int ws, int C,
                             __half* __restrict__ out) {
  const int wo = ws / 2;
  const int c8n = C / 8;
  const long long total = nwin * wo * wo * c8n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c8 = (int)(i % c8n);
    const long long t = i / c8n;
    const int l = (int)(t % (wo * wo));
    const long long w = t / (wo * wo);
    const int oy = l / wo, ox = l - (l / wo) * wo;
    const long long r00 = w * ws * ws + (long long)(2 * oy) * ws + 2 * ox;
    const __half* p = q + c8 * 8;
    const uint4 a = *reinterpret_cast<const uint4*>(p + r00 * ld);
    const uint4 b = *reinterpret_cast<const uint4*>(p + (r00 + 1) * ld);
    const uint4 c = *reinterpret_cast<const uint4*>(p + (r00 + ws) * ld);
    const uint4 d = *reinterpret_cast<const uint4*>(p + (r00 + ws + 1) * ld);
    const __half2* ha = reinterpret_cast<const __half2*>(&a);
    const __half2* hb = reinterpret_cast<const __half2*>(&b);
    const __half2* hc = reinterpret_cast<const __half2*>(&c);
    const __half2* hd = reinterpret_cast<const __half2*>(&d);
    uint4 o;
    __half2* ho = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) ho[e] = __hmax2(__hmax2(ha[e], hb[e]), __hmax2(hc[e], hd[e]));
    *reinterpret_cast<uint4*>(out + t * C + c8 * 8) = o;
  }
}

// Source taps of output index o along one axis (sam3.cpp:3449-3462): half-pixel centre
// (o + 0.5) * s - 0.5 clamped at 0, the next tap clamped at the last index, weight of the next
// tap = the fraction. f64 with every operation rounded on its own (no contraction), as the
// reference's host code does.
__device__ __forceinline__ void bilinear_taps(int o, double s, int n, int& i0, int& i1, double& w) {
  double f = __dadd_rn(__dmul_rn(__dadd_rn((double)o, 0.5), s), -0.5);
  if (f < 0.0) f = 0.0;
  i0 = (int)f;
  i1 = i0 < n - 1 ? i0 + 1 : i0;
  w = __dadd_rn(f, -(double)i0);
}

// Bilinear resize of uint8 HWC frames [B][SH][SW][3] to [B][DH][DW] (sam3.cpp:3441-3481):
// v = wy0 (wx0 p00 + wx p01) + wy (wx0 p10 + wx p11) in f64, then (int)(v + 0.5) clamped to
// [0, 255]. NORM = false stores uint8 HWC; NORM = true stores the normalised f32 CHW frame
// ((q/255 - mean)/std, sam3.cpp:3505-3511 and 3535-3541) of the rounded value q.
template <bool NORM>
__global__ void resize_bilinear_kernel(const uint8_t* __restrict__ src, int B, int SH, int SW, int DH, int DW,
                                       double sy, double sx, float m0, float m1, float m2, float s0, float s1,
                                       float s2, void* __restrict__ out) {
  const long long plane = (long long)DH * DW;
  const long long total = (long long)B * plane;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / plane;
    const long long pix = i - b * plane;
    const int y = (int)(pix / DW), x = (int)(pix - (long long)y * DW);
    int y0, y1, x0, x1;
    double wy, wx;
    bilinear_taps(y, sy, SH, y0, y1, wy);
    bilinear_taps(x, sx, SW, x0, x1, wx);
    const double wy0 = __dadd_rn(1.0, -wy), wx0 = __dadd_rn(1.0, -wx);
    const uint8_t* f = src + b * SH * (long long)SW * 3;
    const uint8_t* r0 = f + (long long)y0 * SW * 3;
    const uint8_t* r1 = f + (long long)y1 * SW * 3;
    uint8_t q[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const double p00 = r0[x0 * 3 + c], p01 = r0[x1 * 3 + c], p10 = r1[x0 * 3 + c], p11 = r1[x1 * 3 + c];
      const double top = __dadd_rn(__dmul_rn(wx0, p00), __dmul_rn(wx, p01));
      const double bot = __dadd_rn(__dmul_rn(wx0, p10), __dmul_rn(wx, p11));
      const double v = __dadd_rn(__dmul_rn(wy0, top), __dmul_rn(wy, bot));
      int iv = (int)__dadd_rn(v, 0.5);
      iv = iv < 0 ? 0 : (iv > 255 ? 255 : iv);
      q[c] = (uint8_t)iv;
    }
    if (NORM) {
      float* o = static_cast<float*>(out);
      o[(b * 3 + 0) * plane + pix] = ((float)q[0] / 255.0f - m0) / s0;
      o[(b * 3 + 1) * plane + pix] = ((float)q[1] / 255.0f - m1) / s1;
      o[(b * 3 + 2) * plane + pix] = ((float)q[2] / 255.0f - m2) / s2;
    } else {
      uint8_t* o = static_cast<uint8_t*>(out) + i * 3;
      o[0] = q[0];
      o[1] = q[1];
      o[2] = q[2];
    }
  }
}

// 4 values per thread (n4 = n / 4 float4 groups), then the n % 4 tail.
__global__ void cast_kernel(const float* __restrict__ x, long long n, __half* __restrict__ y) {
  const long long n4 = n >> 2;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 v = __ldcs(reinterpret_cast<const float4*>(x) + i);
    __half2 h[2] = {__floats2half2_rn(v.x, v.y), __floats2half2_rn(v.z, v.w)};
    reinterpret_cast<uint2*>(y)[i] = *reinterpret_cast<const uint2*>(h);
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) y[4 * n4 + threadIdx.x] = __float2half_rn(x[4 * n4 + threadIdx.x]);
}

__global__ void add_scaled_kernel(const float* __restrict__ a, const float* __restrict__ b, float s, long long n,
                                  float* __restrict__ y) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = a[i] + s * b[i];
}

__global__ void add_scaled_to_f16_kernel(const float* __restrict__ a, const float* __restrict__ b, float s,
                                         long long n, __half* __restrict__ y) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = __float2half_rn(b ? a[i] + s * b[i] : a[i]);
}

// One thread per 32-value block. Values are produced exactly as ggml's
// dequantisers define them: q4_0 (q - 8) * d, q4_1 q * d + m (multiply then
// add, both rounded to f32), q8_0 q * d, with d and m the f16 fields.
__global__ void dequant_kernel(const uint8_t* __restrict__ src, int qtype, long long ne0, long long nrows,
                               long long row_bytes, void* __restrict__ dst, int dst_f32, long long ld_dst) {
  const long long nb = ne0 / 32;
  const long long total = nb * nrows;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / nb, blk = i - r * nb;
    float v[32];
    if (qtype == QT_Q4_0) {
      const uint8_t* p = src + r * row_bytes + blk * 18;
      const float d = __half2float(*reinterpret_cast<const __half*>(p));
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint8_t b = p[2 + j];
        v[j] = (float)((int)(b & 0x0F) - 8) * d;
        v[j + 16] = (float)((int)(b >> 4) - 8) * d;
      }
    } else if (qtype == QT_Q4_1) {
      const uint8_t* p = src + r * row_bytes + blk * 20;
      const float d = __half2float(*reinterpret_cast<const __half*>(p));
      const float m = __half2float(*reinterpret_cast<const __half*>(p + 2));
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint8_t b = p[4 + j];
        v[j] = __fadd_rn(__fmul_rn((float)(b & 0x0F), d), m);
        v[j + 16] = __fadd_rn(__fmul_rn((float)(b >> 4), d), m);
      }
    } else {  // QT_Q8_0
      const uint8_t* p = src + r * row_bytes + blk * 34;
      const float d = __half2float(*reinterpret_cast<const __half*>(p));
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = (float)(reinterpret_cast<const int8_t*>(p + 2)[j]) * d;
    }
    if (dst_f32) {
      float* o = reinterpret_cast<float*>(dst) + r * ld_dst + blk * 32;
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = v[j];
    } else {
      __half* o = reinterpret_cast<__half*>(dst) + r * ld_dst + blk * 32;
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = __float2half_rn(v[j]);
    }
  }
}

inline int grid_for(long long n, int threads) {
  long long g = (n + threads - 1) / threads;
  const long long cap = (long long)num_sms() * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

inline int launch_ok() { return launch_status("elementwise kernel"); }

// Rows whose float4 count is not a multiple of 32 (Hiera widths 96, 144, 192, 288, 576): L lanes per
// row (L = 4, 8 or 16, C = 4 L NV exactly), 32 / L rows per warp side by side, RI such groups per warp
// loaded up front; the reductions are shuffles inside each L-lane group. No lane idles, and every load
// instruction covers 32 / L contiguous 16 L-byte runs.
template <int L, int NV, int RI>
__global__ void __launch_bounds__(256) layernorm_sub_kernel(const float* __restrict__ x, long long ldx,
                                                            void* __restrict__ y, int y_f32, long long ldy,
                                                            long long rows, int C, const float* __restrict__ gamma,
                                                            const float* __restrict__ beta, float eps, RowMap map) {
  constexpr int G = 32 / L;
  const int lane = threadIdx.x & 31;
  const int sub = lane / L, sl = lane % L;
  const long long row0 = ((long long)layernorm_block_rev() * (blockDim.x >> 5) + (threadIdx.x >> 5)) * (G * RI);
  float4 v[RI][NV];
  long long src[RI];
#pragma unroll
  for (int r = 0; r < RI; ++r) {
    const long long row = row0 + r * G + sub;
    src[r] = row < rows ? map_row(map, row) : -2;
    const float* xr = x + (src[r] > 0 ? src[r] : 0) * ldx;
#pragma unroll
    for (int i = 0; i < NV; ++i)
      v[r][i] = src[r] >= 0 ? __ldcs(reinterpret_cast<const float4*>(xr + 4 * (sl + L * i)))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float mean[RI], var[RI];
#pragma unroll
  for (int r = 0; r < RI; ++r) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) s += (v[r][i].x + v[r][i].y) + (v[r][i].z + v[r][i].w);
    mean[r] = s;
  }
#pragma unroll
  for (int o = L / 2; o; o >>= 1)
#pragma unroll
    for (int r = 0; r < RI; ++r) mean[r] += __shfl_xor_sync(0xffffffffu, mean[r], o);
#pragma unroll
  for (int r = 0; r < RI; ++r) {
    mean[r] /= (float)C;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float a = v[r][i].x - mean[r], b = v[r][i].y - mean[r], c = v[r][i].z - mean[r], d = v[r][i].w - mean[r];
      s += (a * a + b * b) + (c * c + d * d);
    }
    var[r] = s;
  }
#pragma unroll
  for (int o = L / 2; o; o >>= 1)
#pragma unroll
    for (int r = 0; r < RI; ++r) var[r] += __shfl_xor_sync(0xffffffffu, var[r], o);
#pragma unroll
  for (int r = 0; r < RI; ++r) {
    if (src[r] == -2) continue;
    const long long row = row0 + r * G + sub;
    const float rs = rsqrtf(var[r] / (float)C + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int vi = sl + L * i;
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);  // padding row of a window partition: zeros
      if (src[r] >= 0) {
        const float4 g = *reinterpret_cast<const float4*>(gamma + 4 * vi);
        const float4 b = beta ? *reinterpret_cast<const float4*>(beta + 4 * vi) : make_float4(0.f, 0.f, 0.f, 0.f);
        o.x = (v[r][i].x - mean[r]) * rs * g.x + b.x;
        o.y = (v[r][i].y - mean[r]) * rs * g.y + b.y;
        o.z = (v[r][i].z - mean[r]) * rs * g.z + b.z;
        o.w = (v[r][i].w - mean[r]) * rs * g.w + b.w;
      }
      if (y_f32) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + row * ldy + 4 * vi) = o;
      } else {
        __half2 h0 = __floats2half2_rn(o.x, o.y), h1 = __floats2half2_rn(o.z, o.w);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&h0);
        u.y = *reinterpret_cast<uint32_t*>(&h1);
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(y) + row * ldy + 4 * vi) = u;
      }
    }
  }
}

}  // namespace

int layernorm(const float* x, long long ldx, void* y, int y_f32, long long ldy, long long rows, int C,
              const float* gamma, const float* beta, float eps, const RowMap& map, cudaStream_t st) {
  if (C % 4 || C > 4 * 32 * kMaxVec || ldx % 4 || ldy % 4 || rows <= 0) return -1;
  const int warps = 8;
  const int c4 = C / 4;
  if (c4 % 32) {
    // sub-warp rows: the largest L in {16, 8, 4} dividing C/4 with at most 12 float4 per lane
    int L = 0;
    for (int l = 16; l >= 4; l >>= 1)
      if (c4 % l == 0 && c4 / l <= 12) { L = l; break; }
    if (L) {
      constexpr int RI = 2;
      const long long rows_per_block = (long long)warps * (32 / L) * RI;
      const long long blocks = (rows + rows_per_block - 1) / rows_per_block;
      if (blocks > 0x7fffffffLL) return -1;
      const int nv = c4 / L;
      bool launched = true;
#define S3B_LNS(LL, NN)                                                                                          \
  if (L == LL && nv == NN)                                                                                       \
    layernorm_sub_kernel<LL, NN, RI><<<(unsigned)blocks, warps * 32, 0, st>>>(x, ldx, y, y_f32, ldy, rows, C,    \
                                                                              gamma, beta, eps, map);            \
  else
      S3B_LNS(16, 1) S3B_LNS(16, 2) S3B_LNS(16, 3) S3B_LNS(16, 5) S3B_LNS(16, 6) S3B_LNS(16, 9)
      S3B_LNS(8, 1) S3B_LNS(8, 3) S3B_LNS(8, 5) S3B_LNS(8, 7) S3B_LNS(8, 9) S3B_LNS(8, 11)
      S3B_LNS(4, 1) S3B_LNS(4, 3) S3B_LNS(4, 5) S3B_LNS(4, 7) S3B_LNS(4, 9) S3B_LNS(4, 11)
      launched = false;
#undef S3B_LNS
      if (launched) return launch_ok();
    }
  }
  const int nv = (C + 127) / 128;
  const int rpw = nv <= 2 ? 4 : nv == 3 ? 2 : 1;  // rows per warp
  const long long blocks = (rows + (long long)warps * rpw - 1) / ((long long)warps * rpw);
  if (blocks > 0x7fffffffLL) return -1;
#define S3B_LN_CASE(N)                                                                                            \
  case N:                                                                                                        \
    layernorm_kernel<N, (N <= 2 ? 4 : N == 3 ? 2 : 1)><<<(unsigned)blocks, warps * 32, 0, st>>>(                 \
        x, ldx, y, y_f32, ldy, rows, C, gamma, beta, eps, map);                                                  \
    break;
  switch (nv) {
    S3B_LN_CASE(1) S3B_LN_CASE(2) S3B_LN_CASE(3) S3B_LN_CASE(4) S3B_LN_CASE(5) S3B_LN_CASE(6) S3B_LN_CASE(7)
    S3B_LN_CASE(8) S3B_LN_CASE(9) S3B_LN_CASE(10) S3B_LN_CASE(11) S3B_LN_CASE(12) S3B_LN_CASE(13)
    S3B_LN_CASE(14) S3B_LN_CASE(15) S3B_LN_CASE(16)
    default:
      return -1;
  }
#undef S3B_LN_CASE
  return launch_ok();
}

static size_t patch_cols_smem(int Cin, int k, int stride, int OW, int Kpad) {
  const size_t Wp = (size_t)(OW - 1) * stride + k;
  return (((size_t)Cin * k * Wp * 2 + 15) & ~(size_t)15) + (size_t)Kpad * 4;
}

template <bool U8>
static int launch_patch_cols(const void* src, int B, int Cin, int H, int W, int k, int stride, int pad, int OH, int OW,
                             __half* out, int Kpad, const float* mean, const float* stdv, cudaStream_t st) {
  if (Kpad < Cin * k * k || Kpad % 8 || (reinterpret_cast<uintptr_t>(out) & 15) || B <= 0 || OH <= 0 || OW <= 0 ||
      (U8 && Cin != 3))
    return -1;
  if ((long long)B * OH > 0x7fffffffLL) return -1;
  const size_t smem = patch_cols_smem(Cin, k, stride, OW, Kpad);
  if (smem > 232448) return -1;
  // the opt-in limit once per device (models with other patch sizes need other amounts)
  if (kernel_setup(patch_cols_kernel<U8>, 232448) <= 0) return -13;
  patch_cols_kernel<U8><<<(unsigned)(B * OH), 256, smem, st>>>(
      src, Cin, H, W, k, stride, pad, OH, OW, out, Kpad, U8 ? mean[0] : 0.f, U8 ? mean[1] : 0.f, U8 ? mean[2] : 0.f,
      U8 ? stdv[0] : 1.f, U8 ? stdv[1] : 1.f, U8 ? stdv[2] : 1.f);
  return launch_ok();
}

int patch_cols_f32(const float* img, int B, int Cin, int H, int W, int k, int stride, int pad, int OH, int OW,
                   __half* out, int Kpad, cudaStream_t st) {
  return launch_patch_cols<false>(img, B, Cin, H, W, k, stride, pad, OH, OW, out, Kpad, nullptr, nullptr, st);
}

int patch_cols_u8(const uint8_t* hwc, int B, int H, int W, const float mean[3], const float stdv[3], int k, int stride,
                  int pad, int OH, int OW, __half* out, int Kpad, cudaStream_t st) {
  return launch_patch_cols<true>(hwc, B, 3, H, W, k, stride, pad, OH, OW, out, Kpad, mean, stdv, st);
}

int im2col_3x3_cl(const __half* x, int B, int H, int W, int C, __half* out, cudaStream_t st) {
  if (C % 8) return -1;
  const long long n = (long long)B * H * W * 9 * (C / 8);
  im2col_3x3_cl_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, B, H, W, C, out);
  return launch_ok();
}

int maxpool2_cl_f16(const __half* x, int B, int H, int W, int C, __half* y, cudaStream_t st) {
  const long long n = (long long)B * (H / 2) * (W / 2) * (C / 8);  // 16-byte groups
  if (C % 8 || n > 0x7fffffffLL || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return -1;
  maxpool2_cl_kernel<__half><<<grid_for(n, 256), 256, 0, st>>>(x, B, H, W, C, y);
  return launch_ok();
}
int maxpool2_cl_f32(const float* x, int B, int H, int W, int C, float* y, cudaStream_t st) {
  const long long n = (long long)B * (H / 2) * (W / 2) * (C / 4);  // 16-byte groups
  if (C % 4 || n > 0x7fffffffLL || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return -1;
  maxpool2_cl_kernel<float><<<grid_for(n, 256), 256, 0, st>>>(x, B, H, W, C, y);
  return launch_ok();
}

int qpool_windows(const __half* q, long long ld, long long nwin, int ws, int C, __half* out, cudaStream_t st) {
  if (C % 8 || ld % 8) return -1;
  const long long n = nwin * (ws / 2) * (ws / 2) * (C / 8);
  qpool_kernel<<<grid_for(n, 256), 256, 0, st>>>(q, ld, nwin, ws, C, out);
  return launch_ok();
}

int resize_bilinear_u8(const uint8_t* src, int B, int SH, int SW, int DH, int DW, const float* mean,
                       const float* stdv, void* out, cudaStream_t st) {
  if (B <= 0 || SH <= 0 || SW <= 0 || DH <= 0 || DW <= 0) return -1;
  const double sy = (double)SH / DH, sx = (double)SW / DW;
  const long long n = (long long)B * DH * DW;
  if (mean && stdv)
    resize_bilinear_kernel<true><<<grid_for(n, 256), 256, 0, st>>>(src, B, SH, SW, DH, DW, sy, sx, mean[0], mean[1],
                                                                   mean[2], stdv[0], stdv[1], stdv[2], out);
  else
    resize_bilinear_kernel<false><<<grid_for(n, 256), 256, 0, st>>>(src, B, SH, SW, DH, DW, sy, sx, 0.f, 0.f, 0.f,
                                                                    1.f, 1.f, 1.f, out);
  return launch_ok();
}

int cast_f32_f16(const float* x, long long n, __half* y, cudaStream_t st) {
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 7)) return -1;
  cast_kernel<<<grid_for((n + 3) / 4, 256), 256, 0, st>>>(x, n, y);
  return launch_ok();
}

int add_scaled_f32(const float* a, const float* b, float s, long long n, float* y, cudaStream_t st) {
  add_scaled_kernel<<<grid_for(n, 256), 256, 0, st>>>(a, b, s, n, y);
  return launch_ok();
}

int add_scaled_to_f16(const float* a, const float* b, float s, long long n, __half* y, cudaStream_t st) {
  add_scaled_to_f16_kernel<<<grid_for(n, 256), 256, 0, st>>>(a, b, s, n, y);
  return launch_ok();
}

// One thread per 4 values of a prompt row (16 per row); float4 loads and stores.
__global__ void build_prompt_kernel(const PromptArgs args, long long rows, void* __restrict__ a,
                                    void* __restrict__ b, int out_f16) {
  const long long m_sp = (long long)args.n_slots * args.slot_tokens;
  const long long n = rows * (kPromptMD / 4);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i >> 4;
    const int c = (int)(i & 15) * 4;
    float4 pr, ps;
    if (r < m_sp) {
      const int s = (int)(r / args.slot_tokens);
      const long long t = r - (long long)s * args.slot_tokens;
      pr = *reinterpret_cast<const float4*>(args.feat[s] + t * kPromptMD + c);
      ps = *reinterpret_cast<const float4*>(args.pe[s] + t * kPromptMD + c);
      if (args.has_tpos[s]) {  // pos[d + n*MD] += tpos_all[d + enc_idx*MD]
        ps.x += args.tpos[s][c];
        ps.y += args.tpos[s][c + 1];
        ps.z += args.tpos[s][c + 2];
        ps.w += args.tpos[s][c + 3];
      }
    } else {
      const long long q = r - m_sp;
      const int k = (int)(q / args.split), t = (int)(q - (long long)k * args.split);
      pr = *reinterpret_cast<const float4*>(args.ptrs + ((long long)args.ptr_src[k] * args.split + t) * kPromptMD + c);
      ps = make_float4(args.ptr_pe[k][c], args.ptr_pe[k][c + 1], args.ptr_pe[k][c + 2], args.ptr_pe[k][c + 3]);
    }
    if (out_f16) {
      __half2* ka = reinterpret_cast<__half2*>(reinterpret_cast<__half*>(a) + r * kPromptMD + c);
      __half2* vb = reinterpret_cast<__half2*>(reinterpret_cast<__half*>(b) + r * kPromptMD + c);
      ka[0] = __halves2half2(__float2half_rn(pr.x + ps.x), __float2half_rn(pr.y + ps.y));
      ka[1] = __halves2half2(__float2half_rn(pr.z + ps.z), __float2half_rn(pr.w + ps.w));
      vb[0] = __halves2half2(__float2half_rn(pr.x), __float2half_rn(pr.y));
      vb[1] = __halves2half2(__float2half_rn(pr.z), __float2half_rn(pr.w));
    } else {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(a) + r * kPromptMD + c) = pr;
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(b) + r * kPromptMD + c) = ps;
    }
  }
}

int build_prompt(const PromptArgs& args, void* a, void* b, int out_f16, cudaStream_t st) {
  if (args.n_slots < 0 || args.n_slots > kPromptMaxSlots || args.n_ptr < 0 || args.n_ptr > kPromptMaxPtrs ||
      args.split <= 0 || (args.n_slots > 0 && args.slot_tokens <= 0) || (args.n_ptr > 0 && !args.ptrs) || !a || !b)
    return -2;
  for (int s = 0; s < args.n_slots; ++s)
    if (!args.feat[s] || !args.pe[s] || (reinterpret_cast<uintptr_t>(args.feat[s]) & 15) ||
        (reinterpret_cast<uintptr_t>(args.pe[s]) & 15))
      return -11;
  if ((args.ptrs && (reinterpret_cast<uintptr_t>(args.ptrs) & 15)) || (reinterpret_cast<uintptr_t>(a) & 15) ||
      (reinterpret_cast<uintptr_t>(b) & 15))
    return -11;
  const long long rows = (long long)args.n_slots * args.slot_tokens + (long long)args.n_ptr * args.split;
  if (rows <= 0) return -2;
  build_prompt_kernel<<<grid_for(rows * 16, 256), 256, 0, st>>>(args, rows, a, b, out_f16);
  return launch_ok();
}

long long qtype_row_bytes(int qtype, long long ne0) {
  switch (qtype) {
    case QT_F32: return ne0 * 4;
    case QT_F16: return ne0 * 2;
    case QT_Q4_0: return (ne0 / 32) * 18;
    case QT_Q4_1: return (ne0 / 32) * 20;
    case QT_Q8_0: return (ne0 / 32) * 34;
    default: return -1;
  }
}

// One thread per 32-value block of row n: the f16 scale goes to scales[blk][n]; q4_0 values to
// 16 bytes of the nibble plane row n, as 4 words of 8 values each (value 2p of a word in nibble p,
// value 2p + 1 in nibble p + 4); q8_0 values to 32 bytes of the int8 plane row n, in order.
__global__ void repack_q_kernel(const uint8_t* __restrict__ src, int qtype, int N, int K, long long row_bytes,
                                uint8_t* __restrict__ values, uint16_t* __restrict__ scales) {
  const int nb = K / 32;
  const long long total = (long long)nb * N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / nb), blk = (int)(i - (long long)n * nb);
    const uint8_t* p = src + n * row_bytes + (long long)blk * (qtype == QT_Q4_0 ? 18 : 34);
    scales[(long long)blk * N + n] = (uint16_t)(p[0] | (p[1] << 8));
    if (qtype == QT_Q4_0) {
      uint8_t q[32];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        q[j] = p[2 + j] & 0x0F;
        q[j + 16] = p[2 + j] >> 4;
      }
      uint32_t* o = reinterpret_cast<uint32_t*>(values + (long long)n * (K / 2) + blk * 16);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t w = 0;
#pragma unroll
        for (int pp = 0; pp < 4; ++pp)
          w |= ((uint32_t)q[8 * g + 2 * pp] << (4 * pp)) | ((uint32_t)q[8 * g + 2 * pp + 1] << (16 + 4 * pp));
        o[g] = w;
      }
    } else {
      uint8_t* o = values + (long long)n * K + blk * 32;
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = p[2 + j];
    }
  }
}

int repack_q_rows(const void* src, int qtype, int N, int K, void* values, __half* scales, cudaStream_t st) {
  if (qtype != QT_Q4_0 && qtype != QT_Q8_0) return -1;
  if (K % 32 || N <= 0 || K <= 0) return -2;
  const long long n = (long long)(K / 32) * N;
  repack_q_kernel<<<grid_for(n, 128), 128, 0, st>>>(reinterpret_cast<const uint8_t*>(src), qtype, N, K,
                                                    qtype_row_bytes(qtype, K), reinterpret_cast<uint8_t*>(values),
                                                    reinterpret_cast<uint16_t*>(scales));
  return launch_ok();
}

int dequant_rows(const void* src, int qtype, long long ne0, long long nrows, void* dst, int dst_f32,
                 long long ld_dst, cudaStream_t st) {
  if (qtype != QT_Q4_0 && qtype != QT_Q4_1 && qtype != QT_Q8_0) return -1;
  if (ne0 % 32 || nrows <= 0) return -2;
  const long long n = (ne0 / 32) * nrows;
  dequant_kernel<<<grid_for(n, 128), 128, 0, st>>>(reinterpret_cast<const uint8_t*>(src), qtype, ne0, nrows,
                                                   qtype_row_bytes(qtype, ne0), dst, dst_f32, ld_dst);
  return launch_ok();
}

}  // namespace s3b
