// Kernels of the tracker's memory encoder (sm_100a).
//
// Replaces the ggml graph of sam3_encode_memory (sam3.cpp:11506-11603) around its tensor-core parts
// (the 64 -> 256 downsampler conv, the 1x1 projections and the CXBlock MLPs run on the tcgen05 GEMM,
// memory_encoder.cpp):
//   - the mask preprocessing (sam3_bilinear_interpolate, 9614-9639, twice, with the sigmoid /
//     scale / bias between): one thread per output pixel, coordinates in f64 and the blend in the
//     reference's f32 order with no fused multiply-adds, so a resize equals the host function's bits;
//   - the first three downsampler stages (3x3 / stride 2 / pad 1 convolutions with 1 -> 4 -> 16 -> 64
//     channels, too narrow for tensor-core tiles): one thread per output pixel with all its output
//     channels in registers, LayerNorm2d (eps 1e-6) and GELU in the same thread;
//   - the stride-2 column matrix of the last stage, a row LayerNorm + GELU, the CXBlock depthwise 7x7
//     conv + LayerNorm2d (one warp per pixel, 8 channels per lane), the object-pointer selection and
//     the no-object embedding, both decided on the device from the decoder's object score.
#include "common.cuh"
#include "kernels.h"

namespace s3b {
namespace {

inline int me_grid(long long n, int threads, int per_sm = 16) {
  long long g = (n + threads - 1) / threads;
  const long long cap = (long long)num_sms() * per_sm;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

inline int me_launch_ok() { return launch_status("memory encoder kernel"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ggml_gelu's tanh form: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  return 0.5f * x * (1.0f + tanhf(u));
}

__device__ __forceinline__ float f16_round(float x) { return __half2float(__float2half_rn(x)); }

// One output pixel per thread. The source coordinate, its clamp and the taps follow the host function
// in f64; the weights are f32 and the blend is (1 - wy)((1 - wx) a + wx b) + wy((1 - wx) c + wx d) with
// each operation rounded on its own. mode 1 applies sigmoid(v) * scale + bias to the result.
__global__ void __launch_bounds__(256) bilinear_kernel(const float* __restrict__ src, int sw, int sh,
                                                       float* __restrict__ dst, int dw, int dh, int mode, float scale,
                                                       float bias) {
  const long long n = (long long)dw * dh;
  const double sx = (double)sw / dw, sy = (double)sh / dh;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int y = (int)(i / dw), x = (int)(i - (long long)y * dw);
    double fy = (y + 0.5) * sy - 0.5;
    fy = fmax(0.0, fmin(fy, (double)(sh - 1)));
    const int y0 = min((int)fy, sh - 2), y1 = y0 + 1;
    const float wy = (float)(fy - y0);
    double fx = (x + 0.5) * sx - 0.5;
    fx = fmax(0.0, fmin(fx, (double)(sw - 1)));
    const int x0 = min((int)fx, sw - 2), x1 = x0 + 1;
    const float wx = (float)(fx - x0);
    const float a = src[(long long)y0 * sw + x0], b = src[(long long)y0 * sw + x1];
    const float c = src[(long long)y1 * sw + x0], d = src[(long long)y1 * sw + x1];
    const float owx = __fsub_rn(1.0f, wx), owy = __fsub_rn(1.0f, wy);
    const float top = __fadd_rn(__fmul_rn(owx, a), __fmul_rn(wx, b));
    const float bot = __fadd_rn(__fmul_rn(owx, c), __fmul_rn(wx, d));
    float v = __fadd_rn(__fmul_rn(owy, top), __fmul_rn(wy, bot));
    if (mode == 1) {
      const float s = 1.0f / (1.0f + expf(-v));
      v = s * scale + bias;
    }
    dst[i] = v;
  }
}

// 3x3 / stride 2 / pad 1 convolution over a channel-last f32 map [Hi][Wi][CIN] into [Ho][Wo][COUT],
// inputs rounded to f16 (the reference's im2col runs in its f16 kernel's type), weights [9][CIN][COUT]
// in shared memory, f32 accumulation; then + bias, LayerNorm over the COUT channels (eps) and GELU-tanh.
template <int CIN, int COUT>
__global__ void __launch_bounds__(128) ds_conv_kernel(const float* __restrict__ x, int Hi, int Wi, const float* w,
                                                      const float* bias, const float* g, const float* beta, float eps,
                                                      float* __restrict__ y, int Ho, int Wo) {
  __shared__ float ws[9 * CIN * COUT];
  __shared__ float bs[COUT], gs[COUT], betas[COUT];
  for (int i = threadIdx.x; i < 9 * CIN * COUT; i += blockDim.x) ws[i] = w[i];
  for (int i = threadIdx.x; i < COUT; i += blockDim.x) {
    bs[i] = bias[i];
    gs[i] = g[i];
    betas[i] = beta[i];
  }
  __syncthreads();
  const long long n = (long long)Ho * Wo;
  for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += (long long)gridDim.x * blockDim.x) {
    const int oy = (int)(p / Wo), ox = (int)(p - (long long)oy * Wo);
    float acc[COUT];
#pragma unroll
    for (int c = 0; c < COUT; ++c) acc[c] = 0.f;
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
      const int iy = 2 * oy - 1 + ky;
      if (iy < 0 || iy >= Hi) continue;
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const int ix = 2 * ox - 1 + kx;
        if (ix < 0 || ix >= Wi) continue;
        const float* xp = x + ((long long)iy * Wi + ix) * CIN;
        const float* wp = ws + (ky * 3 + kx) * CIN * COUT;
#pragma unroll 4
        for (int ci = 0; ci < CIN; ++ci) {
          const float v = f16_round(xp[ci]);
#pragma unroll
          for (int c = 0; c < COUT; ++c) acc[c] = fmaf(v, wp[ci * COUT + c], acc[c]);
        }
      }
    }
    float mean = 0.f;
#pragma unroll
    for (int c = 0; c < COUT; ++c) {
      acc[c] += bs[c];
      mean += acc[c];
    }
    mean *= 1.0f / COUT;
    float var = 0.f;
#pragma unroll
    for (int c = 0; c < COUT; ++c) {
      const float d = acc[c] - mean;
      var = fmaf(d, d, var);
    }
    const float rstd = rsqrtf(var * (1.0f / COUT) + eps);
    float* yp = y + p * COUT;
#pragma unroll
    for (int c = 0; c < COUT; c += 4) {
      float4 o;
      o.x = gelu_tanh_f((acc[c] - mean) * rstd * gs[c] + betas[c]);
      o.y = gelu_tanh_f((acc[c + 1] - mean) * rstd * gs[c + 1] + betas[c + 1]);
      o.z = gelu_tanh_f((acc[c + 2] - mean) * rstd * gs[c + 2] + betas[c + 2]);
      o.w = gelu_tanh_f((acc[c + 3] - mean) * rstd * gs[c + 3] + betas[c + 3]);
      *reinterpret_cast<float4*>(yp + c) = o;
    }
  }
}

// Column matrix of a 3x3 / stride 2 / pad 1 convolution over channel-last f32 [Hi][Wi][C] (C a multiple
// of 8): row (oy, ox), column (ky*3 + kx)*C + c, f16, zeros outside the map.
__global__ void __launch_bounds__(256) im2col_s2_kernel(const float* __restrict__ x, int Hi, int Wi, int C, int Ho,
                                                        int Wo, __half* __restrict__ col) {
  const int vec = C / 8;
  const long long n = (long long)Ho * Wo * 9 * vec;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int v = (int)(i % vec);
    const long long r = i / vec;
    const int tap = (int)(r % 9);
    const long long p = r / 9;
    const int oy = (int)(p / Wo), ox = (int)(p - (long long)oy * Wo);
    const int iy = 2 * oy - 1 + tap / 3, ix = 2 * ox - 1 + tap % 3;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (iy >= 0 && iy < Hi && ix >= 0 && ix < Wi) {
      const float* s = x + ((long long)iy * Wi + ix) * C + v * 8;
      *reinterpret_cast<float4*>(&f[0]) = *reinterpret_cast<const float4*>(s);
      *reinterpret_cast<float4*>(&f[4]) = *reinterpret_cast<const float4*>(s + 4);
    }
    uint4 o;
    __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(f[2 * k], f[2 * k + 1]);
    *reinterpret_cast<uint4*>(col + p * 9 * C + tap * C + v * 8) = o;
  }
}

// One warp per row of C = 32 * NV channels: out = f16(GELU-tanh(LayerNorm(x) * g + beta)).
template <int NV>
__global__ void __launch_bounds__(256) ln_gelu_rows_kernel(const float* __restrict__ x, long long rows, const float* g,
                                                           const float* beta, float eps, __half* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  constexpr int C = 32 * NV;
  for (long long r = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += (long long)gridDim.x * 8) {
    float v[NV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      v[i] = x[r * C + i * 32 + lane];
      s += v[i];
    }
    const float mean = warp_sum(s) * (1.0f / C);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      v[i] -= mean;
      q = fmaf(v[i], v[i], q);
    }
    const float rstd = rsqrtf(warp_sum(q) * (1.0f / C) + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = i * 32 + lane;
      y[r * C + c] = __float2half_rn(gelu_tanh_f(v[i] * rstd * g[c] + beta[c]));
    }
  }
}

// CXBlock depthwise 7x7 / pad 3 convolution (f32 math as ggml_conv_2d_dw_direct) + bias + LayerNorm2d
// over the 256 channels. Persistent CTAs over 4 x 8 pixel tiles: the tile's 10 x 14 input halo (zeros
// outside the map) and the 49 x 256 weights are staged in shared memory; warp w takes 4 consecutive
// pixels of tile row w / 2, lane 8 consecutive channels, so each tap's weights are loaded once for 4
// pixels. Out f16 [H*W][256] (the pointwise MLP's GEMM operand).
constexpr int kDwTY = 4, kDwTX = 8, kDwHY = kDwTY + 6, kDwHX = kDwTX + 6;
constexpr size_t kDwSmem = (size_t)(kDwHY * kDwHX + 49) * 256 * 4;

__global__ void __launch_bounds__(256) dwconv7_ln_kernel(const float* __restrict__ x, int H, int W, const float* w,
                                                         const float* b, const float* g, const float* beta, float eps,
                                                         __half* __restrict__ y) {
  extern __shared__ __align__(16) float dsm[];
  float* xs = dsm;                          // [kDwHY * kDwHX][256]
  float* ws = dsm + kDwHY * kDwHX * 256;    // [49][256]
  for (int i = threadIdx.x; i < 49 * 64; i += blockDim.x)
    reinterpret_cast<float4*>(ws)[i] = reinterpret_cast<const float4*>(w)[i];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, c = lane * 8;
  const int ly = warp >> 1, lx0 = (warp & 1) * 4;
  float bb[8], gg[8], be[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    bb[i] = b[c + i];
    gg[i] = g[c + i];
    be[i] = beta[c + i];
  }
  const int tiles_x = (W + kDwTX - 1) / kDwTX, tiles = tiles_x * ((H + kDwTY - 1) / kDwTY);
  for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int ty0 = (tile / tiles_x) * kDwTY, tx0 = (tile % tiles_x) * kDwTX;
    __syncthreads();
    for (int i = threadIdx.x; i < kDwHY * kDwHX * 64; i += blockDim.x) {
      const int pix = i >> 6, q = i & 63;
      const int iy = ty0 - 3 + pix / kDwHX, ix = tx0 - 3 + pix % kDwHX;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (iy >= 0 && iy < H && ix >= 0 && ix < W)
        v = reinterpret_cast<const float4*>(x + ((long long)iy * W + ix) * 256)[q];
      reinterpret_cast<float4*>(xs + pix * 256)[q] = v;
    }
    __syncthreads();
    float acc[4][8];
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[p][i] = 0.f;
    for (int ky = 0; ky < 7; ++ky) {
#pragma unroll
      for (int kx = 0; kx < 7; ++kx) {
        const float* wk = ws + (ky * 7 + kx) * 256 + c;
        const float4 w0 = *reinterpret_cast<const float4*>(wk);
        const float4 w1 = *reinterpret_cast<const float4*>(wk + 4);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float* xp = xs + ((ly + ky) * kDwHX + lx0 + p + kx) * 256 + c;
          const float4 a0 = *reinterpret_cast<const float4*>(xp);
          const float4 a1 = *reinterpret_cast<const float4*>(xp + 4);
          acc[p][0] = fmaf(a0.x, w0.x, acc[p][0]);
          acc[p][1] = fmaf(a0.y, w0.y, acc[p][1]);
          acc[p][2] = fmaf(a0.z, w0.z, acc[p][2]);
          acc[p][3] = fmaf(a0.w, w0.w, acc[p][3]);
          acc[p][4] = fmaf(a1.x, w1.x, acc[p][4]);
          acc[p][5] = fmaf(a1.y, w1.y, acc[p][5]);
          acc[p][6] = fmaf(a1.z, w1.z, acc[p][6]);
          acc[p][7] = fmaf(a1.w, w1.w, acc[p][7]);
        }
      }
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int py = ty0 + ly, px = tx0 + lx0 + p;
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc[p][i] += bb[i];
        s += acc[p][i];
      }
      const float mean = warp_sum(s) * (1.0f / 256);
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc[p][i] -= mean;
        q = fmaf(acc[p][i], acc[p][i], q);
      }
      const float rstd = rsqrtf(warp_sum(q) * (1.0f / 256) + eps);
      if (py < H && px < W) {
        uint4 o;
        __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          h[k] = __floats2half2_rn(acc[p][2 * k] * rstd * gg[2 * k] + be[2 * k],
                                   acc[p][2 * k + 1] * rstd * gg[2 * k + 1] + be[2 * k + 1]);
        *reinterpret_cast<uint4*>(y + ((long long)py * W + px) * 256 + c) = o;
      }
    }
  }
}

// Object absent (score <= 0, read from device memory): out[p][c] += emb[c] (no_obj_embed_spatial).
__global__ void add_if_absent_kernel(float* out, long long rows, int C, const float* emb, const float* score) {
  if (*score > 0.0f) return;
  const long long n = rows * C;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] += emb[i % C];
}

// Object pointer: the MLP output when the object score is > 0, else no_obj_ptr (sam3.cpp:9353-9390).
__global__ void select_ptr_kernel(const float* mlp, const float* no_obj, const float* score, int n, float* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = (score == nullptr || *score > 0.0f) ? mlp[i] : no_obj[i];
}

}  // namespace

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int bilinear_resize(const float* src, int sw, int sh, float* dst, int dw, int dh, int sigmoid_mode, float scale,
                    float bias, cudaStream_t st) {
  if (!src || !dst || sw < 2 || sh < 2 || dw <= 0 || dh <= 0) return -2;
  bilinear_kernel<<<me_grid((long long)dw * dh, 256), 256, 0, st>>>(src, sw, sh, dst, dw, dh, sigmoid_mode, scale,
                                                                    bias);
  return me_launch_ok();
}

int mask_ds_conv(const float* x, int Hi, int Wi, int cin, int cout, const float* w, const float* bias, const float* g,
                 const float* beta, float eps, float* y, cudaStream_t st) {
  if (!x || !w || !bias || !g || !beta || !y || Hi <= 0 || Wi <= 0) return -2;
  if (!al16(y)) return -11;
  const int Ho = (Hi + 1) / 2, Wo = (Wi + 1) / 2;
  const long long n = (long long)Ho * Wo;
  const int grid = me_grid(n, 128, 8);
  if (cin == 1 && cout == 4)
    ds_conv_kernel<1, 4><<<grid, 128, 0, st>>>(x, Hi, Wi, w, bias, g, beta, eps, y, Ho, Wo);
  else if (cin == 4 && cout == 16)
    ds_conv_kernel<4, 16><<<grid, 128, 0, st>>>(x, Hi, Wi, w, bias, g, beta, eps, y, Ho, Wo);
  else if (cin == 16 && cout == 64)
    ds_conv_kernel<16, 64><<<grid, 128, 0, st>>>(x, Hi, Wi, w, bias, g, beta, eps, y, Ho, Wo);
  else
    return -2;
  return me_launch_ok();
}

int im2col_s2(const float* x, int Hi, int Wi, int C, __half* col, cudaStream_t st) {
  if (!x || !col || C % 8 || Hi <= 0 || Wi <= 0) return -2;
  if (!al16(x) || !al16(col)) return -11;
  const int Ho = (Hi + 1) / 2, Wo = (Wi + 1) / 2;
  im2col_s2_kernel<<<me_grid((long long)Ho * Wo * 9 * (C / 8), 256), 256, 0, st>>>(x, Hi, Wi, C, Ho, Wo, col);
  return me_launch_ok();
}

int ln_gelu_rows(const float* x, long long rows, int C, const float* g, const float* beta, float eps, __half* y,
                 cudaStream_t st) {
  if (!x || !g || !beta || !y || rows <= 0) return -2;
  const int grid = me_grid(rows * 32, 256);
  if (C == 256) ln_gelu_rows_kernel<8><<<grid, 256, 0, st>>>(x, rows, g, beta, eps, y);
  else if (C == 64) ln_gelu_rows_kernel<2><<<grid, 256, 0, st>>>(x, rows, g, beta, eps, y);
  else return -2;
  return me_launch_ok();
}

int dwconv7_ln(const float* x, int H, int W, const float* w, const float* b, const float* g, const float* beta,
               float eps, __half* y, cudaStream_t st) {
  if (!x || !w || !b || !g || !beta || !y || H <= 0 || W <= 0) return -2;
  if (!al16(x) || !al16(w) || !al16(y)) return -11;
  if (kernel_setup(dwconv7_ln_kernel, kDwSmem) < 0) return -13;
  const long long tiles = (long long)((W + kDwTX - 1) / kDwTX) * ((H + kDwTY - 1) / kDwTY);
  const int grid = (int)(tiles < num_sms() ? tiles : num_sms());
  dwconv7_ln_kernel<<<grid, 256, kDwSmem, st>>>(x, H, W, w, b, g, beta, eps, y);
  return me_launch_ok();
}

int add_if_absent(float* out, long long rows, int C, const float* emb, const float* score, cudaStream_t st) {
  if (!out || !emb || !score || rows <= 0 || C <= 0) return -2;
  add_if_absent_kernel<<<me_grid(rows * C, 256), 256, 0, st>>>(out, rows, C, emb, score);
  return me_launch_ok();
}

int select_obj_ptr(const float* mlp, const float* no_obj, const float* score, int n, float* out, cudaStream_t st) {
  if (!mlp || !no_obj || !out || n <= 0) return -2;
  select_ptr_kernel<<<(n + 255) / 256, 256, 0, st>>>(mlp, no_obj, score, n, out);
  return me_launch_ok();
}

}  // namespace s3b
