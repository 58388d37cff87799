// .ggml model file parsing and device weight preparation (host, C++14).
//
// File format (sam3.cpp:3200-3344 loader, convert_sam3_to_ggml.py:160-240 and
// convert_sam2_to_ggml.py:206-318 writers): u32 magic, i32 version, i32 ftype,
// i32 n_tensors, the model's i32 hyper-parameters, then records
//   i32 n_dims, i32 name_len, i32 dtype, i32 ne[n_dims] (ggml order), name,
//   zero padding to a 32-byte file offset, raw data.
// Unlike sam3_load_tensors (sam3.cpp:3091-3194), tensors the encoder engine
// does not use are skipped instead of rejected, so full model files load.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <fstream>
#include <thread>

#include "engine.h"

namespace s3b {

static constexpr uint32_t kMagicSam3 = 0x73616D33;
static constexpr uint32_t kMagicSam2 = 0x73616D32;

int set_error(s3b_ctx* ctx, int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (ctx) ctx->last_error = buf;
  fprintf(stderr, "s3b: %s\n", buf);
  return code;
}

int check_device(s3b_ctx* ctx, const char* where) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(ctx, kErrCuda, "%s: %s", where, cudaGetErrorString(e));
  return kOk;
}

static float h2f(uint16_t h) {
  __half_raw r;
  r.x = h;
  return __half2float(__half(r));
}

// Host restatement of the block dequantisers (same values as the device kernel).
static void dequant_row_host(int dtype, const uint8_t* p, int64_t n, float* y) {
  const int64_t nb = n / 32;
  for (int64_t b = 0; b < nb; ++b) {
    if (dtype == QT_Q4_0) {
      const uint8_t* q = p + b * 18;
      uint16_t dh;
      memcpy(&dh, q, 2);
      const float d = h2f(dh);
      for (int j = 0; j < 16; ++j) {
        y[b * 32 + j] = (float)((int)(q[2 + j] & 0x0F) - 8) * d;
        y[b * 32 + j + 16] = (float)((int)(q[2 + j] >> 4) - 8) * d;
      }
    } else if (dtype == QT_Q4_1) {
      const uint8_t* q = p + b * 20;
      uint16_t dh, mh;
      memcpy(&dh, q, 2);
      memcpy(&mh, q + 2, 2);
      const float d = h2f(dh), m = h2f(mh);
      for (int j = 0; j < 16; ++j) {
        volatile float a = (float)(q[4 + j] & 0x0F) * d;
        volatile float c = (float)(q[4 + j] >> 4) * d;
        y[b * 32 + j] = a + m;
        y[b * 32 + j + 16] = c + m;
      }
    } else {
      const uint8_t* q = p + b * 34;
      uint16_t dh;
      memcpy(&dh, q, 2);
      const float d = h2f(dh);
      for (int j = 0; j < 32; ++j) y[b * 32 + j] = (float)((const int8_t*)(q + 2))[j] * d;
    }
  }
}

// Runs fn(begin, end) over disjoint parts of [0, n) on up to 32 host threads; one call when n is below
// two chunks of min_chunk. Load-time conversions are independent per element or row, so the result does
// not depend on the split.
template <typename F>
static void parallel_for(int64_t n, int64_t min_chunk, F fn) {
  unsigned nt = std::thread::hardware_concurrency();
  nt = std::max(1u, std::min(nt, 32u));
  const int64_t parts = std::min<int64_t>((int64_t)nt, n / std::max<int64_t>(min_chunk, 1));
  if (parts <= 1) {
    fn((int64_t)0, n);
    return;
  }
  // chunks whose thread could not be started (a thread or resource limit) run on this thread, so no
  // exception leaves the C ABI
  std::vector<std::thread> th;
  int64_t started = 0;
  try {
    for (; started < parts; ++started) {
      const int64_t c = started;
      th.emplace_back([&, c]() { fn(n * c / parts, n * (c + 1) / parts); });
    }
  } catch (...) {
  }
  for (int64_t c = started; c < parts; ++c) fn(n * c / parts, n * (c + 1) / parts);
  for (auto& x : th) x.join();
}

void tensor_to_f32(const FileTensor& t, std::vector<float>& out) {
  const int64_t n = t.nelements();
  out.resize(n);
  if (t.dtype == QT_F32) {
    memcpy(out.data(), t.data.data(), n * 4);
  } else if (t.dtype == QT_F16) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(t.data.data());
    parallel_for(n, 1 << 18, [&](int64_t b, int64_t e) {
      for (int64_t i = b; i < e; ++i) out[i] = h2f(h[i]);
    });
  } else {
    const int64_t rows = n / t.ne[0];
    const long long rb = qtype_row_bytes(t.dtype, t.ne[0]);
    parallel_for(rows, (1 << 18) / std::max<int64_t>(t.ne[0], 1) + 1, [&](int64_t b, int64_t e) {
      for (int64_t r = b; r < e; ++r)
        dequant_row_host(t.dtype, t.data.data() + r * rb, t.ne[0], out.data() + r * t.ne[0]);
    });
  }
}

static bool rd32(std::ifstream& f, int32_t& v) {
  f.read(reinterpret_cast<char*>(&v), 4);
  return !f.fail();
}

// Reads the hparam block that follows magic / version / ftype / n_tensors, in file order, through
// next(v) (false when the source is exhausted): sam3_load_hparams (sam3.cpp:1477-1520) for SAM 3,
// sam2_load_hparams (1564-1626) for SAM 2.
template <typename Next>
static int parse_hparams(bool sam2, Next next, HParams& hp, std::string& err) {
  bool ok = true;
  int32_t v = 0;
  auto rd = [&](int& dst) {
    if (!next(v)) {
      ok = false;
      v = 0;
    }
    dst = v;
  };
  if (!sam2) {
    // sam3_load_hparams (sam3.cpp:1477-1520)
    hp.is_sam2 = 0;
    int dummy;
    rd(hp.img_size);
    rd(hp.patch_size);
    rd(hp.vit_embed_dim);
    rd(hp.vit_depth);
    rd(hp.vit_num_heads);
    int mlp_ratio_x1000;
    rd(mlp_ratio_x1000);
    hp.vit_mlp_dim = (int)(hp.vit_embed_dim * (mlp_ratio_x1000 / 1000.0f));
    rd(hp.vit_window_size);
    rd(hp.n_global_attn);
    if (hp.n_global_attn < 0 || hp.n_global_attn > 64) {
      err = "corrupt global-attention count";
      return kErrFormat;
    }
    for (int i = 0; i < hp.n_global_attn; ++i) {
      int g;
      rd(g);
      if (i < 4) hp.global_attn_idx[i] = g;
    }
    for (int i = 0; i < 6; ++i) rd(dummy);  // text_width..text_out_dim
    rd(hp.neck_dim);
    for (int i = 0; i < 10; ++i) rd(dummy);  // fenc (3), ddec (4), geom, presence, geom queries
    for (int i = 0; i < 4; ++i) rd(dummy);   // sam decoder
    rd(hp.mem_out_dim);
    rd(hp.mem_attn_layers);
    rd(hp.num_maskmem);
    rd(hp.max_obj_ptrs);
    rd(dummy);  // n_amb_experts
    rd(hp.visual_only);
  } else {
    // sam2_load_hparams (sam3.cpp:1564-1626)
    hp.is_sam2 = 1;
    int dummy;
    rd(hp.img_size);
    rd(hp.backbone_type);
    rd(hp.hiera_embed_dim);
    rd(hp.hiera_num_heads);
    rd(hp.hiera_num_stages);
    for (int i = 0; i < 4; ++i) rd(hp.hiera_stages[i]);
    rd(hp.hiera_global_n);
    for (int i = 0; i < 8; ++i) rd(hp.hiera_global_idx[i]);
    rd(hp.hiera_q_pool);
    for (int i = 0; i < 4; ++i) rd(hp.hiera_window_spec[i]);
    rd(hp.bkg_h);
    rd(hp.bkg_w);
    rd(hp.scalp);
    rd(hp.neck_dim);
    rd(hp.fpn_top_down_n);
    for (int i = 0; i < 4; ++i) rd(hp.fpn_top_down_levels[i]);
    for (int i = 0; i < 4; ++i) rd(dummy);  // sam decoder
    rd(hp.mem_out_dim);
    rd(hp.mem_attn_layers);
    rd(hp.num_maskmem);
    rd(hp.max_obj_ptrs);
    rd(hp.sigmoid_scale_x100);
    rd(hp.sigmoid_bias_x100);
    for (int i = 0; i < 15; ++i) rd(hp.trk_flags[i]);
    if (ok && hp.backbone_type != 1) {
      err = "only the Hiera backbone (backbone_type 1) is supported by the encoder engine";
      return kErrUnsupported;
    }
  }
  if (!ok) {
    err = "truncated header";
    return kErrFormat;
  }
  return kOk;
}

int read_ggml_file(const std::string& path, HParams& hp, std::vector<FileTensor>& tensors, std::string& err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    err = "cannot open " + path;
    return kErrIO;
  }
  uint32_t magic = 0;
  f.read(reinterpret_cast<char*>(&magic), 4);
  int32_t version = 0, ftype = 0, n_tensors = 0;
  rd32(f, version);
  rd32(f, ftype);
  rd32(f, n_tensors);
  if (f.fail() || (magic != kMagicSam3 && magic != kMagicSam2)) {
    err = "bad magic in " + path;
    return kErrFormat;
  }
  hp.ftype = ftype;
  {
    const int rc = parse_hparams(magic == kMagicSam2, [&](int32_t& v) { return rd32(f, v); }, hp, err);
    if (rc) return rc;
  }
  if (f.fail()) {
    err = "truncated header";
    return kErrFormat;
  }
  tensors.clear();
  tensors.reserve(n_tensors);
  for (int t = 0; t < n_tensors; ++t) {
    int32_t n_dims, name_len, dtype;
    if (!rd32(f, n_dims) || !rd32(f, name_len) || !rd32(f, dtype)) {
      err = "truncated tensor header";
      return kErrFormat;
    }
    if (n_dims < 1 || n_dims > 4 || name_len <= 0 || name_len > 512) {
      err = "corrupt tensor header";
      return kErrFormat;
    }
    FileTensor ft;
    ft.n_dims = n_dims;
    ft.dtype = dtype;
    for (int i = 0; i < n_dims; ++i) {
      int32_t d;
      rd32(f, d);
      if (d <= 0) {
        err = "corrupt tensor shape";
        return kErrFormat;
      }
      ft.ne[i] = d;
    }
    ft.name.resize(name_len);
    f.read(&ft.name[0], name_len);
    const size_t pos = (size_t)f.tellg();
    const size_t pad = (32 - pos % 32) % 32;
    if (pad) f.seekg(pad, std::ios::cur);
    int64_t bytes;
    if (dtype == QT_F32 || dtype == QT_F16) {
      bytes = ft.nelements() * (dtype == QT_F16 ? 2 : 4);
    } else if (dtype == QT_Q4_0 || dtype == QT_Q4_1 || dtype == QT_Q8_0) {
      if (ft.ne[0] % 32) {
        err = "quantised tensor with ne0 % 32 != 0: " + ft.name;
        return kErrFormat;
      }
      bytes = qtype_row_bytes(dtype, ft.ne[0]) * (ft.nelements() / ft.ne[0]);
    } else {
      err = "unsupported dtype in " + ft.name;
      return kErrFormat;
    }
    ft.data.resize(bytes);
    f.read(reinterpret_cast<char*>(ft.data.data()), bytes);
    if (f.fail()) {
      err = "failed to read tensor " + ft.name;
      return kErrIO;
    }
    tensors.push_back(std::move(ft));
  }
  return kOk;
}

// ---------------------------------------------------------------- uploads
static std::shared_ptr<DevBuf> upload_bytes(s3b_ctx* ctx, const void* src, size_t bytes, int* rc) {
  auto b = std::make_shared<DevBuf>();
  if (b->reserve(bytes) != 0) {
    *rc = set_error(ctx, kErrOOM, "cudaMalloc(%zu) failed", bytes);
    return nullptr;
  }
  if ((*rc = upload_sync(ctx, b->p, src, bytes))) return nullptr;
  ctx->model.device_bytes += bytes;
  return b;
}

static Vec upload_vec(s3b_ctx* ctx, const FileTensor& t, int* rc) {
  std::vector<float> f;
  tensor_to_f32(t, f);
  Vec v;
  v.n = (int)f.size();
  v.d = upload_bytes(ctx, f.data(), f.size() * 4, rc);
  return v;
}

// Uploads a GEMM B operand given as f32 [N][K] (row-major), padded to Kpad.
static int upload_b_operand(s3b_ctx* ctx, const std::vector<float>& w, int N, int K, int kpad_to, Linear& L) {
  L.N = N;
  L.K = K;
  L.Kpad = ((K + kpad_to - 1) / kpad_to) * kpad_to;
  std::vector<__half> h((size_t)N * L.Kpad, __float2half_rn(0.f));
  parallel_for(N, (1 << 18) / std::max(K, 1) + 1, [&](int64_t b, int64_t e) {
    for (int64_t n = b; n < e; ++n)
      for (int k = 0; k < K; ++k) h[(size_t)n * L.Kpad + k] = __float2half_rn(w[(size_t)n * K + k]);
  });
  int rc = 0;
  L.w = upload_bytes(ctx, h.data(), h.size() * 2, &rc);
  return rc;
}

int upload_linear(s3b_ctx* ctx, const FileTensor& t, const FileTensor* bias, Linear& L, int kpad_to, int k_dims) {
  // ggml weight [K, N] (ne0 = K contiguous) == row-major [N][K]; a conv kernel
  // [kW, kH, Cin, Cout] folds its first k_dims = 3 dims into K.
  int64_t K64 = 1;
  for (int i = 0; i < k_dims && i < 4; ++i) K64 *= t.ne[i];
  const int K = (int)K64;
  const int N = (int)(t.nelements() / K64);
  int rc = 0;
  L.file_dtype = t.dtype;
  if (ctx->weights_quantised && k_dims == 1 && (t.dtype == QT_Q4_0 || t.dtype == QT_Q8_0) && K % 32 == 0 &&
      N % 8 == 0) {
    // block form on the device: the file's rows go up once and are split into the value and
    // scale planes the GEMM's TMA loads read; no f16 copy of the weight exists
    L.N = N;
    L.K = K;
    L.Kpad = K;
    L.qtype = t.dtype;
    std::shared_ptr<DevBuf> raw = upload_bytes(ctx, t.data.data(), t.data.size(), &rc);
    if (rc) return rc;
    L.qv = std::make_shared<DevBuf>();
    L.qs = std::make_shared<DevBuf>();
    const size_t vbytes = (size_t)N * (t.dtype == QT_Q4_0 ? K / 2 : K);
    if (L.qv->reserve(vbytes) || L.qs->reserve((size_t)N * (K / 32) * 2))
      return set_error(ctx, kErrOOM, "out of device memory for %s", t.name.c_str());
    if (repack_q_rows(raw->p, t.dtype, N, K, L.qv->p, L.qs->as<__half>(), ctx->stream))
      return set_error(ctx, kErrCuda, "repack of %s failed", t.name.c_str());
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess)
      return set_error(ctx, kErrCuda, "repack of %s failed", t.name.c_str());
    ctx->model.device_bytes += vbytes + (size_t)N * (K / 32) * 2;
    ctx->model.qstage_elems = std::max(ctx->model.qstage_elems, (size_t)N * K);
    ctx->model.device_bytes -= t.data.size();  // the uploaded rows are released here
  } else {
    std::vector<float> w;
    tensor_to_f32(t, w);
    rc = upload_b_operand(ctx, w, N, K, kpad_to, L);
    if (rc) return rc;
    if (t.dtype == QT_Q4_0 || t.dtype == QT_Q4_1 || t.dtype == QT_Q8_0) {
      L.raw = upload_bytes(ctx, t.data.data(), t.data.size(), &rc);
      if (rc) return rc;
    }
  }
  if (bias) {
    std::vector<float> b;
    tensor_to_f32(*bias, b);
    if ((int)b.size() != N) return set_error(ctx, kErrFormat, "bias size mismatch for %s", t.name.c_str());
    L.b = upload_bytes(ctx, b.data(), b.size() * 4, &rc);
  }
  return rc;
}

// ConvTranspose2d k=2 s=2, ggml [2, 2, Cout, Cin] -> B[(ky*2+kx)*Cout + co][ci].
// ConvTranspose2d 2x2 stride 2, ggml [2, 2, Cout, Cin] -> rows [(ky*2 + kx)*Cout + co][ci].
static void deconv_rows(const FileTensor& t, std::vector<float>& r) {
  const int Cout = (int)t.ne[2], Cin = (int)t.ne[3];
  std::vector<float> w;
  r.assign((size_t)4 * Cout * Cin, 0.f);
  tensor_to_f32(t, w);
  for (int ci = 0; ci < Cin; ++ci)
    for (int co = 0; co < Cout; ++co)
      for (int ky = 0; ky < 2; ++ky)
        for (int kx = 0; kx < 2; ++kx)
          r[(size_t)((ky * 2 + kx) * Cout + co) * Cin + ci] = w[(size_t)kx + 2 * (ky + 2 * (co + (size_t)Cout * ci))];
}

// A 1x1 conv (c [Co][Cd], bias bc) applied to the output of a 2x2 deconvolution (rows d [4*Cd][Cin],
// bias bd) is one deconvolution: rows f[p*Co + o] = sum_c c[o][c] d[p*Cd + c], bias
// bf[o] = bc[o] + sum_c c[o][c] bd[c] (the deconvolution bias is the same at every kernel position).
// Computed in f32 on the host threads at load.
static void fold_1x1_into_deconv(const std::vector<float>& d, const std::vector<float>& bd, int Cd, int Cin,
                                 const std::vector<float>& c, const std::vector<float>& bc, int Co,
                                 std::vector<float>& f, std::vector<float>& bf) {
  f.assign((size_t)4 * Co * Cin, 0.f);
  bf.assign(Co, 0.f);
  for (int o = 0; o < Co; ++o) {
    double acc = bc[o];
    for (int k = 0; k < Cd; ++k) acc += (double)c[(size_t)o * Cd + k] * bd[k];
    bf[o] = (float)acc;
  }
  const int n_rows = 4 * Co;
  parallel_for(n_rows, 1, [&](int64_t b, int64_t e) {
    for (int64_t row = b; row < e; ++row) {
      const int p = (int)(row / Co), o = (int)(row % Co);
      float* out = f.data() + (size_t)row * Cin;
      for (int k = 0; k < Cd; ++k) {
        const float s = c[(size_t)o * Cd + k];
        const float* in = d.data() + (size_t)(p * Cd + k) * Cin;
        for (int i = 0; i < Cin; ++i) out[i] += s * in[i];
      }
    }
  });
}

static int upload_deconv(s3b_ctx* ctx, const FileTensor& t, const FileTensor& bias, Linear& L) {
  const int Cout = (int)t.ne[2], Cin = (int)t.ne[3];
  std::vector<float> r;
  deconv_rows(t, r);
  int rc = upload_b_operand(ctx, r, 4 * Cout, Cin, 8, L);
  if (rc) return rc;
  std::vector<float> b;
  tensor_to_f32(bias, b);
  L.b = upload_bytes(ctx, b.data(), b.size() * 4, &rc);
  L.file_dtype = t.dtype;
  return rc;
}

// Conv2d kxk, ggml [k, k, Cin, Cout] -> rows [co][(ky*k + kx)*Cin + ci] (channel-last im2col order).
static void conv_rows(const FileTensor& t, std::vector<float>& r) {
  const int k = (int)t.ne[0], Cin = (int)t.ne[2], Cout = (int)t.ne[3];
  std::vector<float> w;
  r.assign((size_t)Cout * k * k * Cin, 0.f);
  tensor_to_f32(t, w);
  for (int co = 0; co < Cout; ++co)
    for (int ci = 0; ci < Cin; ++ci)
      for (int ky = 0; ky < k; ++ky)
        for (int kx = 0; kx < k; ++kx)
          r[(size_t)co * k * k * Cin + (size_t)(ky * k + kx) * Cin + ci] =
              w[(size_t)kx + k * (ky + (size_t)k * (ci + (size_t)Cin * co))];
}

static int upload_conv_cl(s3b_ctx* ctx, const FileTensor& t, const FileTensor& bias, Linear& L) {
  const int k = (int)t.ne[0], Cin = (int)t.ne[2], Cout = (int)t.ne[3];
  std::vector<float> r;
  conv_rows(t, r);
  int rc = upload_b_operand(ctx, r, Cout, k * k * Cin, 8, L);
  if (rc) return rc;
  std::vector<float> b;
  tensor_to_f32(bias, b);
  L.b = upload_bytes(ctx, b.data(), b.size() * 4, &rc);
  L.file_dtype = t.dtype;
  return rc;
}

// ---------------------------------------------------------------- model build
namespace {
struct Index {
  std::map<std::string, const FileTensor*> m;
  const FileTensor* get(const std::string& n) const {
    auto it = m.find(n);
    return it == m.end() ? nullptr : it->second;
  }
};
}  // namespace

#define NEED(var, name)                                                                   \
  const FileTensor* var = idx.get(name);                                                  \
  if (!var) return set_error(ctx, kErrFormat, "missing tensor '%s'", std::string(name).c_str());

// The last deconvolution of scales 0 and 1 is followed by the 1x1 conv with nothing in between, so
// the two are uploaded as one deconvolution (fold_1x1_into_deconv); scales 2 and 3 keep the 1x1 conv.
static int load_neck(s3b_ctx* ctx, const Index& idx, const std::string& pfx, NeckScale* sc) {
  int rc;
  auto fold = [&](const FileTensor& dw, const FileTensor& db, const std::string& conv, Linear& L) -> int {
    NEED(cw, conv + ".conv_1x1.weight");
    NEED(cb, conv + ".conv_1x1.bias");
    const int Cd = (int)dw.ne[2], Cin = (int)dw.ne[3], Co = (int)cw->ne[3];
    if ((int)cw->ne[2] != Cd || cw->ne[0] != 1 || cw->ne[1] != 1)
      return set_error(ctx, kErrFormat, "%s: 1x1 conv does not follow the deconvolution", conv.c_str());
    std::vector<float> d, bd, c, bc, f, bf;
    deconv_rows(dw, d);
    tensor_to_f32(db, bd);
    conv_rows(*cw, c);
    tensor_to_f32(*cb, bc);
    if ((int)bd.size() != Cd || (int)bc.size() != Co) return set_error(ctx, kErrFormat, "%s: bias size", conv.c_str());
    fold_1x1_into_deconv(d, bd, Cd, Cin, c, bc, Co, f, bf);
    int r = upload_b_operand(ctx, f, 4 * Co, Cin, 8, L);
    if (r) return r;
    L.b = upload_bytes(ctx, bf.data(), bf.size() * 4, &r);
    L.file_dtype = dw.dtype;
    return r;
  };
  {
    NEED(w0, pfx + "0.dconv_2x2_0.weight");
    NEED(b0, pfx + "0.dconv_2x2_0.bias");
    NEED(w1, pfx + "0.dconv_2x2_1.weight");
    NEED(b1, pfx + "0.dconv_2x2_1.bias");
    if ((rc = upload_deconv(ctx, *w0, *b0, sc[0].dc1))) return rc;
    if ((rc = fold(*w1, *b1, pfx + "0", sc[0].dcf))) return rc;
  }
  {
    NEED(w, pfx + "1.dconv_2x2.weight");
    NEED(b, pfx + "1.dconv_2x2.bias");
    if ((rc = fold(*w, *b, pfx + "1", sc[1].dcf))) return rc;
  }
  for (int s = 0; s < 4; ++s) {
    const std::string p = pfx + std::to_string(s);
    NEED(w3, p + ".conv_3x3.weight");
    NEED(b3, p + ".conv_3x3.bias");
    if (s >= 2) {
      NEED(w1, p + ".conv_1x1.weight");
      NEED(b1, p + ".conv_1x1.bias");
      if ((rc = upload_conv_cl(ctx, *w1, *b1, sc[s].c1))) return rc;
    }
    if ((rc = upload_conv_cl(ctx, *w3, *b3, sc[s].c3))) return rc;
  }
  return kOk;
}

static int load_mem_attn(s3b_ctx* ctx, const Index& idx) {
  Model& M = ctx->model;
  const HParams& hp = M.hp;
  if (!idx.get("mem_attn.layers.0.sa.q_proj.weight")) return kOk;  // optional
  int rc = 0;
  M.mem.resize(hp.mem_attn_layers);
  for (int i = 0; i < hp.mem_attn_layers; ++i) {
    MemAttnLayer& L = M.mem[i];
    const std::string p = "mem_attn.layers." + std::to_string(i);
    NEED(n1w, p + ".norm1.weight");
    NEED(n1b, p + ".norm1.bias");
    NEED(n2w, p + ".norm2.weight");
    NEED(n2b, p + ".norm2.bias");
    NEED(n3w, p + ".norm3.weight");
    NEED(n3b, p + ".norm3.bias");
    L.n1w = upload_vec(ctx, *n1w, &rc);
    L.n1b = upload_vec(ctx, *n1b, &rc);
    L.n2w = upload_vec(ctx, *n2w, &rc);
    L.n2b = upload_vec(ctx, *n2b, &rc);
    L.n3w = upload_vec(ctx, *n3w, &rc);
    L.n3b = upload_vec(ctx, *n3b, &rc);
    // self-attention q/k/v concatenated into one [3*D][D] GEMM
    {
      NEED(qw, p + ".sa.q_proj.weight");
      NEED(kw, p + ".sa.k_proj.weight");
      NEED(vw, p + ".sa.v_proj.weight");
      NEED(qb, p + ".sa.q_proj.bias");
      NEED(kb, p + ".sa.k_proj.bias");
      NEED(vb, p + ".sa.v_proj.bias");
      const int D = (int)qw->ne[0];
      if (qw->dtype == kw->dtype && qw->dtype == vw->dtype && qw->ne[0] == kw->ne[0] && qw->ne[0] == vw->ne[0] &&
          qw->ne[1] == D && kw->ne[1] == D && vw->ne[1] == D) {
        // the three weights' rows, concatenated in their stored form (f32 / f16 / block rows)
        FileTensor cat;
        cat.name = p + ".sa.qkv_proj.weight";
        cat.dtype = qw->dtype;
        cat.n_dims = 2;
        cat.ne[0] = D;
        cat.ne[1] = 3 * D;
        cat.data.reserve(qw->data.size() * 3);
        for (const FileTensor* t : {qw, kw, vw}) cat.data.insert(cat.data.end(), t->data.begin(), t->data.end());
        if ((rc = upload_linear(ctx, cat, nullptr, L.sa_qkv))) return rc;
      } else {
        std::vector<float> a, b, c, w;
        tensor_to_f32(*qw, a);
        tensor_to_f32(*kw, b);
        tensor_to_f32(*vw, c);
        w.reserve(a.size() * 3);
        w.insert(w.end(), a.begin(), a.end());
        w.insert(w.end(), b.begin(), b.end());
        w.insert(w.end(), c.begin(), c.end());
        if ((rc = upload_b_operand(ctx, w, 3 * D, D, 8, L.sa_qkv))) return rc;
      }
      std::vector<float> ba, bb, bc;
      tensor_to_f32(*qb, ba);
      tensor_to_f32(*kb, bb);
      tensor_to_f32(*vb, bc);
      ba.insert(ba.end(), bb.begin(), bb.end());
      ba.insert(ba.end(), bc.begin(), bc.end());
      L.sa_qkv.b = upload_bytes(ctx, ba.data(), ba.size() * 4, &rc);
    }
    {
      NEED(w, p + ".sa.out_proj.weight");
      NEED(b, p + ".sa.out_proj.bias");
      if ((rc = upload_linear(ctx, *w, b, L.sa_out))) return rc;
    }
    {
      NEED(w, p + ".ca.q_proj.weight");
      NEED(b, p + ".ca.q_proj.bias");
      if ((rc = upload_linear(ctx, *w, b, L.ca_q))) return rc;
    }
    {
      NEED(w, p + ".ca.k_proj.weight");
      NEED(b, p + ".ca.k_proj.bias");
      if ((rc = upload_linear(ctx, *w, b, L.ca_k))) return rc;
    }
    {
      NEED(w, p + ".ca.v_proj.weight");
      NEED(b, p + ".ca.v_proj.bias");
      if ((rc = upload_linear(ctx, *w, b, L.ca_v))) return rc;
    }
    {
      NEED(w, p + ".ca.out_proj.weight");
      NEED(b, p + ".ca.out_proj.bias");
      if ((rc = upload_linear(ctx, *w, b, L.ca_out))) return rc;
    }
    {
      NEED(w, p + ".linear1.weight");
      NEED(b, p + ".linear1.bias");
      if ((rc = upload_linear(ctx, *w, b, L.fc1))) return rc;
    }
    {
      NEED(w, p + ".linear2.weight");
      NEED(b, p + ".linear2.bias");
      if ((rc = upload_linear(ctx, *w, b, L.fc2))) return rc;
    }
  }
  NEED(nw, "mem_attn.norm.weight");
  NEED(nb, "mem_attn.norm.bias");
  M.mem_norm_w = upload_vec(ctx, *nw, &rc);
  M.mem_norm_b = upload_vec(ctx, *nb, &rc);
  if (const FileTensor* t = idx.get("mem_enc.tpos_enc")) tensor_to_f32(*t, M.maskmem_tpos);
  if (const FileTensor* t = idx.get("obj_ptr_tpos_proj.weight")) tensor_to_f32(*t, M.obj_ptr_tpos_w);
  if (const FileTensor* t = idx.get("obj_ptr_tpos_proj.bias")) tensor_to_f32(*t, M.obj_ptr_tpos_b);
  M.has_mem_attn = true;
  return rc;
}

// SAM prompt encoder + mask decoder weights (sam3.cpp:1848-1966; optional: files without them load the
// encoder path alone). Every linear and 1x1 weight is dequantised to f16 at load whatever the file's type:
// the decoder is a few MB and its token-side layers read their weights with plain loads.
static int load_sam_dec(s3b_ctx* ctx, const Index& idx) {
  // dense PE grids cached for the previous model's Gaussian matrix
  for (auto it = ctx->ws.begin(); it != ctx->ws.end();)
    it = it->first.compare(0, 7, "dec_pe_") == 0 ? ctx->ws.erase(it) : std::next(it);
  if (!idx.get("sam_dec.iou_token.weight")) return kOk;
  SamDecoder& d = ctx->model.dec;
  d = SamDecoder();
  const int saved_q = ctx->weights_quantised;
  ctx->weights_quantised = 0;
  struct Restore {
    s3b_ctx* c;
    int v;
    ~Restore() { c->weights_quantised = v; }
  } restore{ctx, saved_q};
  int rc = 0;
  auto lin = [&](const std::string& p, Linear& L, int k_dims = 1) -> int {
    NEED(w, p + ".weight");
    NEED(b, p + ".bias");
    return upload_linear(ctx, *w, b, L, 8, k_dims);
  };
  auto vec = [&](const std::string& n, Vec& v) -> int {
    NEED(t, n);
    v = upload_vec(ctx, *t, &rc);
    return rc;
  };
  auto host = [&](const std::string& n, std::vector<float>& v, size_t want) -> int {
    NEED(t, n);
    tensor_to_f32(*t, v);
    if (want && v.size() != want) return set_error(ctx, kErrFormat, "%s: %zu values, expected %zu", n.c_str(), v.size(), want);
    return kOk;
  };
  NEED(mt, "sam_dec.mask_tokens.weight");
  d.D = (int)mt->ne[0];
  d.n_mask = (int)mt->ne[1];
  const int D = d.D;
  if (D != 256 || d.n_mask != 4) return set_error(ctx, kErrFormat, "mask decoder: D %d / %d mask tokens unsupported", D, d.n_mask);
  d.has_obj = idx.get("sam_dec.obj_score_token.weight") != nullptr;
  if ((rc = host("sam_pe.pe_gaussian", d.pe_gauss, (size_t)D))) return rc;
  for (int i = 0; i < 4; ++i)
    if ((rc = host("sam_pe.point_embeddings." + std::to_string(i) + ".weight", d.point_emb[i], D))) return rc;
  if ((rc = host("sam_pe.not_a_point_embed.weight", d.not_a_point, D))) return rc;
  if ((rc = host("sam_pe.no_mask_embed.weight", d.no_mask, D))) return rc;
  if (idx.get("no_mem_embed")) {
    if ((rc = host("no_mem_embed", d.no_mem, D))) return rc;
  } else {
    d.no_mem.assign(D, 0.f);
  }
  {
    // output tokens in the decoder's order: [obj_score?], iou, mask tokens (sam3.cpp:10575-10590)
    std::vector<float> tok, t;
    if (d.has_obj) {
      if ((rc = host("sam_dec.obj_score_token.weight", t, D))) return rc;
      tok.insert(tok.end(), t.begin(), t.end());
    }
    if ((rc = host("sam_dec.iou_token.weight", t, D))) return rc;
    tok.insert(tok.end(), t.begin(), t.end());
    if ((rc = host("sam_dec.mask_tokens.weight", t, (size_t)D * d.n_mask))) return rc;
    tok.insert(tok.end(), t.begin(), t.end());
    d.tokens = upload_bytes(ctx, tok.data(), tok.size() * 4, &rc);
    if (rc) return rc;
    d.d_no_mask.n = d.d_no_mem.n = d.d_not_a_point.n = D;
    d.d_no_mask.d = upload_bytes(ctx, d.no_mask.data(), D * 4, &rc);
    if (!rc) d.d_no_mem.d = upload_bytes(ctx, d.no_mem.data(), D * 4, &rc);
    if (!rc) d.d_not_a_point.d = upload_bytes(ctx, d.not_a_point.data(), D * 4, &rc);
    if (rc) return rc;
  }
  int depth = 0;
  while (idx.get("sam_dec.twoway." + std::to_string(depth) + ".norm1.weight")) ++depth;
  if (depth == 0) return set_error(ctx, kErrFormat, "mask decoder without TwoWay blocks");
  d.blocks.resize(depth);
  for (int i = 0; i < depth; ++i) {
    SamTwoWay& B = d.blocks[i];
    const std::string p = "sam_dec.twoway." + std::to_string(i);
    if ((rc = lin(p + ".sa.q_proj", B.sa_q)) || (rc = lin(p + ".sa.k_proj", B.sa_k)) ||
        (rc = lin(p + ".sa.v_proj", B.sa_v)) || (rc = lin(p + ".sa.out_proj", B.sa_out)) ||
        (rc = lin(p + ".cross_attn_token_to_image.q_proj", B.t2i_q)) ||
        (rc = lin(p + ".cross_attn_token_to_image.v_proj", B.t2i_v)) ||
        (rc = lin(p + ".cross_attn_token_to_image.out_proj", B.t2i_out)) ||
        (rc = lin(p + ".cross_attn_image_to_token.k_proj", B.i2t_k)) ||
        (rc = lin(p + ".cross_attn_image_to_token.v_proj", B.i2t_v)) ||
        (rc = lin(p + ".cross_attn_image_to_token.out_proj", B.i2t_out)) || (rc = lin(p + ".mlp.lin1", B.mlp1)) ||
        (rc = lin(p + ".mlp.lin2", B.mlp2)))
      return rc;
    {
      // the two image-side projections of keys + key_pe share one GEMM: rows [t2i k ; i2t q]
      NEED(kw, p + ".cross_attn_token_to_image.k_proj.weight");
      NEED(kb, p + ".cross_attn_token_to_image.k_proj.bias");
      NEED(qw, p + ".cross_attn_image_to_token.q_proj.weight");
      NEED(qb, p + ".cross_attn_image_to_token.q_proj.bias");
      std::vector<float> a, b, ba, bb;
      tensor_to_f32(*kw, a);
      tensor_to_f32(*qw, b);
      tensor_to_f32(*kb, ba);
      tensor_to_f32(*qb, bb);
      const int K = (int)kw->ne[0];
      if (qw->ne[0] != K || (int)ba.size() * K != (int)a.size() || (int)bb.size() * K != (int)b.size())
        return set_error(ctx, kErrFormat, "%s: cross-attention projection shapes", p.c_str());
      const int N = (int)(ba.size() + bb.size());
      a.insert(a.end(), b.begin(), b.end());
      ba.insert(ba.end(), bb.begin(), bb.end());
      if ((rc = upload_b_operand(ctx, a, N, K, 8, B.kq))) return rc;
      B.kq.b = upload_bytes(ctx, ba.data(), ba.size() * 4, &rc);
      if (rc) return rc;
    }
    if ((rc = vec(p + ".norm1.weight", B.n1w)) || (rc = vec(p + ".norm1.bias", B.n1b)) ||
        (rc = vec(p + ".norm2.weight", B.n2w)) || (rc = vec(p + ".norm2.bias", B.n2b)) ||
        (rc = vec(p + ".norm3.weight", B.n3w)) || (rc = vec(p + ".norm3.bias", B.n3b)) ||
        (rc = vec(p + ".norm4.weight", B.n4w)) || (rc = vec(p + ".norm4.bias", B.n4b)))
      return rc;
    if (B.sa_q.N != D || B.t2i_q.N != 128 || B.kq.N != 256 || B.t2i_v.N != 128 || B.i2t_k.N != 128 ||
        B.i2t_out.K != 128 || B.mlp2.N != D)
      return set_error(ctx, kErrFormat, "%s: unsupported attention dims", p.c_str());
  }
  if ((rc = lin("sam_dec.final_attn.q_proj", d.fin_q)) || (rc = lin("sam_dec.final_attn.k_proj", d.fin_k)) ||
      (rc = lin("sam_dec.final_attn.v_proj", d.fin_v)) || (rc = lin("sam_dec.final_attn.out_proj", d.fin_out)) ||
      (rc = vec("sam_dec.final_norm.weight", d.fin_nw)) || (rc = vec("sam_dec.final_norm.bias", d.fin_nb)))
    return rc;
  {
    NEED(w0, "sam_dec.upscale.0.weight");
    NEED(b0, "sam_dec.upscale.0.bias");
    NEED(w3, "sam_dec.upscale.3.weight");
    NEED(b3, "sam_dec.upscale.3.bias");
    if ((rc = upload_deconv(ctx, *w0, *b0, d.up1)) || (rc = upload_deconv(ctx, *w3, *b3, d.up2))) return rc;
    if ((rc = vec("sam_dec.upscale.1.weight", d.up1_nw)) || (rc = vec("sam_dec.upscale.1.bias", d.up1_nb))) return rc;
    if ((rc = lin("sam_dec.conv_s0", d.conv_s0, 3)) || (rc = lin("sam_dec.conv_s1", d.conv_s1, 3))) return rc;
    if (d.up1.N != 4 * 64 || d.up1.K != D || d.up2.N != 4 * 32 || d.up2.K != 64 || d.conv_s0.N != 32 ||
        d.conv_s0.K != D || d.conv_s1.N != 64 || d.conv_s1.K != D || d.up1_nw.n != 64)
      return set_error(ctx, kErrFormat, "mask decoder: unsupported upscaling shapes");
  }
  d.hyper.resize((size_t)d.n_mask * 3);
  for (int m = 0; m < d.n_mask; ++m)
    for (int j = 0; j < 3; ++j)
      if ((rc = lin("sam_dec.hyper." + std::to_string(m) + ".layers." + std::to_string(j), d.hyper[m * 3 + j])))
        return rc;
  for (int j = 0; j < 3; ++j) {
    if ((rc = lin("sam_dec.iou_prediction_head.layers." + std::to_string(j), d.iou[j]))) return rc;
    if (d.has_obj && (rc = lin("sam_dec.pred_obj_score_head.layers." + std::to_string(j), d.obj[j]))) return rc;
  }
  if (d.hyper[2].N != 32 || d.iou[2].N != d.n_mask) return set_error(ctx, kErrFormat, "mask decoder: head shapes");
  d.loaded = true;
  return kOk;
}

// Memory encoder + object-pointer MLP weights (optional). The downsampler's narrow stages keep f32
// copies of their (f16-stored) weights for the direct convolution kernels; the CXBlocks' layer scale
// gamma is multiplied into pwconv2's rows and bias (gamma (W t + b) = (gamma W) t + gamma b), rounded
// to f16 once.
static int load_mem_enc(s3b_ctx* ctx, const Index& idx) {
  if (!idx.get("mem_enc.ds.0.weight") || !idx.get("obj_ptr_proj.layers.0.weight")) return kOk;
  MemEncoder& E = ctx->model.menc;
  E = MemEncoder();
  const int saved_q = ctx->weights_quantised;
  ctx->weights_quantised = 0;
  struct Restore {
    s3b_ctx* c;
    int v;
    ~Restore() { c->weights_quantised = v; }
  } restore{ctx, saved_q};
  int rc = 0;
  auto vec = [&](const std::string& n, Vec& v) -> int {
    NEED(t, n);
    v = upload_vec(ctx, *t, &rc);
    return rc;
  };
  const int ch[5] = {1, 4, 16, 64, 256};
  const int conv_id[4] = {0, 3, 6, 9}, norm_id[4] = {1, 4, 7, 10};
  for (int s = 0; s < 4; ++s) {
    const std::string c = "mem_enc.ds." + std::to_string(conv_id[s]), nm = "mem_enc.ds." + std::to_string(norm_id[s]);
    NEED(w, c + ".weight");
    NEED(b, c + ".bias");
    if (w->ne[0] != 3 || w->ne[1] != 3 || w->ne[2] != ch[s] || w->ne[3] != ch[s + 1])
      return set_error(ctx, kErrFormat, "%s: unexpected shape", c.c_str());
    if ((rc = vec(nm + ".weight", E.ds_nw[s])) || (rc = vec(nm + ".bias", E.ds_nb[s]))) return rc;
    if (s < 3) {
      // ggml [3, 3, cin, cout] -> [ky*3 + kx][ci][co]
      std::vector<float> f, r((size_t)9 * ch[s] * ch[s + 1]);
      tensor_to_f32(*w, f);
      for (int co = 0; co < ch[s + 1]; ++co)
        for (int ci = 0; ci < ch[s]; ++ci)
          for (int t = 0; t < 9; ++t)
            r[((size_t)t * ch[s] + ci) * ch[s + 1] + co] = f[(size_t)t + 9 * (ci + (size_t)ch[s] * co)];
      E.ds_w[s].n = (int)r.size();
      E.ds_w[s].d = upload_bytes(ctx, r.data(), r.size() * 4, &rc);
      if (rc || (rc = vec(c + ".bias", E.ds_b[s]))) return rc;
    } else if ((rc = upload_conv_cl(ctx, *w, *b, E.ds3))) {
      return rc;
    }
  }
  {
    NEED(w, "mem_enc.ds.12.weight");
    NEED(b, "mem_enc.ds.12.bias");
    NEED(pw, "mem_enc.pix_feat_proj.weight");
    NEED(pb, "mem_enc.pix_feat_proj.bias");
    NEED(ow, "mem_enc.out_proj.weight");
    NEED(ob, "mem_enc.out_proj.bias");
    if ((rc = upload_linear(ctx, *w, b, E.ds12, 8, 3)) || (rc = upload_linear(ctx, *pw, pb, E.pix, 8, 3)) ||
        (rc = upload_linear(ctx, *ow, ob, E.out, 8, 3)))
      return rc;
  }
  for (int i = 0; i < 2; ++i) {
    const std::string p = "mem_enc.fuser." + std::to_string(i);
    MemEncoder::Fuser& F = E.fuser[i];
    NEED(dw, p + ".dwconv.weight");
    if (dw->ne[0] != 7 || dw->ne[1] != 7 || dw->ne[2] != 1) return set_error(ctx, kErrFormat, "%s.dwconv: shape", p.c_str());
    {
      // ggml [7, 7, 1, C] -> [ky*7 + kx][c]
      const int C = (int)dw->ne[3];
      std::vector<float> f, r((size_t)49 * C);
      tensor_to_f32(*dw, f);
      for (int c = 0; c < C; ++c)
        for (int t = 0; t < 49; ++t) r[(size_t)t * C + c] = f[(size_t)c * 49 + t];
      F.dw.n = (int)r.size();
      F.dw.d = upload_bytes(ctx, r.data(), r.size() * 4, &rc);
      if (rc) return rc;
    }
    if ((rc = vec(p + ".dwconv.bias", F.dw_b)) || (rc = vec(p + ".norm.weight", F.nw)) ||
        (rc = vec(p + ".norm.bias", F.nb)))
      return rc;
    NEED(w1, p + ".pwconv1.weight");
    NEED(b1, p + ".pwconv1.bias");
    if ((rc = upload_linear(ctx, *w1, b1, F.fc1))) return rc;
    NEED(w2, p + ".pwconv2.weight");
    NEED(b2, p + ".pwconv2.bias");
    NEED(gm, p + ".gamma");
    std::vector<float> w, b, g;
    tensor_to_f32(*w2, w);
    tensor_to_f32(*b2, b);
    tensor_to_f32(*gm, g);
    const int K = (int)w2->ne[0], N = (int)(w.size() / K);
    if ((int)g.size() != N || (int)b.size() != N) return set_error(ctx, kErrFormat, "%s: gamma / bias size", p.c_str());
    for (int n = 0; n < N; ++n) {
      for (int k = 0; k < K; ++k) w[(size_t)n * K + k] *= g[n];
      b[n] *= g[n];
    }
    if ((rc = upload_b_operand(ctx, w, N, K, 8, F.fc2))) return rc;
    F.fc2.b = upload_bytes(ctx, b.data(), b.size() * 4, &rc);
    if (rc) return rc;
  }
  for (int j = 0; j < 3; ++j) {
    const std::string p = "obj_ptr_proj.layers." + std::to_string(j);
    NEED(w, p + ".weight");
    NEED(b, p + ".bias");
    if ((rc = upload_linear(ctx, *w, b, E.ptr[j]))) return rc;
  }
  if ((rc = vec("no_obj_ptr", E.no_obj_ptr))) return rc;
  if (idx.get("no_obj_embed_spatial") && (rc = vec("no_obj_embed_spatial", E.no_obj_spatial))) return rc;
  E.D = E.pix.N;
  E.MD = E.out.N;
  const HParams& hp = ctx->model.hp;
  if (hp.is_sam2) {
    E.sig_scale = hp.sigmoid_scale_x100 / 100.0f;
    E.sig_bias = hp.sigmoid_bias_x100 / 100.0f;
  }
  if (E.D != 256 || E.ds3.N != 256 || E.ds3.K != 9 * 64 || E.ds12.K != 256 || E.fuser[0].fc1.K != 256 ||
      E.no_obj_ptr.n != E.D || (E.no_obj_spatial.n && E.no_obj_spatial.n != E.MD))
    return set_error(ctx, kErrFormat, "memory encoder: unsupported shapes");
  E.loaded = true;
  return kOk;
}

static int load_sam3(s3b_ctx* ctx, const Index& idx) {
  Model& M = ctx->model;
  const HParams& hp = M.hp;
  const int E = hp.vit_embed_dim;
  int rc = 0;
  {
    NEED(pw, "vit.patch_embed.proj.weight");
    // ggml [p, p, 3, E] == [E][3][p][p]: row co, column (ci*p + ky)*p + kx (the im2col order)
    if ((rc = upload_linear(ctx, *pw, nullptr, M.patch, 16, 3))) return rc;
  }
  {
    NEED(pos, "vit.pos_embed");
    std::vector<float> p;
    tensor_to_f32(*pos, p);
    const int G = (int)pos->ne[1], H = hp.n_img_embd();
    // ggml_repeat of [E, G, G] to [E, H, H] (sam3.cpp:3817-3822), plus 128 rows repeating the first
    // (the patch-embedding GEMM adds it per frame as a wrap-padded residual table)
    std::vector<float> tiled(((size_t)H * H + 128) * E);
    for (int y = 0; y < H; ++y)
      for (int x = 0; x < H; ++x)
        memcpy(&tiled[((size_t)y * H + x) * E], &p[((size_t)(y % G) * G + (x % G)) * E], E * 4);
    for (int r = 0; r < 128; ++r)
      memcpy(&tiled[((size_t)H * H + r) * E], &tiled[(size_t)(r % (H * H)) * E], E * 4);
    M.pos_tiled = upload_bytes(ctx, tiled.data(), tiled.size() * 4, &rc);
    if (rc) return rc;
  }
  {
    NEED(w, "vit.ln_pre.weight");
    NEED(b, "vit.ln_pre.bias");
    M.ln_pre_w = upload_vec(ctx, *w, &rc);
    M.ln_pre_b = upload_vec(ctx, *b, &rc);
  }
  M.vit.resize(hp.vit_depth);
  for (int i = 0; i < hp.vit_depth; ++i) {
    VitBlock& B = M.vit[i];
    const std::string p = "vit.blocks." + std::to_string(i);
    NEED(n1w, p + ".norm1.weight");
    NEED(n1b, p + ".norm1.bias");
    NEED(n2w, p + ".norm2.weight");
    NEED(n2b, p + ".norm2.bias");
    B.n1w = upload_vec(ctx, *n1w, &rc);
    B.n1b = upload_vec(ctx, *n1b, &rc);
    B.n2w = upload_vec(ctx, *n2w, &rc);
    B.n2b = upload_vec(ctx, *n2b, &rc);
    NEED(qw, p + ".attn.qkv.weight");
    NEED(qb, p + ".attn.qkv.bias");
    NEED(pw, p + ".attn.proj.weight");
    NEED(pb, p + ".attn.proj.bias");
    NEED(f1w, p + ".mlp.lin1.weight");
    NEED(f1b, p + ".mlp.lin1.bias");
    NEED(f2w, p + ".mlp.lin2.weight");
    NEED(f2b, p + ".mlp.lin2.bias");
    if ((rc = upload_linear(ctx, *qw, qb, B.qkv))) return rc;
    if ((rc = upload_linear(ctx, *pw, pb, B.proj))) return rc;
    if ((rc = upload_linear(ctx, *f1w, f1b, B.fc1))) return rc;
    if ((rc = upload_linear(ctx, *f2w, f2b, B.fc2))) return rc;
    B.global = hp.is_global(i);
    if (const FileTensor* fc = idx.get(p + ".attn.freqs_cis")) {
      std::vector<float> f, fp;
      tensor_to_f32(*fc, f);
      B.rope_n = (int)fc->ne[2];
      if (f.size() % ((size_t)B.rope_n * 2)) return set_error(ctx, kErrFormat, "%s: bad freqs_cis shape", p.c_str());
      rope_position_major(f, B.rope_n, (int)(f.size() / ((size_t)B.rope_n * 2)), fp);
      B.rope = upload_bytes(ctx, fp.data(), fp.size() * 4, &rc);
    }
  }
  if (idx.get("neck.trk.0.conv_1x1.weight")) {
    if ((rc = load_neck(ctx, idx, "neck.trk.", M.neck_trk))) return rc;
    M.has_neck_trk = true;
  }
  if (!hp.visual_only && idx.get("neck.det.0.conv_1x1.weight")) {
    if ((rc = load_neck(ctx, idx, "neck.det.", M.neck_det))) return rc;
    M.has_neck_det = true;
  }
  if ((rc = load_mem_attn(ctx, idx)) || (rc = load_mem_enc(ctx, idx))) return rc;
  return load_sam_dec(ctx, idx);
}

// Per-block Hiera metadata (sam2_precompute_hiera_metadata, sam3.cpp:1676-1742):
// stage dims double at stage starts, q-stride on the first block of stages
// 1..q_pool, and the window size "lags" one block at stage transitions.
// Keys cubic convolution (a = -0.75), half-pixel centres, clamped taps: the
// resampling of sam2_bicubic_interpolate_cpu (sam3.cpp:4072-4109).
static float cubic_w(float x) {
  x = fabsf(x);
  if (x < 1.0f) return (1.25f * x - 2.25f) * x * x + 1.0f;
  if (x < 2.0f) return ((-0.75f * x + 3.75f) * x - 6.0f) * x + 3.0f;
  return 0.0f;
}

// Hiera PE (sam2_compute_pos_embed, sam3.cpp:4114-4171): background PE
// [E][bh][bw] resized to S x S plus the window PE [E][ws][ws] tiled, written
// channel-last [S][S][E].
void hiera_pos_embed(const std::vector<float>& bkg, int bh, int bw, const std::vector<float>& win, int ws, int E,
                     int S, std::vector<float>& pe) {
  pe.assign((size_t)S * S * E, 0.f);
  for (int y = 0; y < S; ++y) {
    const float fy = ((float)y + 0.5f) * (float)bh / (float)S - 0.5f;
    const int iy = (int)floorf(fy);
    const float dy = fy - iy;
    for (int x = 0; x < S; ++x) {
      const float fx = ((float)x + 0.5f) * (float)bw / (float)S - 0.5f;
      const int ix = (int)floorf(fx);
      const float dx = fx - ix;
      float* dst = &pe[((size_t)y * S + x) * E];
      for (int jj = -1; jj <= 2; ++jj) {
        const float wy = cubic_w(dy - jj);
        const int sy = std::min(std::max(iy + jj, 0), bh - 1);
        for (int ii = -1; ii <= 2; ++ii) {
          const float wx = cubic_w(dx - ii);
          const int sx = std::min(std::max(ix + ii, 0), bw - 1);
          for (int e = 0; e < E; ++e) dst[e] += wy * wx * bkg[((size_t)e * bh + sy) * bw + sx];
        }
      }
      for (int e = 0; e < E; ++e) dst[e] += win[((size_t)e * ws + (y % ws)) * ws + (x % ws)];
    }
  }
}

static void hiera_metadata(Model& M) {
  const HParams& hp = M.hp;
  int total = 0;
  for (int s = 0; s < hp.hiera_num_stages; ++s) total += hp.hiera_stages[s];
  M.hiera.resize(total);
  int cum = 0;
  for (int s = 0; s < hp.hiera_num_stages; ++s) {
    cum += hp.hiera_stages[s];
    M.stage_ends[s] = cum - 1;
  }
  std::vector<int> qpool_blocks;
  for (int s = 0; s < hp.hiera_num_stages - 1 && (int)qpool_blocks.size() < hp.hiera_q_pool; ++s)
    qpool_blocks.push_back(M.stage_ends[s] + 1);
  int cur_stage = 0, embed = hp.hiera_embed_dim, heads = hp.hiera_num_heads;
  for (int i = 0; i < total; ++i) {
    HieraBlock& B = M.hiera[i];
    int ws = hp.hiera_window_spec[cur_stage];
    if (hp.is_hiera_global(i)) ws = 0;
    B.window = ws;
    int dout = embed;
    if (i > 0 && i - 1 == M.stage_ends[cur_stage]) {
      dout = embed * 2;
      heads *= 2;
      cur_stage++;
    }
    B.stage = cur_stage;
    B.dim_in = embed;
    B.dim_out = dout;
    B.heads = heads;
    B.q_stride = false;
    for (int qb : qpool_blocks)
      if (qb == i) B.q_stride = true;
    embed = dout;
  }
}

static int load_sam2(s3b_ctx* ctx, const Index& idx) {
  Model& M = ctx->model;
  const HParams& hp = M.hp;
  int rc = 0;
  hiera_metadata(M);
  {
    NEED(w, "hiera.patch_embed.weight");
    NEED(b, "hiera.patch_embed.bias");
    if ((rc = upload_linear(ctx, *w, b, M.hpatch, 8, 3))) return rc;
  }
  {
    NEED(pb, "hiera.pos_embed");
    NEED(pw, "hiera.pos_embed_window");
    tensor_to_f32(*pb, M.pos_bkg);
    tensor_to_f32(*pw, M.pos_win);
    // The PE is the same for every frame of a given size: computed once here
    // instead of per frame (sam3.cpp:5928-5934 recomputes it on the host each frame).
    const int E0 = hp.hiera_embed_dim, S = hp.img_size / 4;
    std::vector<float> pe;
    hiera_pos_embed(M.pos_bkg, (int)pb->ne[1], (int)pb->ne[0], M.pos_win, (int)pw->ne[0], E0, S, pe);
    M.hiera_pe = upload_bytes(ctx, pe.data(), pe.size() * 4, &rc);
    if (rc) return rc;
    M.hiera_pe_size = S;
  }
  for (size_t i = 0; i < M.hiera.size(); ++i) {
    HieraBlock& B = M.hiera[i];
    const std::string p = "hiera.blocks." + std::to_string(i);
    NEED(n1w, p + ".norm1.weight");
    NEED(n1b, p + ".norm1.bias");
    NEED(n2w, p + ".norm2.weight");
    NEED(n2b, p + ".norm2.bias");
    B.n1w = upload_vec(ctx, *n1w, &rc);
    B.n1b = upload_vec(ctx, *n1b, &rc);
    B.n2w = upload_vec(ctx, *n2w, &rc);
    B.n2b = upload_vec(ctx, *n2b, &rc);
    NEED(qw, p + ".attn.qkv.weight");
    NEED(qb, p + ".attn.qkv.bias");
    NEED(pw, p + ".attn.proj.weight");
    NEED(pb, p + ".attn.proj.bias");
    NEED(f1w, p + ".mlp.fc1.weight");
    NEED(f1b, p + ".mlp.fc1.bias");
    NEED(f2w, p + ".mlp.fc2.weight");
    NEED(f2b, p + ".mlp.fc2.bias");
    if ((rc = upload_linear(ctx, *qw, qb, B.qkv))) return rc;
    if ((rc = upload_linear(ctx, *pw, pb, B.proj))) return rc;
    if ((rc = upload_linear(ctx, *f1w, f1b, B.fc1))) return rc;
    if ((rc = upload_linear(ctx, *f2w, f2b, B.fc2))) return rc;
    if (B.dim_in != B.dim_out) {
      NEED(dw, p + ".proj.weight");
      NEED(db, p + ".proj.bias");
      if ((rc = upload_linear(ctx, *dw, db, B.dim_proj))) return rc;
      B.has_dim_proj = true;
    }
  }
  for (int i = 0; i < 4; ++i) {
    const std::string p = "fpn.convs." + std::to_string(i);
    NEED(w, p + ".weight");
    NEED(b, p + ".bias");
    if ((rc = upload_linear(ctx, *w, b, M.fpn[i], 8, 3))) return rc;
  }
  if ((rc = load_mem_attn(ctx, idx)) || (rc = load_mem_enc(ctx, idx))) return rc;
  return load_sam_dec(ctx, idx);
}

int parse_hparams_array(int is_sam2, const int32_t* v, int n, HParams& hp, std::string& err) {
  int i = 0;
  const int rc = parse_hparams(is_sam2 != 0, [&](int32_t& x) {
    if (i >= n) return false;
    x = v[i++];
    return true;
  }, hp, err);
  if (rc) return rc;
  if (i != n) {
    err = "hparams: " + std::to_string(n) + " values given, the header has " + std::to_string(i);
    return kErrFormat;
  }
  return kOk;
}

int load_model(s3b_ctx* ctx, const std::string& path) {
  HParams hp;
  std::vector<FileTensor> tensors;
  std::string err;
  int rc = read_ggml_file(path, hp, tensors, err);
  if (rc) return set_error(ctx, rc, "%s", err.c_str());
  return load_model_tensors(ctx, hp, tensors);
}

int load_model_tensors(s3b_ctx* ctx, const HParams& hp, const std::vector<FileTensor>& tensors) {
  int rc = 0;
  ctx->model = Model();
  ctx->model.hp = hp;
  Index idx;
  for (const FileTensor& t : tensors) idx.m[t.name] = &t;
  cudaSetDevice(ctx->device);
  rc = hp.is_sam2 ? load_sam2(ctx, idx) : load_sam3(ctx, idx);
  if (rc) return rc;
  if (const size_t elems = stage_arena_elems(ctx->model)) {
    // the staging buffers are sized once here, so they never move under a captured graph: the arena
    // of the staged groups and a buffer for a single weight outside them
    ctx->buf("wq_stage", elems * 2, &rc);
    if (rc) return rc;
    ctx->buf("wq_stage1", ctx->model.qstage_elems * 2, &rc);
    if (rc) return rc;
  }
  ctx->model.loaded = true;
  return kOk;
}

}  // namespace s3b
