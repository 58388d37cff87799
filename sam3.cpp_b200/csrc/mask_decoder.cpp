// SAM prompt encoder + mask decoder on B200 (host orchestration, C++14).
//
// Replaces sam3_build_sam_dec_graph (sam3.cpp:10544-10757) with its ggml compute, as
// sam3_segment_pvs (10760-10990, the image predictor: image features = neck_trk_2 + no_mem_embed,
// point / box prompt tokens) and sam3_propagate_single (11171-11453, tracking: image features =
// the memory-attention output, one not_a_point token) call it, plus the prompt encoder's host
// parts: sam3_pe_encode_coord (10269-10282), the dense PE grid of sam3_populate_pe_cache
// (10288-10345) and the sparse tokens of sam3_collect_pvs_prompt_tokens + sam3_segment_pvs
// (10361-10391, 10877-10900).
//
// Per TwoWay block (sam3_twoway_block_forward, 10436-10500) the image side is three tcgen05 GEMMs
// (keys + key_pe -> [t2i k | i2t q], keys -> t2i v, i2t attention output -> out proj with the
// residual into the keys), the i2t attention and one pass that LayerNorms the keys and writes the
// next GEMMs' f16 operands; the token side (at most kTokMaxRows rows) is tok_linear / tok_attention /
// tok_layernorm launches and the split-key t2i attention. The upscaling runs the first transposed
// convolution on the tcgen05 pixel-block GEMM and the rest in two fused per-pixel kernels whose last
// step is the hypernetwork mask products.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "engine.h"

namespace s3b {

#define CKL(call)                                                                                  \
  do {                                                                                             \
    int _rc = (call);                                                                              \
    count_launch(ctx);                                                                             \
    if (_rc) return set_error(ctx, launcher_status_code(_rc), "%s failed (%d)", #call, _rc);  \
  } while (0)
#define CKR(call)        \
  do {                   \
    int _rc = (call);    \
    if (_rc) return _rc; \
  } while (0)

// sam3_pe_encode_coord (sam3.cpp:10269-10282): coordinates in [0, 1] -> [sin(128) ; cos(128)], in the
// reference's f32 steps.
static void pe_encode_coord(float* out, float x_norm, float y_norm, const float* g, int npf) {
  const float cx = 2.0f * x_norm - 1.0f, cy = 2.0f * y_norm - 1.0f;
  for (int i = 0; i < npf; ++i) {
    float dot = cx * g[i] + cy * g[npf + i];
    dot *= 2.0f * (float)M_PI;
    out[i] = sinf(dot);
    out[i + npf] = cosf(dot);
  }
}

const float* sam_dec_dense_pe(s3b_ctx* ctx, int H, int* rc) {
  const SamDecoder& d = ctx->model.dec;
  const std::string key = "dec_pe_" + std::to_string(H);
  auto it = ctx->ws.find(key);
  if (it != ctx->ws.end() && it->second) return it->second->as<float>();
  const int D = d.D, npf = D / 2;
  std::vector<float> pe((size_t)H * H * D);
  for (int row = 0; row < H; ++row)
    for (int col = 0; col < H; ++col)
      pe_encode_coord(&pe[((size_t)row * H + col) * D], ((float)col + 0.5f) / (float)H, ((float)row + 0.5f) / (float)H,
                      d.pe_gauss.data(), npf);
  DevBuf* b = ctx->buf(key, pe.size() * 4, rc);
  if (*rc) return nullptr;
  if ((*rc = upload_sync(ctx, b->p, pe.data(), pe.size() * 4))) return nullptr;
  return b->as<float>();
}

int sam_prompt_tokens(const SamDecoder& d, const float* box, const float* pos, int n_pos, const float* neg, int n_neg,
                      float orig_w, float orig_h, int input_size, float* out, int capacity) {
  if (!d.loaded || n_pos < 0 || n_neg < 0 || (n_pos && !pos) || (n_neg && !neg) || orig_w <= 0 || orig_h <= 0 ||
      input_size <= 0 || !out)
    return kErrArg;
  std::vector<float> coords;
  std::vector<int> labels;
  if (box) {
    coords.insert(coords.end(), {box[0], box[1], box[2], box[3]});
    labels.insert(labels.end(), {2, 3});
  }
  for (int i = 0; i < n_pos; ++i) {
    coords.insert(coords.end(), {pos[2 * i], pos[2 * i + 1]});
    labels.push_back(1);
  }
  for (int i = 0; i < n_neg; ++i) {
    coords.insert(coords.end(), {neg[2 * i], neg[2 * i + 1]});
    labels.push_back(0);
  }
  coords.insert(coords.end(), {0.0f, 0.0f});
  labels.push_back(-1);
  const int n = (int)labels.size(), D = d.D;
  if (n > capacity) return kErrArg;
  const float s = (float)input_size;
  for (int p = 0; p < n; ++p) {
    float* o = out + (size_t)p * D;
    if (labels[p] == -1) {
      memcpy(o, d.not_a_point.data(), D * 4);
      continue;
    }
    const float px = coords[2 * p] / orig_w * s + 0.5f, py = coords[2 * p + 1] / orig_h * s + 0.5f;
    float pe[512];
    pe_encode_coord(pe, px / s, py / s, d.pe_gauss.data(), D / 2);
    for (int c = 0; c < D; ++c) o[c] = pe[c] + d.point_emb[labels[p]][c];
  }
  return n;
}

static TokJob tj(const float* x, const float* x2, long long ldx, int R, const Linear& L, float* y, long long ldy,
                 const float* resid = nullptr, int act = 0) {
  TokJob j;
  j.x = x;
  j.x2 = x2;
  j.ldx = ldx;
  j.R = R;
  j.W = L.w->as<__half>();
  j.ldw = L.Kpad;
  j.b = L.b ? L.b->as<float>() : nullptr;
  j.N = L.N;
  j.K = L.K;
  j.y = y;
  j.ldy = ldy;
  j.resid = resid;
  j.ldr = ldy;
  j.act = act;
  return j;
}

int sam_dec_run(s3b_ctx* ctx, int H, const float* image_feats, const float* feat_s0, const float* feat_s1,
                const float* sparse, int n_sparse, int add_no_mem, float* masks, float* iou, float* obj,
                float* mask_tokens) {
  const SamDecoder& d = ctx->model.dec;
  if (!d.loaded) return set_error(ctx, kErrState, "the model has no SAM mask decoder");
  if (H <= 0 || H > 1024 || !image_feats || !feat_s0 || !feat_s1 || n_sparse < 0 || (n_sparse && !sparse))
    return set_error(ctx, kErrArg, "sam_decode: bad arguments");
  const int D = d.D, ns = d.n_special(), s = d.has_obj ? 1 : 0;
  const int npts = n_sparse ? n_sparse : 1;
  const int NT = ns + npts;
  if (NT > kTokMaxRows)
    return set_error(ctx, kErrArg, "sam_decode: %d prompt tokens (at most %d)", n_sparse, kTokMaxRows - ns);
  const long long HH = (long long)H * H, H1 = 4 * HH;
  const int heads = d.heads;
  int rc = 0;
  const float* pe = sam_dec_dense_pe(ctx, H, &rc);
  if (rc) return rc;
  DevBuf* keys = ctx->buf("dec_keys", HH * D * 4, &rc);
  DevBuf* k16 = ctx->buf("dec_k16", HH * D * 2, &rc);
  DevBuf* kpe16 = ctx->buf("dec_kpe16", HH * D * 2, &rc);
  DevBuf* kq = ctx->buf("dec_kq", HH * 256 * 2, &rc);
  DevBuf* vimg = ctx->buf("dec_v", HH * 128 * 2, &rc);
  DevBuf* oimg = ctx->buf("dec_o", HH * 128 * 2, &rc);
  DevBuf* up1 = ctx->buf("dec_up1", H1 * 64 * 4, &rc);
  DevBuf* u1 = ctx->buf("dec_u1", H1 * 64 * 2, &rc);
  DevBuf* tws = ctx->buf("dec_t2i_ws", t2i_ws_floats(NT, heads, HH) * 4, &rc);
  // token buffers (f32): T0 (initial tokens = query PE), T, QKV [NT][768], AO, Qt, Ot, Hd [NT][2048],
  // Kt, Vt, head hidden rows x 2, hyper [n_mask][32], iou, obj
  const int FFN = d.blocks[0].mlp1.N;
  const size_t tok_floats = (size_t)NT * (D * 4 + 768 + 128 * 4 + FFN) + 2 * 8 * 256 + 4 * 32 + 64;
  DevBuf* tb = ctx->buf("dec_tok", tok_floats * 4 + 256, &rc);
  if (rc) return rc;
  float* T0 = tb->as<float>();
  float* T = T0 + NT * D;
  float* AO = T + NT * D;
  float* QKV = AO + NT * D;
  float* Qt = QKV + NT * 768;
  float* Ot = Qt + NT * 128;
  float* Kt = Ot + NT * 128;
  float* Vt = Kt + NT * 128;
  float* Hd = Vt + NT * 128;
  float* HA = Hd + (size_t)NT * FFN;
  float* HB = HA + 8 * 256;
  float* hyper = HB + 8 * 256;
  float* iou_d = hyper + 4 * 32;
  float* obj_d = iou_d + 8;
  cudaStream_t st = ctx->stream;

  // tokens = [special tokens ; prompt tokens]; the query PE is this initial copy (sam3.cpp:10575-10604)
  if (cudaMemcpyAsync(T0, d.tokens->p, (size_t)ns * D * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(T0 + (size_t)ns * D, n_sparse ? sparse : d.d_not_a_point.ptr(), (size_t)npts * D * 4,
                      cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(T, T0, (size_t)NT * D * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return set_error(ctx, kErrCuda, "sam_decode: token copies failed");
  // keys = image_feats (+ no_mem_embed) + no_mask dense embedding; key PE = the dense grid
  CKL(dec_keys(image_feats, HH, 0, d.d_no_mask.ptr(), add_no_mem ? d.d_no_mem.ptr() : nullptr, nullptr, nullptr,
               0.f, pe, keys->as<float>(), k16->as<__half>(), kpe16->as<__half>(), st));
  float* K32 = keys->as<float>();
  __half* K16 = k16->as<__half>();
  __half* KPE = kpe16->as<__half>();
  __half* KQ = kq->as<__half>();
  __half* V = vimg->as<__half>();
  __half* O = oimg->as<__half>();
  const float sa_scale = 1.0f / sqrtf((float)(D / heads));
  const float x_scale = 1.0f / sqrtf((float)(128 / heads));
  for (size_t i = 0; i < d.blocks.size(); ++i) {
    const SamTwoWay& B = d.blocks[i];
    // image side of both cross-attentions from the block's input keys
    CKR(run_gemm(ctx, KPE, D, B.kq, HH, epi_store(B.kq, KQ, 0, 256)));
    CKR(run_gemm(ctx, K16, D, B.t2i_v, HH, epi_store(B.t2i_v, V, 0, 128)));
    // 1. token self-attention (block 0: q = k = v = queries, no residual)
    {
      const float* pe_in = i == 0 ? nullptr : T0;
      TokJob j[3] = {tj(T, pe_in, D, NT, B.sa_q, QKV, 768), tj(T, pe_in, D, NT, B.sa_k, QKV + 256, 768),
                     tj(T, nullptr, D, NT, B.sa_v, QKV + 512, 768)};
      CKL(tok_linear(j, 3, st));
      CKL(tok_attention(QKV, 768, QKV + 256, 768, QKV + 512, 768, NT, heads, D / heads, sa_scale, AO, D, st));
      TokJob o = tj(AO, nullptr, D, NT, B.sa_out, T, D, i == 0 ? nullptr : T);
      CKL(tok_linear(&o, 1, st));
      CKL(tok_layernorm(T, nullptr, D, NT, D, B.n1w.ptr(), B.n1b.ptr(), 1e-5f, T, st));
    }
    // 2. tokens -> image
    {
      TokJob q = tj(T, T0, D, NT, B.t2i_q, Qt, 128);
      CKL(tok_linear(&q, 1, st));
      CKL(t2i_attention(Qt, 128, KQ, 256, V, 128, NT, heads, HH, x_scale, tws->as<float>(), Ot, 128, st));
      TokJob o = tj(Ot, nullptr, 128, NT, B.t2i_out, T, D, T);
      CKL(tok_linear(&o, 1, st));
      CKL(tok_layernorm(T, nullptr, D, NT, D, B.n2w.ptr(), B.n2b.ptr(), 1e-5f, T, st));
    }
    // 3. token MLP (ReLU)
    {
      TokJob a = tj(T, nullptr, D, NT, B.mlp1, Hd, FFN, nullptr, 1);
      CKL(tok_linear(&a, 1, st));
      TokJob b = tj(Hd, nullptr, FFN, NT, B.mlp2, T, D, T);
      CKL(tok_linear(&b, 1, st));
      CKL(tok_layernorm(T, nullptr, D, NT, D, B.n3w.ptr(), B.n3b.ptr(), 1e-5f, T, st));
    }
    // 4. image -> tokens: k from queries + query PE, v from queries; keys += out proj, LayerNorm
    {
      TokJob j[2] = {tj(T, T0, D, NT, B.i2t_k, Kt, 128), tj(T, nullptr, D, NT, B.i2t_v, Vt, 128)};
      CKL(tok_linear(j, 2, st));
      CKL(i2t_attention(KQ + 128, 256, Kt, 128, Vt, 128, NT, heads, HH, x_scale, O, 128, st));
      EpiParams r = epi_store(B.i2t_out, K32, 1, D);
      r.resid = K32;
      r.ldr = D;
      CKR(run_gemm(ctx, O, 128, B.i2t_out, HH, r));
      CKL(dec_keys(K32, HH, 1, nullptr, nullptr, B.n4w.ptr(), B.n4b.ptr(), 1e-5f, pe, K32, K16, KPE, st));
    }
  }
  // final tokens -> image attention + LayerNorm (sam3.cpp:10620-10627)
  {
    CKR(run_gemm(ctx, KPE, D, d.fin_k, HH, epi_store(d.fin_k, KQ, 0, 128)));
    CKR(run_gemm(ctx, K16, D, d.fin_v, HH, epi_store(d.fin_v, V, 0, 128)));
    TokJob q = tj(T, T0, D, NT, d.fin_q, Qt, 128);
    CKL(tok_linear(&q, 1, st));
    CKL(t2i_attention(Qt, 128, KQ, 128, V, 128, NT, heads, HH, x_scale, tws->as<float>(), Ot, 128, st));
    TokJob o = tj(Ot, nullptr, 128, NT, d.fin_out, T, D, T);
    CKL(tok_linear(&o, 1, st));
    CKL(tok_layernorm(T, nullptr, D, NT, D, d.fin_nw.ptr(), d.fin_nb.ptr(), 1e-5f, T, st));
  }
  // hypernetwork MLPs (mask tokens s+1 .. s+4), IoU head (token s), object-score head (token 0)
  {
    const int nm = d.n_mask;
    float* in_rows[2] = {HA, HB};
    for (int layer = 0; layer < 3; ++layer) {
      TokJob j[kTokMaxJobs];
      int n = 0;
      const bool last = layer == 2;
      for (int m = 0; m < nm; ++m) {
        const float* x = layer == 0 ? T + (size_t)(s + 1 + m) * D : in_rows[(layer - 1) & 1] + (size_t)m * 256;
        float* y = last ? hyper + m * 32 : in_rows[layer & 1] + (size_t)m * 256;
        j[n++] = tj(x, nullptr, D, 1, d.hyper[m * 3 + layer], y, 256, nullptr, last ? 0 : 1);
      }
      {
        const float* x = layer == 0 ? T + (size_t)s * D : in_rows[(layer - 1) & 1] + (size_t)nm * 256;
        float* y = last ? iou_d : in_rows[layer & 1] + (size_t)nm * 256;
        j[n++] = tj(x, nullptr, D, 1, d.iou[layer], y, 256, nullptr, last ? 2 : 1);
      }
      if (d.has_obj) {
        const float* x = layer == 0 ? T : in_rows[(layer - 1) & 1] + (size_t)(nm + 1) * 256;
        float* y = last ? obj_d : in_rows[layer & 1] + (size_t)(nm + 1) * 256;
        j[n++] = tj(x, nullptr, D, 1, d.obj[layer], y, 256, nullptr, last ? 0 : 1);
      }
      CKL(tok_linear(j, n, st));
    }
  }
  // upscaling: deconv(keys) -> + conv_s1(feat_s1) -> LayerNorm2d -> GELU -> deconv -> + conv_s0(feat_s0)
  // -> GELU -> mask products (sam3.cpp:10650-10730)
  {
    EpiParams e = epi_store(d.up1, up1->p, 1, 64);
    e.bias = d.up1.b->as<float>();
    CKR(run_deconv2x2(ctx, d.up1, K16, 1, H, H, e));
    CKL(dec_upscale1(up1->as<float>(), feat_s1, d.conv_s1.w->as<__half>(), d.conv_s1.b->as<float>(), d.up1_nw.ptr(),
                     d.up1_nb.ptr(), 1e-6f, H1, u1->as<__half>(), st));
    if (masks)
      CKL(dec_masks(u1->as<__half>(), d.up2.w->as<__half>(), d.up2.b->as<float>(), feat_s0,
                    d.conv_s0.w->as<__half>(), d.conv_s0.b->as<float>(), hyper, 4 * H, masks, st));
  }
  const int nm = d.n_mask;
  if (iou && cudaMemcpyAsync(iou, iou_d, nm * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return set_error(ctx, kErrCuda, "sam_decode: output copy failed");
  if (obj) {
    // without an object-score token the score is the constant logit 10 (sam3.cpp:10740-10746)
    if (!d.has_obj) {
      const float ten = 10.0f;
      CKR(upload_sync(ctx, obj_d, &ten, 4));
    }
    if (cudaMemcpyAsync(obj, obj_d, 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return set_error(ctx, kErrCuda, "sam_decode: output copy failed");
  }
  if (mask_tokens &&
      cudaMemcpyAsync(mask_tokens, T + (size_t)(s + 1) * D, (size_t)nm * D * 4, cudaMemcpyDeviceToDevice, st) !=
          cudaSuccess)
    return set_error(ctx, kErrCuda, "sam_decode: output copy failed");
  return check_device(ctx, "sam_decode");
}

}  // namespace s3b
