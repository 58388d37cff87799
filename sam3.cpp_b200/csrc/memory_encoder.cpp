// Memory encoder and object-pointer MLP on B200 (host orchestration, C++14).
//
// Replaces sam3_encode_memory (sam3.cpp:11506-11603), its ggml graph and host loops, and
// sam3_extract_obj_ptr_cpu (9344-9418). The mask preprocessing and the three narrow downsampler stages
// run as direct kernels (mem_enc.cu); the 64 -> 256 stage, the 1x1 convolutions and the CXBlock MLPs
// are tcgen05 GEMMs; the no-object embedding and the pointer's no-object replacement are decided on the
// device from the decoder's object score, so a tracking step needs no host round trip.
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

int mem_encode_run(s3b_ctx* ctx, int H, const float* pix_feat, const float* mask_logits, int mask_h, int mask_w,
                   const float* obj_score, float* out) {
  const MemEncoder& E = ctx->model.menc;
  if (!E.loaded) return set_error(ctx, kErrState, "the model has no memory encoder");
  const int img = ctx->model.hp.img_size;
  if (H <= 0 || H > 512 || mask_h < 2 || mask_w < 2 || !pix_feat || !mask_logits || !out || img < 2)
    return set_error(ctx, kErrArg, "mem_encode: bad arguments");
  const int S = 16 * H;  // the downsampler's input size (sam3.cpp:11514)
  const long long HH = (long long)H * H;
  int rc = 0;
  DevBuf* hires = ctx->buf("me_hires", (size_t)img * img * 4, &rc);
  DevBuf* m0 = ctx->buf("me_m0", (size_t)S * S * 4, &rc);
  DevBuf* s0 = ctx->buf("me_s0", (size_t)(S / 2) * (S / 2) * 4 * 4, &rc);
  DevBuf* s1 = ctx->buf("me_s1", (size_t)(S / 4) * (S / 4) * 16 * 4, &rc);
  DevBuf* s2 = ctx->buf("me_s2", (size_t)(S / 8) * (S / 8) * 64 * 4, &rc);
  DevBuf* col = ctx->buf("me_col", (size_t)HH * 9 * 64 * 2, &rc);
  DevBuf* x32 = ctx->buf("me_x32", (size_t)HH * 256 * 4, &rc);
  DevBuf* x16 = ctx->buf("me_x16", (size_t)HH * 256 * 2, &rc);
  DevBuf* h32 = ctx->buf("me_h32", (size_t)HH * 256 * 4, &rc);
  DevBuf* t16 = ctx->buf("me_t16", (size_t)HH * 1024 * 2, &rc);
  if (rc) return rc;
  cudaStream_t st = ctx->stream;
  // mask logits -> input size -> sigmoid * scale + bias -> 16 H (sam3.cpp:11516-11520)
  CKL(bilinear_resize(mask_logits, mask_w, mask_h, hires->as<float>(), img, img, 1, E.sig_scale, E.sig_bias, st));
  CKL(bilinear_resize(hires->as<float>(), img, img, m0->as<float>(), S, S, 0, 0.f, 0.f, st));
  // downsampler stages 0-2 (direct), stage 3 (column matrix + GEMM, LayerNorm2d + GELU), 1x1 conv
  const float* in = m0->as<float>();
  float* outs[3] = {s0->as<float>(), s1->as<float>(), s2->as<float>()};
  const int ch[4] = {1, 4, 16, 64};
  int side = S;
  for (int s = 0; s < 3; ++s) {
    CKL(mask_ds_conv(in, side, side, ch[s], ch[s + 1], E.ds_w[s].ptr(), E.ds_b[s].ptr(), E.ds_nw[s].ptr(),
                     E.ds_nb[s].ptr(), 1e-6f, outs[s], st));
    in = outs[s];
    side = (side + 1) / 2;
  }
  if ((side + 1) / 2 != H) return set_error(ctx, kErrArg, "mem_encode: downsampler size %d != %d", (side + 1) / 2, H);
  CKL(im2col_s2(in, side, side, 64, col->as<__half>(), st));
  CKR(run_gemm(ctx, col->as<__half>(), 9 * 64, E.ds3, HH, epi_store(E.ds3, x32->p, 1, 256)));
  CKL(ln_gelu_rows(x32->as<float>(), HH, 256, E.ds_nw[3].ptr(), E.ds_nb[3].ptr(), 1e-6f, x16->as<__half>(), st));
  CKR(run_gemm(ctx, x16->as<__half>(), 256, E.ds12, HH, epi_store(E.ds12, x32->p, 1, 256)));
  // fused = pix_feat_proj(neck_trk_2) + downsampled mask (sam3.cpp:11550-11561)
  CKL(cast_f32_f16(pix_feat, HH * 256, x16->as<__half>(), st));
  {
    EpiParams e = epi_store(E.pix, h32->p, 1, 256);
    e.resid = x32->as<float>();
    e.ldr = 256;
    CKR(run_gemm(ctx, x16->as<__half>(), 256, E.pix, HH, e));
  }
  // two CXBlocks (sam3_cxblock_forward, 9058-9104): x + gamma * pwconv2(GELU(pwconv1(LN2d(dwconv(x)))))
  for (int i = 0; i < 2; ++i) {
    const MemEncoder::Fuser& F = E.fuser[i];
    CKL(dwconv7_ln(h32->as<float>(), H, H, F.dw.ptr(), F.dw_b.ptr(), F.nw.ptr(), F.nb.ptr(), 1e-6f,
                   x16->as<__half>(), st));
    CKR(run_gemm(ctx, x16->as<__half>(), 256, F.fc1, HH, epi_store(F.fc1, t16->p, 0, F.fc1.N, ACT_GELU_TANH)));
    EpiParams e = epi_store(F.fc2, h32->p, 1, 256);
    e.resid = h32->as<float>();
    e.ldr = 256;
    CKR(run_gemm(ctx, t16->as<__half>(), F.fc1.N, F.fc2, HH, e));
  }
  // out projection to the memory dim; no_obj_embed_spatial when the object is absent (11575-11589)
  CKL(cast_f32_f16(h32->as<float>(), HH * 256, x16->as<__half>(), st));
  CKR(run_gemm(ctx, x16->as<__half>(), 256, E.out, HH, epi_store(E.out, out, 1, E.MD)));
  if (obj_score && E.no_obj_spatial.n) CKL(add_if_absent(out, HH, E.MD, E.no_obj_spatial.ptr(), obj_score, st));
  return check_device(ctx, "mem_encode");
}

int obj_ptr_run(s3b_ctx* ctx, const float* sam_token, const float* obj_score, float* out) {
  const MemEncoder& E = ctx->model.menc;
  if (!E.loaded) return set_error(ctx, kErrState, "the model has no object-pointer MLP");
  if (!sam_token || !out) return set_error(ctx, kErrArg, "obj_ptr: bad arguments");
  int rc = 0;
  DevBuf* hb = ctx->buf("op_h", 3 * 256 * 4, &rc);
  if (rc) return rc;
  float* h = hb->as<float>();
  const float* x = sam_token;
  for (int j = 0; j < 3; ++j) {
    const Linear& L = E.ptr[j];
    TokJob jb;
    jb.x = x;
    jb.ldx = L.K;
    jb.R = 1;
    jb.W = L.w->as<__half>();
    jb.ldw = L.Kpad;
    jb.b = L.b->as<float>();
    jb.N = L.N;
    jb.K = L.K;
    jb.y = h + j * 256;
    jb.ldy = L.N;
    jb.act = j < 2 ? 1 : 0;
    CKL(tok_linear(&jb, 1, ctx->stream));
    x = h + j * 256;
  }
  CKL(select_obj_ptr(h + 512, E.no_obj_ptr.ptr(), obj_score, E.D, out, ctx->stream));
  return check_device(ctx, "obj_ptr");
}

}  // namespace s3b
