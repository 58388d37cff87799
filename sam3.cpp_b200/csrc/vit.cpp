// SAM 3 image encoder on B200: ViT backbone + SimpleFPN neck (host
// orchestration, C++14). Replaces sam3_build_vit_graph (sam3.cpp:3835-3849),
// sam3_build_vit_prefix_graph (3806-3830), sam3_vit_block_forward (3710-3801)
// and sam3_build_neck_graph (3863-3921) with a fixed sequence of kernel
// launches on the context's stream; nothing is re-planned per frame.
//
// Activation layout: token-major, channel-last (ggml [C, W, H, B] memory),
// rows = frame * H*W + y*W + x. The residual stream stays f32; GEMM inputs
// are f16; window partition / unpartition are folded into the LayerNorm row
// gather and the projection epilogue's row map.
#include <math.h>
#include <string.h>

#include "engine.h"

namespace s3b {

#define CK(call)                                                                                          \
  do {                                                                                                    \
    int _rc = (call);                                                                                     \
    count_launch(ctx);                                                                                    \
    if (_rc) return set_error(ctx, launcher_status_code(_rc), "%s failed (%d) at %s:%d", #call, _rc, \
                              __FILE__, __LINE__);                                                        \
  } while (0)
#define CKG(call)                                                                                         \
  do {                                                                                                    \
    int _rc = (call);                                                                                     \
    if (_rc) return _rc;                                                                                  \
  } while (0)

static int gemm(s3b_ctx* ctx, const __half* A, long long lda, const Linear& L, long long M, const EpiParams& ep) {
  return run_gemm(ctx, A, lda, L, M, ep);
}

// One ViT block (sam3_vit_block_forward, sam3.cpp:3710-3801) on T tokens.
static int vit_block(s3b_ctx* ctx, const VitBlock& B, int F, float* x, __half* xn, __half* qkv, __half* ao,
                     __half* hbuf) {
  const HParams& hp = ctx->model.hp;
  const int E = hp.vit_embed_dim, NH = hp.vit_num_heads, HD = E / NH, G = hp.n_img_embd();
  const long long T = (long long)F * G * G;
  RowMap wmap;
  int ntok, nwin;
  if (!B.global) {
    const int ws = hp.vit_window_size;
    const int nw = (G + ws - 1) / ws;
    wmap.kind = 1;
    wmap.ws = ws;
    wmap.nww = wmap.nwh = nw;
    wmap.W = wmap.H = G;
    ntok = ws * ws;
    nwin = F * nw * nw;
  } else {
    ntok = G * G;
    nwin = F;
  }
  const long long Tw = (long long)nwin * ntok;  // rows in window order (>= T when padded)
  // norm1 + window partition (ggml_win_part, sam3.cpp:3730)
  CK(run_ln(ctx, x, E, xn, 0, E, Tw, E, B.n1w.ptr(), B.n1b.ptr(), 1e-5f, wmap));
  // qkv + bias + RoPE(q, k) into [Tw][3E] f16 (sam3.cpp:3738-3771); the attention
  // kernel reads q / k / v of each (window, head) with strides, so no split copies
  EpiParams ep = epi_store(B.qkv, qkv, 0, 3LL * E);
  if (B.rope) {
    if (B.rope_n != ntok)
      return set_error(ctx, kErrFormat, "freqs_cis has %d positions, attention has %d", B.rope_n, ntok);
    ep.rope = B.rope->as<float>();
    ep.rope_D = HD;
    ep.rope_cols = 2 * E;
    ep.rope_rows = Tw;
    ep.rope_mod = ntok;
  }
  CKG(gemm(ctx, xn, E, B.qkv, Tw, ep));
  // flash attention, scale 1/sqrt(HD) (sam3.cpp:3773-3774); rows leave in spatial
  // order (window unpartition, sam3.cpp:3784) so the projection needs no remap
  AttnParams ap;
  ap.q = qkv;
  ap.k = qkv + E;
  ap.v = qkv + 2 * E;
  ap.o = ao;
  ap.q_b = ap.k_b = ap.v_b = (long long)ntok * 3 * E;
  ap.q_h = ap.k_h = ap.v_h = HD;
  ap.q_n = ap.k_n = ap.v_n = 3LL * E;
  ap.heads = NH;
  ap.nq = ap.nk = ntok;
  ap.o_n = E;
  ap.omap = wmap;
  ap.scale = 1.0f / sqrtf((float)HD);
  CKG(run_attn(ctx, ap, HD, nwin * NH));
  // proj + bias, residual added in place (x chunk TMA-loaded in the epilogue) (sam3.cpp:3779-3787)
  EpiParams pe = epi_store(B.proj, x, 1, E);
  pe.resid = x;
  pe.ldr = E;
  CKG(gemm(ctx, ao, E, B.proj, T, pe));
  // norm2 -> fc1 + GELU(erf) -> fc2 + residual (sam3.cpp:3789-3798)
  RowMap id;
  CK(run_ln(ctx, x, E, xn, 0, E, T, E, B.n2w.ptr(), B.n2b.ptr(), 1e-5f, id));
  const int MLP = B.fc1.N;
  CKG(gemm(ctx, xn, E, B.fc1, T, epi_store(B.fc1, hbuf, 0, MLP, ACT_GELU_ERF)));
  EpiParams f2 = epi_store(B.fc2, x, 1, E);
  f2.resid = x;
  f2.ldr = E;
  CKG(gemm(ctx, hbuf, MLP, B.fc2, T, f2));
  return kOk;
}

// conv 3x3 (pad 1), channel-last f16 in -> f32 out: implicit GEMM (im2col + GEMM when disabled).
static int conv3x3(s3b_ctx* ctx, const Linear& L, const __half* in, int F, int S, float* out, __half* col) {
  return run_conv3x3(ctx, L, in, F, S, S, epi_store(L, out, 1, L.N), col);
}

// One SimpleFPN path (sam3_build_neck_graph, sam3.cpp:3863-3921) for F frames.
static int vit_neck(s3b_ctx* ctx, const NeckScale* sc, const __half* xh, int F, float* const outs[4]) {
  const HParams& hp = ctx->model.hp;
  const int G = hp.n_img_embd();
  int rc = 0;
  const long long T = (long long)F * G * G;
  const int c_mid = sc[0].dc1.N / 4;  // 512
  const int D = sc[0].c3.N;           // 256
  DevBuf* d1 = ctx->buf("neck_d1", (size_t)T * 4 * c_mid * 2, &rc);
  DevBuf* c1 = ctx->buf("neck_c1", (size_t)T * 16 * D * 2, &rc);
  // im2col workspace only when the implicit convolution is switched off
  DevBuf* col = ctx->conv_implicit ? nullptr : ctx->buf("neck_col", (size_t)T * 16 * 9 * D * 2, &rc);
  __half* colp = col ? col->as<__half>() : nullptr;
  DevBuf* mp = ctx->buf("neck_mp", (size_t)T / 4 * hp.vit_embed_dim * 2, &rc);
  if (rc) return rc;
  // scale 0: deconv(E->512) + GELU(erf) -> [deconv(512->D) -> 1x1, folded into one deconv] -> 3x3  (4x)
  {
    if ((rc = run_deconv2x2(ctx, sc[0].dc1, xh, F, G, G, epi_store(sc[0].dc1, d1->p, 0, c_mid, ACT_GELU_ERF))))
      return rc;
    if ((rc = run_deconv2x2(ctx, sc[0].dcf, d1->as<__half>(), F, 2 * G, 2 * G, epi_store(sc[0].dcf, c1->p, 0, D))))
      return rc;
    if ((rc = conv3x3(ctx, sc[0].c3, c1->as<__half>(), F, 4 * G, outs[0], colp))) return rc;
  }
  // scale 1: [deconv(E->512) -> 1x1 (512->D), folded into one deconv] -> 3x3  (2x)
  {
    if ((rc = run_deconv2x2(ctx, sc[1].dcf, xh, F, G, G, epi_store(sc[1].dcf, c1->p, 0, D)))) return rc;
    if ((rc = conv3x3(ctx, sc[1].c3, c1->as<__half>(), F, 2 * G, outs[1], colp))) return rc;
  }
  // scale 2: 1x1 (E->D) -> 3x3  (1x)
  {
    CKG(gemm(ctx, xh, hp.vit_embed_dim, sc[2].c1, T, epi_store(sc[2].c1, c1->p, 0, D)));
    if ((rc = conv3x3(ctx, sc[2].c3, c1->as<__half>(), F, G, outs[2], colp))) return rc;
  }
  // scale 3: maxpool 2x2 -> 1x1 -> 3x3  (0.5x)
  {
    CK(maxpool2_cl_f16(xh, F, G, G, hp.vit_embed_dim, mp->as<__half>(), ctx->stream));
    CKG(gemm(ctx, mp->as<__half>(), hp.vit_embed_dim, sc[3].c1, T / 4, epi_store(sc[3].c1, c1->p, 0, D)));
    if ((rc = conv3x3(ctx, sc[3].c3, c1->as<__half>(), F, G / 2, outs[3], colp))) return rc;
  }
  return kOk;
}

int vit_encode(s3b_ctx* ctx, const float* d_chw, int n_frames, int flags, const uint8_t* d_u8) {
  Model& M = ctx->model;
  const HParams& hp = M.hp;
  const int E = hp.vit_embed_dim, G = hp.n_img_embd(), P = hp.patch_size, S = hp.img_size;
  const long long tok_per_frame = (long long)G * G;
  int rc = 0;
  Outputs& O = ctx->out;
  const bool want_neck = !(flags & 1) && M.has_neck_trk && ctx->stop_after_blocks < 0;
  const bool want_det = want_neck && M.has_neck_det && !(flags & 2);
  // outputs
  if (O.n_frames != n_frames || O.img_size != S || !O.backbone) {
    O = Outputs();
    O.n_frames = n_frames;
    O.img_size = S;
    O.backbone = std::make_shared<DevBuf>();
    if (O.backbone->reserve((size_t)n_frames * tok_per_frame * E * 4)) return set_error(ctx, kErrOOM, "out alloc");
  }
  const int sizes[4] = {4 * G, 2 * G, G, G / 2};
  if (want_neck) {
    O.n_fpn = 4;
    for (int i = 0; i < 4; ++i) {
      O.fpn_size[i] = sizes[i];
      if (!O.fpn[i]) O.fpn[i] = std::make_shared<DevBuf>();
      if (O.fpn[i]->reserve((size_t)n_frames * sizes[i] * sizes[i] * hp.neck_dim * 4))
        return set_error(ctx, kErrOOM, "out alloc");
      if (want_det) {
        if (!O.det[i]) O.det[i] = std::make_shared<DevBuf>();
        if (O.det[i]->reserve((size_t)n_frames * sizes[i] * sizes[i] * hp.neck_dim * 4))
          return set_error(ctx, kErrOOM, "out alloc");
      }
    }
    O.n_det = want_det ? 4 : 0;
  }
  const int FB = ctx->max_frames_per_pass;
  // rows per frame in window order (>= G*G when the grid is padded to whole windows)
  const int nwv = (G + hp.vit_window_size - 1) / hp.vit_window_size;
  const long long win_per_frame = (long long)nwv * nwv * hp.vit_window_size * hp.vit_window_size;
  const long long Tmax = (long long)FB * (win_per_frame > tok_per_frame ? win_per_frame : tok_per_frame);
  const int Kp = M.patch.Kpad;
  DevBuf* col = ctx->buf("vit_col", (size_t)Tmax * Kp * 2, &rc);
  DevBuf* xp = ctx->buf("vit_xp", (size_t)Tmax * E * 4, &rc);
  DevBuf* xn = ctx->buf("vit_xn", (size_t)Tmax * E * 2, &rc);
  DevBuf* qkv = ctx->buf("vit_qkv", (size_t)Tmax * 3 * E * 2, &rc);
  DevBuf* ao = ctx->buf("vit_ao", (size_t)Tmax * E * 2, &rc);
  DevBuf* hb = ctx->buf("vit_h", (size_t)Tmax * hp.vit_mlp_dim * 2, &rc);
  if (rc) return rc;
  // Passes of at most FB frames. The blocks run layer-major: block b on every pass, then block b + 1,
  // so each block's block-form weights are staged once per call and stay hot in L2 across the passes.
  const int n_pass = (n_frames + FB - 1) / FB;
  const bool bound_backbone = ctx->host_bind.count("vit_output") || ctx->host_bind.count("backbone");
  auto pass_frames = [&](int p) { return (n_frames - p * FB) < FB ? (n_frames - p * FB) : FB; };
  auto pass_x = [&](int p) { return O.backbone->as<float>() + (size_t)p * FB * tok_per_frame * E; };
  for (int p = 0; p < n_pass; ++p) {
    const int f0 = p * FB, F = pass_frames(p);
    const long long T = (long long)F * tok_per_frame;
    if (bound_backbone && (rc = outputs_pass_begin(ctx, p, FB))) return rc;
    // patch embed (conv 14x14/s14, no bias) + tiled abs pos (sam3.cpp:3815-3822)
    if (d_u8)
      CK(patch_cols_u8(d_u8 + (size_t)f0 * S * S * 3, F, S, S, kMeanSam3, kStdSam3, P, P, 0, G, G, col->as<__half>(), Kp,
                       ctx->stream));
    else
      CK(patch_cols_f32(d_chw + (size_t)f0 * 3 * S * S, F, 3, S, S, P, P, 0, G, G, col->as<__half>(), Kp, ctx->stream));
    EpiParams pe = epi_store(M.patch, xp->p, 1, E);
    pe.resid = M.pos_tiled->as<float>();
    pe.ldr = E;
    pe.resid_mod = tok_per_frame;
    pe.resid_wrap_pad = 1;
    CKG(gemm(ctx, col->as<__half>(), Kp, M.patch, T, pe));
    // ln_pre (sam3.cpp:3825-3827)
    RowMap id;
    CK(run_ln(ctx, xp->as<float>(), E, pass_x(p), 1, E, T, E, M.ln_pre_w.ptr(), M.ln_pre_b.ptr(), 1e-5f, id));
  }
  // stage runner (test hook, like sam3_test_run_vit_block_stage): stop after `stop_after_blocks`
  const int n_blocks = ctx->stop_after_blocks >= 0 && ctx->stop_after_blocks < hp.vit_depth
                           ? ctx->stop_after_blocks
                           : hp.vit_depth;
  for (int b = 0; b < n_blocks; ++b) {
    VitBlock Bs = M.vit[b];
    const Linear* in[4] = {&M.vit[b].qkv, &M.vit[b].proj, &M.vit[b].fc1, &M.vit[b].fc2};
    Linear* outl[4] = {&Bs.qkv, &Bs.proj, &Bs.fc1, &Bs.fc2};
    if ((rc = stage_linears(ctx, in, outl, 4))) return rc;
    for (int p = 0; p < n_pass; ++p) {
      if ((rc = vit_block(ctx, Bs, pass_frames(p), pass_x(p), xn->as<__half>(), qkv->as<__half>(), ao->as<__half>(),
                          hb->as<__half>())))
        return rc;
    }
  }
  for (int p = 0; p < n_pass; ++p) {
    const int f0 = p * FB, F = pass_frames(p);
    const long long T = (long long)F * tok_per_frame;
    if (!bound_backbone && (rc = outputs_pass_begin(ctx, p, FB))) return rc;
    if (want_neck) {
      // neck input in f16 (ggml converts the conv input to the f16 kernel type)
      __half* xh = xn->as<__half>();
      CK(cast_f32_f16(pass_x(p), T * E, xh, ctx->stream));
      float* outs[4];
      for (int i = 0; i < 4; ++i) outs[i] = O.fpn[i]->as<float>() + (size_t)f0 * sizes[i] * sizes[i] * hp.neck_dim;
      if ((rc = vit_neck(ctx, M.neck_trk, xh, F, outs))) return rc;
      if (want_det) {
        for (int i = 0; i < 4; ++i) outs[i] = O.det[i]->as<float>() + (size_t)f0 * sizes[i] * sizes[i] * hp.neck_dim;
        if ((rc = vit_neck(ctx, M.neck_det, xh, F, outs))) return rc;
      }
    }
    if ((rc = outputs_pass_end(ctx, p, f0, F))) return rc;
  }
  return check_device(ctx, "vit_encode");
}

}  // namespace s3b
