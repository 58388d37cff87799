// SAM 2 / 2.1 image encoder on B200: Hiera backbone + FPN neck (host
// orchestration, C++14). Replaces sam2_build_hiera_graph (sam3.cpp:4462-4527),
// sam2_hiera_block_forward (4295-4457), sam2_build_fpn_neck_graph (4532-4603)
// and the per-frame host PE of sam2_encode_image_hiera (5857-6018).
//
// Layout: channel-last token maps [frames][S][S][C] (ggml [C, W, H, B]); the
// residual stream is f32, GEMM / attention operands f16. Window partition
// with its zero padding is folded into the LayerNorm row gather; Q pooling
// inside windows is one strided kernel; the window unpartition (ws, or ws/2
// after pooling) is the attention kernel's output row map; residuals are
// added in place by the projection / fc2 epilogues.
#include <math.h>
#include <string.h>

#include <algorithm>

#include "engine.h"

namespace s3b {

#define CKH(call)                                                                                          \
  do {                                                                                                     \
    int _rc = (call);                                                                                      \
    count_launch(ctx);                                                                                     \
    if (_rc) return set_error(ctx, launcher_status_code(_rc), "%s failed (%d)", #call, _rc);          \
  } while (0)
#define CKR(call)        \
  do {                   \
    int _rc = (call);    \
    if (_rc) return _rc; \
  } while (0)

namespace {

struct BlockGeom {
  int S = 0, S2 = 0;        // input / output spatial size
  int ws = 0, ws_eff = 0;   // window (0 = global) and the grid the attention sees
  int nw = 1;               // windows per side
  long long ntok = 0, ntok_q = 0;
  RowMap wmap, omap;
};

BlockGeom geom(const HieraBlock& B, int S) {
  BlockGeom g;
  g.S = S;
  g.S2 = B.q_stride ? S / 2 : S;
  g.ws = B.window;
  if (B.window > 0) {
    g.ws_eff = B.window;
    g.nw = (S + B.window - 1) / B.window;
    g.wmap.kind = 1;
    g.wmap.ws = B.window;
    g.wmap.nww = g.wmap.nwh = g.nw;
    g.wmap.W = g.wmap.H = S;
    if (B.q_stride) {
      // unpartition after pooling: windows of ws/2 over the halved grid (sam3.cpp:4414-4430)
      g.omap.kind = 1;
      g.omap.ws = B.window / 2;
      g.omap.nww = g.omap.nwh = g.nw;
      g.omap.W = g.omap.H = g.S2;
    } else {
      g.omap = g.wmap;
    }
  } else {
    g.ws_eff = S;
    g.nw = 1;
  }
  g.ntok = (long long)g.ws_eff * g.ws_eff;
  g.ntok_q = B.q_stride ? (long long)(g.ws_eff / 2) * (g.ws_eff / 2) : g.ntok;
  return g;
}

}  // namespace

static int hiera_block(s3b_ctx* ctx, const HieraBlock& B0, int F, int S, float* x, float* xalt, float** x_out,
                       __half* xn, __half* xw, __half* qkv, __half* qp, __half* ao, __half* hbuf, float* tmp) {
  // block-form weights of the block staged in f16 in one launch (weights_quantised = 1)
  HieraBlock B = B0;
  {
    const Linear* in[5] = {&B0.qkv, &B0.proj, &B0.fc1, &B0.fc2, &B0.dim_proj};
    Linear* outl[5] = {&B.qkv, &B.proj, &B.fc1, &B.fc2, &B.dim_proj};
    const int rc = stage_linears(ctx, in, outl, 5);
    if (rc) return rc;
  }
  const BlockGeom g = geom(B, S);
  const int din = B.dim_in, dout = B.dim_out, hd = dout / B.heads;
  const long long T = (long long)F * S * S, T2 = (long long)F * g.S2 * g.S2;
  const long long nwin = (long long)F * g.nw * g.nw, Tw = nwin * g.ntok;
  RowMap id;
  // shortcut (sam3.cpp:4312-4327): dim projection of the normed input and/or 2x2 max pool
  float* xnew = x;
  if (din != dout) {
    CKH(run_ln(ctx, x, din, xn, 0, din, T, din, B.n1w.ptr(), B.n1b.ptr(), 1e-6f, id));
    xnew = xalt;
    if (B.q_stride) {
      CKR(run_gemm(ctx, xn, din, B.dim_proj, T, epi_store(B.dim_proj, tmp, 1, dout)));
      CKH(maxpool2_cl_f32(tmp, F, S, S, dout, xnew, ctx->stream));
    } else {
      CKR(run_gemm(ctx, xn, din, B.dim_proj, T, epi_store(B.dim_proj, xnew, 1, dout)));
    }
  } else if (B.q_stride) {
    xnew = xalt;
    CKH(maxpool2_cl_f32(x, F, S, S, dout, xnew, ctx->stream));
  }
  // norm1 + zero-padded window partition (sam3.cpp:4306-4337)
  CKH(run_ln(ctx, x, din, xw, 0, din, Tw, din, B.n1w.ptr(), B.n1b.ptr(), 1e-6f, g.wmap));
  // qkv (sam3.cpp:4344-4357)
  CKR(run_gemm(ctx, xw, din, B.qkv, Tw, epi_store(B.qkv, qkv, 0, 3LL * dout)));
  AttnParams a;
  if (B.q_stride) {
    // Q max-pooled inside each window (sam3.cpp:4363-4371)
    CKH(qpool_windows(qkv, 3LL * dout, nwin, g.ws_eff, dout, qp, ctx->stream));
    a.q = qp;
    a.q_n = dout;
    a.q_b = g.ntok_q * dout;
  } else {
    a.q = qkv;
    a.q_n = 3LL * dout;
    a.q_b = g.ntok * 3 * dout;
  }
  a.q_h = hd;
  a.k = qkv + dout;
  a.v = qkv + 2 * dout;
  a.k_n = a.v_n = 3LL * dout;
  a.k_h = a.v_h = hd;
  a.k_b = a.v_b = g.ntok * 3 * dout;
  a.heads = B.heads;
  a.nq = (int)g.ntok_q;
  a.nk = (int)g.ntok;
  a.o = ao;
  a.o_n = dout;
  a.omap = g.omap;  // window unpartition (and crop of padding) on the way out
  a.scale = 1.0f / sqrtf((float)hd);
  CKR(run_attn(ctx, a, hd, (int)(nwin * B.heads)));
  // proj + bias + residual (sam3.cpp:4401-4436)
  EpiParams pr = epi_store(B.proj, xnew, 1, dout);
  pr.resid = xnew;
  pr.ldr = dout;
  CKR(run_gemm(ctx, ao, dout, B.proj, T2, pr));
  // MLP with tanh GELU + residual (sam3.cpp:4440-4454)
  CKH(run_ln(ctx, xnew, dout, xn, 0, dout, T2, dout, B.n2w.ptr(), B.n2b.ptr(), 1e-6f, id));
  CKR(run_gemm(ctx, xn, dout, B.fc1, T2, epi_store(B.fc1, hbuf, 0, 4LL * dout, ACT_GELU_TANH)));
  EpiParams f2 = epi_store(B.fc2, xnew, 1, dout);
  f2.resid = xnew;
  f2.ldr = dout;
  CKR(run_gemm(ctx, hbuf, 4LL * dout, B.fc2, T2, f2));
  *x_out = xnew;
  return kOk;
}

int hiera_encode(s3b_ctx* ctx, const float* d_chw, int n_frames, int flags, const uint8_t* d_u8) {
  Model& M = ctx->model;
  const HParams& hp = M.hp;
  const int E0 = hp.hiera_embed_dim, S0 = hp.img_size / 4, img = hp.img_size;
  if (!M.hiera_pe || M.hiera_pe_size != S0) return set_error(ctx, kErrState, "Hiera PE not prepared");
  int rc = 0;
  Outputs& O = ctx->out;
  const bool want_neck = !(flags & 1) && ctx->stop_after_blocks < 0;
  const int n_out = 4 - hp.scalp;
  if (O.n_frames != n_frames || O.img_size != img) {
    O = Outputs();
    O.n_frames = n_frames;
    O.img_size = img;
  }
  O.backbone_c = 0;
  O.n_fpn = n_out;
  for (int i = 0; i < n_out; ++i) {
    O.fpn_size[i] = S0 >> i;
    if (!O.fpn[i]) O.fpn[i] = std::make_shared<DevBuf>();
    if (O.fpn[i]->reserve((size_t)n_frames * O.fpn_size[i] * O.fpn_size[i] * hp.neck_dim * 4))
      return set_error(ctx, kErrOOM, "out alloc");
  }
  // workspace sizes: the largest per-frame footprint over all blocks
  const int FB = ctx->max_frames_per_pass;
  long long mx_x = (long long)S0 * S0 * E0, mx_xw = 0, mx_qkv = 0, mx_qp = 0, mx_h = 0, mx_tmp = 0, mx_ao = 0;
  long long stage_sz[4] = {0, 0, 0, 0};
  {
    int S = S0, st = 0;
    for (size_t i = 0; i < M.hiera.size(); ++i) {
      const HieraBlock& B = M.hiera[i];
      const BlockGeom g = geom(B, S);
      const long long nwin = (long long)g.nw * g.nw, Tw = nwin * g.ntok;
      mx_x = std::max(mx_x, (long long)S * S * std::max(B.dim_in, B.dim_out));
      mx_xw = std::max(mx_xw, std::max(Tw, (long long)S * S) * B.dim_in);
      mx_qkv = std::max(mx_qkv, Tw * 3 * B.dim_out);
      mx_qp = std::max(mx_qp, nwin * g.ntok_q * B.dim_out);
      mx_ao = std::max(mx_ao, (long long)g.S2 * g.S2 * B.dim_out);
      mx_h = std::max(mx_h, (long long)g.S2 * g.S2 * 4 * B.dim_out);
      mx_tmp = std::max(mx_tmp, (long long)S * S * B.dim_out);
      S = g.S2;
      if ((int)i == M.stage_ends[st]) stage_sz[st++] = (long long)S * S * B.dim_out;
    }
  }
  const int Kp = M.hpatch.Kpad;
  DevBuf* col = ctx->buf("hi_col", (size_t)FB * S0 * S0 * Kp * 2, &rc);
  DevBuf* xa = ctx->buf("hi_xa", (size_t)FB * mx_x * 4, &rc);
  DevBuf* xb = ctx->buf("hi_xb", (size_t)FB * mx_x * 4, &rc);
  DevBuf* xn = ctx->buf("hi_xn", (size_t)FB * mx_xw * 2, &rc);
  DevBuf* xw = ctx->buf("hi_xw", (size_t)FB * mx_xw * 2, &rc);
  DevBuf* qkv = ctx->buf("hi_qkv", (size_t)FB * mx_qkv * 2, &rc);
  DevBuf* qp = ctx->buf("hi_qp", (size_t)FB * mx_qp * 2, &rc);
  DevBuf* ao = ctx->buf("hi_ao", (size_t)FB * mx_ao * 2, &rc);
  DevBuf* hb = ctx->buf("hi_h", (size_t)FB * mx_h * 2, &rc);
  DevBuf* tmp = ctx->buf("hi_tmp", (size_t)FB * mx_tmp * 4, &rc);
  DevBuf* stg[4];
  for (int s = 0; s < 4; ++s) stg[s] = ctx->buf("hi_stage" + std::to_string(s), (size_t)FB * stage_sz[s] * 2, &rc);
  DevBuf* lat3 = ctx->buf("hi_lat3", (size_t)FB * (S0 >> 3) * (S0 >> 3) * hp.neck_dim * 4, &rc);
  if (rc) return rc;

  for (int f0 = 0; f0 < n_frames; f0 += FB) {
    const int F = (n_frames - f0) < FB ? (n_frames - f0) : FB;
    const long long T0 = (long long)F * S0 * S0;
    if ((rc = outputs_pass_begin(ctx, f0 / FB, FB))) return rc;
    // patch embed: conv 7x7 / s4 / p3 + bias, + PE (sam3.cpp:4469-4490)
    if (d_u8)
      CKH(patch_cols_u8(d_u8 + (size_t)f0 * img * img * 3, F, img, img, kMeanSam2, kStdSam2, 7, 4, 3, S0, S0,
                        col->as<__half>(), Kp, ctx->stream));
    else
      CKH(patch_cols_f32(d_chw + (size_t)f0 * 3 * img * img, F, 3, img, img, 7, 4, 3, S0, S0, col->as<__half>(), Kp,
                         ctx->stream));
    EpiParams pe = epi_store(M.hpatch, xa->p, 1, E0);
    pe.resid = M.hiera_pe->as<float>();
    pe.ldr = E0;
    pe.resid_mod = (long long)S0 * S0;
    CKR(run_gemm(ctx, col->as<__half>(), Kp, M.hpatch, T0, pe));
    float* x = xa->as<float>();
    float* other = xb->as<float>();
    int S = S0, st = 0;
    const int n_blocks = ctx->stop_after_blocks >= 0 && ctx->stop_after_blocks < (int)M.hiera.size()
                             ? ctx->stop_after_blocks
                             : (int)M.hiera.size();
    for (int i = 0; i < n_blocks; ++i) {
      const HieraBlock& B = M.hiera[i];
      float* xo = nullptr;
      CKR(hiera_block(ctx, B, F, S, x, other, &xo, xn->as<__half>(), xw->as<__half>(), qkv->as<__half>(),
                      qp->as<__half>(), ao->as<__half>(), hb->as<__half>(), tmp->as<float>()));
      if (xo != x) std::swap(x, other);
      if (B.q_stride) S /= 2;
      if (i == M.stage_ends[st]) {
        // stage output -> f16 FPN input
        CKH(cast_f32_f16(x, (long long)F * S * S * B.dim_out, stg[st]->as<__half>(), ctx->stream));
        ++st;
      }
    }
    if (!want_neck) {
      // backbone state after `stop_after_blocks` blocks (stage-runner test hook), output "backbone"
      const int C = n_blocks ? M.hiera[n_blocks - 1].dim_out : E0;
      const long long per_frame = (long long)S * S * C;
      if (!O.backbone) O.backbone = std::make_shared<DevBuf>();
      if (O.backbone->reserve((size_t)n_frames * per_frame * 4)) return set_error(ctx, kErrOOM, "out alloc");
      O.backbone_c = C;
      O.backbone_s = S;
      if (cudaMemcpyAsync(O.backbone->as<float>() + (size_t)f0 * per_frame, x, (size_t)F * per_frame * 4,
                          cudaMemcpyDeviceToDevice, ctx->stream) != cudaSuccess)
        return set_error(ctx, kErrCuda, "backbone copy failed");
      CKR(outputs_pass_end(ctx, f0 / FB, f0, F));
      continue;
    }
    // FPN neck (sam3.cpp:4532-4603): lateral 1x1 convs, nearest 2x top-down adds, scalp
    const float* prev = nullptr;
    int prev_S = 0;
    for (int i = 3; i >= 0; --i) {
      const int Si = S0 >> i;
      const Linear& L = M.fpn[3 - i];
      float* dst = i < n_out ? O.fpn[i]->as<float>() + (size_t)f0 * Si * Si * hp.neck_dim : lat3->as<float>();
      bool td = false;
      for (int j = 0; j < hp.fpn_top_down_n && j < 4; ++j) td |= hp.fpn_top_down_levels[j] == i;
      EpiParams ep = epi_store(L, dst, 1, hp.neck_dim);
      if (td && prev) {
        ep.resid = prev;
        ep.ldr = hp.neck_dim;
        ep.resid_up = 1;
        ep.map.W = ep.map.H = Si;
        (void)prev_S;
      }
      CKR(run_gemm(ctx, stg[i]->as<__half>(), L.K, L, (long long)F * Si * Si, ep));
      if (td || !prev) {
        prev = dst;
        prev_S = Si;
      }
    }
    CKR(outputs_pass_end(ctx, f0 / FB, f0, F));
  }
  if (!want_neck) O.n_fpn = 0;
  return check_device(ctx, "hiera_encode");
}

}  // namespace s3b
