// Launch helpers shared by the encoders: launch accounting and optional
// CUDA-event timing of each GEMM / attention launch on the context stream.
#include <algorithm>

#include "engine.h"

cudaEvent_t s3b_ctx::next_event() {
  if (event_next == event_pool.size()) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    event_pool.push_back(e);
  }
  return event_pool[event_next++];
}

namespace s3b {

void rope_position_major(const std::vector<float>& in, int npos, int half_d, std::vector<float>& out) {
  out.resize((size_t)npos * half_d * 2);
  for (int p = 0; p < npos; ++p)
    for (int i = 0; i < half_d; ++i) {
      out[((size_t)i * npos + p) * 2] = in[((size_t)p * half_d + i) * 2];
      out[((size_t)i * npos + p) * 2 + 1] = in[((size_t)p * half_d + i) * 2 + 1];
    }
}

void count_launch(s3b_ctx* ctx, int n) { ctx->n_launches += n; }

int upload_sync(s3b_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess ||
      cudaStreamSynchronize(ctx->stream) != cudaSuccess)
    return set_error(ctx, kErrCuda, "upload of %zu bytes failed: %s", bytes, cudaGetErrorString(cudaGetLastError()));
  return kOk;
}

EpiParams epi_store(const Linear& L, void* out, int out_f32, long long ldo, int act) {
  EpiParams ep;
  ep.mode = EPI_STORE;
  ep.bias = L.b ? L.b->as<float>() : nullptr;
  ep.out = out;
  ep.out_f32 = out_f32;
  ep.ldo = ldo;
  ep.act = act;
  return ep;
}

int run_gemm(s3b_ctx* ctx, const __half* A, long long lda, const Linear& L, long long M, const EpiParams& ep) {
  cudaEvent_t a = nullptr, b = nullptr;
  if (ctx->prof) {
    a = ctx->next_event();
    b = ctx->next_event();
    cudaEventRecord(a, ctx->stream);
  }
  int rc;
  if (L.staged) {
    // block-form weight staged in f16 for this block / layer (stage_linears)
    rc = gemm_f16(A, lda, L.staged, L.K, (int)M, L.N, L.K, ep, ctx->d_err, ctx->stream);
  } else if (L.qtype) {
    QWeight qw;
    qw.type = L.qtype;
    qw.values = L.qv->p;
    qw.scales = L.qs->as<__half>();
    if (ctx->weights_quantised == 2) {
      rc = gemm_q(A, lda, qw, (int)M, L.N, L.K, ep, ctx->d_err, ctx->stream);
    } else {
      // a block-form weight outside a staged group: read from HBM in block form once and written as
      // f16 into its own staging buffer, which the GEMM then reads from L2 across its tile sweep
      const auto it = ctx->ws.find("wq_stage1");
      if (it == ctx->ws.end() || !it->second || it->second->bytes < (size_t)L.N * L.K * 2)
        return set_error(ctx, kErrState, "no staging buffer for block-form weights (model not loaded with it)");
      __half* stage = it->second->as<__half>();
      cudaEvent_t da = nullptr, db = nullptr;
      if (ctx->prof) {
        da = ctx->next_event();
        db = ctx->next_event();
        cudaEventRecord(da, ctx->stream);
      }
      rc = dequant_planes_f16(qw, L.N, L.K, stage, L.K, ctx->stream);
      count_launch(ctx);
      if (rc) return set_error(ctx, launcher_status_code(rc), "weight staging N=%d K=%d failed (%d)", L.N, L.K, rc);
      if (ctx->prof) {
        cudaEventRecord(db, ctx->stream);
        const double qbytes = L.qtype == QT_Q4_0 ? L.N * (L.K / 2.0 + L.K / 16.0) : L.N * (L.K + L.K / 16.0);
        ctx->prof_entries.push_back({3, 0.0, qbytes + 2.0 * L.N * L.K, da, db});
      }
      if (ctx->prof) cudaEventRecord(a, ctx->stream);  // the GEMM's own time starts after the staging
      rc = gemm_f16(A, lda, stage, L.K, (int)M, L.N, L.K, ep, ctx->d_err, ctx->stream);
    }
  } else {
    rc = gemm_f16(A, lda, L.w->as<__half>(), L.Kpad, (int)M, L.N, L.Kpad, ep, ctx->d_err, ctx->stream);
  }
  count_launch(ctx);
  if (rc) return set_error(ctx, launcher_status_code(rc), "gemm M=%lld N=%d K=%d failed (%d)", M, L.N, L.Kpad, rc);
  if (ctx->prof) {
    cudaEventRecord(b, ctx->stream);
    // algorithmic work: 2*M*N*K flops; bytes: A + B (f16, or the block values + f16 scales) + output
    const double wbytes = L.qtype == QT_Q4_0   ? L.N * (L.K / 2.0 + L.K / 16.0)
                          : L.qtype == QT_Q8_0 ? L.N * (L.K + L.K / 16.0)
                                               : 2.0 * L.N * L.K;
    const double bytes = 2.0 * M * L.K + wbytes + (ep.out_f32 ? 4.0 : 2.0) * M * L.N;
    ctx->prof_entries.push_back({0, 2.0 * M * L.N * L.K, bytes, a, b});
  }
  return kOk;
}

size_t stage_arena_elems(const Model& M) {
  auto q = [](const Linear& L) -> size_t { return L.qtype ? (size_t)L.N * L.K : 0; };
  size_t best = M.qstage_elems;
  for (const VitBlock& B : M.vit) best = std::max(best, q(B.qkv) + q(B.proj) + q(B.fc1) + q(B.fc2));
  for (const HieraBlock& B : M.hiera)
    best = std::max(best, q(B.qkv) + q(B.proj) + q(B.fc1) + q(B.fc2) + q(B.dim_proj));
  for (const MemAttnLayer& L : M.mem)
    best = std::max(best, q(L.sa_qkv) + q(L.sa_out) + q(L.ca_q) + q(L.ca_k) + q(L.ca_v) + q(L.ca_out) + q(L.fc1) +
                              q(L.fc2));
  // every region starts on a 256-byte boundary
  return best ? best + 128 * kMaxStageJobs : 0;
}

int stage_linears(s3b_ctx* ctx, const Linear* const* in, Linear* const* out, int n) {
  StageJob jobs[kMaxStageJobs];
  int nj = 0;
  size_t off = 0;
  DevBuf* arena = nullptr;
  for (int i = 0; i < n; ++i) {
    *out[i] = *in[i];
    out[i]->staged = nullptr;
    const Linear& L = *in[i];
    if (!L.qtype || ctx->weights_quantised == 2) continue;
    if (!arena) {
      const auto it = ctx->ws.find("wq_stage");
      if (it == ctx->ws.end() || !it->second) return set_error(ctx, kErrState, "no staging arena for block-form weights");
      arena = it->second.get();
    }
    if (nj == kMaxStageJobs) return set_error(ctx, kErrArg, "more than %d weights staged at once", kMaxStageJobs);
    const size_t elems = (size_t)L.N * L.K;
    if ((off + elems) * 2 > arena->bytes) return set_error(ctx, kErrState, "staging arena too small");
    __half* dst = arena->as<__half>() + off;
    off += (elems + 127) / 128 * 128;
    jobs[nj].w.type = L.qtype;
    jobs[nj].w.values = L.qv->p;
    jobs[nj].w.scales = L.qs->as<__half>();
    jobs[nj].N = L.N;
    jobs[nj].K = L.K;
    jobs[nj].out = dst;
    ++nj;
    out[i]->staged = dst;
  }
  if (!nj) return kOk;
  cudaEvent_t a = nullptr, b = nullptr;
  if (ctx->prof) {
    a = ctx->next_event();
    b = ctx->next_event();
    cudaEventRecord(a, ctx->stream);
  }
  const int rc = dequant_planes_multi(jobs, nj, ctx->stream);
  count_launch(ctx);
  if (rc) return set_error(ctx, launcher_status_code(rc), "weight staging failed (%d)", rc);
  if (ctx->prof) {
    cudaEventRecord(b, ctx->stream);
    double bytes = 0;
    for (int j = 0; j < nj; ++j) {
      const double nk = (double)jobs[j].N * jobs[j].K;
      bytes += (jobs[j].w.type == QT_Q4_0 ? nk * (0.5 + 1.0 / 16) : nk * (1.0 + 1.0 / 16)) + 2.0 * nk;
    }
    ctx->prof_entries.push_back({3, 0.0, bytes, a, b});
  }
  return kOk;
}

// 3x3 / pad 1 conv of a channel-last f16 map as an implicit GEMM when the option and the shapes allow,
// else im2col into `col` + GEMM. Counted and timed as a GEMM (algorithmic flops 2*pixels*N*9C).
int run_conv3x3(s3b_ctx* ctx, const Linear& L, const __half* x, int F, int H, int W, const EpiParams& ep,
                __half* col) {
  const int C = L.K / 9;
  const long long M = (long long)F * H * W;
  if (ctx->conv_implicit && L.Kpad == L.K && C % 64 == 0) {
    cudaEvent_t a = nullptr, b = nullptr;
    if (ctx->prof) {
      a = ctx->next_event();
      b = ctx->next_event();
      cudaEventRecord(a, ctx->stream);
    }
    const int rc = gemm_conv3x3(x, F, H, W, C, L.w->as<__half>(), L.Kpad, L.N, ep, ctx->d_err, ctx->stream);
    if (rc != -2) {
      count_launch(ctx);
      if (rc) return set_error(ctx, launcher_status_code(rc), "implicit conv3x3 failed (%d)", rc);
      if (ctx->prof) {
        cudaEventRecord(b, ctx->stream);
        const double bytes = 2.0 * M * C + 2.0 * L.N * L.K + (ep.out_f32 ? 4.0 : 2.0) * M * L.N;
        ctx->prof_entries.push_back({0, 2.0 * M * L.N * L.K, bytes, a, b});
      }
      return kOk;
    }
  }
  if (!col) return set_error(ctx, kErrArg, "conv3x3: no column workspace for the im2col path");
  int rc = im2col_3x3_cl(x, F, H, W, C, col, ctx->stream);
  count_launch(ctx);
  if (rc) return set_error(ctx, kErrCuda, "im2col_3x3 failed (%d)", rc);
  return run_gemm(ctx, col, L.Kpad, L, M, ep);
}

// 2x2 / stride 2 deconvolution of a channel-last f16 map [F][H][W][Cin] into [F][2H][2W][cout]
// (cout = L.N / 4): pixel-block GEMM with 5-D TMA output stores when the option and the shapes
// allow, else the GEMM with scattered 16-value stores (EPI_DECONV2). Counted and timed as a GEMM.
int run_deconv2x2(s3b_ctx* ctx, const Linear& L, const __half* x, int F, int H, int W, EpiParams ep) {
  const int cout = L.N / 4;
  const long long M = (long long)F * H * W;
  if (ctx->conv_implicit && L.Kpad == L.K) {
    cudaEvent_t a = nullptr, b = nullptr;
    if (ctx->prof) {
      a = ctx->next_event();
      b = ctx->next_event();
      cudaEventRecord(a, ctx->stream);
    }
    const int rc = gemm_deconv2x2(x, F, H, W, L.K, L.w->as<__half>(), L.Kpad, cout, ep, ctx->d_err, ctx->stream);
    if (rc != -2) {
      count_launch(ctx);
      if (rc) return set_error(ctx, launcher_status_code(rc), "deconv2x2 failed (%d)", rc);
      if (ctx->prof) {
        cudaEventRecord(b, ctx->stream);
        const double bytes = 2.0 * M * L.K + 2.0 * L.N * L.K + (ep.out_f32 ? 4.0 : 2.0) * M * L.N;
        ctx->prof_entries.push_back({0, 2.0 * M * L.N * L.K, bytes, a, b});
      }
      return kOk;
    }
  }
  ep.mode = EPI_DECONV2;
  ep.cout = cout;
  ep.map.W = W;
  ep.map.H = H;
  return run_gemm(ctx, x, L.Kpad, L, M, ep);
}

// LayerNorm (HBM-bound): algorithmic bytes = f32 rows in + rows out (f16 / f32) + gamma, beta.
int run_ln(s3b_ctx* ctx, const float* x, long long ldx, void* y, int y_f32, long long ldy, long long rows, int C,
           const float* g, const float* b, float eps, const RowMap& map) {
  cudaEvent_t ea = nullptr, eb = nullptr;
  if (ctx->prof) {
    ea = ctx->next_event();
    eb = ctx->next_event();
    cudaEventRecord(ea, ctx->stream);
  }
  const int rc = layernorm(x, ldx, y, y_f32, ldy, rows, C, g, b, eps, map, ctx->stream);
  if (!rc && ctx->prof) {
    cudaEventRecord(eb, ctx->stream);
    const double bytes = (4.0 + (y_f32 ? 4.0 : 2.0)) * rows * C + 8.0 * C;
    ctx->prof_entries.push_back({2, 0.0, bytes, ea, eb});
  }
  return rc;
}

int run_attn(s3b_ctx* ctx, const AttnParams& p, int D, int batch_heads) {
  cudaEvent_t a = nullptr, b = nullptr;
  if (ctx->prof) {
    a = ctx->next_event();
    b = ctx->next_event();
    cudaEventRecord(a, ctx->stream);
  }
  // the tcgen05 kernel serves d = 64 attention over one fused qkv buffer (the ViT blocks)
  const long long kq = p.k - p.q, vq = p.v - p.q;
  const bool tc_ok = (ctx->attention_impl == 0 || ctx->attention_impl == 3 || ctx->attention_impl == 4) && D == 64 &&
                     p.nq == p.nk && p.q_n == p.k_n && p.q_n == p.v_n &&
                     p.q_b == p.k_b && p.q_b == p.v_b && p.q_b == (long long)p.nq * p.q_n && p.q_h == 64 &&
                     p.k_h == 64 && p.v_h == 64 && kq > 0 && vq > 0 && kq + 64LL * p.heads <= p.q_n &&
                     vq + 64LL * p.heads <= p.q_n && batch_heads % p.heads == 0;
  int rc;
  // d = 64: the persistent two-tile kernel (measured faster than the one-tile-per-CTA kernel for the
  // ViT windows, 499 against 408 TF/s, and for the global rows, 680 against 667 TF/s); attention_impl 3
  // selects the one-tile kernel
  const bool fa = tc_ok && (ctx->attention_impl == 4 || ctx->attention_impl == 0);
  if (fa) {
    rc = attention_fa64(p.q, p.q_n, 0, (int)kq, (int)vq, p.heads, p.nq, batch_heads / p.heads, p.o, p.o_n, p.omap,
                        p.scale, ctx->attention_fa_exp_poly, ctx->d_err, ctx->stream);
  } else if (tc_ok) {
    rc = attention_tc64(p.q, p.q_n, 0, (int)kq, (int)vq, p.heads, p.nq, batch_heads / p.heads, p.o, p.o_n, p.omap,
                        p.scale, ctx->attention_exp_poly, 1, ctx->d_err,
                        ctx->stream);
  } else {
    // d = 256 (memory attention) and d = 72 / 96 (Hiera) with at least one full query tile on the
    // tcgen05 kernel when its layout rules hold, else mma.sync
    rc = -2;
    if (ctx->attention_impl != 1 &&
        (D == 256 || ((D == 72 || D == 96 || (D == 64 && ctx->attention_impl == 2)) && p.nq >= 128))) {
      // workspace for key splits (used when the query tiles leave SMs idle)
      const long long units = (long long)((p.nq + 127) / 128) * batch_heads;
      const int max_split = attention_wide_max_split(D, units);
      float* ws = nullptr;
      size_t ws_bytes = 0;
      if (max_split > 1) {
        ws_bytes = attention_wide_ws_bytes(D, max_split, batch_heads, p.nq);
        int brc = 0;
        DevBuf* buf = ctx->buf("attn_wide_split", ws_bytes, &brc);
        if (brc) return brc;
        ws = buf->as<float>();
      }
      // d = 72 / 96: 128-key tiles for long rows (the Hiera global blocks: 4096 keys, measured 560 -> 674
      // TF/s at d = 96, 410 -> 449 at d = 72), 64-key tiles and two CTAs per SM for the windows (196 / 256
      // keys: 208 against 140 TF/s at d = 96)
      const int k128 = ctx->attention_wide_k128 >= 0 ? ctx->attention_wide_k128 : (p.nk >= 1024 ? 1 : 0);
      rc = attention_wide(p, D, batch_heads, ws, ws_bytes, k128, ctx->d_err, ctx->stream);
    }
    if (rc == -2) rc = attention(p, D, batch_heads, ctx->stream);
  }
  count_launch(ctx);
  if (rc) return set_error(ctx, launcher_status_code(rc), "attention D=%d failed (%d)", D, rc);
  if (ctx->prof) {
    cudaEventRecord(b, ctx->stream);
    const double flops = 4.0 * p.nq * (double)p.nk * D * batch_heads;
    const double bytes = 2.0 * batch_heads * D * (2.0 * p.nq + 2.0 * p.nk);
    ctx->prof_entries.push_back({1, flops, bytes, a, b});
  }
  return kOk;
}

}  // namespace s3b
