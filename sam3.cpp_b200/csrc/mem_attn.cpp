// Memory attention on B200 (host orchestration, C++14).
//
// Replaces sam3_build_mem_attn_graph (sam3.cpp:9224-9337) and its ggml
// compute inside sam3_propagate_single (sam3.cpp:11171-11453): per layer a
// single-head (d = 256) RoPE self-attention over the N = feat^2 current
// tokens, a RoPE cross-attention to the M memory tokens (K projected from
// prompt + prompt_pos, V from prompt; RoPE on the spatial keys only, their
// table repeated per memory slot), and a ReLU FFN, each pre-normed with a
// residual; a final LayerNorm. The RoPE table follows
// sam3_ensure_tracker_pe_caches (sam3.cpp:11126-11169) and is cached on the
// device per feature size.
#include <math.h>

#include <vector>

#include "engine.h"

namespace s3b {

#define CKL(call)                                                                                          \
  do {                                                                                                     \
    int _rc = (call);                                                                                      \
    count_launch(ctx);                                                                                     \
    if (_rc) return set_error(ctx, launcher_status_code(_rc), "%s failed (%d)", #call, _rc);          \
  } while (0)
#define CKR(call)           \
  do {                      \
    int _rc = (call);       \
    if (_rc) return _rc;    \
  } while (0)

// Axial RoPE table (sam3_compute_axial_cis, sam3.cpp:3555-3586) as [N][dim/2][2].
static void axial_cis(int dim, int end_x, int end_y, float theta, float scale, std::vector<float>& out) {
  const int q = dim / 4;
  std::vector<float> freqs(q);
  for (int i = 0; i < q; ++i) freqs[i] = 1.0f / powf(theta, (float)(i * 4) / (float)dim);
  const int N = end_x * end_y;
  out.assign((size_t)N * dim, 0.f);
  for (int idx = 0; idx < N; ++idx) {
    const float tx = (float)(idx % end_x) * scale, ty = (float)(idx / end_x) * scale;
    for (int i = 0; i < q; ++i) {
      out[(size_t)idx * dim + 2 * i] = cosf(tx * freqs[i]);
      out[(size_t)idx * dim + 2 * i + 1] = sinf(tx * freqs[i]);
      out[(size_t)idx * dim + 2 * q + 2 * i] = cosf(ty * freqs[i]);
      out[(size_t)idx * dim + 2 * q + 2 * i + 1] = sinf(ty * freqs[i]);
    }
  }
}

static const float* rope_table(s3b_ctx* ctx, int feat, int D, int* rc) {
  const std::string key = "ma_rope_" + std::to_string(feat) + "_" + std::to_string(D);
  auto it = ctx->ws.find(key);
  if (it != ctx->ws.end() && it->second) return it->second->as<float>();
  std::vector<float> t0, t;
  axial_cis(D, feat, feat, 10000.0f, 1.0f, t0);
  rope_position_major(t0, feat * feat, D / 2, t);
  DevBuf* b = ctx->buf(key, t.size() * 4, rc);
  if (*rc) return nullptr;
  if ((*rc = upload_sync(ctx, b->p, t.data(), t.size() * 4))) return nullptr;
  return b->as<float>();
}

// The layers of memory attention (sam3.cpp:9245-9327) on the context's work buffers: every launch
// reads and writes only buffers of the context and the model, so the sequence can be captured once
// and replayed.
struct MemAttnBufs {
  float* X;
  __half *XN, *qkv, *ao, *hb, *kvin, *pin, *kb, *vb;
  const float* rope;
  long long N, Mt, m_sp;
  int D, FFN;
};

static int mem_attn_layers(s3b_ctx* ctx, const MemAttnBufs& b) {
  const Model& M = ctx->model;
  const int D = b.D, FFN = b.FFN, MD = M.hp.mem_out_dim;
  const long long N = b.N, Mt = b.Mt, m_sp = b.m_sp;
  float* X = b.X;
  __half* XN = b.XN;
  const float* rope = b.rope;
  const float scale = 1.0f / sqrtf((float)D);
  RowMap id;
  for (size_t l = 0; l < M.mem.size(); ++l) {
    // block-form weights of the layer staged in f16 in one launch (weights_quantised = 1)
    const MemAttnLayer& L0 = M.mem[l];
    MemAttnLayer L = L0;
    const Linear* in[8] = {&L0.sa_qkv, &L0.sa_out, &L0.ca_q, &L0.ca_k, &L0.ca_v, &L0.ca_out, &L0.fc1, &L0.fc2};
    Linear* outl[8] = {&L.sa_qkv, &L.sa_out, &L.ca_q, &L.ca_k, &L.ca_v, &L.ca_out, &L.fc1, &L.fc2};
    CKR(stage_linears(ctx, in, outl, 8));
    // self-attention with RoPE on q and k (sam3.cpp:9247-9271)
    CKL(run_ln(ctx, X, D, XN, 0, D, N, D, L.n1w.ptr(), L.n1b.ptr(), 1e-5f, id));
    EpiParams e = epi_store(L.sa_qkv, (void*)b.qkv, 0, 3LL * D);
    e.rope = rope;
    e.rope_D = D;
    e.rope_cols = 2 * D;
    e.rope_rows = N;
    e.rope_mod = N;
    CKR(run_gemm(ctx, XN, D, L.sa_qkv, N, e));
    AttnParams a;
    a.q = b.qkv;
    a.k = a.q + D;
    a.v = a.q + 2 * D;
    a.q_n = a.k_n = a.v_n = 3LL * D;
    a.heads = 1;
    a.nq = a.nk = (int)N;
    a.o = b.ao;
    a.o_n = D;
    a.scale = scale;
    CKR(run_attn(ctx, a, D, 1));
    EpiParams r = epi_store(L.sa_out, X, 1, D);
    r.resid = X;
    r.ldr = D;
    CKR(run_gemm(ctx, b.ao, D, L.sa_out, N, r));
    // cross-attention to the memory (sam3.cpp:9274-9316)
    CKL(run_ln(ctx, X, D, XN, 0, D, N, D, L.n2w.ptr(), L.n2b.ptr(), 1e-5f, id));
    EpiParams eq = epi_store(L.ca_q, (void*)b.qkv, 0, D);
    eq.rope = rope;
    eq.rope_D = D;
    eq.rope_cols = D;
    eq.rope_rows = N;
    eq.rope_mod = N;
    CKR(run_gemm(ctx, XN, D, L.ca_q, N, eq));
    EpiParams ek = epi_store(L.ca_k, (void*)b.kb, 0, D);
    if (m_sp > 0) {
      ek.rope = rope;
      ek.rope_D = D;
      ek.rope_cols = D;
      ek.rope_rows = m_sp;  // pointer tokens at the end get no RoPE
      ek.rope_mod = N;      // the table repeats for every memory slot
    }
    CKR(run_gemm(ctx, b.kvin, MD, L.ca_k, Mt, ek));
    CKR(run_gemm(ctx, b.pin, MD, L.ca_v, Mt, epi_store(L.ca_v, (void*)b.vb, 0, D)));
    AttnParams c;
    c.q = b.qkv;
    c.k = b.kb;
    c.v = b.vb;
    c.q_n = c.k_n = c.v_n = D;
    c.heads = 1;
    c.nq = (int)N;
    c.nk = (int)Mt;
    c.o = b.ao;
    c.o_n = D;
    c.scale = scale;
    CKR(run_attn(ctx, c, D, 1));
    EpiParams r2 = epi_store(L.ca_out, X, 1, D);
    r2.resid = X;
    r2.ldr = D;
    CKR(run_gemm(ctx, b.ao, D, L.ca_out, N, r2));
    // FFN (sam3.cpp:9318-9326)
    CKL(run_ln(ctx, X, D, XN, 0, D, N, D, L.n3w.ptr(), L.n3b.ptr(), 1e-5f, id));
    CKR(run_gemm(ctx, XN, D, L.fc1, N, epi_store(L.fc1, (void*)b.hb, 0, FFN, ACT_RELU)));
    EpiParams r3 = epi_store(L.fc2, X, 1, D);
    r3.resid = X;
    r3.ldr = D;
    CKR(run_gemm(ctx, b.hb, FFN, L.fc2, N, r3));
  }
  return kOk;
}

// Memory attention with its cross-attention inputs built by `prep` (prompt + prompt_pos -> kvin,
// prompt -> pin, both f16 [Mt][64]) from the caller's prompt arrays or on the device from the memory bank.
template <typename Prep>
static int mem_attn_body(s3b_ctx* ctx, const float* curr, const float* src_pos, int feat, int m_total, int n_ptr,
                         float* out, Prep prep) {
  const Model& M = ctx->model;
  const int D = M.hp.neck_dim, MD = M.hp.mem_out_dim;
  const long long N = (long long)feat * feat;
  const long long Mt = m_total, m_sp = m_total - n_ptr;
  if (M.mem.empty()) return set_error(ctx, kErrState, "no memory-attention layers");
  if (M.mem[0].ca_k.K != MD) return set_error(ctx, kErrFormat, "cross-attention kv dim %d != %d", M.mem[0].ca_k.K, MD);
  int rc = 0;
  const float* rope = rope_table(ctx, feat, D, &rc);
  if (rc) return rc;
  const int FFN = M.mem[0].fc1.N;
  DevBuf* x = ctx->buf("ma_x", (size_t)N * D * 4, &rc);
  DevBuf* xn = ctx->buf("ma_xn", (size_t)N * D * 2, &rc);
  DevBuf* qkv = ctx->buf("ma_qkv", (size_t)N * 3 * D * 2, &rc);
  DevBuf* ao = ctx->buf("ma_ao", (size_t)N * D * 2, &rc);
  DevBuf* hb = ctx->buf("ma_h", (size_t)N * FFN * 2, &rc);
  DevBuf* kvin = ctx->buf("ma_kvin", (size_t)Mt * MD * 2, &rc);
  DevBuf* pin = ctx->buf("ma_pin", (size_t)Mt * MD * 2, &rc);
  DevBuf* kb = ctx->buf("ma_k", (size_t)Mt * D * 2, &rc);
  DevBuf* vb = ctx->buf("ma_v", (size_t)Mt * D * 2, &rc);
  if (rc) return rc;
  float* X = x->as<float>();
  __half* XN = xn->as<__half>();
  RowMap id;
  // pos_enc_at_input: x = curr + 0.1 * src_pos (sam3.cpp:9243)
  CKL(add_scaled_f32(curr, src_pos, 0.1f, N * D, X, ctx->stream));
  // memory keys see prompt + prompt_pos, values see prompt (sam3.cpp:9278-9283)
  CKR(prep(kvin->as<__half>(), pin->as<__half>()));
  MemAttnBufs mb;
  mb.X = X;
  mb.XN = XN;
  mb.qkv = qkv->as<__half>();
  mb.ao = ao->as<__half>();
  mb.hb = hb->as<__half>();
  mb.kvin = kvin->as<__half>();
  mb.pin = pin->as<__half>();
  mb.kb = kb->as<__half>();
  mb.vb = vb->as<__half>();
  mb.rope = rope;
  mb.N = N;
  mb.Mt = Mt;
  mb.m_sp = m_sp;
  mb.D = D;
  mb.FFN = FFN;
  // The layers are about 50 launches of short kernels. With profiling off and a capturable stream,
  // the second call with the same shapes, buffers and options captures them into a CUDA graph (the
  // first call has allocated every workspace and set every kernel attribute) and later calls replay
  // it, which removes the host launch work and most of the gaps between the kernels.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(ctx->stream, &cap);
  // inside a capture of the whole call (a tracking step) the layers are recorded eagerly into that graph
  const bool can_graph = ctx->graphs && !ctx->prof && ctx->stream != nullptr && cap == cudaStreamCaptureStatusNone;
  // every buffer the layers touch is in the key, the attention's key-split workspace included (an
  // encoder call on the same context may grow and so move it)
  const auto ws_it = ctx->ws.find("attn_wide_split");
  const uintptr_t split_ws = (ws_it != ctx->ws.end() && ws_it->second) ? (uintptr_t)ws_it->second->p : 0;
  const std::vector<uintptr_t> key = {(uintptr_t)ctx->graph_epoch, (uintptr_t)gemm_config_id(), (uintptr_t)N,
                                      (uintptr_t)Mt, (uintptr_t)m_sp, (uintptr_t)X, (uintptr_t)XN,
                                      (uintptr_t)mb.qkv, (uintptr_t)mb.ao, (uintptr_t)mb.hb, (uintptr_t)mb.kvin,
                                      (uintptr_t)mb.pin, (uintptr_t)mb.kb, (uintptr_t)mb.vb, (uintptr_t)rope,
                                      split_ws};
  if (key != ctx->ma_key) {
    if (ctx->ma_exec) cudaGraphExecDestroy(ctx->ma_exec);
    ctx->ma_exec = nullptr;
    ctx->ma_key = key;
    ctx->ma_seen = 0;
  }
  if (can_graph && !ctx->ma_exec && ctx->ma_seen >= 1) {
    const long long n0 = ctx->n_launches;
    cudaGraph_t g = nullptr;
    bool ok = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    const int lrc = ok ? mem_attn_layers(ctx, mb) : kOk;
    if (ok) ok = cudaStreamEndCapture(ctx->stream, &g) == cudaSuccess && lrc == kOk;
    cudaGraphExec_t exec = nullptr;
    if (ok) ok = cudaGraphInstantiate(&exec, g, 0) == cudaSuccess;
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();  // a failed capture leaves its error here; the eager path below reports real faults
    const long long captured = ctx->n_launches - n0;
    ctx->n_launches = n0;  // nothing ran during the capture
    if (ok) {
      ctx->ma_exec = exec;
      ctx->ma_launches = captured;
    } else {
      if (exec) cudaGraphExecDestroy(exec);
      ctx->ma_seen = -(1 << 30);  // not capturable on this stream: stay eager for this key
    }
  }
  if (can_graph && ctx->ma_exec) {
    if (cudaGraphLaunch(ctx->ma_exec, ctx->stream) != cudaSuccess)
      return set_error(ctx, kErrCuda, "memory-attention graph launch failed");
    count_launch(ctx, (int)ctx->ma_launches);
  } else {
    ++ctx->ma_seen;
    CKR(mem_attn_layers(ctx, mb));
  }
  // final norm (sam3.cpp:9330-9334)
  CKL(run_ln(ctx, X, D, out, 1, D, N, D, M.mem_norm_w.ptr(), M.mem_norm_b.ptr(), 1e-5f, id));
  return check_device(ctx, "mem_attn");
}

int mem_attn_run(s3b_ctx* ctx, const float* curr, const float* src_pos, int feat, const float* prompt,
                 const float* prompt_pos, int m_total, int n_ptr, float* out) {
  const long long n = (long long)m_total * ctx->model.hp.mem_out_dim;
  return mem_attn_body(ctx, curr, src_pos, feat, m_total, n_ptr, out, [&](__half* kvin, __half* pin) {
    CKL(add_scaled_to_f16(prompt, prompt_pos, 1.0f, n, kvin, ctx->stream));
    CKL(add_scaled_to_f16(prompt, nullptr, 0.0f, n, pin, ctx->stream));
    return (int)kOk;
  });
}

int mem_attn_run_bank(s3b_ctx* ctx, const float* curr, const float* src_pos, int feat, const PromptArgs& pa,
                      float* out) {
  const int m_total = pa.n_slots * pa.slot_tokens + pa.n_ptr * pa.split;
  return mem_attn_body(ctx, curr, src_pos, feat, m_total, pa.n_ptr * pa.split, out, [&](__half* kvin, __half* pin) {
    CKL(build_prompt(pa, kvin, pin, 1, ctx->stream));
    return (int)kOk;
  });
}

}  // namespace s3b
