// extern "C" entry points of the engine (include/sam3_b200.h).
#include <math.h>
#include <string.h>

#include <algorithm>
#include <functional>
#include <string>
#include <vector>

#include "../../include/sam3_b200.h"
#include "engine.h"

namespace s3b {
void quantize_row_host(int type, const float* x, int64_t n, uint8_t* dst);
}  // namespace s3b

using namespace s3b;

s3b::DevBuf* s3b_ctx::buf(const std::string& name, size_t bytes, int* rc) {
  auto& b = ws[name];
  if (!b) b = std::make_shared<DevBuf>();
  if (b->reserve(bytes)) {
    *rc = set_error(this, kErrOOM, "workspace '%s': cudaMalloc(%zu) failed", name.c_str(), bytes);
    return b.get();
  }
  return b.get();
}

namespace {

int ctx_enter(s3b_ctx* ctx) {
  if (!ctx) return kErrArg;
  if (cudaSetDevice(ctx->device) != cudaSuccess) return set_error(ctx, kErrCuda, "cudaSetDevice(%d)", ctx->device);
  return kOk;
}

// Reads the device error word; a non-zero value means a bounded wait expired.
int read_dev_err(s3b_ctx* ctx) {
  int h = 0;
  if (cudaMemcpy(&h, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return set_error(ctx, kErrCuda, "reading the device error word: %s", cudaGetErrorString(cudaGetLastError()));
  if (h != 0) {
    // cleared in the context stream's order, so no later kernel's code can be wiped by it
    cudaMemsetAsync(ctx->d_err, 0, sizeof(int), ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    return set_error(ctx, kErrDevice, "device-side wait timed out (code %d)", h);
  }
  return kOk;
}

// Sinusoidal 2D PE (sam3_sinusoidal_pe_2d, sam3.cpp:3597-3633), channel-last [H][W][d].
void sine_pe_2d(int H, int W, int d_model, float* pe) {
  const int half = d_model / 2;
  const float scale = 2.0f * (float)M_PI;
  for (int y = 0; y < H; ++y)
    for (int x = 0; x < W; ++x) {
      const float py = ((float)(y + 1) / (float)H) * scale;
      const float px = ((float)(x + 1) / (float)W) * scale;
      for (int i = 0; i < half; ++i) {
        const int paired = i & ~1;
        const float dim_t = powf(10000.0f, (float)paired / (float)half);
        float vx, vy;
        if (i % 2 == 0) {
          vx = sinf(px / dim_t);
          vy = sinf(py / dim_t);
        } else {
          vx = cosf(px / dim_t);
          vy = cosf(py / dim_t);
        }
        pe[((size_t)y * W + x) * d_model + i] = vy;
        pe[((size_t)y * W + x) * d_model + i + half] = vx;
      }
    }
}

// 1-D sine PE (sam3_get_1d_sine_pe, sam3.cpp:3636-3647): [dim], first dim/2 sin, then cos.
void sine_pe_1d(float* out, float pos_ind, int dim) {
  const int pe_dim = dim / 2;
  for (int i = 0; i < pe_dim; ++i) {
    const int paired = i & ~1;
    const float dim_t = powf(10000.0f, (float)paired / (float)pe_dim);
    const float val = pos_ind / dim_t;
    out[i] = sinf(val);
    out[pe_dim + i] = cosf(val);
  }
}

// Device copy of the sinusoidal PE [S][S][d] (computed on the host once per size, like the tracker's
// cached_sinpe_256 / cached_sinpe_64, sam3.cpp:11137-11138).
const float* device_sine_pe(s3b_ctx* ctx, int S, int d, int* rc) {
  const std::string key = "sine_pe_" + std::to_string(S) + "_" + std::to_string(d);
  auto it = ctx->ws.find(key);
  if (it != ctx->ws.end() && it->second && it->second->p) return it->second->as<float>();
  std::vector<float> pe((size_t)S * S * d);
  sine_pe_2d(S, S, d, pe.data());
  DevBuf* b = ctx->buf(key, pe.size() * 4, rc);
  if (*rc) return nullptr;
  if ((*rc = upload_sync(ctx, b->p, pe.data(), pe.size() * 4))) return nullptr;
  return b->as<float>();
}

// Parameters of the device prompt build from a memory bank (sam3_build_prompt_and_pos,
// sam3.cpp:9123-9209, with the inputs sam3_propagate_single gathers at 11186-11228).
int prompt_args(s3b_ctx* ctx, int feat, const float* const* slot_feats, const float* const* slot_pes,
                const int* slot_tpos, int n_slots, const float* obj_ptrs, const int* ptr_tpos, int n_ptrs,
                PromptArgs& pa) {
  const Model& M = ctx->model;
  const HParams& hp = M.hp;
  const int D = hp.neck_dim, MD = hp.mem_out_dim;
  if (MD != kPromptMD || D % MD) return set_error(ctx, kErrUnsupported, "memory dim %d / %d", MD, D);
  if (n_slots < 0 || n_slots > kPromptMaxSlots || n_ptrs < 0 || n_ptrs > kPromptMaxPtrs || feat <= 0 ||
      (n_slots > 0 && (!slot_feats || !slot_tpos)) || (n_ptrs > 0 && (!obj_ptrs || !ptr_tpos)))
    return set_error(ctx, kErrArg, "bad memory-bank arguments (at most %d slots and %d pointers)", kPromptMaxSlots,
                     kPromptMaxPtrs);
  pa.n_slots = n_slots;
  pa.slot_tokens = feat * feat;
  pa.split = D / MD;
  int rc = 0;
  for (int s = 0; s < n_slots; ++s) {
    pa.feat[s] = slot_feats[s];
    pa.pe[s] = slot_pes && slot_pes[s] ? slot_pes[s] : device_sine_pe(ctx, feat, MD, &rc);  // cached_sinpe_64
    if (rc) return rc;
    if (!pa.feat[s]) return set_error(ctx, kErrArg, "null memory slot %d", s);
    const int tp = slot_tpos[s];
    pa.has_tpos[s] = 0;
    if (tp >= 0 && tp < hp.num_maskmem) {
      const int enc_idx = hp.num_maskmem - tp - 1;  // maskmem_tpos_enc[num_maskmem - tpos - 1]
      if ((int)M.maskmem_tpos.size() < (enc_idx + 1) * MD)
        return set_error(ctx, kErrState, "model has no temporal encodings (mem_enc.tpos_enc)");
      memcpy(pa.tpos[s], M.maskmem_tpos.data() + (size_t)enc_idx * MD, MD * sizeof(float));
      pa.has_tpos[s] = 1;
    }
  }
  pa.ptrs = obj_ptrs;
  pa.n_ptr = 0;
  for (int p = 0; p < n_ptrs; ++p) {
    const int rel = ptr_tpos[p];
    if (rel < 0) continue;  // skipped pointers (sam3.cpp:9181)
    auto it = ctx->ptr_pe_cache.find(rel);
    if (it == ctx->ptr_pe_cache.end()) {
      if ((int)M.obj_ptr_tpos_w.size() != D * MD || (int)M.obj_ptr_tpos_b.size() != MD)
        return set_error(ctx, kErrState, "model has no obj_ptr_tpos_proj weights");
      // 1-D sine PE of rel / 15 projected 256 -> 64 in f32, bias first then i in order (9182-9195)
      std::vector<float> sine(D), proj(MD);
      sine_pe_1d(sine.data(), (float)rel / 15.0f, D);
      for (int j = 0; j < MD; ++j) {
        float sum = M.obj_ptr_tpos_b[j];
        for (int i = 0; i < D; ++i) sum += M.obj_ptr_tpos_w[(size_t)i + (size_t)j * D] * sine[i];
        proj[j] = sum;
      }
      it = ctx->ptr_pe_cache.emplace(rel, proj).first;
    }
    memcpy(pa.ptr_pe[pa.n_ptr], it->second.data(), MD * sizeof(float));
    pa.ptr_src[pa.n_ptr] = p;
    ++pa.n_ptr;
  }
  if (pa.n_slots * pa.slot_tokens + pa.n_ptr * pa.split <= 0) return set_error(ctx, kErrArg, "empty memory");
  return kOk;
}

struct OutRef {
  const float* dev = nullptr;  // frame 0
  int64_t ne[4] = {1, 1, 1, 1};
  int64_t frame_elems = 0;
  bool is_pe = false;
  int pe_size = 0;
};

int resolve_output(s3b_ctx* ctx, const char* name, OutRef& r) {
  const Outputs& O = ctx->out;
  const HParams& hp = ctx->model.hp;
  std::string n(name ? name : "");
  if (O.n_frames <= 0) return set_error(ctx, kErrState, "no encode has run");
  if (n == "backbone" && O.backbone && hp.is_sam2 && O.backbone_c > 0) {
    r.dev = O.backbone->as<float>();
    r.ne[0] = O.backbone_c;
    r.ne[1] = r.ne[2] = O.backbone_s;
    r.frame_elems = (int64_t)O.backbone_s * O.backbone_s * O.backbone_c;
    return kOk;
  }
  if ((n == "vit_output" || n == "backbone") && O.backbone && !hp.is_sam2) {
    const int G = hp.n_img_embd();
    r.dev = O.backbone->as<float>();
    r.ne[0] = hp.vit_embed_dim;
    r.ne[1] = G;
    r.ne[2] = G;
    r.frame_elems = (int64_t)G * G * hp.vit_embed_dim;
    return kOk;
  }
  for (int i = 0; i < 4; ++i) {
    const std::string si = std::to_string(i);
    if (n == "neck_trk_" + si && i < O.n_fpn) {
      r.dev = O.fpn[i]->as<float>();
      r.ne[0] = hp.neck_dim;
      r.ne[1] = r.ne[2] = O.fpn_size[i];
      r.frame_elems = (int64_t)O.fpn_size[i] * O.fpn_size[i] * hp.neck_dim;
      return kOk;
    }
    if (n == "neck_det_" + si && i < O.n_det) {
      r.dev = O.det[i]->as<float>();
      r.ne[0] = hp.neck_dim;
      r.ne[1] = r.ne[2] = O.fpn_size[i];
      r.frame_elems = (int64_t)O.fpn_size[i] * O.fpn_size[i] * hp.neck_dim;
      return kOk;
    }
    if ((n == "neck_trk_pe_" + si || n == "neck_det_pe_" + si) && i < O.n_fpn) {
      r.is_pe = true;
      r.pe_size = O.fpn_size[i];
      r.ne[0] = hp.neck_dim;
      r.ne[1] = r.ne[2] = O.fpn_size[i];
      r.frame_elems = (int64_t)O.fpn_size[i] * O.fpn_size[i] * hp.neck_dim;
      return kOk;
    }
  }
  return set_error(ctx, kErrArg, "unknown output '%s'", n.c_str());
}

template <typename T>
int stage_host(s3b_ctx* ctx, const T* host, size_t n, const char* name, T** dev) {
  int rc = 0;
  DevBuf* b = ctx->buf(name, n * sizeof(T), &rc);
  if (rc) return rc;
  if (cudaMemcpyAsync(b->p, host, n * sizeof(T), cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess)
    return set_error(ctx, kErrCuda, "host-to-device copy failed");
  *dev = b->as<T>();
  return kOk;
}

// d_u8 (uint8 HWC frames at the model size) instead of d_chw: the preprocessing (sam3_preprocess_image /
// sam2_preprocess_image, sam3.cpp:3486-3544, normalisation only) runs inside the patch-column kernel.
int encode_device_chw(s3b_ctx* ctx, const float* d_chw, int n_frames, int img_size, int flags,
                      const uint8_t* d_u8 = nullptr) {
  if (!ctx->model.loaded) return set_error(ctx, kErrState, "no model loaded");
  if (n_frames <= 0) return set_error(ctx, kErrArg, "n_frames must be > 0");
  if (img_size != ctx->model.hp.img_size)
    return set_error(ctx, kErrUnsupported, "img_size %d != model img_size %d (resize is done by the caller)", img_size,
                     ctx->model.hp.img_size);
  return ctx->model.hp.is_sam2 ? hiera_encode(ctx, d_chw, n_frames, flags, d_u8)
                               : vit_encode(ctx, d_chw, n_frames, flags, d_u8);
}

int encode_device_u8(s3b_ctx* ctx, const uint8_t* d_u8, int n_frames, int img_size, int flags) {
  if (!ctx->model.loaded) return set_error(ctx, kErrState, "no model loaded");
  if (n_frames <= 0 || img_size <= 0) return set_error(ctx, kErrArg, "bad frame count / size");
  return encode_device_chw(ctx, nullptr, n_frames, img_size, flags, d_u8);
}

// Frames of any size: resized on the device to the model size and normalised in the same pass
// (sam3_preprocess_image / sam2_preprocess_image, sam3.cpp:3486-3544); frames already at the
// model size skip the resize, as the reference does (3496).
int encode_device_image_u8(s3b_ctx* ctx, const uint8_t* d_u8, int n_frames, int width, int height, int flags) {
  if (!ctx->model.loaded) return set_error(ctx, kErrState, "no model loaded");
  if (n_frames <= 0 || width <= 0 || height <= 0) return set_error(ctx, kErrArg, "bad frame count / size");
  const int S = ctx->model.hp.img_size;
  if (width == S && height == S) return encode_device_u8(ctx, d_u8, n_frames, S, flags);
  int rc = 0;
  DevBuf* chw = ctx->buf("frames_chw", (size_t)n_frames * 3 * S * S * 4, &rc);
  if (rc) return rc;
  const bool sam2 = ctx->model.hp.is_sam2 != 0;
  rc = resize_bilinear_u8(d_u8, n_frames, height, width, S, S, sam2 ? kMeanSam2 : kMeanSam3,
                          sam2 ? kStdSam2 : kStdSam3, chw->p, ctx->stream);
  if (rc) return set_error(ctx, kErrCuda, "resize launch failed");
  return encode_device_chw(ctx, chw->as<float>(), n_frames, S, flags);
}

constexpr size_t kMaxEncGraphs = 16;

// Runs one call (`body`: all of its work on the context stream; an encoder call or a tracking step)
// eagerly, or replays it from a CUDA graph. Such a call is a fixed sequence of tens to hundreds of
// launches; from the second call with the same key (`key` + the option epoch, the GEMM configuration and
// the DevBuf generation, so every pointer the launches hold is unchanged) the sequence is captured once
// and replayed, which removes the host launch work and most of the gaps between kernels (the batch-1
// latency). Calls with profiling on, with host-bound outputs (their per-pass copies run on a second
// stream), behind pending output copies or on the legacy default stream stay eager, and so does a key
// whose capture failed.
int run_graphed(s3b_ctx* ctx, std::vector<uintptr_t> key, const std::function<int()>& body) {
  if (!ctx->graphs || ctx->prof || !ctx->stream || !ctx->host_bind.empty()) return body();
  // output copies of an earlier host-bound call still pending: the eager call orders itself after them
  for (char pending : ctx->copy_pending)
    if (pending) return body();
  key.push_back((uintptr_t)ctx->graph_epoch);
  key.push_back((uintptr_t)gemm_config_id());
  key.push_back((uintptr_t)devbuf_generation().load());
  auto& G = ctx->enc_graphs;
  auto it = std::find_if(G.begin(), G.end(), [&](const s3b_ctx::EncGraph& g) { return g.key == key; });
  if (it == G.end()) {
    if (G.size() >= kMaxEncGraphs) {
      if (G.front().exec) cudaGraphExecDestroy(G.front().exec);
      G.erase(G.begin());
    }
    G.push_back(s3b_ctx::EncGraph());
    G.back().key = key;
    it = G.end() - 1;
  } else if (it != G.end() - 1) {
    std::rotate(it, it + 1, G.end());  // most recently used last
    it = G.end() - 1;
  }
  s3b_ctx::EncGraph& g = *it;
  if (!g.exec && g.seen >= 1) {
    const long long n0 = ctx->n_launches;
    cudaGraph_t graph = nullptr;
    bool ok = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    const int brc = ok ? body() : kOk;
    if (ok) ok = cudaStreamEndCapture(ctx->stream, &graph) == cudaSuccess && brc == kOk;
    cudaGraphExec_t exec = nullptr;
    if (ok) ok = cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();  // a failed capture leaves its error here; the eager run below reports real faults
    const long long captured = ctx->n_launches - n0;
    ctx->n_launches = n0;  // nothing ran during the capture
    // the capture is valid only if the body allocated nothing (a DevBuf growing inside it fails the
    // capture anyway; this also covers one that was released)
    if (ok && (uintptr_t)devbuf_generation().load() == key.back()) {
      g.exec = exec;
      g.launches = captured;
    } else {
      if (exec) cudaGraphExecDestroy(exec);
      g.seen = -(1 << 30);  // not capturable: stay eager for this key
    }
  }
  if (g.exec) {
    if (cudaGraphLaunch(g.exec, ctx->stream) != cudaSuccess)
      return set_error(ctx, kErrCuda, "encoder graph launch failed");
    count_launch(ctx, (int)g.launches);
    return check_device(ctx, "encoder graph");
  }
  ++g.seen;
  return body();
}

}  // namespace

namespace s3b {

const float* sine_pe_device(s3b_ctx* ctx, int S, int d, int* rc) { return device_sine_pe(ctx, S, d, rc); }

int outputs_pass_begin(s3b_ctx* ctx, int pass, int fb) {
  if (ctx->copy_done.empty()) return kOk;
  if (fb != ctx->copy_fb) {
    // another pass size: any pending copy may read frames this call writes
    for (size_t p = 0; p < ctx->copy_done.size(); ++p)
      if (ctx->copy_pending[p]) {
        if (cudaStreamWaitEvent(ctx->stream, ctx->copy_done[p], 0) != cudaSuccess)
          return set_error(ctx, kErrCuda, "waiting for output copies failed");
        ctx->copy_pending[p] = 0;
      }
    return kOk;
  }
  if (pass < (int)ctx->copy_done.size() && ctx->copy_pending[pass]) {
    if (cudaStreamWaitEvent(ctx->stream, ctx->copy_done[pass], 0) != cudaSuccess)
      return set_error(ctx, kErrCuda, "waiting for output copies failed");
    ctx->copy_pending[pass] = 0;
  }
  return kOk;
}

int outputs_pass_end(s3b_ctx* ctx, int pass, int f0, int F) {
  if (ctx->host_bind.empty()) return kOk;
  if (!ctx->copy_stream &&
      cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking) != cudaSuccess)
    return set_error(ctx, kErrCuda, "copy stream creation failed");
  while ((int)ctx->copy_done.size() <= pass) {
    cudaEvent_t a, b;
    if (cudaEventCreateWithFlags(&a, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&b, cudaEventDisableTiming) != cudaSuccess)
      return set_error(ctx, kErrCuda, "event creation failed");
    ctx->pass_done.push_back(a);
    ctx->copy_done.push_back(b);
    ctx->copy_pending.push_back(0);
  }
  if (cudaEventRecord(ctx->pass_done[pass], ctx->stream) != cudaSuccess ||
      cudaStreamWaitEvent(ctx->copy_stream, ctx->pass_done[pass], 0) != cudaSuccess)
    return set_error(ctx, kErrCuda, "output copy ordering failed");
  for (const auto& kv : ctx->host_bind) {
    OutRef r;
    int rc = resolve_output(ctx, kv.first.c_str(), r);
    if (rc) return rc;
    if (r.is_pe) return set_error(ctx, kErrArg, "'%s' is host-computed and cannot be bound", kv.first.c_str());
    if (kv.second.n < (int64_t)ctx->out.n_frames * r.frame_elems)
      return set_error(ctx, kErrArg, "host buffer of '%s' holds %lld floats, the call needs %lld", kv.first.c_str(),
                       (long long)kv.second.n, (long long)ctx->out.n_frames * r.frame_elems);
    const size_t off = (size_t)f0 * r.frame_elems;
    if (cudaMemcpyAsync(kv.second.host + off, r.dev + off, (size_t)F * r.frame_elems * 4, cudaMemcpyDeviceToHost,
                        ctx->copy_stream) != cudaSuccess)
      return set_error(ctx, kErrCuda, "output copy of '%s' failed", kv.first.c_str());
  }
  if (cudaEventRecord(ctx->copy_done[pass], ctx->copy_stream) != cudaSuccess)
    return set_error(ctx, kErrCuda, "output copy ordering failed");
  ctx->copy_pending[pass] = 1;
  ctx->copy_fb = ctx->max_frames_per_pass;
  return kOk;
}

}  // namespace s3b

extern "C" {

int s3b_create(int device, s3b_ctx** out) {
  if (!out) return kErrArg;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    fprintf(stderr, "s3b: no CUDA device %d (count %d)\n", device, n);
    return kErrCuda;
  }
  s3b_ctx* ctx = new s3b_ctx();
  ctx->device = device;
  if (cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->d_err, sizeof(int)) != cudaSuccess || cudaMemset(ctx->d_err, 0, sizeof(int)) != cudaSuccess) {
    fprintf(stderr, "s3b: context creation failed on device %d\n", device);
    delete ctx;
    return kErrCuda;
  }
  ctx->own_stream = true;
  *out = ctx;
  return kOk;
}

void s3b_destroy(s3b_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->copy_stream) cudaStreamSynchronize(ctx->copy_stream);
  for (cudaEvent_t e : ctx->pass_done) cudaEventDestroy(e);
  for (cudaEvent_t e : ctx->copy_done) cudaEventDestroy(e);
  if (ctx->copy_stream) cudaStreamDestroy(ctx->copy_stream);
  if (ctx->ma_exec) cudaGraphExecDestroy(ctx->ma_exec);
  for (auto& g : ctx->enc_graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  ctx->enc_graphs.clear();
  for (void* p : ctx->ipc_mapped) cudaIpcCloseMemHandle(p);
  ctx->ipc_mapped.clear();
  ctx->user_allocs.clear();
  ctx->ws.clear();
  ctx->out = Outputs();
  ctx->model = Model();
  for (cudaEvent_t e : ctx->event_pool) cudaEventDestroy(e);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

const char* s3b_last_error(const s3b_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

int s3b_set_stream(s3b_ctx* ctx, void* stream) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  cudaStreamSynchronize(ctx->stream);
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  ctx->own_stream = false;
  ctx->stream = reinterpret_cast<cudaStream_t>(stream);
  return kOk;
}

int s3b_reset_stream(s3b_ctx* ctx) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (ctx->own_stream) return kOk;
  cudaStreamSynchronize(ctx->stream);
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess)
    return set_error(ctx, kErrCuda, "stream creation failed");
  ctx->own_stream = true;
  return kOk;
}

int s3b_sync(s3b_ctx* ctx) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return set_error(ctx, kErrCuda, "stream synchronize: %s", cudaGetErrorString(e));
  if (ctx->copy_stream) {
    e = cudaStreamSynchronize(ctx->copy_stream);
    if (e != cudaSuccess) return set_error(ctx, kErrCuda, "output copies: %s", cudaGetErrorString(e));
    for (auto& p : ctx->copy_pending) p = 0;
  }
  return read_dev_err(ctx);
}

int s3b_output_host_bind(s3b_ctx* ctx, const char* name, float* host, int64_t n_floats) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!name) return set_error(ctx, kErrArg, "null output name");
  const std::string n(name);
  bool known = n == "vit_output" || n == "backbone";
  for (int i = 0; i < 4; ++i)
    known = known || n == "neck_trk_" + std::to_string(i) || n == "neck_det_" + std::to_string(i);
  if (!known) return set_error(ctx, kErrArg, "output '%s' cannot be bound to host memory", name);
  // copies still reading the previous binding finish first
  if (ctx->copy_stream && cudaStreamSynchronize(ctx->copy_stream) != cudaSuccess)
    return set_error(ctx, kErrCuda, "output copies failed");
  for (auto& p : ctx->copy_pending) p = 0;
  if (!host) {
    ctx->host_bind.erase(n);
    return kOk;
  }
  if (n_floats <= 0) return set_error(ctx, kErrArg, "bad host buffer size");
  ctx->host_bind[n] = s3b_ctx::HostBind{host, n_floats};
  return kOk;
}

int s3b_set_option(s3b_ctx* ctx, const char* key, int64_t value) {
  if (!ctx || !key) return kErrArg;
  const std::string k(key);
  ++ctx->graph_epoch;  // kernel choices may change: recapture graphs
  if (k == "graphs") {
    if (value < 0 || value > 1) return set_error(ctx, kErrArg, "graphs must be 0 or 1");
    ctx->graphs = (int)value;
    return kOk;
  }
  if (k == "frames_per_pass") {
    if (value < 1 || value > 256) return set_error(ctx, kErrArg, "frames_per_pass out of range");
    ctx->max_frames_per_pass = (int)value;
    return kOk;
  }
  if (k == "attention_impl") {
    if (value < 0 || value > 4) return set_error(ctx, kErrArg, "attention_impl must be in [0, 4]");
    ctx->attention_impl = (int)value;
    return kOk;
  }
  if (k == "gemm_pairs") {
    if (value < 0 || value > 2) return set_error(ctx, kErrArg, "gemm_pairs must be 0, 1 or 2");
    set_gemm_pairs((int)value);
    return kOk;
  }
  if (k == "gemm_wide_epilogue") {
    if (value < 0 || value > 1) return set_error(ctx, kErrArg, "gemm_wide_epilogue must be 0 or 1");
    set_gemm_wide_epilogue((int)value);
    return kOk;
  }
  if (k == "weights_quantised") {
    if (value < 0 || value > 2) return set_error(ctx, kErrArg, "weights_quantised must be 0, 1 or 2");
    ctx->weights_quantised = (int)value;
    return kOk;
  }
  if (k == "conv_implicit") {
    if (value < 0 || value > 1) return set_error(ctx, kErrArg, "conv_implicit must be 0 or 1");
    ctx->conv_implicit = (int)value;
    return kOk;
  }
  if (k == "attention_wide_k128") {
    if (value < -1 || value > 1) return set_error(ctx, kErrArg, "attention_wide_k128 must be -1, 0 or 1");
    ctx->attention_wide_k128 = (int)value;
    return kOk;
  }
  if (k == "attention_fa_exp_poly") {
    if (value < 0 || value > 4) return set_error(ctx, kErrArg, "attention_fa_exp_poly must be in [0, 4]");
    ctx->attention_fa_exp_poly = (int)value;
    return kOk;
  }
  if (k == "attention_exp_poly") {
    if (value < 0 || value > 4) return set_error(ctx, kErrArg, "attention_exp_poly must be in [0, 4]");
    ctx->attention_exp_poly = (int)value;
    return kOk;
  }
  if (k == "stop_after_blocks") {
    if (value < -1 || value > 1024) return set_error(ctx, kErrArg, "stop_after_blocks out of range");
    ctx->stop_after_blocks = (int)value;
    return kOk;
  }
  return set_error(ctx, kErrArg, "unknown option '%s'", key);
}

int s3b_profile_begin(s3b_ctx* ctx, int with_events) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  ctx->prof = with_events != 0;
  ctx->prof_entries.clear();
  ctx->event_next = 0;
  ctx->n_launches = 0;
  return kOk;
}

int s3b_profile_end(s3b_ctx* ctx, double* out, int n) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) return set_error(ctx, kErrCuda, "synchronize failed");
  double v[17] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
  for (const auto& e : ctx->prof_entries) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e.a, e.b);
    const int base = e.kind == 0 ? 0 : e.kind == 1 ? 4 : e.kind == 2 ? 9 : 13;
    v[base + 0] += 1;
    v[base + 1] += ms;
    v[base + 2] += e.flops;
    v[base + 3] += e.bytes;
  }
  v[8] = (double)ctx->n_launches;
  for (int i = 0; i < n && i < 17; ++i) out[i] = v[i];
  ctx->prof = false;
  ctx->prof_entries.clear();
  ctx->event_next = 0;
  return read_dev_err(ctx);
}

int s3b_load_model(s3b_ctx* ctx, const char* path) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!path) return set_error(ctx, kErrArg, "null path");
  ctx->out = Outputs();
  ctx->ptr_pe_cache.clear();
  ++ctx->graph_epoch;  // graphs hold the old weights' addresses
  return load_model(ctx, path);
}

int s3b_load_model_cached(s3b_ctx* ctx, const char* model_path, const char* cache_path) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!model_path || !cache_path) return set_error(ctx, kErrArg, "null path");
  ctx->out = Outputs();
  ctx->ptr_pe_cache.clear();
  for (auto it = ctx->ws.begin(); it != ctx->ws.end();)  // dense PE grids of the previous decoder
    it = it->first.compare(0, 7, "dec_pe_") == 0 ? ctx->ws.erase(it) : std::next(it);
  ++ctx->graph_epoch;  // graphs hold the old weights' addresses
  return load_model_cached(ctx, model_path, cache_path);
}

int s3b_load_weights(s3b_ctx* ctx, int is_sam2, const int32_t* hparams, int n_hparams, int ftype,
                     const s3b_tensor_desc* descs, int n) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!hparams || n_hparams <= 0 || !descs || n <= 0) return set_error(ctx, kErrArg, "bad load_weights arguments");
  HParams hp;
  std::string err;
  if ((rc = parse_hparams_array(is_sam2, hparams, n_hparams, hp, err))) return set_error(ctx, rc, "%s", err.c_str());
  hp.ftype = ftype;
  // the caller's tensors as the file reader would return them (sam3_load_tensors, sam3.cpp:3091-3194):
  // same names, ggml shapes and dtypes, data in ggml row layout
  std::vector<FileTensor> tensors(n);
  for (int i = 0; i < n; ++i) {
    const s3b_tensor_desc& d = descs[i];
    FileTensor& t = tensors[i];
    if (!d.name || !d.data || d.n_dims < 1 || d.n_dims > 4)
      return set_error(ctx, kErrArg, "tensor %d: bad descriptor", i);
    t.name = d.name;
    t.dtype = d.dtype;
    t.n_dims = d.n_dims;
    for (int k = 0; k < 4; ++k) {
      t.ne[k] = k < d.n_dims ? d.ne[k] : 1;
      if (t.ne[k] <= 0) return set_error(ctx, kErrArg, "tensor %s: bad shape", d.name);
    }
    int64_t bytes;
    if (d.dtype == QT_F32 || d.dtype == QT_F16) {
      bytes = t.nelements() * (d.dtype == QT_F16 ? 2 : 4);
    } else if (d.dtype == QT_Q4_0 || d.dtype == QT_Q4_1 || d.dtype == QT_Q8_0) {
      if (t.ne[0] % 32) return set_error(ctx, kErrFormat, "quantised tensor with ne0 %% 32 != 0: %s", d.name);
      bytes = qtype_row_bytes(d.dtype, t.ne[0]) * (t.nelements() / t.ne[0]);
    } else {
      return set_error(ctx, kErrFormat, "unsupported dtype %d in %s", d.dtype, d.name);
    }
    const uint8_t* src = static_cast<const uint8_t*>(d.data);
    t.data.assign(src, src + bytes);
  }
  ctx->out = Outputs();
  ctx->ptr_pe_cache.clear();
  ++ctx->graph_epoch;
  return load_model_tensors(ctx, hp, tensors);
}

int s3b_inspect_model(const char* path, int32_t* info, int n, char* err, int err_len) {
  if (!path) return kErrArg;
  HParams hp;
  std::vector<FileTensor> tensors;
  std::string e;
  const int rc = read_ggml_file(path, hp, tensors, e);
  if (rc) {
    if (err && err_len > 0) snprintf(err, err_len, "%s", e.c_str());
    return rc;
  }
  int nq = 0;
  for (const auto& t : tensors) nq += (t.dtype == QT_Q4_0 || t.dtype == QT_Q4_1 || t.dtype == QT_Q8_0) ? 1 : 0;
  int depth = 0;
  for (int s = 0; s < hp.hiera_num_stages && s < 4; ++s) depth += hp.hiera_stages[s];
  const int32_t v[7] = {hp.is_sam2, hp.img_size, (int32_t)tensors.size(), hp.ftype,
                        hp.is_sam2 ? depth : hp.vit_depth, hp.is_sam2 ? hp.hiera_embed_dim : hp.vit_embed_dim, nq};
  for (int i = 0; i < n && i < 7; ++i) info[i] = v[i];
  if (err && err_len > 0) err[0] = 0;
  return kOk;
}

int s3b_model_info(s3b_ctx* ctx, int32_t* info, int n) {
  if (!ctx || !info) return kErrArg;
  if (!ctx->model.loaded) return set_error(ctx, kErrState, "no model loaded");
  const HParams& hp = ctx->model.hp;
  int32_t v[7] = {hp.is_sam2, hp.img_size, hp.is_sam2 ? (int32_t)ctx->model.hiera.size() : hp.vit_depth,
                  hp.is_sam2 ? hp.hiera_embed_dim : hp.vit_embed_dim, hp.neck_dim,
                  ctx->model.has_mem_attn ? hp.mem_attn_layers : 0,
                  (int32_t)((ctx->model.device_bytes >> 20) & 0x7fffffff)};
  for (int i = 0; i < n && i < 7; ++i) info[i] = v[i];
  return kOk;
}

int s3b_encode_u8(s3b_ctx* ctx, const uint8_t* frames, int n_frames, int img_size, int flags) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!frames || n_frames <= 0 || img_size <= 0) return set_error(ctx, kErrArg, "bad arguments");
  uint8_t* d = nullptr;
  if ((rc = stage_host(ctx, frames, (size_t)n_frames * img_size * img_size * 3, "frames_u8", &d))) return rc;
  return run_graphed(ctx, {1, (uintptr_t)d, (uintptr_t)n_frames, (uintptr_t)img_size, (uintptr_t)flags},
                    [&] { return encode_device_u8(ctx, d, n_frames, img_size, flags); });
}

int s3b_encode_image_u8(s3b_ctx* ctx, const uint8_t* frames, int n_frames, int width, int height, int flags) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!frames || n_frames <= 0 || width <= 0 || height <= 0) return set_error(ctx, kErrArg, "bad arguments");
  uint8_t* d = nullptr;
  if ((rc = stage_host(ctx, frames, (size_t)n_frames * width * height * 3, "frames_u8", &d))) return rc;
  return run_graphed(ctx, {2, (uintptr_t)d, (uintptr_t)n_frames, (uintptr_t)width, (uintptr_t)height, (uintptr_t)flags},
                    [&] { return encode_device_image_u8(ctx, d, n_frames, width, height, flags); });
}

int s3b_encode_image_u8_device(s3b_ctx* ctx, const uint8_t* d_frames, int n_frames, int width, int height,
                               int flags) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!d_frames) return set_error(ctx, kErrArg, "null frames");
  return run_graphed(ctx,
                     {2, (uintptr_t)d_frames, (uintptr_t)n_frames, (uintptr_t)width, (uintptr_t)height, (uintptr_t)flags},
                     [&] { return encode_device_image_u8(ctx, d_frames, n_frames, width, height, flags); });
}

int s3b_encode_chw(s3b_ctx* ctx, const float* chw, int n_frames, int img_size, int flags) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!chw || n_frames <= 0 || img_size <= 0) return set_error(ctx, kErrArg, "bad arguments");
  float* d = nullptr;
  if ((rc = stage_host(ctx, chw, (size_t)n_frames * 3 * img_size * img_size, "frames_chw_in", &d))) return rc;
  return run_graphed(ctx, {3, (uintptr_t)d, (uintptr_t)n_frames, (uintptr_t)img_size, (uintptr_t)flags},
                    [&] { return encode_device_chw(ctx, d, n_frames, img_size, flags); });
}

int s3b_encode_u8_device(s3b_ctx* ctx, const uint8_t* d_frames, int n_frames, int img_size, int flags) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!d_frames) return set_error(ctx, kErrArg, "null frames");
  return run_graphed(ctx, {1, (uintptr_t)d_frames, (uintptr_t)n_frames, (uintptr_t)img_size, (uintptr_t)flags},
                    [&] { return encode_device_u8(ctx, d_frames, n_frames, img_size, flags); });
}

int s3b_encode_chw_device(s3b_ctx* ctx, const float* d_chw, int n_frames, int img_size, int flags) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!d_chw) return set_error(ctx, kErrArg, "null frames");
  return run_graphed(ctx, {3, (uintptr_t)d_chw, (uintptr_t)n_frames, (uintptr_t)img_size, (uintptr_t)flags},
                    [&] { return encode_device_chw(ctx, d_chw, n_frames, img_size, flags); });
}

int s3b_output_shape(s3b_ctx* ctx, const char* name, int64_t ne[4]) {
  if (!ctx || !ne) return kErrArg;
  OutRef r;
  int rc = resolve_output(ctx, name, r);
  if (rc) return rc;
  for (int i = 0; i < 4; ++i) ne[i] = r.ne[i];
  return kOk;
}

int s3b_output_copy(s3b_ctx* ctx, const char* name, int frame, float* dst, int64_t n) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  OutRef r;
  if ((rc = resolve_output(ctx, name, r))) return rc;
  if (!dst || n != r.frame_elems) return set_error(ctx, kErrArg, "output '%s' has %lld elements per frame", name,
                                                   (long long)r.frame_elems);
  if (r.is_pe) {
    sine_pe_2d(r.pe_size, r.pe_size, (int)r.ne[0], dst);
    return kOk;
  }
  if (frame < 0 || frame >= ctx->out.n_frames) return set_error(ctx, kErrArg, "frame %d out of range", frame);
  if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) return set_error(ctx, kErrCuda, "synchronize failed");
  if ((rc = read_dev_err(ctx))) return rc;
  if (cudaMemcpy(dst, r.dev + (size_t)frame * r.frame_elems, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return set_error(ctx, kErrCuda, "device-to-host copy failed");
  return kOk;
}

int s3b_output_device_ptr(s3b_ctx* ctx, const char* name, int frame, const float** dptr) {
  if (!ctx || !dptr) return kErrArg;
  OutRef r;
  int rc = resolve_output(ctx, name, r);
  if (rc) return rc;
  if (frame < 0 || frame >= ctx->out.n_frames) return set_error(ctx, kErrArg, "frame out of range");
  if (r.is_pe) {
    // the same PE for every frame, kept on the device once per size
    if ((rc = ctx_enter(ctx))) return rc;
    const float* pe = device_sine_pe(ctx, r.pe_size, (int)r.ne[0], &rc);
    if (rc) return rc;
    *dptr = pe;
    return kOk;
  }
  *dptr = r.dev + (size_t)frame * r.frame_elems;
  return kOk;
}

int s3b_peer_copy_output(s3b_ctx* ctx, const char* name, int frame, void* dst, int dst_device, int64_t dst_bytes) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!dst || dst_device < 0) return set_error(ctx, kErrArg, "bad peer copy destination");
  OutRef r;
  if ((rc = resolve_output(ctx, name, r))) return rc;
  if (r.is_pe) return set_error(ctx, kErrArg, "PE outputs are host-computed; use s3b_output_copy");
  if (frame < 0 || frame >= ctx->out.n_frames) return set_error(ctx, kErrArg, "frame out of range");
  const size_t bytes = (size_t)r.frame_elems * sizeof(float);
  if (dst_bytes < (int64_t)bytes) return set_error(ctx, kErrArg, "destination holds %lld bytes, need %zu",
                                                   (long long)dst_bytes, bytes);
  const float* src = r.dev + (size_t)frame * r.frame_elems;
  cudaError_t e;
  if (dst_device == ctx->device) {
    e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream);
  } else {
    int can = 0;
    if (cudaDeviceCanAccessPeer(&can, ctx->device, dst_device) != cudaSuccess)
      return set_error(ctx, kErrCuda, "cudaDeviceCanAccessPeer(%d, %d)", ctx->device, dst_device);
    if (can) {
      const cudaError_t pe = cudaDeviceEnablePeerAccess(dst_device, 0);
      if (pe != cudaSuccess && pe != cudaErrorPeerAccessAlreadyEnabled)
        return set_error(ctx, kErrCuda, "cudaDeviceEnablePeerAccess(%d): %s", dst_device, cudaGetErrorString(pe));
      cudaGetLastError();  // clears "already enabled"
    }
    // without peer access the driver stages the copy through host memory
    e = cudaMemcpyPeerAsync(dst, dst_device, src, ctx->device, bytes, ctx->stream);
  }
  if (e != cudaSuccess) return set_error(ctx, kErrCuda, "peer copy: %s", cudaGetErrorString(e));
  return kOk;
}

int s3b_device_alloc(s3b_ctx* ctx, int64_t bytes, void** dptr) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!dptr || bytes <= 0) return set_error(ctx, kErrArg, "bad allocation arguments");
  auto b = std::make_shared<DevBuf>();
  if (cudaMalloc(&b->p, (size_t)bytes) != cudaSuccess) {
    b->p = nullptr;
    cudaGetLastError();
    return set_error(ctx, kErrCuda, "cudaMalloc(%lld) failed", (long long)bytes);
  }
  b->bytes = (size_t)bytes;
  *dptr = b->p;
  ctx->user_allocs[b->p] = b;
  return kOk;
}

int s3b_device_free(s3b_ctx* ctx, void* dptr) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  auto it = ctx->user_allocs.find(dptr);
  if (it == ctx->user_allocs.end()) return set_error(ctx, kErrArg, "not an s3b_device_alloc allocation");
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  ctx->user_allocs.erase(it);
  return kOk;
}

int s3b_ipc_export(s3b_ctx* ctx, const void* dptr, void* handle64) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!handle64 || ctx->user_allocs.find(const_cast<void*>(dptr)) == ctx->user_allocs.end())
    return set_error(ctx, kErrArg, "IPC export needs an s3b_device_alloc allocation");
  cudaIpcMemHandle_t h;
  static_assert(sizeof(h) == 64, "CUDA IPC handle size");
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(dptr)) != cudaSuccess)
    return set_error(ctx, kErrCuda, "cudaIpcGetMemHandle: %s", cudaGetErrorString(cudaGetLastError()));
  memcpy(handle64, &h, sizeof(h));
  return kOk;
}

int s3b_ipc_open(s3b_ctx* ctx, const void* handle64, void** dptr) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!handle64 || !dptr) return set_error(ctx, kErrArg, "bad IPC arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  if (cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return set_error(ctx, kErrCuda, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(cudaGetLastError()));
  ctx->ipc_mapped.insert(*dptr);
  return kOk;
}

int s3b_ipc_close(s3b_ctx* ctx, void* dptr) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  auto it = ctx->ipc_mapped.find(dptr);
  if (it == ctx->ipc_mapped.end()) return set_error(ctx, kErrArg, "not an s3b_ipc_open mapping");
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  cudaIpcCloseMemHandle(dptr);
  ctx->ipc_mapped.erase(it);
  return kOk;
}

int s3b_mem_attn(s3b_ctx* ctx, const float* curr, const float* src_pos, int feat, const float* prompt,
                 const float* prompt_pos, int m_total, int n_ptr_tokens, float* out, int device_ptrs) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!ctx->model.has_mem_attn) return set_error(ctx, kErrState, "model has no memory-attention weights");
  if (!curr || !src_pos || !prompt || !prompt_pos || !out || feat <= 0 || m_total <= 0 || n_ptr_tokens < 0 ||
      n_ptr_tokens > m_total)
    return set_error(ctx, kErrArg, "bad memory-attention arguments");
  const int D = ctx->model.hp.neck_dim, MD = ctx->model.hp.mem_out_dim;
  const size_t N = (size_t)feat * feat;
  if (device_ptrs) return mem_attn_run(ctx, curr, src_pos, feat, prompt, prompt_pos, m_total, n_ptr_tokens, out);
  float *dc, *dp, *dpr, *dpp;
  if ((rc = stage_host(ctx, curr, N * D, "ma_h_curr", &dc))) return rc;
  if ((rc = stage_host(ctx, src_pos, N * D, "ma_h_pos", &dp))) return rc;
  if ((rc = stage_host(ctx, prompt, (size_t)m_total * MD, "ma_h_prompt", &dpr))) return rc;
  if ((rc = stage_host(ctx, prompt_pos, (size_t)m_total * MD, "ma_h_ppos", &dpp))) return rc;
  DevBuf* o = ctx->buf("ma_h_out", N * D * 4, &rc);
  if (rc) return rc;
  if ((rc = mem_attn_run(ctx, dc, dp, feat, dpr, dpp, m_total, n_ptr_tokens, o->as<float>()))) return rc;
  if (cudaMemcpyAsync(out, o->p, N * D * 4, cudaMemcpyDeviceToHost, ctx->stream) != cudaSuccess)
    return set_error(ctx, kErrCuda, "device-to-host copy failed");
  return s3b_sync(ctx);
}

int s3b_mem_attn_bank(s3b_ctx* ctx, const float* curr, const float* src_pos, int feat,
                      const float* const* slot_feats, const float* const* slot_pes, const int* slot_tpos, int n_slots,
                      const float* obj_ptrs, const int* ptr_tpos, int n_ptrs, float* out) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!ctx->model.has_mem_attn) return set_error(ctx, kErrState, "model has no memory-attention weights");
  if (!curr || !out || feat <= 0) return set_error(ctx, kErrArg, "bad memory-attention arguments");
  PromptArgs pa;
  if ((rc = prompt_args(ctx, feat, slot_feats, slot_pes, slot_tpos, n_slots, obj_ptrs, ptr_tpos, n_ptrs, pa)))
    return rc;
  if (!src_pos) {
    src_pos = device_sine_pe(ctx, feat, ctx->model.hp.neck_dim, &rc);  // cached_sinpe_256
    if (rc) return rc;
  }
  return mem_attn_run_bank(ctx, curr, src_pos, feat, pa, out);
}

int s3b_op_build_prompt(s3b_ctx* ctx, int feat, const float* const* slot_feats, const float* const* slot_pes,
                        const int* slot_tpos, int n_slots, const float* obj_ptrs, const int* ptr_tpos, int n_ptrs,
                        float* prompt, float* prompt_pos, int64_t capacity_rows, int* m_total, int* n_ptr_tokens) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!prompt || !prompt_pos) return set_error(ctx, kErrArg, "null prompt outputs");
  PromptArgs pa;
  if ((rc = prompt_args(ctx, feat, slot_feats, slot_pes, slot_tpos, n_slots, obj_ptrs, ptr_tpos, n_ptrs, pa)))
    return rc;
  const int64_t rows = (int64_t)pa.n_slots * pa.slot_tokens + (int64_t)pa.n_ptr * pa.split;
  if (m_total) *m_total = (int)rows;
  if (n_ptr_tokens) *n_ptr_tokens = pa.n_ptr * pa.split;
  if (rows > capacity_rows) return set_error(ctx, kErrArg, "prompt needs %lld rows, buffers hold %lld",
                                             (long long)rows, (long long)capacity_rows);
  rc = build_prompt(pa, prompt, prompt_pos, 0, ctx->stream);
  if (rc) return set_error(ctx, launcher_status_code(rc), "prompt build launch failed (%d)", rc);
  return kOk;
}

int s3b_sam_decode(s3b_ctx* ctx, int feat, const float* image_feats, const float* feat_s0, const float* feat_s1,
                   const float* sparse, int n_sparse, int flags, float* masks, float* iou, float* obj_score,
                   float* mask_tokens) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  const SamDecoder& d = ctx->model.dec;
  if (!d.loaded) return set_error(ctx, kErrState, "model has no SAM mask decoder weights");
  if (feat <= 0 || feat > 1024 || !image_feats || !feat_s0 || !feat_s1 || n_sparse < 0 || (n_sparse && !sparse) ||
      (flags & ~(S3B_DEC_ADD_NO_MEM | S3B_DEC_DEVICE_PTRS)))
    return set_error(ctx, kErrArg, "bad mask-decoder arguments");
  const int add_no_mem = (flags & S3B_DEC_ADD_NO_MEM) ? 1 : 0;
  if (flags & S3B_DEC_DEVICE_PTRS)
    return sam_dec_run(ctx, feat, image_feats, feat_s0, feat_s1, sparse, n_sparse, add_no_mem, masks, iou, obj_score,
                       mask_tokens);
  const size_t D = d.D, HH = (size_t)feat * feat, nm = d.n_mask;
  float *di, *d0, *d1, *dsp = nullptr;
  if ((rc = stage_host(ctx, image_feats, HH * D, "dec_h_img", &di))) return rc;
  if ((rc = stage_host(ctx, feat_s0, 16 * HH * D, "dec_h_s0", &d0))) return rc;
  if ((rc = stage_host(ctx, feat_s1, 4 * HH * D, "dec_h_s1", &d1))) return rc;
  if (n_sparse && (rc = stage_host(ctx, sparse, (size_t)n_sparse * D, "dec_h_sparse", &dsp))) return rc;
  DevBuf* o = ctx->buf("dec_h_out", (16 * HH * nm + nm + 1 + nm * D) * 4, &rc);
  if (rc) return rc;
  float* om = o->as<float>();
  float* oi = om + 16 * HH * nm;
  float* oo = oi + nm;
  float* ot = oo + 1;
  if ((rc = sam_dec_run(ctx, feat, di, d0, d1, dsp, n_sparse, add_no_mem, om, oi, oo, ot))) return rc;
  struct Out {
    float* dst;
    const float* src;
    size_t n;
  } outs[4] = {{masks, om, 16 * HH * nm}, {iou, oi, nm}, {obj_score, oo, 1}, {mask_tokens, ot, nm * D}};
  for (const Out& x : outs)
    if (x.dst && cudaMemcpyAsync(x.dst, x.src, x.n * 4, cudaMemcpyDeviceToHost, ctx->stream) != cudaSuccess)
      return set_error(ctx, kErrCuda, "device-to-host copy failed");
  return s3b_sync(ctx);
}

int s3b_sam_prompt_tokens(s3b_ctx* ctx, const float* box, const float* pos_points, int n_pos, const float* neg_points,
                          int n_neg, int orig_width, int orig_height, float* out, int capacity) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!ctx->model.dec.loaded) return set_error(ctx, kErrState, "model has no SAM prompt encoder weights");
  const int n = sam_prompt_tokens(ctx->model.dec, box, pos_points, n_pos, neg_points, n_neg, (float)orig_width,
                                  (float)orig_height, ctx->model.hp.img_size, out, capacity);
  if (n < 0) return set_error(ctx, kErrArg, "bad prompt arguments (or more than %d tokens)", capacity);
  return n;
}

int s3b_sam_dense_pe(s3b_ctx* ctx, int feat, float* out) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!ctx->model.dec.loaded) return set_error(ctx, kErrState, "model has no SAM prompt encoder weights");
  if (feat <= 0 || feat > 1024 || !out) return set_error(ctx, kErrArg, "bad dense-PE arguments");
  const float* pe = sam_dec_dense_pe(ctx, feat, &rc);
  if (rc) return rc;
  if (cudaMemcpyAsync(out, pe, (size_t)feat * feat * ctx->model.dec.D * 4, cudaMemcpyDeviceToHost, ctx->stream) !=
      cudaSuccess)
    return set_error(ctx, kErrCuda, "device-to-host copy failed");
  return s3b_sync(ctx);
}

int s3b_mem_encode(s3b_ctx* ctx, int feat, const float* pix_feat, const float* mask_logits, int mask_h, int mask_w,
                   const float* obj_score, float* out, int flags) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  const MemEncoder& E = ctx->model.menc;
  if (!E.loaded) return set_error(ctx, kErrState, "model has no memory-encoder weights");
  if (feat <= 0 || feat > 512 || !pix_feat || !mask_logits || mask_h < 2 || mask_w < 2 || !out ||
      (flags & ~S3B_MEMENC_DEVICE_PTRS))
    return set_error(ctx, kErrArg, "bad memory-encoder arguments");
  if (flags & S3B_MEMENC_DEVICE_PTRS) return mem_encode_run(ctx, feat, pix_feat, mask_logits, mask_h, mask_w, obj_score, out);
  const size_t HH = (size_t)feat * feat;
  float *dp, *dm, *ds = nullptr;
  if ((rc = stage_host(ctx, pix_feat, HH * E.D, "me_h_pix", &dp))) return rc;
  if ((rc = stage_host(ctx, mask_logits, (size_t)mask_h * mask_w, "me_h_mask", &dm))) return rc;
  if (obj_score && (rc = stage_host(ctx, obj_score, 1, "me_h_score", &ds))) return rc;
  DevBuf* o = ctx->buf("me_h_out", HH * E.MD * 4, &rc);
  if (rc) return rc;
  if ((rc = mem_encode_run(ctx, feat, dp, dm, mask_h, mask_w, ds, o->as<float>()))) return rc;
  if (cudaMemcpyAsync(out, o->p, HH * E.MD * 4, cudaMemcpyDeviceToHost, ctx->stream) != cudaSuccess)
    return set_error(ctx, kErrCuda, "device-to-host copy failed");
  return s3b_sync(ctx);
}

int s3b_obj_ptr(s3b_ctx* ctx, const float* sam_token, const float* obj_score, float* out, int flags) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  const MemEncoder& E = ctx->model.menc;
  if (!E.loaded) return set_error(ctx, kErrState, "model has no object-pointer weights");
  if (!sam_token || !out || (flags & ~S3B_MEMENC_DEVICE_PTRS)) return set_error(ctx, kErrArg, "bad obj_ptr arguments");
  if (flags & S3B_MEMENC_DEVICE_PTRS) return obj_ptr_run(ctx, sam_token, obj_score, out);
  float *dt, *ds = nullptr;
  if ((rc = stage_host(ctx, sam_token, (size_t)E.D, "op_h_tok", &dt))) return rc;
  if (obj_score && (rc = stage_host(ctx, obj_score, 1, "op_h_score", &ds))) return rc;
  DevBuf* o = ctx->buf("op_h_out", (size_t)E.D * 4, &rc);
  if (rc) return rc;
  if ((rc = obj_ptr_run(ctx, dt, ds, o->as<float>()))) return rc;
  if (cudaMemcpyAsync(out, o->p, (size_t)E.D * 4, cudaMemcpyDeviceToHost, ctx->stream) != cudaSuccess)
    return set_error(ctx, kErrCuda, "device-to-host copy failed");
  return s3b_sync(ctx);
}

int s3b_track_step(s3b_ctx* ctx, int feat, const float* neck_trk_0, const float* neck_trk_1, const float* neck_trk_2,
                   const float* const* slot_feats, const float* const* slot_pes, const int* slot_tpos, int n_slots,
                   const float* obj_ptrs, const int* ptr_tpos, int n_ptrs, float* mask_logits, float* scores,
                   float* mem_feats, float* obj_ptr) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (feat <= 0 || feat > 512 || !neck_trk_0 || !neck_trk_1 || !neck_trk_2)
    return set_error(ctx, kErrArg, "bad tracking-step arguments");
  PromptArgs pa;
  if ((rc = prompt_args(ctx, feat, slot_feats, slot_pes, slot_tpos, n_slots, obj_ptrs, ptr_tpos, n_ptrs, pa)))
    return rc;
  // a tracker that keeps its memory bank and feature maps in the same buffers from frame to frame replays
  // the step (about 130 launches) from a CUDA graph; the key holds every pointer and position it depends on
  std::vector<uintptr_t> key = {10,
                                (uintptr_t)feat,
                                (uintptr_t)neck_trk_0,
                                (uintptr_t)neck_trk_1,
                                (uintptr_t)neck_trk_2,
                                (uintptr_t)n_slots,
                                (uintptr_t)obj_ptrs,
                                (uintptr_t)n_ptrs,
                                (uintptr_t)mask_logits,
                                (uintptr_t)scores,
                                (uintptr_t)mem_feats,
                                (uintptr_t)obj_ptr};
  for (int s = 0; s < n_slots; ++s) {
    key.push_back((uintptr_t)slot_feats[s]);
    key.push_back((uintptr_t)(slot_pes ? slot_pes[s] : nullptr));
    key.push_back((uintptr_t)(intptr_t)slot_tpos[s]);
  }
  for (int p = 0; p < n_ptrs; ++p) key.push_back((uintptr_t)(intptr_t)ptr_tpos[p]);
  return run_graphed(ctx, key, [&] {
    return track_step_run(ctx, feat, neck_trk_0, neck_trk_1, neck_trk_2, pa, mask_logits, scores, mem_feats, obj_ptr);
  });
}

int s3b_sam_best_mask(const float* iou, int n_masks, int multimask) {
  if (!iou || n_masks <= 0) return S3B_ERR_ARG;
  if (!multimask || n_masks < 2) return 0;
  // multimask output: the best of the tokens 1 .. n-1 by predicted IoU, first one on ties
  int best = 1;
  for (int m = 2; m < n_masks; ++m)
    if (iou[m] > iou[best]) best = m;
  return best;
}

int s3b_test_wait_timeout(s3b_ctx* ctx, int64_t limit_ns, int withhold) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  rc = wait_probe(ctx->d_err, limit_ns, withhold, ctx->stream);
  count_launch(ctx);
  if (rc) return set_error(ctx, launcher_status_code(rc), "wait probe: limit_ns must be in (0, 2e9] (%d)", rc);
  return kOk;
}

int s3b_select_memory_frames(int bank_size, int max_slots, int* out_idx, int capacity) {
  if (bank_size < 0 || max_slots < 0 || (!out_idx && capacity > 0)) return kErrArg;
  // sam3_select_memory_frames (sam3.cpp:9423-9447): all slots when they fit, else the first, the
  // last and max_slots - 2 evenly spaced between them, sorted and unique
  std::vector<int> sel;
  if (bank_size <= max_slots) {
    for (int i = 0; i < bank_size; ++i) sel.push_back(i);
  } else {
    sel.push_back(0);
    sel.push_back(bank_size - 1);
    const int remaining = max_slots - 2;
    if (remaining > 0) {
      const float step = (float)(bank_size - 2) / (float)(remaining + 1);
      for (int i = 0; i < remaining; ++i) {
        int idx = 1 + (int)((float)(i + 1) * step);
        if (idx > bank_size - 2) idx = bank_size - 2;
        sel.push_back(idx);
      }
    }
    std::sort(sel.begin(), sel.end());
    sel.erase(std::unique(sel.begin(), sel.end()), sel.end());
  }
  if ((int)sel.size() > capacity) return kErrArg;
  for (size_t i = 0; i < sel.size(); ++i) out_idx[i] = sel[i];
  return (int)sel.size();
}

int s3b_sine_pe_2d(int H, int W, int d_model, float* out) {
  if (H <= 0 || W <= 0 || d_model <= 0 || (d_model & 1) || !out) return kErrArg;
  sine_pe_2d(H, W, d_model, out);
  return kOk;
}

int s3b_op_gemm(s3b_ctx* ctx, const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K,
                const float* bias, int act, void* out, int out_f32, int64_t ldo, const float* resid, int64_t ldr) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!A || !B || !out || M <= 0 || N <= 0 || K <= 0) return set_error(ctx, kErrArg, "bad gemm arguments");
  EpiParams ep;
  ep.mode = EPI_STORE;
  ep.act = act;
  ep.bias = bias;
  ep.out = out;
  ep.out_f32 = out_f32;
  ep.ldo = ldo;
  ep.resid = resid;
  ep.ldr = ldr;
  rc = gemm_f16(reinterpret_cast<const __half*>(A), lda, reinterpret_cast<const __half*>(B), ldb, M, N, K, ep,
                ctx->d_err, ctx->stream);
  if (rc) return set_error(ctx, launcher_status_code(rc), "gemm launch failed (%d)", rc);
  return kOk;
}

int s3b_op_gemm_rope(s3b_ctx* ctx, const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K,
                     const float* bias, const float* table, int rope_d, int rope_cols, int64_t rope_mod, void* out,
                     int out_f32, int64_t ldo) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!A || !B || !out || !table || M <= 0 || N <= 0 || K <= 0 || rope_d <= 0 || (rope_d & 1) || rope_mod <= 0)
    return set_error(ctx, kErrArg, "bad gemm_rope arguments");
  // the epilogue reads the table position-major: re-lay the caller's [positions][rope_d/2][2] table
  // into a context buffer, one strided copy per frequency
  const int half_d = rope_d / 2;
  DevBuf* tb = ctx->buf("gemm_rope_table", (size_t)rope_mod * half_d * 8, &rc);
  if (rc) return rc;
  for (int i = 0; i < half_d; ++i) {
    if (cudaMemcpy2DAsync(static_cast<char*>(tb->p) + (size_t)i * rope_mod * 8, 8, table + 2 * i, (size_t)half_d * 8, 8,
                          (size_t)rope_mod, cudaMemcpyDeviceToDevice, ctx->stream) != cudaSuccess)
      return set_error(ctx, kErrCuda, "gemm_rope: table copy failed");
  }
  EpiParams ep;
  ep.mode = EPI_STORE;
  ep.bias = bias;
  ep.out = out;
  ep.out_f32 = out_f32;
  ep.ldo = ldo;
  ep.rope = tb->as<float>();
  ep.rope_D = rope_d;
  ep.rope_cols = rope_cols;
  ep.rope_rows = M;
  ep.rope_mod = rope_mod;
  rc = gemm_f16(reinterpret_cast<const __half*>(A), lda, reinterpret_cast<const __half*>(B), ldb, M, N, K, ep,
                ctx->d_err, ctx->stream);
  if (rc) return set_error(ctx, launcher_status_code(rc), "gemm_rope launch failed (%d)", rc);
  return kOk;
}

int s3b_op_attention(s3b_ctx* ctx, const void* q, const void* k, const void* v, void* out, int batch, int heads,
                     int nq, int nk, int d, float scale) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!q || !k || !v || !out) return set_error(ctx, kErrArg, "null pointer");
  AttnParams p;
  p.q = reinterpret_cast<const __half*>(q);
  p.k = reinterpret_cast<const __half*>(k);
  p.v = reinterpret_cast<const __half*>(v);
  p.o = reinterpret_cast<__half*>(out);
  p.q_b = (long long)heads * nq * d;
  p.q_h = (long long)nq * d;
  p.k_b = p.v_b = (long long)heads * nk * d;
  p.k_h = p.v_h = (long long)nk * d;
  p.q_n = p.k_n = p.v_n = d;
  p.heads = heads;
  p.nq = nq;
  p.nk = nk;
  p.o_n = (long long)heads * d;
  p.scale = scale;
  // the engine's own dispatch (tcgen05 kernels where their layout rules hold, else mma.sync)
  return run_attn(ctx, p, d, batch * heads);
}

int s3b_op_attention_qkv(s3b_ctx* ctx, const void* qkv, int64_t ld, void* out, int64_t ld_out, int nwin, int heads,
                         int ntok, int d, float scale) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!qkv || !out || nwin <= 0 || heads <= 0 || ntok <= 0 || d <= 0 || ld < 3LL * heads * d || ld_out < (int64_t)heads * d)
    return set_error(ctx, kErrArg, "bad attention_qkv arguments");
  AttnParams p;
  p.q = reinterpret_cast<const __half*>(qkv);
  p.k = p.q + (long long)heads * d;
  p.v = p.q + 2LL * heads * d;
  p.q_b = p.k_b = p.v_b = (long long)ntok * ld;
  p.q_h = p.k_h = p.v_h = d;
  p.q_n = p.k_n = p.v_n = ld;
  p.heads = heads;
  p.nq = p.nk = ntok;
  p.o = reinterpret_cast<__half*>(out);
  p.o_n = ld_out;
  p.scale = scale;
  return run_attn(ctx, p, d, nwin * heads);
}

int s3b_op_resize_bilinear_u8(s3b_ctx* ctx, const uint8_t* src, int n_frames, int src_w, int src_h, uint8_t* dst,
                              int dst_w, int dst_h) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!src || !dst || n_frames <= 0 || src_w <= 0 || src_h <= 0 || dst_w <= 0 || dst_h <= 0)
    return set_error(ctx, kErrArg, "bad resize arguments");
  rc = resize_bilinear_u8(src, n_frames, src_h, src_w, dst_h, dst_w, nullptr, nullptr, dst, ctx->stream);
  if (rc) return set_error(ctx, kErrCuda, "resize launch failed (%d)", rc);
  return kOk;
}

int s3b_op_layernorm(s3b_ctx* ctx, const float* x, void* out, int out_f32, int64_t rows, int C, const float* g,
                     const float* b, float eps) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!x || !out || !g) return set_error(ctx, kErrArg, "null pointer");
  RowMap id;
  rc = layernorm(x, C, out, out_f32, C, rows, C, g, b, eps, id, ctx->stream);
  if (rc) return set_error(ctx, kErrArg, "layernorm launch failed (%d)", rc);
  return kOk;
}

int s3b_op_conv3x3(s3b_ctx* ctx, const void* x, int B, int H, int W, int C, const void* w, const float* bias,
                   float* out, int Cout) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!x || !w || !out || B <= 0 || H <= 0 || W <= 0 || C <= 0 || Cout <= 0 || C % 8 || Cout % 8)
    return set_error(ctx, kErrArg, "bad conv3x3 arguments");
  const long long M = (long long)B * H * W;
  EpiParams ep;
  ep.mode = EPI_STORE;
  ep.bias = bias;
  ep.out = out;
  ep.out_f32 = 1;
  ep.ldo = Cout;
  if (ctx->conv_implicit && C % 64 == 0) {
    // implicit GEMM: no column matrix
    rc = gemm_conv3x3(reinterpret_cast<const __half*>(x), B, H, W, C, reinterpret_cast<const __half*>(w), 9LL * C,
                      Cout, ep, ctx->d_err, ctx->stream);
    if (rc != -2) {
      if (rc) return set_error(ctx, launcher_status_code(rc), "implicit conv3x3 launch failed (%d)", rc);
      return kOk;
    }
  }
  DevBuf* col = ctx->buf("op_conv_col", (size_t)M * 9 * C * 2, &rc);
  if (rc) return rc;
  rc = im2col_3x3_cl(reinterpret_cast<const __half*>(x), B, H, W, C, col->as<__half>(), ctx->stream);
  if (rc) return set_error(ctx, kErrCuda, "im2col launch failed (%d)", rc);
  rc = gemm_f16(col->as<__half>(), 9LL * C, reinterpret_cast<const __half*>(w), 9LL * C, (int)M, Cout, 9 * C, ep,
                ctx->d_err, ctx->stream);
  if (rc) return set_error(ctx, launcher_status_code(rc), "conv gemm launch failed (%d)", rc);
  return kOk;
}

int s3b_op_deconv2x2(s3b_ctx* ctx, const void* x, int B, int H, int W, int Cin, const void* w, const float* bias,
                     int act, void* out, int out_f32, int Cout) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!x || !w || !out || B <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cout <= 0 || Cin % 8 || Cout % 32 ||
      (act != 0 && act != 1))
    return set_error(ctx, kErrArg, "bad deconv2x2 arguments");
  EpiParams ep;
  ep.mode = EPI_STORE;
  ep.bias = bias;
  ep.act = act ? ACT_GELU_ERF : ACT_NONE;
  ep.out = out;
  ep.out_f32 = out_f32 ? 1 : 0;
  ep.ldo = Cout;
  const __half* xh = reinterpret_cast<const __half*>(x);
  const __half* wh = reinterpret_cast<const __half*>(w);
  if (ctx->conv_implicit) {
    rc = gemm_deconv2x2(xh, B, H, W, Cin, wh, Cin, Cout, ep, ctx->d_err, ctx->stream);
    if (rc != -2) {
      if (rc) return set_error(ctx, launcher_status_code(rc), "deconv2x2 launch failed (%d)", rc);
      return kOk;
    }
  }
  // scattered 16-value stores of each (ky, kx) group at pixel (2y + ky, 2x + kx)
  ep.mode = EPI_DECONV2;
  ep.cout = Cout;
  ep.map.W = W;
  ep.map.H = H;
  rc = gemm_f16(xh, Cin, wh, Cin, B * H * W, 4 * Cout, Cin, ep, ctx->d_err, ctx->stream);
  if (rc) return set_error(ctx, launcher_status_code(rc), "deconv2x2 gemm launch failed (%d)", rc);
  return kOk;
}

int s3b_op_gemm_q(s3b_ctx* ctx, const void* A, int64_t lda, const void* blocks, int type, int M, int N, int K,
                  const float* bias, int act, void* out, int out_f32, int64_t ldo, const float* resid, int64_t ldr) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  if (!A || !blocks || !out || M <= 0 || N <= 0 || K <= 0) return set_error(ctx, kErrArg, "bad gemm_q arguments");
  if (type != QT_Q4_0 && type != QT_Q8_0) return set_error(ctx, kErrUnsupported, "gemm_q takes q4_0 or q8_0 rows");
  if (K % 32 || N % 8) return set_error(ctx, kErrArg, "gemm_q needs K %% 32 == 0 and N %% 8 == 0");
  // the rows are split into the value and scale planes in context workspaces, then multiplied
  const size_t vbytes = (size_t)N * (type == QT_Q4_0 ? K / 2 : K);
  DevBuf* qv = ctx->buf("gemm_q_values", vbytes, &rc);
  if (rc) return rc;
  DevBuf* qs = ctx->buf("gemm_q_scales", (size_t)N * (K / 32) * 2, &rc);
  if (rc) return rc;
  rc = repack_q_rows(blocks, type, N, K, qv->p, qs->as<__half>(), ctx->stream);
  if (rc) return set_error(ctx, kErrArg, "gemm_q repack launch failed (%d)", rc);
  EpiParams ep;
  ep.mode = EPI_STORE;
  ep.act = act;
  ep.bias = bias;
  ep.out = out;
  ep.out_f32 = out_f32;
  ep.ldo = ldo;
  ep.resid = resid;
  ep.ldr = ldr;
  QWeight w;
  w.type = type;
  w.values = qv->p;
  w.scales = qs->as<__half>();
  rc = gemm_q(reinterpret_cast<const __half*>(A), lda, w, M, N, K, ep, ctx->d_err, ctx->stream);
  if (rc) return set_error(ctx, launcher_status_code(rc), "gemm_q launch failed (%d)", rc);
  return kOk;
}

int s3b_op_dequantize(s3b_ctx* ctx, const void* src, int type, int64_t ne0, int64_t nrows, float* dst) {
  int rc = ctx_enter(ctx);
  if (rc) return rc;
  rc = dequant_rows(src, type, ne0, nrows, dst, 1, ne0, ctx->stream);
  if (rc) return set_error(ctx, kErrArg, "dequantize launch failed (%d)", rc);
  return kOk;
}

int64_t s3b_row_size(int type, int64_t ne0) { return qtype_row_bytes(type, ne0); }

int s3b_quantize_rows(int type, const float* src, int64_t ne0, int64_t nrows, void* dst) {
  if (!src || !dst || ne0 % 32 || nrows < 0) return kErrArg;
  if (type != QT_Q4_0 && type != QT_Q4_1 && type != QT_Q8_0) return kErrUnsupported;
  const int64_t rb = qtype_row_bytes(type, ne0);
  for (int64_t r = 0; r < nrows; ++r)
    quantize_row_host(type, src + r * ne0, ne0, reinterpret_cast<uint8_t*>(dst) + r * rb);
  return kOk;
}

int s3b_dequantize_rows(int type, const void* src, int64_t ne0, int64_t nrows, float* dst) {
  if (!src || !dst || ne0 % 32 || nrows < 0) return kErrArg;
  if (type != QT_Q4_0 && type != QT_Q4_1 && type != QT_Q8_0) return kErrUnsupported;
  FileTensor t;
  t.dtype = type;
  t.ne[0] = ne0;
  t.ne[1] = nrows;
  const int64_t bytes = qtype_row_bytes(type, ne0) * nrows;
  t.data.assign(reinterpret_cast<const uint8_t*>(src), reinterpret_cast<const uint8_t*>(src) + bytes);
  std::vector<float> f;
  tensor_to_f32(t, f);
  memcpy(dst, f.data(), f.size() * 4);
  return kOk;
}

}  // extern "C"
