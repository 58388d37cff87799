// One tracking step of one object on B200 (host orchestration, C++14).
//
// Composes what sam3_propagate_frame (sam3.cpp:12128-12203) runs per object on a frame the encoder has
// already processed: sam3_propagate_single (11171-11453: memory prompt from the object's memory bank,
// memory attention on neck_trk_2, the SAM mask decoder on its output with neck_trk_0 / 1 and the single
// not_a_point token, the mask choice by IoU), then sam3_encode_memory (11506-11603) of the kept mask
// and sam3_extract_obj_ptr_cpu (9344-9418) of its SAM token. Everything stays on the device and on the
// context stream: the kept mask's index is chosen by a kernel, the object score is read by the kernels
// that depend on it, and nothing is copied to the host. The tracker's bookkeeping around it (masklet
// confirmation, bank eviction, the binary mask at the original resolution) stays with the caller.
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

int track_step_run(s3b_ctx* ctx, int H, const float* trk0, const float* trk1, const float* trk2, const PromptArgs& pa,
                   float* mask_out, float* scores_out, float* mem_out, float* ptr_out) {
  const Model& M = ctx->model;
  if (!M.has_mem_attn || !M.dec.loaded || !M.menc.loaded)
    return set_error(ctx, kErrState, "tracking needs memory attention, the mask decoder and the memory encoder");
  const int D = M.hp.neck_dim, nm = M.dec.n_mask;
  const long long HH = (long long)H * H, plane = 16 * HH;
  int rc = 0;
  DevBuf* cond = ctx->buf("trk_cond", (size_t)HH * D * 4, &rc);
  DevBuf* outs = ctx->buf("trk_dec", ((size_t)nm * plane + nm + 4 + (size_t)nm * 256 + 256 + 4) * 4, &rc);
  if (rc) return rc;
  float* masks = outs->as<float>();
  float* iou = masks + (size_t)nm * plane;
  float* obj = iou + nm;
  float* toks = obj + 4;
  float* tok = toks + (size_t)nm * 256;
  float* sc = tok + 256;
  const float* src_pos = sine_pe_device(ctx, H, D, &rc);  // cached_sinpe_256
  if (rc) return rc;
  CKR(mem_attn_run_bank(ctx, trk2, src_pos, H, pa, cond->as<float>()));
  CKR(sam_dec_run(ctx, H, cond->as<float>(), trk0, trk1, nullptr, 0, 0, masks, iou, obj, toks));
  // SAM 2 with multimask output picks the best of the three multimask tokens (and uses its token for the
  // object pointer when use_multimask_token_for_obj_ptr); SAM 3 keeps token 0 (sam3.cpp:11395-11430)
  const int multimask = M.hp.is_sam2 && M.hp.trk_flags[13];
  const int mm_token = multimask && M.hp.trk_flags[3];
  float* kept = mask_out;
  DevBuf* kb = nullptr;
  if (!kept) {
    kb = ctx->buf("trk_kept", (size_t)plane * 4, &rc);
    if (rc) return rc;
    kept = kb->as<float>();
  }
  CKL(pick_mask(masks, plane, iou, toks, nm, multimask, mm_token, kept, tok, scores_out ? scores_out : sc, obj,
                ctx->stream));
  if (mem_out) CKR(mem_encode_run(ctx, H, trk2, kept, 4 * H, 4 * H, obj, mem_out));
  if (ptr_out) CKR(obj_ptr_run(ctx, tok, obj, ptr_out));
  return check_device(ctx, "track_step");
}

}  // namespace s3b
