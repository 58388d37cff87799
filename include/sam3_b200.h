/*
 * sam3_b200.h - C ABI of the B200 encoder engine for sam3.cpp.
 *
 * The engine replaces the ggml graph builders of the per-frame backbone
 * forward and of memory attention in sam3.cpp (PABannier/sam3.cpp) with
 * hand-written sm_100a CUDA kernels. Signatures use plain pointers and sizes
 * only. Every function returns S3B_OK (0) or a negative S3B_ERR_* code; the
 * message of the last error is available from s3b_last_error(), and is also
 * printed to stderr, following the reference's "return false + stderr"
 * convention (sam3.cpp:1021-1022).
 *
 * Layouts follow ggml's memory order: a feature map [C, W, H, B] in ggml
 * notation is channel-last, row index = (b*H + y)*W + x, C contiguous.
 */
#ifndef SAM3_B200_H
#define SAM3_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct s3b_ctx s3b_ctx;

enum {
    S3B_OK = 0,
    S3B_ERR_ARG = -1,
    S3B_ERR_IO = -2,
    S3B_ERR_FORMAT = -3,
    S3B_ERR_CUDA = -4,
    S3B_ERR_STATE = -5,
    S3B_ERR_UNSUPPORTED = -6,
    S3B_ERR_DEVICE = -7, /* a kernel's bounded wait expired; see s3b_last_error */
    S3B_ERR_OOM = -8
};

/* ggml tensor types used by the .ggml files (sam3.cpp:3242-3251). */
enum { S3B_F32 = 0, S3B_F16 = 1, S3B_Q4_0 = 2, S3B_Q4_1 = 3, S3B_Q8_0 = 8 };

/* Epilogue activations of s3b_op_gemm. */
enum { S3B_ACT_NONE = 0, S3B_ACT_GELU_ERF = 1, S3B_ACT_GELU_TANH = 2, S3B_ACT_RELU = 3 };

/* Flags of the encode calls. */
enum {
    S3B_ENCODE_NO_NECK = 1, /* backbone only (no FPN / SimpleFPN neck) */
    S3B_ENCODE_NO_DET = 2   /* SAM 3: skip the detector neck path */
};

/* ---------------------------------------------------------------- context */

/* Creates a context bound to CUDA device `device` with its own stream.
 * Replaces the backend set-up of sam3_load_model (sam3.cpp:3275-3288). */
int s3b_create(int device, s3b_ctx** out);
void s3b_destroy(s3b_ctx* ctx);
const char* s3b_last_error(const s3b_ctx* ctx);
/* Uses `cuda_stream` (a cudaStream_t; NULL = the legacy default stream) for
 * all work of the context; s3b_reset_stream returns to a stream owned by the
 * context. */
int s3b_set_stream(s3b_ctx* ctx, void* cuda_stream);
int s3b_reset_stream(s3b_ctx* ctx);
/* Waits for all work of the context and checks the device error word. */
int s3b_sync(s3b_ctx* ctx);
/* Options: "frames_per_pass" (encoder micro-batch, default 8);
 * "attention_impl" (0: tcgen05 flash attention where eligible: for d = 64
 * the persistent kernel with two 128-query tiles per CTA (one thread per
 * query row, 96-key tiles), windows and global rows alike; 1: always the
 * mma.sync kernel, 2: as 0 but d = 64 on the 64-key-tile tcgen05 kernel,
 * 3: as 0 but d = 64 on the one-tile-per-CTA kernel (two threads per query
 * row, 128-key tiles), 4: the same as 0);
 * "attention_wide_k128" (-1, default: d = 72 / 96 attention over rows of at
 * least 1024 keys, the Hiera global blocks, on the 128-key-tile tcgen05
 * kernel, shorter rows on the 64-key-tile kernel with two CTAs per SM; 1
 * always the 128-key kernel; 0 never; d = 256 always uses it);
 * "attention_fa_exp_poly" (0-4, default 1: of every 8 exponentials of the
 * persistent two-tile kernel, how many are evaluated on the FMA pipe);
 * "gemm_pairs" (which wide GEMMs run 256-row tiles on pairs of SMs, tcgen05
 * cta_group::2: 2, default, all; 1 those with K >= 2048 and the f16-output
 * ones with 16 epilogue warps; 0 none, 128-row tiles on single SMs;
 * applies to every context of the process);
 * "gemm_wide_epilogue" (1, default: GEMMs with K < 2048 run 16 epilogue
 * warps instead of 8; 0: all run 8; process-wide);
 * "weights_quantised" (read by s3b_load_model; q4_0 / q8_0 linear weights
 * stay in block form in device memory, read from HBM only in that form:
 * 1: right before each GEMM one kernel dequantises the layer's weight into
 * an f16 staging buffer sized for the largest layer, which stays in L2 while
 * the unchanged f16 GEMM reads it; 2: the GEMM's own warps dequantise each
 * weight tile in shared memory; 0, default: dequantised to f16 once at load;
 * results are identical in all three);
 * "conv_implicit" (1, default: 3x3 convolutions with C a multiple of 64 run
 * as implicit GEMMs whose TMA loads fetch the shifted pixel blocks, no
 * column matrix, and the neck's 2x2 deconvolutions store their outputs
 * through 5-D TMA; 0: im2col + GEMM and scattered deconvolution stores);
 * "attention_exp_poly" (0-4: of every 8 softmax exponentials in the tcgen05
 * kernel, how many are evaluated by a polynomial on the FMA pipe instead of
 * the MUFU unit; a tuning knob, results agree to f16 rounding);
 * "graphs" (1, default: s3b_mem_attn replays its per-layer body, and the
 * s3b_encode_* calls their whole launch sequence, from a CUDA graph captured
 * on the second call with the same shapes, input pointer, buffers and
 * options, when the context's stream is not the legacy default stream,
 * profiling is off and (encoder) no output is host-bound; 0: every launch
 * issued from the host);
 * "stop_after_blocks" (test hook: run only the first n backbone blocks and
 * no neck, -1 = all; the stage runners of sam3.h:441-496 play this role in
 * the reference). */
int s3b_set_option(s3b_ctx* ctx, const char* key, int64_t value);

/* Profiling (CUDA events on the context stream around every GEMM, attention
 * and LayerNorm launch; the reference times compute with std::chrono around
 * ggml_backend_graph_compute, sam3.cpp:6118-6131). s3b_profile_end waits for
 * the stream and writes the first n (up to 17) of: out[0..3] GEMM {launches,
 * ms, flops, bytes}, out[4..7] attention {launches, ms, flops, bytes},
 * out[8] the total number of kernel launches since s3b_profile_begin,
 * out[9..12] LayerNorm {launches, ms, 0, bytes}, out[13..16] block-form
 * weight staging {launches, ms, 0, bytes}. Bytes and flops are algorithmic
 * (operands and results once). */
int s3b_profile_begin(s3b_ctx* ctx, int with_events);
int s3b_profile_end(s3b_ctx* ctx, double* out, int n);

/* ---------------------------------------------------------------- model */

/* Loads the encoder / memory-attention weights of a .ggml file (SAM 3 or
 * SAM 2.x Hiera; f32, f16, q4_0, q4_1, q8_0 tensors) onto the device.
 * Replaces sam3_load_model + sam3_load_tensors (sam3.cpp:3091-3344);
 * tensors outside the engine's scope are skipped. */
int s3b_load_model(s3b_ctx* ctx, const char* path);

/* s3b_load_model through a persistent cache of the model's device form
 * (the row layouts, block-form planes, folded and fused weights and tables
 * that loading computes from the file; sam3_load_tensors, sam3.cpp:3091-3194,
 * redoes its conversions at every start). When cache_path holds a cache made
 * from the same file (size, modification time and a hash of its first and
 * last MiB), the same engine format and the same "weights_quantised" option,
 * the model is copied from it to the device with no conversion and 1 is
 * returned. Otherwise the file is loaded as s3b_load_model does, the cache is
 * (re)written and 0 is returned; a cache that cannot be written is reported
 * on stderr and does not fail the load. Negative: the load failed. */
int s3b_load_model_cached(s3b_ctx* ctx, const char* model_path, const char* cache_path);

/* A weight tensor in the caller's host memory, as sam3.cpp holds it after
 * sam3_load_tensors (sam3.cpp:3091-3194): the .ggml tensor name, its ggml
 * type, shape in ggml order (ne[0] contiguous; unused dims 1) and data in
 * ggml row layout (s3b_row_size(dtype, ne[0]) bytes per row). */
typedef struct s3b_tensor_desc {
    const char* name;
    int32_t dtype;
    int32_t n_dims;
    int64_t ne[4];
    const void* data;
} s3b_tensor_desc;

/* Loads the weights from tensors the caller already holds (copied to the
 * device, the host memory stays the caller's), so a sam3.cpp that has
 * loaded its model does not parse the file a second time. hparams are the
 * n_hparams i32 values of the file header after magic / version / ftype /
 * n_tensors, in file order (SAM 3: sam3.cpp:1477-1520, is_sam2 = 0;
 * SAM 2: 1564-1626, is_sam2 = 1); ftype is the file type. The result is the
 * same device model as s3b_load_model on the file the tensors came from;
 * tensors outside the engine's scope are skipped. */
int s3b_load_weights(s3b_ctx* ctx, int is_sam2, const int32_t* hparams, int n_hparams, int ftype,
                     const s3b_tensor_desc* descs, int n);

/* Parses a .ggml file on the host only (no device needed) and checks every
 * record: info[0] = 1 for SAM 2 else 0, info[1] = img_size, info[2] = number
 * of tensor records, info[3] = file ftype, info[4] = backbone depth,
 * info[5] = backbone embed dim, info[6] = records with quantised dtypes.
 * Returns S3B_ERR_FORMAT / S3B_ERR_IO on corrupt or truncated files. */
int s3b_inspect_model(const char* path, int32_t* info, int n, char* err, int err_len);

/* info[0] = 1 for SAM 2 (Hiera) else 0, info[1] = img_size, info[2] = number
 * of backbone blocks, info[3] = backbone embed dim, info[4] = neck dim,
 * info[5] = memory-attention layers (0 if absent), info[6] = device bytes of
 * weights (low 31 bits, MiB). */
int s3b_model_info(s3b_ctx* ctx, int32_t* info, int n);

/* ---------------------------------------------------------------- encoder */

/* Encodes n_frames uint8 HWC frames of img_size^2 (host memory): SAM 3
 * normalisation (p/255-0.5)/0.5 or SAM 2 ImageNet mean/std
 * (sam3.cpp:3486-3544), then backbone + neck. Replaces sam3_encode_image
 * (sam3.cpp:6024-6212, 5857-6018) for frames already at the model size. */
int s3b_encode_u8(s3b_ctx* ctx, const uint8_t* frames_hwc, int n_frames, int img_size, int flags);

/* Encodes n_frames uint8 HWC frames of width x height (host memory), resized
 * on the device to the model size by the reference's bilinear (f64 weights,
 * half-pixel centres, rounded to uint8: sam3_resize_bilinear,
 * sam3.cpp:3441-3481) and normalised in the same pass; frames already at the
 * model size skip the resize (sam3.cpp:3496). All frames share one size.
 * Replaces sam3_encode_image (sam3.cpp:6024-6212, 5857-6018) for any image. */
int s3b_encode_image_u8(s3b_ctx* ctx, const uint8_t* frames_hwc, int n_frames, int width, int height, int flags);
int s3b_encode_image_u8_device(s3b_ctx* ctx, const uint8_t* d_frames_hwc, int n_frames, int width, int height,
                               int flags);

/* Same from preprocessed f32 CHW frames in host memory; replaces
 * sam3_encode_image_from_preprocessed (sam3.h:426-435, sam3.cpp:6997-7481). */
int s3b_encode_chw(s3b_ctx* ctx, const float* frames_chw, int n_frames, int img_size, int flags);

/* Same with device pointers (frames already resident in HBM). */
int s3b_encode_u8_device(s3b_ctx* ctx, const uint8_t* d_frames_hwc, int n_frames, int img_size, int flags);
int s3b_encode_chw_device(s3b_ctx* ctx, const float* d_frames_chw, int n_frames, int img_size, int flags);

/* Shape (ggml order ne[0..3]) of an output of the last encode call. Names
 * follow sam3_dump_state_tensor (sam3.cpp:14334-14376): "vit_output",
 * "neck_trk_0".."neck_trk_3", "neck_det_0".."neck_det_3", "neck_trk_pe_i".
 * For SAM 2 the FPN levels are "neck_trk_0".."neck_trk_2". */
int s3b_output_shape(s3b_ctx* ctx, const char* name, int64_t ne[4]);
/* Copies frame `frame` of an output to host memory (n floats). */
int s3b_output_copy(s3b_ctx* ctx, const char* name, int frame, float* dst, int64_t n);
/* Device pointer of frame `frame` of an output (valid until the next encode;
 * the "neck_*_pe_i" outputs are one device table per size, the same for
 * every frame, valid until the context is destroyed). */
int s3b_output_device_ptr(s3b_ctx* ctx, const char* name, int frame, const float** dptr);

/* Binds host memory (`n_floats` floats, pinned by the caller for the copies
 * to overlap) to output `name` ("vit_output", "neck_trk_i", "neck_det_i"):
 * every later encode call copies each pass's frames of that output (f32,
 * frame f at host + f * frame_elems) to it on a copy stream of the context,
 * while the next pass computes; the next call's pass waits only for the copy
 * of the frames it overwrites. s3b_sync waits for the copies. host = NULL
 * unbinds. An encode call fails with S3B_ERR_ARG if a bound buffer is
 * smaller than n_frames * frame_elems. This is the host hand-off of
 * state.neck_trk that sam3_propagate_single does with ggml_backend_tensor_get
 * (sam3.cpp:11378-11391), moved off the critical path. */
int s3b_output_host_bind(s3b_ctx* ctx, const char* name, float* host, int64_t n_floats);

/* ---------------------------------------------------------------- features to the tracking GPU */

/* Copies frame `frame` of output `name` (as s3b_output_device_ptr) into
 * device memory `dst` of GPU `dst_device`: over NVLink peer access
 * (cudaMemcpyPeerAsync, peer access enabled on first use) when dst_device is
 * not the context's GPU, else a device-to-device copy. dst may be another
 * GPU's buffer of this process or a pointer from s3b_ipc_open (one process
 * per GPU). Enqueued on the context stream after the encode that produced
 * the output; s3b_sync(ctx) waits for it. dst_bytes must hold the frame's
 * output. This is the hand-off of per-frame features from an encoding GPU to
 * the tracking GPU, which the reference does through host copies of
 * state.neck_trk (sam3_propagate_single, sam3.cpp:11378-11391). */
int s3b_peer_copy_output(s3b_ctx* ctx, const char* name, int frame, void* dst, int dst_device, int64_t dst_bytes);

/* Device memory owned by the context's GPU (cudaMalloc'd, so it has its own
 * base address and can be shared by s3b_ipc_export), freed by
 * s3b_device_free or with the context. */
int s3b_device_alloc(s3b_ctx* ctx, int64_t bytes, void** dptr);
int s3b_device_free(s3b_ctx* ctx, void* dptr);
/* CUDA IPC for the one-process-per-GPU layout: export writes the 64-byte
 * handle of an allocation made by s3b_device_alloc; another process opens it
 * (its context on any GPU of the box) and gets a device pointer it can pass
 * to s3b_peer_copy_output; close releases the mapping. */
int s3b_ipc_export(s3b_ctx* ctx, const void* dptr, void* handle64);
int s3b_ipc_open(s3b_ctx* ctx, const void* handle64, void** dptr);
int s3b_ipc_close(s3b_ctx* ctx, void* dptr);

/* ---------------------------------------------------------------- memory attention */

/* Memory attention (sam3_build_mem_attn_graph, sam3.cpp:9224-9337) on one
 * feature map of side `feat` (N = feat^2 tokens, D = 256):
 *   curr       [N][D]  current-frame features (neck_trk level 2, channel-last)
 *   src_pos    [N][D]  sinusoidal PE of the current tokens
 *   prompt     [M][64] memory tokens (spatial slots then object-pointer tokens)
 *   prompt_pos [M][64]
 *   n_ptr_tokens: trailing pointer tokens excluded from RoPE
 *   out        [N][D]
 * RoPE tables (axial, dim 256, theta 1e4, feat x feat; sam3.cpp:11126-11169)
 * are computed by the engine. `device_ptrs` = 1 if all pointers are device
 * pointers, 0 if they are host pointers. */
int s3b_mem_attn(s3b_ctx* ctx, const float* curr, const float* src_pos, int feat, const float* prompt,
                 const float* prompt_pos, int m_total, int n_ptr_tokens, float* out, int device_ptrs);

/* Memory attention with the memory prompt built on the device from a
 * memory bank in device memory: replaces sam3_build_prompt_and_pos
 * (sam3.cpp:9123-9209) + sam3_build_mem_attn_graph (9224-9337) as
 * sam3_propagate_single calls them (11182-11307), with no host loop, host
 * GEMV or host-to-device copy of the prompt. All pointers are device
 * pointers except the int arrays and the two pointer arrays themselves:
 *   curr [N][256], N = feat^2; src_pos [N][256] or NULL (the engine's sine
 *     PE of the feat x feat grid, tracker.cached_sinpe_256);
 *   slot_feats[s]: [N][64] f32 spatial memory features of selected slot s
 *     (s < n_slots <= 16, in prompt order); slot_pes[s]: [N][64] or NULL
 *     (the 64-channel sine PE, tracker.cached_sinpe_64); slot_pes may be NULL;
 *   slot_tpos[s]: temporal position (0 = conditioning frame); when
 *     0 <= tpos < num_maskmem the PE row maskmem_tpos_enc[num_maskmem -
 *     tpos - 1] is added to the slot's PE;
 *   obj_ptrs [n_ptrs][256] f32 (n_ptrs <= 16); ptr_tpos[p]: frame distance
 *     of pointer p (< 0: skipped); each kept pointer becomes 4 tokens of 64
 *     with the 256 -> 64 projection of the 1-D sine PE of distance / 15;
 *   out [N][256].
 * Results equal s3b_mem_attn on the prompt the reference builds. */
int s3b_mem_attn_bank(s3b_ctx* ctx, const float* curr, const float* src_pos, int feat,
                      const float* const* slot_feats, const float* const* slot_pes, const int* slot_tpos, int n_slots,
                      const float* obj_ptrs, const int* ptr_tpos, int n_ptrs, float* out);

/* The device prompt build of s3b_mem_attn_bank alone: writes prompt and
 * prompt_pos (device f32 [m_total][64], capacity_rows rows each) as
 * sam3_build_prompt_and_pos (sam3.cpp:9123-9209) returns them, and
 * m_total / n_ptr_tokens (either may be NULL). */
int s3b_op_build_prompt(s3b_ctx* ctx, int feat, const float* const* slot_feats, const float* const* slot_pes,
                        const int* slot_tpos, int n_slots, const float* obj_ptrs, const int* ptr_tpos, int n_ptrs,
                        float* prompt, float* prompt_pos, int64_t capacity_rows, int* m_total, int* n_ptr_tokens);

/* ---------------------------------------------------------------- SAM mask decoder */

/* SAM mask decoder (sam3_build_sam_dec_graph, sam3.cpp:10544-10757, with the
 * prompt encoder's dense inputs of sam3_populate_pe_cache, 10288-10345) on
 * one frame, as the image predictor (sam3_segment_pvs, 10760-10990) and the
 * tracker (sam3_propagate_single, 11171-11453) call it:
 *   image_feats [feat*feat][256] f32: neck_trk_2 (image predictor, with
 *     S3B_DEC_ADD_NO_MEM: no_mem_embed is added as sam3.cpp:10922-10931 does)
 *     or the memory-attention output (tracker);
 *   feat_s0 [(4 feat)^2][256], feat_s1 [(2 feat)^2][256]: neck_trk_0 / 1;
 *   sparse [n_sparse][256]: prompt tokens (s3b_sam_prompt_tokens); n_sparse
 *     = 0 uses the single not_a_point token of the tracker (11311-11314);
 *     at most 26 tokens;
 *   outputs (each may be NULL): masks [4][(4 feat)^2] mask logits, iou [4]
 *     (sigmoid), obj_score [1] (logit; 10 without an object-score head),
 *     mask_tokens [4][256] (token 0 is the SAM output token of the object
 *     pointer).
 * With S3B_DEC_DEVICE_PTRS every array is device memory and the call is
 * asynchronous on the context stream; otherwise they are host arrays and the
 * call returns when the outputs are written. */
#define S3B_DEC_ADD_NO_MEM 1
#define S3B_DEC_DEVICE_PTRS 2
int s3b_sam_decode(s3b_ctx* ctx, int feat, const float* image_feats, const float* feat_s0, const float* feat_s1,
                   const float* sparse, int n_sparse, int flags, float* masks, float* iou, float* obj_score,
                   float* mask_tokens);

/* Sparse prompt tokens of the image predictor (sam3_collect_pvs_prompt_tokens,
 * sam3.cpp:10361-10391, encoded as sam3_segment_pvs does at 10877-10900):
 * box corners (labels 2, 3; box = {x0, y0, x1, y1} or NULL), positive points,
 * negative points, then one padding token, in original-image pixels
 * (orig_width x orig_height). Writes [n][256] host floats and returns n, or a
 * negative status (S3B_ERR_ARG also when n > capacity). */
int s3b_sam_prompt_tokens(s3b_ctx* ctx, const float* box, const float* pos_points, int n_pos, const float* neg_points,
                          int n_neg, int orig_width, int orig_height, float* out, int capacity);

/* The decoder's dense image PE of a feat x feat grid (the dense_pe_cache of
 * sam3_populate_pe_cache, sam3.cpp:10330-10341) into host floats
 * [feat*feat][256]. */
int s3b_sam_dense_pe(s3b_ctx* ctx, int feat, float* out);

/* Mask choice of sam3_propagate_single (sam3.cpp:11395-11420): 0 without
 * multimask output, else the index in 1 .. n_masks-1 with the highest IoU
 * (first on ties). S3B_ERR_ARG on bad arguments. */
int s3b_sam_best_mask(const float* iou, int n_masks, int multimask);

/* ---------------------------------------------------------------- memory encoder */

/* Memory encoder of the tracker (sam3_encode_memory, sam3.cpp:11506-11603):
 * the frame's mask logits [mask_h][mask_w] (the decoder's chosen mask) are
 * resized to the model input size, mapped through sigmoid * scale + bias
 * (20 / -10, or the SAM 2 file's values), resized to 16 feat, downsampled
 * (4 conv stages + 1x1), added to the 1x1 projection of pix_feat
 * [feat*feat][256] (neck_trk_2), fused by two CXBlocks and projected to the
 * memory features out [feat*feat][64]. obj_score (one float, may be NULL =
 * object present): when <= 0, no_obj_embed_spatial is added (11575-11589).
 * With S3B_MEMENC_DEVICE_PTRS all pointers are device memory (asynchronous on
 * the context stream, the score is read on the device); otherwise host
 * memory and the call returns when out is written. The slot's spatial PE is
 * the 64-channel sine PE (s3b_sine_pe_2d, or NULL slot_pes in
 * s3b_mem_attn_bank). */
#define S3B_MEMENC_DEVICE_PTRS 2
int s3b_mem_encode(s3b_ctx* ctx, int feat, const float* pix_feat, const float* mask_logits, int mask_h, int mask_w,
                   const float* obj_score, float* out, int flags);

/* Object pointer (sam3_extract_obj_ptr_cpu, sam3.cpp:9344-9418): the 3-layer
 * ReLU MLP of the SAM output token sam_token [256] (s3b_sam_decode's
 * mask_tokens[0]), replaced by no_obj_ptr when *obj_score <= 0 (NULL: object
 * present); out [256]. Pointers as in s3b_mem_encode. */
int s3b_obj_ptr(s3b_ctx* ctx, const float* sam_token, const float* obj_score, float* out, int flags);

/* ---------------------------------------------------------------- tracking step */

/* One tracking step of one object on a frame the encoder has processed, as
 * sam3_propagate_frame runs it per object (sam3.cpp:12128-12203):
 * sam3_propagate_single (11171-11453: memory attention on neck_trk_2 with the
 * prompt built from the object's memory bank, the SAM mask decoder on its
 * output with neck_trk_0 / 1 and the single not_a_point token, the mask kept
 * by IoU: token 0 for SAM 3, the best of tokens 1-3 for SAM 2 with multimask
 * output), then sam3_encode_memory of the kept mask (11506-11603) and
 * sam3_extract_obj_ptr_cpu of its SAM token (9344-9418). The bank arguments
 * are those of s3b_mem_attn_bank. Every array is device memory and the step
 * is asynchronous on the context stream; outputs (each may be NULL):
 *   mask_logits [(4 feat)^2] the kept mask; scores [3] = {its IoU, the object
 *   score logit, its token index}; mem_feats [feat*feat][64] the frame's
 *   memory features (its spatial PE is the 64-channel sine PE); obj_ptr [256].
 * The caller keeps the tracker's bookkeeping: it appends mem_feats / obj_ptr
 * to the bank and thresholds the mask at the original resolution. */
int s3b_track_step(s3b_ctx* ctx, int feat, const float* neck_trk_0, const float* neck_trk_1, const float* neck_trk_2,
                   const float* const* slot_feats, const float* const* slot_pes, const int* slot_tpos, int n_slots,
                   const float* obj_ptrs, const int* ptr_tpos, int n_ptrs, float* mask_logits, float* scores,
                   float* mem_feats, float* obj_ptr);

/* Test hook for the engine's failure detection: enqueues on the context
 * stream one kernel that waits on a device barrier with the same bounded
 * wait every GEMM / attention kernel uses, limited to limit_ns (0 < limit_ns
 * <= 2e9). With withhold = 1 nothing completes the barrier, so the wait
 * runs out, records its code in the context's device error word and the
 * kernel returns; the next s3b_sync then reports S3B_ERR_DEVICE and clears
 * the word, and the context stays usable. With withhold = 0 the barrier
 * completes and s3b_sync returns S3B_OK. The reference has no device waits
 * (its error path is "return false + stderr", sam3.cpp:1021-1022). */
int s3b_test_wait_timeout(s3b_ctx* ctx, int64_t limit_ns, int withhold);

/* Host helper: memory-bank slots memory attention reads
 * (sam3_select_memory_frames, sam3.cpp:9423-9447): every slot when
 * bank_size <= max_slots, else the first, the last and max_slots - 2 evenly
 * spaced ones, ascending and unique. Writes at most `capacity` indices and
 * returns their count, or S3B_ERR_ARG. */
int s3b_select_memory_frames(int bank_size, int max_slots, int* out_idx, int capacity);

/* Host helper: sinusoidal 2D PE, channel-last [H][W][d_model], first half
 * of the channels encoding y, second half x (sam3_sinusoidal_pe_2d,
 * sam3.cpp:3597-3633); the values of the "neck_trk_pe_i" outputs. */
int s3b_sine_pe_2d(int H, int W, int d_model, float* out);

/* ---------------------------------------------------------------- operators (device pointers) */

/* out[M][N] = act(A[M][K] * B[N][K]^T + bias) (+ resid), A/B f16 row-major
 * with row strides lda/ldb (multiples of 8 elements); out f16 or f32 with row
 * stride ldo; resid f32 [M][ldr] or NULL. Replaces ggml_mul_mat + ggml_add
 * (+ activation) pairs such as sam3.cpp:3738-3739, 3792-3796. */
int s3b_op_gemm(s3b_ctx* ctx, const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K,
                const float* bias, int act, void* out, int out_f32, int64_t ldo, const float* resid, int64_t ldr);

/* Fused projection + 2D RoPE: out = A B^T + bias, then columns < rope_cols
 * are rotated in pairs (2i, 2i+1) by table [positions][rope_d/2][2] (cos,
 * sin) at position (row % rope_mod) and pair ((col % rope_d) / 2). This is
 * the qkv projection of a ViT block followed by sam3_apply_rope on q and k
 * (sam3.cpp:3738-3771, 3667-3706). */
int s3b_op_gemm_rope(s3b_ctx* ctx, const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K,
                     const float* bias, const float* table, int rope_d, int rope_cols, int64_t rope_mod, void* out,
                     int out_f32, int64_t ldo);

/* softmax(q k^T * scale) v for q [B*H][nq][d], k/v [B*H][nk][d] (f16),
 * out [B][nq][H*d] f16. Replaces ggml_flash_attn_ext (sam3.cpp:3774, 4395,
 * 9267, 9312) with no mask. d in {64, 72, 80, 96, 128, 256}; the engine's
 * dispatch picks the kernel (tcgen05 for d = 256, and for d = 72 / 96 with at
 * least 128 queries; mma.sync otherwise). */
int s3b_op_attention(s3b_ctx* ctx, const void* q, const void* k, const void* v, void* out, int batch, int heads,
                     int nq, int nk, int d, float scale);

/* Attention over a fused qkv buffer, the layout the ViT blocks use:
 * q / k / v of head h of window w at qkv[(w*ntok + n)*ld + {0, E, 2E} + h*d]
 * with E = heads*d (ld >= 3E), nq = nk = ntok; out [nwin*ntok][ld_out] f16 at
 * columns h*d. d = 64 runs the tcgen05 kernel (unless the context option
 * "attention_impl" is 1), other d the mma.sync kernel. Replaces the
 * qkv split + permute + ggml_flash_attn_ext of sam3.cpp:3738-3774. */
int s3b_op_attention_qkv(s3b_ctx* ctx, const void* qkv, int64_t ld, void* out, int64_t ld_out, int nwin, int heads,
                         int ntok, int d, float scale);

/* Bilinear resize of uint8 HWC frames (device pointers) [n][src_h][src_w][3]
 * -> [n][dst_h][dst_w][3]: sam3_resize_bilinear (sam3.cpp:3441-3481), f64
 * arithmetic in the reference's order, (int)(v + 0.5) clamped to [0, 255]. */
int s3b_op_resize_bilinear_u8(s3b_ctx* ctx, const uint8_t* src, int n_frames, int src_w, int src_h, uint8_t* dst,
                              int dst_w, int dst_h);

/* LayerNorm over C of f32 rows: out = (x-mean)/sqrt(var+eps)*g + b, f16 or
 * f32 out. Replaces ggml_norm + mul + add (sam3.cpp:1036-1060). */
int s3b_op_layernorm(s3b_ctx* ctx, const float* x, void* out, int out_f32, int64_t rows, int C, const float* g,
                     const float* b, float eps);

/* 3x3 / stride 1 / pad 1 convolution on channel-last f16 maps x [B][H][W][C]
 * with weights w f16 [Cout][3][3][C] (ky, kx, ci order, i.e. the ggml kernel
 * [3, 3, C, Cout] repacked channel-last), bias f32 [Cout] or NULL, out f32
 * [B][H][W][Cout]. An implicit tensor-core GEMM (C a multiple of 64), else
 * im2col (context workspace) + GEMM.
 * Replaces ggml_conv_2d_s1_ph + bias add (sam3.cpp:3887-3918). C and Cout
 * multiples of 8. */
int s3b_op_conv3x3(s3b_ctx* ctx, const void* x, int B, int H, int W, int C, const void* w, const float* bias,
                   float* out, int Cout);

/* 2x2 / stride 2 transposed convolution on channel-last f16 maps x
 * [B][H][W][Cin] with weights w f16 [2][2][Cout][Cin] (rows (ky*2 + kx)*Cout +
 * co of Cin values, i.e. the ggml kernel [2, 2, Cout, Cin] repacked), bias
 * f32 [Cout] or NULL, act 0 (none) or 1 (GELU, erf form), out f16 (out_f32 =
 * 0) or f32 [B][2H][2W][Cout]. Cin a multiple of 8, Cout of 32. A GEMM over
 * 8 x 16 input-pixel blocks whose outputs leave through 5-D TMA stores
 * (option "conv_implicit" = 0: scattered stores). Replaces
 * ggml_conv_transpose_2d_p0 + bias (+ ggml_gelu_erf) of the SimpleFPN
 * neck (sam3_build_neck_graph, sam3.cpp:3863-3921). */
int s3b_op_deconv2x2(s3b_ctx* ctx, const void* x, int B, int H, int W, int Cin, const void* w, const float* bias,
                     int act, void* out, int out_f32, int Cout);

/* Size of the static device scratch used by s3b_conv3x3_noalloc (32 MiB). */
#define S3B_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* Same computation as s3b_op_conv3x3, for callers that cannot allocate
 * device memory (a host whose GPU memory is pre-sized and owned by another
 * allocator, a plugin whose CUDA context forbids cudaMalloc, or a real-time
 * thread where cudaMalloc/cudaFree would synchronise the device). It needs no
 * s3b_ctx and calls no cudaMalloc, cudaFree or allocating library routine:
 * the im2col workspace and the kernels' error word live in one file-scope
 * __device__ array of S3B_NOALLOC_SCRATCH_BYTES (+256) bytes that every GPU
 * loading the library holds until exit. The caller passes inputs, outputs
 * and a cudaStream_t (NULL = legacy default stream); work is only enqueued.
 * B*H*W*9*C*2 must not exceed S3B_NOALLOC_SCRATCH_BYTES (S3B_ERR_ARG and a
 * message on stderr otherwise). The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress), so make it before any
 * stream capture. All calls share the array: calls that overlap on the GPU
 * race and must be ordered by the caller.
 * No counterpart in the reference (sam3.cpp always allocates through ggml). */
int s3b_conv3x3_noalloc(const void* x, int B, int H, int W, int C, const void* w, const float* bias, float* out,
                        int Cout, void* cuda_stream);

/* Device-side status of s3b_conv3x3_noalloc on the current device. The conv
 * call only enqueues work, so a failure inside its kernels (a bounded wait
 * that timed out, leaving `out` incomplete) cannot reach its return code;
 * it is recorded in the error word of the static scratch instead. After the
 * caller has waited for the stream of the last call (cudaStreamSynchronize),
 * this reads the word: *code = 0 and S3B_OK when every wait finished, else
 * *code = the kernel's code and S3B_ERR_DEVICE, and the word is cleared.
 * S3B_ERR_CUDA if the word cannot be read. Allocates nothing (a 4-byte
 * cudaMemcpyFromSymbol). No counterpart in the reference. */
int s3b_conv3x3_noalloc_status(int* code);

/* As s3b_op_gemm with B given as N rows of K values in q4_0 or q8_0 blocks
 * (device memory, ggml row layout; K a multiple of 32, N of 8): the rows are
 * split into a block-value plane and an f16 scale plane (context workspace)
 * and the GEMM dequantises each weight tile in shared memory, so weights are
 * read from HBM only in block form. Results equal s3b_op_gemm on the
 * dequantised (f16-rounded) weights. Replaces ggml_mul_mat on a quantised
 * weight (sam3.cpp:3738, 3792-3795, 4345, 4447-4450, 9250-9324). */
int s3b_op_gemm_q(s3b_ctx* ctx, const void* A, int64_t lda, const void* blocks, int type, int M, int N, int K,
                  const float* bias, int act, void* out, int out_f32, int64_t ldo, const float* resid, int64_t ldr);

/* Dequantises nrows rows of ne0 values of q4_0 / q4_1 / q8_0 blocks to f32,
 * bit-exactly as ggml's type-traits to_float (sam3.cpp:1076-1077). */
int s3b_op_dequantize(s3b_ctx* ctx, const void* src, int type, int64_t ne0, int64_t nrows, float* dst);

/* ---------------------------------------------------------------- host format helpers */

/* Bytes of one row of ne0 values of `type` (ggml_row_size, sam3.cpp:3133-3135). */
int64_t s3b_row_size(int type, int64_t ne0);
/* Quantises f32 rows to q4_0 / q4_1 / q8_0 with ggml's reference rounding
 * (ggml_quantize_chunk as called by examples/quantize.cpp:244-245). */
int s3b_quantize_rows(int type, const float* src, int64_t ne0, int64_t nrows, void* dst);
/* Host dequantisation (same values as s3b_op_dequantize). */
int s3b_dequantize_rows(int type, const void* src, int64_t ne0, int64_t nrows, float* dst);

#ifdef __cplusplus
}
#endif

#endif /* SAM3_B200_H */
