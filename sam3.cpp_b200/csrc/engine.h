// Internal host-side (C++14) structures of the B200 encoder engine.
//
// The engine replaces the ggml graph builders of sam3.cpp for the per-frame
// backbone forward (SAM 3 ViT + SimpleFPN neck, SAM 2 Hiera + FPN neck) and
// for memory attention, keeping the reference's .ggml files, dtypes and
// ownership rules: the model owns device weights (sam3.cpp:884-887), the
// context owns per-frame outputs (sam3.cpp:911-918) and frees them on destroy.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "kernels.h"

namespace s3b {

// ---------------------------------------------------------------- errors
enum Status : int {
  kOk = 0,
  kErrArg = -1,
  kErrIO = -2,
  kErrFormat = -3,
  kErrCuda = -4,
  kErrState = -5,
  kErrUnsupported = -6,
  kErrDevice = -7,   // a kernel reported a device-side error (bounded wait expired)
  kErrOOM = -8,
};

// ---------------------------------------------------------------- .ggml file
// One tensor record of a .ggml file (sam3.cpp:3093-3143): ne in ggml order
// (ne[0] contiguous), dtype in {0 F32, 1 F16, 2 Q4_0, 3 Q4_1, 8 Q8_0}.
struct FileTensor {
  std::string name;
  int dtype = 0;
  int n_dims = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  std::vector<uint8_t> data;  // raw bytes as stored
  int64_t nelements() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
};

// Hyper-parameters read from the file header (subset of sam3_hparams,
// sam3.cpp:70-242, needed by the encoder and memory attention).
struct HParams {
  int is_sam2 = 0;
  int ftype = 1;
  // SAM 3 (sam3.cpp:1477-1520)
  int img_size = 1008, patch_size = 14, vit_embed_dim = 1024, vit_depth = 32, vit_num_heads = 16;
  int vit_mlp_dim = 4736, vit_window_size = 24, n_global_attn = 4;
  int global_attn_idx[4] = {7, 15, 23, 31};
  int neck_dim = 256, mem_out_dim = 64, mem_attn_layers = 4, num_maskmem = 7, max_obj_ptrs = 16;
  int visual_only = 0;
  // SAM 2 (sam3.cpp:1564-1626)
  int backbone_type = 1;
  int hiera_embed_dim = 144, hiera_num_heads = 2, hiera_num_stages = 4;
  int hiera_stages[4] = {2, 6, 36, 4};
  int hiera_global_n = 3;
  int hiera_global_idx[8] = {23, 33, 43, 0, 0, 0, 0, 0};
  int hiera_q_pool = 3;
  int hiera_window_spec[4] = {8, 4, 16, 8};
  int bkg_h = 7, bkg_w = 7;
  int scalp = 1;
  int fpn_top_down_n = 2;
  int fpn_top_down_levels[4] = {2, 3, 0, 0};
  // SAM 2 tracking fields (sam3.cpp:137-153): sigmoid scale / bias of the memory mask (x100) and the
  // 15 flags after them in file order
  int sigmoid_scale_x100 = 2000, sigmoid_bias_x100 = -1000;
  int trk_flags[15] = {1, 1, 1, 1, 1, 1, 0, 1, 0, 1, 1, 1, 1, 1, 1};

  bool is_global(int layer) const {
    for (int i = 0; i < n_global_attn && i < 4; ++i)
      if (global_attn_idx[i] == layer) return true;
    return false;
  }
  bool is_hiera_global(int b) const {
    for (int i = 0; i < hiera_global_n && i < 8; ++i)
      if (hiera_global_idx[i] == b) return true;
    return false;
  }
  int n_img_embd() const { return img_size / patch_size; }
};

int read_ggml_file(const std::string& path, HParams& hp, std::vector<FileTensor>& tensors, std::string& err);
// The hparam block of a .ggml header given as n i32 values in file order.
int parse_hparams_array(int is_sam2, const int32_t* v, int n, HParams& hp, std::string& err);

// f32 values of a file tensor (f32 / f16 / q4_0 / q4_1 / q8_0).
void tensor_to_f32(const FileTensor& t, std::vector<float>& out);

// ---------------------------------------------------------------- device memory
// Counts every allocation and release of a DevBuf in the process: a CUDA graph captured while the
// count had one value holds only pointers that are still valid while it has that value.
inline std::atomic<long long>& devbuf_generation() {
  static std::atomic<long long> g{0};
  return g;
}

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() { release(); }
  void release() {
    if (p) {
      cudaFree(p);
      ++devbuf_generation();
    }
    p = nullptr;
    bytes = 0;
  }
  // Grows the buffer to at least n bytes (contents are not preserved).
  int reserve(size_t n) {
    if (n <= bytes) return 0;
    release();
    if (cudaMalloc(&p, n) != cudaSuccess) {
      p = nullptr;
      return kErrOOM;
    }
    ++devbuf_generation();
    bytes = n;
    return 0;
  }
  template <typename T>
  T* as() const { return reinterpret_cast<T*>(p); }
};

// A linear weight prepared for the tensor-core GEMM: B operand [N][Kpad] f16
// (K-major), plus the bias and, for quantised files, the raw blocks.
// With the context option weights_quantised, a q4_0 / q8_0 weight keeps its block form on the
// device instead (qtype != 0, w null): value plane qv and f16 scale plane qs in the QWeight
// layout, dequantised before (1) or inside (2) the GEMM.
struct Linear {
  int N = 0, K = 0, Kpad = 0;
  int file_dtype = 0;
  std::shared_ptr<DevBuf> w;     // f16 [N][Kpad]
  std::shared_ptr<DevBuf> b;     // f32 [N] (may be null)
  std::shared_ptr<DevBuf> raw;   // raw quantised rows as in the file (q4_0/q4_1/q8_0), else null
  int qtype = 0;                 // QT_Q4_0 / QT_Q8_0 when the weight is kept in block form
  std::shared_ptr<DevBuf> qv;    // q4_0 nibble plane [N][K/2] or q8_0 int8 plane [N][K]
  std::shared_ptr<DevBuf> qs;    // f16 block scales [K/32][N]
  // set on a per-call copy by stage_linears: the f16 [N][K] staging copy the GEMM reads instead
  const __half* staged = nullptr;
};

struct Vec {
  std::shared_ptr<DevBuf> d;  // f32
  int n = 0;
  const float* ptr() const { return d ? d->as<float>() : nullptr; }
};

struct VitBlock {
  Vec n1w, n1b, n2w, n2b;
  Linear qkv, proj, fc1, fc2;
  std::shared_ptr<DevBuf> rope;  // f32 [32][N][2] (position-major)
  int rope_n = 0;
  bool global = false;
};

struct NeckScale {
  // dc1: first deconvolution of scale 0 as [4*Cout][Cin]; dcf: the last deconvolution of scales 0 / 1
  // with the following 1x1 conv folded in, [4*D][Cin]; c1: 1x1 conv of scales 2 / 3 [D][Cin];
  // c3: 3x3 conv [D][9*D]
  Linear dc1, dcf, c1, c3;
};

struct HieraBlock {
  Vec n1w, n1b, n2w, n2b;
  Linear qkv, proj, fc1, fc2, dim_proj;
  int dim_in = 0, dim_out = 0, heads = 0, window = 0, stage = 0;
  bool q_stride = false, has_dim_proj = false;
};

struct MemAttnLayer {
  Vec n1w, n1b, n2w, n2b, n3w, n3b;
  Linear sa_qkv, sa_out, ca_q, ca_k, ca_v, ca_out, fc1, fc2;
};

// SAM mask decoder (sam3.cpp:563-599, registered at 1848-1966). Token-side weights are read by
// tok_linear, image-side weights by the tcgen05 GEMM; all f16 [N][Kpad] (dequantised at load).
struct SamTwoWay {
  Linear sa_q, sa_k, sa_v, sa_out;  // token self-attention (256 -> 256, 8 heads)
  Linear t2i_q, t2i_out;            // token side of tokens -> image (256 -> 128, 128 -> 256)
  Linear kq;                        // image side, input keys + key_pe: [t2i k ; i2t q] (256 rows)
  Linear t2i_v;                     // image side, input keys: t2i v (128 rows)
  Linear i2t_k, i2t_v;              // token side of image -> tokens (256 -> 128)
  Linear i2t_out;                   // image side, 128 -> 256 (residual into the keys)
  Linear mlp1, mlp2;                // token MLP 256 -> 2048 -> 256 (ReLU)
  Vec n1w, n1b, n2w, n2b, n3w, n3b, n4w, n4b;
};

struct SamDecoder {
  bool loaded = false;
  int D = 256, n_mask = 4, has_obj = 1, heads = 8;
  std::vector<SamTwoWay> blocks;
  Linear fin_q, fin_k, fin_v, fin_out;
  Vec fin_nw, fin_nb;
  Linear up1;      // deconv 2x2 D -> D/4, rows [(ky*2 + kx)*64 + co][D]
  Vec up1_nw, up1_nb;
  Linear up2;      // deconv 2x2 D/4 -> D/8, rows [(ky*2 + kx)*32 + co][64]
  Linear conv_s0;  // 1x1 D -> D/8 on neck_trk_0
  Linear conv_s1;  // 1x1 D -> D/4 on neck_trk_1
  std::vector<Linear> hyper;  // n_mask x 3 layers
  Linear iou[3], obj[3];
  // prompt encoder values kept on the host (sam3_populate_pe_cache, sam3.cpp:10288-10345)
  std::vector<float> pe_gauss, point_emb[4], not_a_point, no_mask, no_mem;
  // device: the special output tokens [obj?, iou, masks] [n_special][D], no_mask, no_mem, not_a_point
  std::shared_ptr<DevBuf> tokens;
  Vec d_no_mask, d_no_mem, d_not_a_point;
  int n_special() const { return (has_obj ? 1 : 0) + 1 + n_mask; }
};

// Memory encoder + object-pointer MLP (sam3.cpp:1968-2056 / 3060-3085).
struct MemEncoder {
  bool loaded = false;
  int D = 256, MD = 64;
  // mask downsampler: stages 0-2 direct convs (f32 [9][cin][cout] weights), stage 3 a GEMM over the
  // stride-2 column matrix [256][9*64] in (ky, kx, ci) order; LayerNorm2d of every stage; 1x1 conv ds12
  Vec ds_w[3], ds_b[3];
  Linear ds3;
  Vec ds_nw[4], ds_nb[4];
  Linear ds12, pix;
  struct Fuser {
    Vec dw, dw_b, nw, nb;  // dw f32 [49][256]
    Linear fc1, fc2;       // fc2 rows and bias scaled by the layer scale gamma at load
  } fuser[2];
  Linear out;
  Vec no_obj_spatial;  // [MD] (may be empty)
  Linear ptr[3];
  Vec no_obj_ptr;      // [D]
  float sig_scale = 20.0f, sig_bias = -10.0f;
};

struct Model {
  HParams hp;
  bool loaded = false;
  // SAM 3 ViT
  Linear patch;                      // [1024][Kpad=592]
  std::shared_ptr<DevBuf> pos_tiled; // f32 [72*72 + 128][1024] (last 128 rows repeat the first)
  Vec ln_pre_w, ln_pre_b;
  std::vector<VitBlock> vit;
  NeckScale neck_trk[4], neck_det[4];
  bool has_neck_trk = false, has_neck_det = false;
  // SAM 2 Hiera
  Linear hpatch;                     // [E0][Kpad=152]
  std::vector<float> pos_bkg, pos_win;  // host copies (CHW) for the PE
  std::shared_ptr<DevBuf> hiera_pe;     // f32 [S][S][E0], S = img_size / 4 (computed at load)
  int hiera_pe_size = 0;
  std::vector<HieraBlock> hiera;
  int stage_ends[4] = {0, 0, 0, 0};
  Linear fpn[4];
  // memory attention
  std::vector<MemAttnLayer> mem;
  Vec mem_norm_w, mem_norm_b;
  bool has_mem_attn = false;
  std::vector<float> maskmem_tpos;   // [num_maskmem][64]
  std::vector<float> obj_ptr_tpos_w, obj_ptr_tpos_b;  // [64][256], [64]
  SamDecoder dec;
  MemEncoder menc;
  size_t device_bytes = 0;
  // largest N*K of a weight kept in block form; the f16 staging arena of weights_quantised = 1 holds
  // the block-form weights of one ViT / Hiera block or memory-attention layer (stage_arena_elems)
  size_t qstage_elems = 0;
};

// Per-frame outputs of one encode call (device, channel-last f32 maps).
struct Outputs {
  int n_frames = 0;
  int img_size = 0;
  std::shared_ptr<DevBuf> backbone;  // ViT output [F][72][72][1024], or the Hiera state (stage runner)
  int backbone_c = 0, backbone_s = 0;  // Hiera stage-runner state: channels, spatial size
  std::shared_ptr<DevBuf> fpn[4];    // neck_trk / fpn levels [F][S][S][256]
  int fpn_size[4] = {0, 0, 0, 0};
  int n_fpn = 0;
  std::shared_ptr<DevBuf> det[4];    // neck_det (SAM 3, non visual-only)
  int n_det = 0;
  std::map<int, std::shared_ptr<DevBuf>> pe_cache;  // sinusoidal PE per size, [S][S][256]
};

}  // namespace s3b

// Opaque context of the C-ABI (one per device).
struct s3b_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int* d_err = nullptr;  // device error word of the bounded waits
  std::string last_error;
  s3b::Model model;
  s3b::Outputs out;
  // workspace (grown on demand, reused across calls)
  std::map<std::string, std::shared_ptr<s3b::DevBuf>> ws;
  // host destinations bound with s3b_output_host_bind: after each encoder pass, that pass's frames
  // of these outputs are copied to host memory on copy_stream while the next pass computes
  struct HostBind {
    float* host = nullptr;
    int64_t n = 0;  // floats the host buffer holds
  };
  std::map<std::string, HostBind> host_bind;
  cudaStream_t copy_stream = nullptr;
  std::vector<cudaEvent_t> pass_done, copy_done;  // per pass index of the encode call
  std::vector<char> copy_pending;                  // copy_done[p] recorded and not yet waited for
  int copy_fb = 0;                                 // frames per pass of the pending copies
  // projected 1-D sine PE of an object pointer at frame distance `rel` (s3b_mem_attn_bank), per rel;
  // cleared when a model is loaded
  std::map<int, std::vector<float>> ptr_pe_cache;
  // s3b_device_alloc allocations and s3b_ipc_open mappings, released with the context
  std::map<void*, std::shared_ptr<s3b::DevBuf>> user_allocs;
  std::set<void*> ipc_mapped;
  int max_frames_per_pass = 8;
  int stop_after_blocks = -1;  // test hook: run only the first n backbone blocks (-1: all)
  int attention_impl = 0;      // 0 (or 4): tcgen05 where eligible, d = 64 on the persistent two-tile kernel;
                               // 1: always mma.sync; 2: d = 64 on the wide tcgen05 kernel; 3: d = 64 on the
                               // one-tile-per-CTA kernel
  int weights_quantised = 0;   // q4_0 / q8_0 linear weights stay in block form in device memory: 1 each is
                               // dequantised into an f16 staging buffer (L2-resident) right before its GEMM,
                               // 2 the GEMM dequantises each weight tile in shared memory; 0 f16 at load
  int conv_implicit = 1;       // pixel-block GEMMs: implicit 3x3 convs, TMA-stored deconvs (0: im2col / scatter)
  int attention_exp_poly = 0;  // of every 8 softmax exponentials in the tcgen05 kernel, how many use the FMA pipe
  int attention_fa_exp_poly = 1;  // the same for the persistent two-tile d = 64 kernel
  int attention_wide_k128 = -1;   // d = 72 / 96 on the 128-key-tile kernel: 1 always, 0 never, -1 rows of >= 1024 keys
  // memory attention: its per-layer body replayed from a CUDA graph (mem_attn.cpp)
  int graphs = 1;               // option "graphs"
  long long graph_epoch = 0;    // bumped by every option change and model load: cached graphs are stale
  cudaGraphExec_t ma_exec = nullptr;
  std::vector<uintptr_t> ma_key;  // shapes, buffers, epoch and kernel choices the graph was captured with
  long long ma_launches = 0;      // kernel launches inside the graph
  int ma_seen = 0;                // eager calls with ma_key so far (the graph is captured on the second)
  // encoder calls and tracking steps replayed from CUDA graphs (capi.cpp run_graphed): one per key (entry point, input
  // pointer, frame count and size, flags, option epoch, GEMM configuration, DevBuf generation), most
  // recently used last
  struct EncGraph {
    std::vector<uintptr_t> key;
    cudaGraphExec_t exec = nullptr;
    long long launches = 0;  // kernel launches inside the graph
    int seen = 0;            // eager calls with this key so far (the graph is captured on the second)
  };
  std::vector<EncGraph> enc_graphs;
  // launch accounting + optional per-kernel CUDA-event timing (s3b_profile_*)
  long long n_launches = 0;
  bool prof = false;
  struct Prof {
    int kind;  // 0 GEMM, 1 attention, 2 LayerNorm, 3 block-form weight staging
    double flops, bytes;
    cudaEvent_t a, b;
  };
  std::vector<Prof> prof_entries;
  std::vector<cudaEvent_t> event_pool;
  size_t event_next = 0;
  cudaEvent_t next_event();

  s3b::DevBuf* buf(const std::string& name, size_t bytes, int* rc);
};

namespace s3b {
// C-ABI status of a kernel launcher's negative code: -1..-9 argument checks and -11 (a pointer or
// row stride that is not 16-byte aligned) are the caller's arguments; -10 (no tensor-map encoder
// from the driver) and below -11 are CUDA failures.
inline int launcher_status_code(int rc) { return (rc == -10 || rc < -11) ? kErrCuda : kErrArg; }
int set_error(s3b_ctx* ctx, int code, const char* fmt, ...);
// Host -> device copy ordered on the context stream and complete on return. A plain cudaMemcpy from
// pageable memory may return before its DMA has landed, and kernels on the context's non-blocking
// stream do not wait for it, so every upload a kernel reads goes through this.
int upload_sync(s3b_ctx* ctx, void* dst, const void* src, size_t bytes);
int check_device(s3b_ctx* ctx, const char* where);

// weight preparation (model.cpp)
int load_model(s3b_ctx* ctx, const std::string& path);
// load_model through the device-weight cache (weight_cache.cpp): 1 = loaded from a valid cache file,
// 0 = loaded from the model file (and the cache written), < 0 = error.
int load_model_cached(s3b_ctx* ctx, const std::string& model_path, const std::string& cache_path);
// Prepares the device weights from parsed tensors (the file reader's or the caller's).
int load_model_tensors(s3b_ctx* ctx, const HParams& hp, const std::vector<FileTensor>& tensors);
int upload_linear(s3b_ctx* ctx, const FileTensor& t, const FileTensor* bias, Linear& L, int kpad_to = 8,
                  int k_dims = 1);

// launch helpers shared by the encoders (ops.cpp): count launches and, when
// profiling is on, bracket the launch with CUDA events on the context stream.
int run_gemm(s3b_ctx* ctx, const __half* A, long long lda, const Linear& L, long long M, const EpiParams& ep);
int run_attn(s3b_ctx* ctx, const AttnParams& p, int D, int batch_heads);
int run_conv3x3(s3b_ctx* ctx, const Linear& L, const __half* x, int F, int H, int W, const EpiParams& ep,
                __half* col);
int run_deconv2x2(s3b_ctx* ctx, const Linear& L, const __half* x, int F, int H, int W, EpiParams ep);
// layernorm() on the context stream, timed when profiling; returns layernorm's status (the caller counts the launch)
int run_ln(s3b_ctx* ctx, const float* x, long long ldx, void* y, int y_f32, long long ldy, long long rows, int C,
           const float* g, const float* b, float eps, const RowMap& map);
void count_launch(s3b_ctx* ctx, int n = 1);
// weights_quantised = 1: dequantises the block-form weights among in[0..n) in one launch into
// consecutive regions of the staging arena and sets out[i]->staged (out[i] starts as a copy of
// *in[i]); f16 weights, and every weight under weights_quantised = 2, pass through unchanged.
// The staged copies stay valid until the next stage_linears call on the context.
int stage_linears(s3b_ctx* ctx, const Linear* const* in, Linear* const* out, int n);
// f16 elements of the staging arena the loaded model needs (0 without block-form weights).
size_t stage_arena_elems(const Model& M);
EpiParams epi_store(const Linear& L, void* out, int out_f32, long long ldo, int act = ACT_NONE);
// RoPE table [npos][half_d][2] (cos, sin) -> the position-major [half_d][npos][2] the GEMM epilogue reads
void rope_position_major(const std::vector<float>& in, int npos, int half_d, std::vector<float>& out);

// Host-bound outputs (s3b_output_host_bind, capi.cpp). pass_begin: before pass `pass` (frames_per_pass
// fb) writes its outputs, the context stream waits for the previous call's copy of the same frames.
// pass_end: enqueues the copies of frames [f0, f0 + F) of every bound output on the copy stream after
// the pass's work. Both are no-ops without bindings.
int outputs_pass_begin(s3b_ctx* ctx, int pass, int fb);
int outputs_pass_end(s3b_ctx* ctx, int pass, int f0, int F);

// memory attention (mem_attn.cpp): from the caller's prompt arrays, or with the prompt built on the
// device from the memory bank
int mem_attn_run(s3b_ctx* ctx, const float* curr, const float* src_pos, int feat, const float* prompt,
                 const float* prompt_pos, int m_total, int n_ptr, float* out);
int mem_attn_run_bank(s3b_ctx* ctx, const float* curr, const float* src_pos, int feat, const PromptArgs& pa,
                      float* out);

// SAM mask decoder (mask_decoder.cpp). Inputs are device pointers: image_feats [H*H][256] (memory-attention
// output or neck_trk_2), feat_s0 [(4H)^2][256], feat_s1 [(2H)^2][256] (neck_trk_0 / 1), sparse [n_sparse][256]
// prompt tokens (n_sparse = 0: the single not_a_point token of the tracker's propagation). Outputs (device):
// masks [n_mask][(4H)^2], iou [n_mask], obj [1], mask_tokens [n_mask][256] (each may be null).
int sam_dec_run(s3b_ctx* ctx, int H, const float* image_feats, const float* feat_s0, const float* feat_s1,
                const float* sparse, int n_sparse, int add_no_mem, float* masks, float* iou, float* obj,
                float* mask_tokens);
// dense image PE of the H x H grid (sam3_populate_pe_cache's dense_pe_cache), device f32 [H*H][256], cached
const float* sam_dec_dense_pe(s3b_ctx* ctx, int H, int* rc);
// sparse prompt tokens of the image predictor (sam3_segment_pvs, sam3.cpp:10877-10900) on the host
int sam_prompt_tokens(const SamDecoder& dec, const float* box, const float* pos, int n_pos, const float* neg,
                      int n_neg, float orig_w, float orig_h, int input_size, float* out, int capacity);

// memory encoder (memory_encoder.cpp), device pointers: pix_feat [H*H][256] (neck_trk_2), mask_logits
// [mask_h][mask_w], obj_score (device float or null: object present) -> out [H*H][64]; obj_ptr: sam_token
// [256] -> out [256].
int mem_encode_run(s3b_ctx* ctx, int H, const float* pix_feat, const float* mask_logits, int mask_h, int mask_w,
                   const float* obj_score, float* out);
int obj_ptr_run(s3b_ctx* ctx, const float* sam_token, const float* obj_score, float* out);

// sinusoidal PE [S][S][d] on the device, computed once per size (sam3_sinusoidal_pe_2d)
const float* sine_pe_device(s3b_ctx* ctx, int S, int d, int* rc);
// One tracking step of one object (tracker.cpp): memory attention from the bank, the mask decoder on its
// output, the kept mask, the memory encoder and the object pointer, all on the context stream.
int track_step_run(s3b_ctx* ctx, int H, const float* trk0, const float* trk1, const float* trk2, const PromptArgs& pa,
                   float* mask_out, float* scores_out, float* mem_out, float* ptr_out);

// encoders
// The backbone input is the f32 CHW batch d_chw, or, when d_u8 is given, the uint8 HWC frames themselves,
// normalised inside the patch-column kernel (the preprocessing fused into the first launch).
int vit_encode(s3b_ctx* ctx, const float* d_chw, int n_frames, int flags, const uint8_t* d_u8 = nullptr);
int hiera_encode(s3b_ctx* ctx, const float* d_chw, int n_frames, int flags, const uint8_t* d_u8 = nullptr);
// SAM 3 normalisation (p/255 - 0.5)/0.5 (sam3.cpp:3505-3511); SAM 2 ImageNet mean/std (3519-3520).
constexpr float kMeanSam3[3] = {0.5f, 0.5f, 0.5f}, kStdSam3[3] = {0.5f, 0.5f, 0.5f};
constexpr float kMeanSam2[3] = {0.485f, 0.456f, 0.406f}, kStdSam2[3] = {0.229f, 0.224f, 0.225f};

}  // namespace s3b
