// Host-visible launchers and parameter blocks of the sm_100a kernels.
// Every launcher returns 0 on success or a negative error code and never
// allocates device memory; buffers are owned by the caller (engine.cpp).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace s3b {

// Maps a row of a GEMM / attention operand, in "work order", to a row of a
// spatial token map [frames][H][W] (or -1 for a padding row that is dropped).
//   kind 0: identity.
//   kind 1: work rows are window-partitioned: frame-major, then windows in
//           (wy, wx) order, then tokens (ly, lx) inside a ws x ws window; the
//           spatial grid is padded up to (nwh*ws, nww*ws) and padded
//           positions map to -1 (sam3.cpp:4190-4277 window partition).
struct RowMap {
  int kind = 0;
  int ws = 0;
  int nww = 0, nwh = 0;
  int W = 0, H = 0;  // spatial grid of the token map (unpadded)
};

__host__ __device__ inline long long map_row(const RowMap& m, long long r) {
  if (m.kind == 0) return r;
  const long long per_win = (long long)m.ws * m.ws;
  const long long per_frame = per_win * m.nww * m.nwh;
  const long long f = r / per_frame;
  const long long rr = r - f * per_frame;
  const int win = (int)(rr / per_win);
  const int l = (int)(rr - (long long)win * per_win);
  const int wy = win / m.nww, wx = win - wy * m.nww;
  const int y = wy * m.ws + l / m.ws, x = wx * m.ws + l % m.ws;
  if (y >= m.H || x >= m.W) return -1;
  return (f * m.H + y) * m.W + x;
}

enum EpiMode : int { EPI_STORE = 0, EPI_DECONV2 = 2 };
enum Act : int { ACT_NONE = 0, ACT_GELU_ERF = 1, ACT_GELU_TANH = 2, ACT_RELU = 3 };

// Epilogue of the tensor-core GEMM C[M,N] = A[M,K] * B[N,K]^T (f32 acc):
//   v = act(C + bias[n]) (+ resid)  then a mode-specific store.
struct EpiParams {
  int mode = EPI_STORE;
  int act = ACT_NONE;
  const float* bias = nullptr;  // [N] (EPI_DECONV2: [cout])
  void* out = nullptr;          // EPI_STORE / EPI_DECONV2 destination
  int out_f32 = 0;              // 1: f32 output, 0: f16 output
  long long ldo = 0;            // row stride of `out` (elements)
  RowMap map;                   // EPI_STORE: GEMM row -> output row
  // residual (f32) added after the activation, indexed by the output row:
  //   resid_up == 0: row' = (resid_mod ? row % resid_mod : row)
  //   resid_up == 1: nearest 2x upsample of a (W/2, H/2) map (FPN top-down)
  const float* resid = nullptr;
  long long ldr = 0;
  long long resid_mod = 0;
  int resid_up = 0;
  // resid_mod tables only: the table holds resid_mod + 128 rows, the last 128 repeating the first
  // (a 128-row output tile then reads its rows contiguously even across the repeat)
  int resid_wrap_pad = 0;
  // EPI_STORE only: out = v * out_scale; RoPE on column pairs (2i, 2i+1) of
  // columns < rope_cols and GEMM rows < rope_rows: head dim rope_D, position
  // (row % rope_mod), position-major table [rope_D/2][rope_mod][2] (cos, sin).
  float out_scale = 1.0f;
  const float* rope = nullptr;
  int rope_D = 0, rope_cols = 0;
  long long rope_rows = 0, rope_mod = 1;
  // EPI_DECONV2: row = input pixel (f, y, x) of a (map.W x map.H) grid,
  // column = (ky*2 + kx)*cout + co, stored at pixel (2y+ky, 2x+kx).
  int cout = 0;
  // implicit 3x3 convolution (gemm_conv3x3 sets these): channel-last f16 input [F][H][W][C]
  int conv_F = 0, conv_H = 0, conv_W = 0, conv_C = 0;
};

// Tensor-core GEMM (tcgen05 + TMA): A f16 [M][lda] K-major, B f16 [N][ldb]
// K-major. lda, ldb multiples of 8; pointers 16-byte aligned.
int gemm_f16(const __half* A, long long lda, const __half* B, long long ldb, int M, int N, int K,
             const EpiParams& ep, int* err, cudaStream_t st);
// 3x3 / stride 1 / pad 1 convolution as an implicit GEMM (no column matrix): x channel-last f16
// [F][H][W][C] (C a multiple of 64), weights Bw [N][9*C] in (ky, kx, c) order, output
// [F][H][W][N] through ep (EPI_STORE with ldo == N, bias / activation / f16 or f32; no residual,
// RoPE or row map). Returns -2 when those conditions do not hold (callers fall back to im2col).
int gemm_conv3x3(const __half* x, int F, int H, int W, int C, const __half* Bw, long long ldb, int N,
                 const EpiParams& ep, int* err, cudaStream_t st);
// 2x2 / stride 2 deconvolution (ConvTranspose2d) as a GEMM over pixel blocks whose outputs leave
// through 5-D TMA stores: x channel-last f16 [F][H][W][Cin] (Cin a multiple of 8), weights Bw
// [4*cout][Cin] with rows (ky*2 + kx)*cout + co, output [F][2H][2W][cout] (cout a multiple of 32)
// through ep (bias per co, activation, f16 or f32). Returns -2 when the conditions do not hold.
int gemm_deconv2x2(const __half* x, int F, int H, int W, int Cin, const __half* Bw, long long ldb, int cout,
                   const EpiParams& ep, int* err, cudaStream_t st);
// Process-wide: which wide TMA-epilogue GEMMs use 256-row tiles on SM pairs:
// 0 none, 1 (default) those with K >= 2048 or f16 outputs on 16 epilogue warps, 2 all.
void set_gemm_pairs(int mode);
// Process-wide: which short-K (K < 2048) GEMMs use 16 epilogue warps: 0 none,
// 1 (default) those with f16 outputs, 2 all.
void set_gemm_wide_epilogue(int mode);
// The current process-wide GEMM variant choices (pairs, epilogue warps) as one number.
int gemm_config_id();

// Flash attention (online softmax, f16 in / f32 acc / f16 out).
struct AttnParams {
  const __half* q = nullptr;
  const __half* k = nullptr;
  const __half* v = nullptr;
  __half* o = nullptr;
  // element strides: q + b*q_b + h*q_h + n*q_n (same for k, v)
  long long q_b = 0, q_h = 0, q_n = 0;
  long long k_b = 0, k_h = 0, k_n = 0;
  long long v_b = 0, v_h = 0, v_n = 0;
  int heads = 1;
  int nq = 0, nk = 0;
  // out row = map_row(omap, b*nq + n): o + row*o_n + h*D + d (rows mapped to -1 are dropped)
  long long o_n = 0;
  RowMap omap;
  float scale = 1.0f;  // softmax scale applied to q.k
};
int attention(const AttnParams& p, int D, int batch_heads, cudaStream_t st);

// Tensor-core (tcgen05) flash attention, head dim 64, q / k / v of head h of
// window w at base[(w*ntok + n)*ld + {q,k,v}_col + h*64] (one fused qkv
// buffer), nq == nk == ntok; output rows map_row(omap, w*ntok + n).
int attention_tc64(const __half* base, long long ld, int q_col, int k_col, int v_col, int heads, int ntok, int nwin,
                   __half* o, long long o_n, const RowMap& omap, float scale, int exp_poly, int p_mode,
                   int* err, cudaStream_t st);
// The same attention (d = 64, fused qkv buffer) on one persistent CTA per SM, two 128-query tiles
// per work unit whose softmax warpgroups (one thread per query row) interleave with the tensor-core
// products of the other tile.
int attention_fa64(const __half* base, long long ld, int q_col, int k_col, int v_col, int heads, int ntok, int nwin,
                   __half* o, long long o_n, const RowMap& omap, float scale, int exp_poly, int* err,
                   cudaStream_t st);
// Tensor-core (tcgen05) flash attention for head dims d = 72, 96, 256
// (Hiera-L, Hiera-T, memory attention): q / k / v with their own row strides
// and row counts (nq, nk), heads as column offsets (q_h etc. < row length) or
// as row blocks ([B][H][n][d]). Returns -2 for layouts or d it does not take.
// When the query tiles alone would leave SMs idle, the keys are split over
// several CTAs whose partial results (in `ws`: attention_wide_ws_bytes(d,
// n_split, ...) bytes for n_split up to attention_wide_max_split(d, query
// tiles x batch_heads)) a second kernel merges; ws = NULL disables splitting.
// d = 256 runs 128-key tiles with P in TMEM; d = 72 / 96 too when bk128 is set (else 64-key tiles, two
// CTAs per SM).
int attention_wide(const AttnParams& p, int d, int batch_heads, float* ws, size_t ws_bytes, int bk128, int* err,
                   cudaStream_t st);
size_t attention_wide_ws_bytes(int d, int n_split, int batch_heads, int nq);
int attention_wide_max_split(int d, long long units);
void* tensor_map_encoder();

// LayerNorm over the last dim (C) of f32 rows, eps as given; out f16 or f32.
// Output row r reads input row map_row(map, r) (or writes zeros for -1).
int layernorm(const float* x, long long ldx, void* y, int y_f32, long long ldy, long long rows, int C,
              const float* gamma, const float* beta, float eps, const RowMap& map, cudaStream_t st);

// Patch columns of a stride-s image convolution over an f32 CHW batch [B][Cin][H][W]: out f16
// [B*OH*OW][Kpad], column = (ci*k + ky)*k + kx, zeros beyond K; staged through shared memory, one block
// per (frame, output row). patch_cols_u8 reads uint8 HWC frames and applies the preprocessing's
// normalisation (p / 255 - mean) / std in f32 first (sam3_preprocess_image / sam2_preprocess_image,
// sam3.cpp:3486-3544), so it gives the bits of normalising into f32 CHW and then taking the columns.
int patch_cols_f32(const float* img, int B, int Cin, int H, int W, int k, int stride, int pad, int OH, int OW,
                   __half* out, int Kpad, cudaStream_t st);
int patch_cols_u8(const uint8_t* hwc, int B, int H, int W, const float mean[3], const float stdv[3], int k, int stride,
                  int pad, int OH, int OW, __half* out, int Kpad, cudaStream_t st);

// im2col for a 3x3 / pad 1 / stride 1 convolution over channel-last f16
// maps [B][H][W][C]: out [B*H*W][9*C], column = (ky*3 + kx)*C + ci.
int im2col_3x3_cl(const __half* x, int B, int H, int W, int C, __half* out, cudaStream_t st);

// 2x2 / stride 2 max pool over channel-last maps [B][H][W][C].
int maxpool2_cl_f16(const __half* x, int B, int H, int W, int C, __half* y, cudaStream_t st);
int maxpool2_cl_f32(const float* x, int B, int H, int W, int C, float* y, cudaStream_t st);

// Q pooling inside windows (sam3.cpp:4363-4371): rows w*ws*ws + (y*ws + x) of
// q (row stride ld elements, C channels) -> out [nwin][(ws/2)^2][C] contiguous.
int qpool_windows(const __half* q, long long ld, long long nwin, int ws, int C, __half* out, cudaStream_t st);

// Bilinear resize of uint8 HWC frames [B][SH][SW][3] to DH x DW (sam3.cpp:3441-3481: half-pixel
// centres, f64 weights, rounded to uint8). mean / stdv null: uint8 HWC out; else the rounded
// frame normalised to f32 CHW [B][3][DH][DW] ((p / 255 - mean) / std in f32).
int resize_bilinear_u8(const uint8_t* src, int B, int SH, int SW, int DH, int DW, const float* mean,
                       const float* stdv, void* out, cudaStream_t st);

int cast_f32_f16(const float* x, long long n, __half* y, cudaStream_t st);
int add_scaled_f32(const float* a, const float* b, float s, long long n, float* y, cudaStream_t st);
// y = f16(a + s*b) (b may be null: y = f16(a)).
int add_scaled_to_f16(const float* a, const float* b, float s, long long n, __half* y, cudaStream_t st);

// Memory-attention prompt (sam3_build_prompt_and_pos, sam3.cpp:9123-9209) built on the device from
// the memory bank: rows [0, n_slots*slot_tokens) are the spatial memory tokens of the slots in
// order (prompt = slot features, prompt_pos = slot PE + the slot's temporal PE row when it has
// one), then n_ptr kept object pointers, each split into `split` tokens of 64 values (prompt = the
// pointer's values t*64..t*64+63, prompt_pos = its projected 1-D sine PE). The temporal and
// pointer PE rows are host-computed and travel in the parameter block.
constexpr int kPromptMaxSlots = 16, kPromptMaxPtrs = 16, kPromptMD = 64;
struct PromptArgs {
  const float* feat[kPromptMaxSlots];  // [slot_tokens][64] f32 each
  const float* pe[kPromptMaxSlots];    // [slot_tokens][64] f32 each
  float tpos[kPromptMaxSlots][kPromptMD];
  int has_tpos[kPromptMaxSlots];
  int n_slots = 0, slot_tokens = 0;
  const float* ptrs = nullptr;  // [n_src][split*64] f32
  int ptr_src[kPromptMaxPtrs];  // source row of the k-th kept pointer
  float ptr_pe[kPromptMaxPtrs][kPromptMD];
  int n_ptr = 0, split = 4;
};
// out_f16 = 0: a = prompt, b = prompt_pos (f32 [M][64]); out_f16 = 1: a = f16(prompt + prompt_pos),
// b = f16(prompt) (the cross-attention key and value inputs, sam3.cpp:9278-9283).
int build_prompt(const PromptArgs& args, void* a, void* b, int out_f16, cudaStream_t st);

// ---------------------------------------------------------------- SAM mask decoder (sam_dec.cu)
// Token-side linear layers of the decoder: a few rows (the output + prompt tokens) times an f16
// weight [N][ldw] (K-major, K and ldw multiples of 8, rows 16-byte aligned):
//   y[r][n] = act((x[r] (+ x2[r])) . W[n] + b[n]) (+ resid[r][n]),  r < R <= kTokMaxRows.
// Up to kTokMaxJobs independent layers run in one launch. act: 0 none, 1 ReLU, 2 sigmoid.
constexpr int kTokMaxRows = 32, kTokMaxJobs = 8;
struct TokJob {
  const float* x = nullptr;
  const float* x2 = nullptr;  // optional second input added to x (the token PE), row stride ldx too
  long long ldx = 0;
  int R = 0;
  const __half* W = nullptr;
  long long ldw = 0;
  const float* b = nullptr;
  int N = 0, K = 0;
  float* y = nullptr;
  long long ldy = 0;
  const float* resid = nullptr;  // may equal y (in-place residual)
  long long ldr = 0;
  int act = 0;
};
int tok_linear(const TokJob* jobs, int n_jobs, cudaStream_t st);
// y[r] = LayerNorm(a[r] (+ b[r])) * g + beta over C (<= 1024, a multiple of 32) channels; y may equal a.
int tok_layernorm(const float* a, const float* b, long long ld, int rows, int C, const float* g, const float* beta,
                  float eps, float* y, cudaStream_t st);
// Multi-head attention among the tokens: q / k / v f32 rows [nt][ld*] with head h in columns h*hd ..,
// out [nt][ldo]; nt <= kTokMaxRows, heads * nt <= 256, hd <= 32.
int tok_attention(const float* q, long long ldq, const float* k, long long ldk, const float* v, long long ldv,
                  int nt, int heads, int hd, float scale, float* out, long long ldo, cudaStream_t st);
// Tokens -> image cross-attention with head dim 16: q f32 [nt][ldq], k / v f16 image rows [nkv][ldk / ldv]
// (head h in columns h*16 ..), out f32 [nt][ldo]. Keys are split over CTAs in chunks of kT2iChunk whose
// partial (max, sum, 16 outputs) per (token, head) go to ws (t2i_ws_floats floats) and are merged by a
// second kernel.
constexpr int kT2iChunk = 64;
long long t2i_ws_floats(int nt, int heads, long long nkv);
int t2i_attention(const float* q, long long ldq, const __half* k, long long ldk, const __half* v, long long ldv,
                  int nt, int heads, long long nkv, float scale, float* ws, float* out, long long ldo,
                  cudaStream_t st);
// Image -> tokens cross-attention with head dim 16: one thread per (image row, head); q f16 [n][ldq],
// k / v f32 token rows [nt][ldk / ldv], out f16 [n][ldo].
int i2t_attention(const __half* q, long long ldq, const float* k, long long ldk, const float* v, long long ldv,
                  int nt, int heads, long long n, float scale, __half* out, long long ldo, cudaStream_t st);
// Image keys of the decoder, one row of C = 256 channels per token:
//   mode 0: v = (x + add1) + add0 (add1 optional);  mode 1: v = LayerNorm(x) * g + beta (eps)
// keys = v (f32, may equal x), k16 = f16(v), kpe16 = f16(v + pe[row]).
int dec_keys(const float* x, long long rows, int mode, const float* add0, const float* add1, const float* g,
             const float* beta, float eps, const float* pe, float* keys, __half* k16, __half* kpe16, cudaStream_t st);
// First upscaling stage at the 2H x 2H grid (n = (2H)^2 pixels): v = up1[p] + (feat_s1[p] . Ws1 + bs1),
// out[p] = f16(GELU-erf(LayerNorm2d(v) * g + beta)), 64 channels; feat_s1 f32 [n][256], Ws1 f16 [64][256].
int dec_upscale1(const float* up1, const float* feat_s1, const __half* ws1, const float* bs1, const float* g,
                 const float* beta, float eps, long long n, __half* out, cudaStream_t st);
// Second upscaling stage and the mask products at the S x S grid (S = 4H): per pixel (y, x),
// u = GELU-erf((u1[y/2][x/2] . W2[(y%2)*2 + x%2] + b2) + (feat_s0[p] . Ws0 + bs0)) (32 channels), then
// masks[m][p] = hyper[m] . u for m < 4. u1 f16 [S/2][S/2][64], W2 f16 rows [(ky*2 + kx)*32 + co][64],
// feat_s0 f32 [S*S][256], Ws0 f16 [32][256], hyper f32 [4][32], masks f32 [4][S*S].
int dec_masks(const __half* u1, const __half* w2, const float* b2, const float* feat_s0, const __half* ws0,
              const float* bs0, const float* hyper, int S, float* masks, cudaStream_t st);

// The mask a tracking step keeps: masks [n_masks][plane], iou [n_masks], tokens [n_masks][256] (device).
// Index 0, or with multimask the best IoU among 1 .. n-1; out_mask = that plane, out_token = that token
// (use_mm_token) or token 0, out_scores = {iou, *obj, index}. Outputs may be null.
int pick_mask(const float* masks, long long plane, const float* iou, const float* tokens, int n_masks, int multimask,
              int use_mm_token, float* out_mask, float* out_token, float* out_scores, const float* obj,
              cudaStream_t st);

// ---------------------------------------------------------------- memory encoder (mem_enc.cu)
// sam3_bilinear_interpolate (sam3.cpp:9614-9639) of an f32 [sh][sw] map to [dh][dw] (sw, sh >= 2), bit for
// bit; sigmoid_mode 1 then maps v -> sigmoid(v) * scale + bias (sam3.cpp:11518-11519).
int bilinear_resize(const float* src, int sw, int sh, float* dst, int dw, int dh, int sigmoid_mode, float scale,
                    float bias, cudaStream_t st);
// One mask-downsampler stage with cin -> cout in {1 -> 4, 4 -> 16, 16 -> 64}: 3x3 / stride 2 / pad 1 conv
// of channel-last f32 x [Hi][Wi][cin] (inputs rounded to f16) with weights w [9][cin][cout] (f32) + bias,
// LayerNorm2d (eps) and GELU-tanh -> y [(Hi+1)/2][(Wi+1)/2][cout] f32.
int mask_ds_conv(const float* x, int Hi, int Wi, int cin, int cout, const float* w, const float* bias, const float* g,
                 const float* beta, float eps, float* y, cudaStream_t st);
// Column matrix [(Hi+1)/2 * (Wi+1)/2][9*C] f16 of a 3x3 / stride 2 / pad 1 conv over f32 [Hi][Wi][C].
int im2col_s2(const float* x, int Hi, int Wi, int C, __half* col, cudaStream_t st);
// y = f16(GELU-tanh(LayerNorm(x) * g + beta)) over rows of C in {64, 256} channels.
int ln_gelu_rows(const float* x, long long rows, int C, const float* g, const float* beta, float eps, __half* y,
                 cudaStream_t st);
// CXBlock depthwise 7x7 / pad 3 conv of f32 [H][W][256] (w f32 [49][256]) + b, LayerNorm2d -> f16 [H*W][256].
int dwconv7_ln(const float* x, int H, int W, const float* w, const float* b, const float* g, const float* beta,
               float eps, __half* y, cudaStream_t st);
// out[r][c] += emb[c] for all rows when *score <= 0 (device value).
int add_if_absent(float* out, long long rows, int C, const float* emb, const float* score, cudaStream_t st);
// out = mlp if score is null or *score > 0, else no_obj (n floats).
int select_obj_ptr(const float* mlp, const float* no_obj, const float* score, int n, float* out, cudaStream_t st);

// ggml block formats (32 values per block along the row).
enum QType : int { QT_F32 = 0, QT_F16 = 1, QT_Q4_0 = 2, QT_Q4_1 = 3, QT_Q8_0 = 8 };
long long qtype_row_bytes(int qtype, long long ne0);
// Dequantise `nrows` rows of `ne0` values: raw blocks -> f32 (bit-exact ggml
// semantics) or -> f16 (rounded from the exact f32 value).
int dequant_rows(const void* src, int qtype, long long ne0, long long nrows, void* dst, int dst_f32,
                 long long ld_dst, cudaStream_t st);

// A q4_0 / q8_0 weight [N][K] kept in block form for the GEMM (K a multiple of 32, N of 8):
// values = q4_0 nibble plane [N][K/2] (per 8 values one 32-bit word, value 2p in nibble p and value
// 2p + 1 in nibble p + 4) or q8_0 int8 plane [N][K]; scales = f16 block scales [K/32][N].
struct QWeight {
  int type = QT_F16;
  const void* values = nullptr;
  const __half* scales = nullptr;
};
// ggml rows of q4_0 / q8_0 blocks [N][row_bytes(K)] -> the QWeight planes (bytes: N*K/2 or N*K
// values, 2*N*K/32 scales).
int repack_q_rows(const void* src, int qtype, int N, int K, void* values, __half* scales, cudaStream_t st);
// C[M,N] = A[M,K] B[N,K]^T with B in block form, dequantised inside the GEMM (its shared-memory
// stages receive the block values and scales and dequantising warps write the f16 tile the
// tensor cores read); same epilogues and results as gemm_f16 on the dequantised weight.
int gemm_q(const __half* A, long long lda, const QWeight& w, int M, int N, int K, const EpiParams& ep, int* err,
           cudaStream_t st);
// Block-form planes of a q4_0 / q8_0 weight -> f16 rows out [N][ldo] (K a multiple of 32, ldo a
// multiple of 8, out 16-byte aligned), values round_f16(q * d) as the load-time dequantisation.
int dequant_planes_f16(const QWeight& w, int N, int K, __half* out, long long ldo, cudaStream_t st);
// Up to kMaxStageJobs such weights (out [N][K] each) in one launch.
constexpr int kMaxStageJobs = 8;
struct StageJob {
  QWeight w;
  int N = 0, K = 0;
  __half* out = nullptr;
};
int dequant_planes_multi(const StageJob* jobs, int n, cudaStream_t st);

// Self-test of the bounded device waits: one CTA waits on an mbarrier (limit_ns <= 2 s) whose only arrive
// is withheld (withhold = 1) or made (0); a wait that runs out records its code in *err and the kernel
// returns.
int wait_probe(int* err, long long limit_ns, int withhold, cudaStream_t st);

// Returns the number of SMs of the current device (cached per device).
int num_sms();

// Once per (current device, kernel): sets the kernel's dynamic shared-memory limit to `smem` (a
// per-device-context attribute) and, when `units` is given, computes and caches an integer (e.g.
// co-resident CTAs) on that device. Later calls on the same device return the cached value.
// Thread-safe. Returns the value (1 without `units`) or -13 when CUDA refuses the set-up.
int kernel_setup(const void* kernel, size_t smem, int (*units)(const void* kernel, size_t smem, int threads),
                 int threads);
template <typename K>
inline int kernel_setup(K* kernel, size_t smem) {
  return kernel_setup(reinterpret_cast<const void*>(kernel), smem, nullptr, 0);
}

// Status of the last launch: 0, or -14 after printing the CUDA error (a
// failed launch, or an earlier asynchronous fault reported at this point).
int launch_status(const char* what);

}  // namespace s3b
