// sdg_kernels.h — host-side launch interface of the engine's CUDA kernels.
// All activations are fp16 NHWC ([B, H, W, C] == token-major [B*H*W, C]).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace sdg {

enum EpiMode : int {
  kEpiPlain = 0,    // out[m, n] fp16 (row stride ld_out)
  kEpiGeglu = 1,    // W rows interleave 16 value and 16 gate rows; out[m, n/2] = value * gelu(gate)
  kEpiHeads = 2,    // scatter into padded per-head layout [B*heads, S, dp] (Q/K/V for attention)
  kEpiNchwF32 = 3,  // out_f32[b, n, p] fp32 (final conv_out)
};

// One GEMM / implicit-GEMM convolution: D[M,N] = A[M,K] * W[N,K]^T with the
// fused epilogue  act(D + bias[n] + rowbias[img(m), n] + residual[m, n]).
// A is either a row-major [M, K] activation matrix (taps == 1) or, for a
// pad-1 3x3 convolution of stride 1 or 2 (taps == 9), gathered on the fly from the
// NHWC input by 4D TMA boxes shifted per tap (out-of-range rows/columns read
// as zero == the convolution's zero padding). A may come from two sources
// (channel concat [src0 ; src1]): K-chunks with channel < cin0 read src0.
struct GemmArgs {
  int M = 0, N = 0, K = 0;
  int taps = 1;
  const __half* a0 = nullptr;  // source 0: [M, cin0] (taps 1) or NHWC [B,H,W,cin0] (taps 9)
  const __half* a1 = nullptr;  // source 1 (concat) or null
  int cin0 = 0, cin1 = 0;      // channels per tap from each source
  int lda0 = 0, lda1 = 0;      // row strides (elements) for taps == 1 (default cin)
  int B = 1, H = 1, W = 1;     // conv geometry (taps == 9): the INPUT image
  int stride = 1;              // taps == 9: 1, or 2 (output H/2 x W/2, pad 1; M = B * H/2 * W/2)
  // taps == 4: nearest-2x upsample followed by a 3x3 pad-1 convolution, as four 2x2 convolutions of the
  // low-resolution input (one per output phase (py, px)). H, W are the INPUT's; M = B * H * W rows (one
  // per input pixel); N = 4 * up_co columns, phase-major (column ph * up_co + c is output channel c of
  // phase ph = 2 py + px); w = [4 * up_co][4 taps][Cin] (pack_upsample_conv_weights); the output is NHWC
  // [B, 2H, 2W, up_co]; bias [4 * up_co] (the conv bias repeated per phase).
  int up_co = 0;
  const __half* w = nullptr;   // [N, K] K-major (conv: [Co][tap][Cin])
  const int8_t* w8 = nullptr;  // weight-only int8 alternative to w: [N, K] ...
  const float* wscale = nullptr;  // ... with per-row (output channel) scale [N]
  // epilogue
  int epi = kEpiPlain;
  int act = 0;                      // 0 none, 1 SiLU
  const float* bias = nullptr;      // [N]
  const float* rowbias = nullptr;   // [images, rowbias_ld]
  int rowbias_ld = 0;
  int rows_per_image = 1;           // m / rows_per_image = image index (rowbias, heads, nchw)
  const __half* residual = nullptr; // [M, ld_res]
  int ld_res = 0;
  __half* out = nullptr;
  int ld_out = 0;
  float* out_f32 = nullptr;
  __half* head_out[3] = {nullptr, nullptr, nullptr};
  int head_C = 0, heads = 0, head_d = 0, head_dp = 0;
  int head_vt = -1;                 // index of the output stored transposed [BH, d16, head_spad]
  int head_d16 = 0, head_spad = 0;
  int bn = 0;                       // tile N (0 = choose)
  float* ws = nullptr;              // split-K workspace (fp32); split-K only when large enough
  size_t ws_bytes = 0;
  // LayerNorm folded into the neighbouring GEMMs (single-pass 1-CTA fp16 plans only; launch_gemm refuses
  // other plans). Producer (plain output, no row bias, no activation): per output row, one (sum, sum of
  // squares) partial per epilogue warp and tile column block at ln_stat_out[m * ln_stat_ld + 2 * n_blk + w],
  // ln_stat_ld = 2 * N / tile width. Consumer (attention-head epilogue): A = the raw rows, w with
  // gamma folded in (w * gamma per input column), bias = b + w beta, ln_colsum[n] = sum_k of the folded fp16
  // w row; the epilogue applies rstd * (acc - mean * colsum) + bias with mean / rstd over ln_C columns
  // from the ln_stat_parts partials of each row.
  float2* ln_stat_out = nullptr;
  int ln_stat_ld = 0;
  const float2* ln_stat_in = nullptr;
  int ln_stat_parts = 0;
  int ln_C = 0;
  float ln_eps = 0.f;
  const float* ln_colsum = nullptr;
  // Failure-path test only (sdg_selftest_stalled_gemm): the producer leaves the pipeline stage of this
  // k-block iteration (counted per CTA) unloaded, so the waits on it expire after wait_limit_ns.
  int test_stall_iter = -1;
  unsigned long long wait_limit_ns = 0;  // 0: the default 2 s limit of every bounded wait
};

cudaError_t launch_gemm(const GemmArgs& a, int* dev_err, cudaStream_t s);
// Workspace the tile chooser wants for split-K (0 = single pass).
size_t gemm_workspace_bytes(const GemmArgs& a);
// Kernel launches launch_gemm issues for these arguments (1, or 2 with split-K).
int gemm_launch_count(const GemmArgs& a);
// The tile chooser's decision: tile width, CTA pair, workspace K splits, cluster K splits.
struct GemmPlan {
  int bn, pair, splits, csplit;
};
GemmPlan gemm_plan(const GemmArgs& a, bool with_workspace);

// Weights of the taps == 4 GEMM (nearest-2x upsample + 3x3 pad-1 conv as four 2x2 convolutions of the
// low-resolution input) from a 3x3 kernel in the reference's layout w3[Co][Ci][3][3] (fp16 bits):
// wp[(ph * Co + co) * 4 * Ci + (ty * 2 + tx) * Ci + ci], ph = 2 py + px, is the fp32 sum of the 3x3 taps
// (ky, kx) with ky in R(py, ty), kx in R(px, tx), rounded once to fp16, where R(0,0) = {0},
// R(0,1) = {1,2}, R(1,0) = {0,1}, R(1,1) = {2}: output row 2i + py reads input rows i + ty + py - 1.
void pack_upsample_conv_weights(const uint16_t* w3, int Co, int Ci, uint16_t* wp);

// GroupNorm(32) (+SiLU) over NHWC input that may be a channel concat of two
// tensors. stats: groupnorm_scratch_bytes() bytes; receives (mean, rstd) per
// (image, group) as float2 [B][groups].
struct GroupNormArgs {
  const __half* x0 = nullptr; const __half* x1 = nullptr;
  int C0 = 0, C1 = 0, B = 1, HW = 1, groups = 32;
  const float* gamma = nullptr; const float* beta = nullptr;
  float eps = 1e-5f; int silu = 1;
  __half* y = nullptr;
  float* stats = nullptr;
};
cudaError_t launch_groupnorm(const GroupNormArgs& a, cudaStream_t s);
size_t groupnorm_scratch_bytes(int B, int HW, int C, int groups);
int groupnorm_launch_count(const GroupNormArgs& a);

cudaError_t launch_layernorm(const __half* x, int M, int C, const float* gamma, const float* beta, float eps,
                             __half* y, cudaStream_t s);

// Flash attention over padded per-head layouts: q [BH, Sq, dp], k [BH, Sk, dp]
// (dp = d rounded up to 64), v transposed [BH, d16, vt_ld] (d16 = d rounded up
// to 16, vt_ld >= Sk, multiple of 8); fp16, zero in every padding column/row.
// out o[(b*Sq + i)*ld_o + h*d + j] fp16.
struct AttnArgs {
  const __half* q = nullptr; const __half* k = nullptr; const __half* v = nullptr;
  int BH = 0, heads = 0, Sq = 0, Sk = 0, d = 0, dp = 0, d16 = 0, vt_ld = 0;
  __half* o = nullptr; int ld_o = 0;
  float scale = 0.f;
};
cudaError_t launch_attention(const AttnArgs& a, int* dev_err, cudaStream_t s);

// small kernels (sdg_misc.cu)
cudaError_t launch_time_embedding(const float* timesteps, int n_t, int B, const float* temb_proj_in, float* out320,
                                  cudaStream_t s);
// y[m, n] = act(x[m,:] . w[n,:] + bias[n]) for small M; x fp32 [M,K], y fp32. Weights are
// either fp16 w [N,K], or int8 w8 [N,K] with per-row scale ws [N] (exactly one of w / w8).
cudaError_t launch_gemv(const float* x, int M, int K, const __half* w, const int8_t* w8, const float* ws,
                        const float* bias, int N, int act_in, int act_out, float* y, int ldy, cudaStream_t s);
cudaError_t launch_latent_im2col(const float* lat_nchw, int B, int C, int H, int W, int Kpad, __half* col,
                                 cudaStream_t s);
cudaError_t launch_upsample2x(const __half* x, int B, int H, int W, int C, __half* y, cudaStream_t s);
cudaError_t launch_concat(const __half* a, int Ca, const __half* b, int Cb, int rows, __half* y, cudaStream_t s);
cudaError_t launch_add(const __half* a, const __half* b, size_t n, __half* y, cudaStream_t s);
cudaError_t launch_f32_to_f16(const float* x, size_t n, __half* y, cudaStream_t s);
// Fused CFG combine + LCM step over n_img images of L latent elements.
// eps: [n_img, 2, L] (cond, uncond) when eps_pairs (combined with cfg), else
// [n_img, L] (cond only). latents [n_img, L] are updated in place; lat_next
// (optional) receives the new latents laid out for the next forward: twice
// per image when next_pairs, else once.
cudaError_t launch_cfg_lcm(const float* eps, int eps_pairs, float* latents, const float* noise, int n_img, int L,
                           float cfg, double c_skip, double c_out, double sqrt_alpha, double sqrt_beta,
                           double sqrt_alpha_prev, double sqrt_beta_prev, int last, float* lat_next, int next_pairs,
                           cudaStream_t s);

int num_sms();

}  // namespace sdg
