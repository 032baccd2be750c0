/* sdg.h — C ABI of the B200 SD1.5 UNet engine (libsdg.so).
 *
 * Drop-in for the JNI surface of the reference's Vulkan engine
 * (Shoolife/sd-vulkan-pixel10-tensor-g5, app/src/main/cpp/vk_engine.cpp and
 * app/src/main/java/.../sd/VulkanBench.kt:10-27). Every entry point returns an
 * int status (SDG_OK == 0); sdg_last_error() gives the message of the last
 * failure on the calling thread.
 *
 * Conventions
 *   - Host arrays are caller-owned and copied in/out within the call.
 *   - "Device" pointers are CUDA device pointers on the engine's device.
 *   - Activations in the op surface are fp16 NHWC (== token-major [B*H*W, C]).
 *   - Weights handed to sdg_upload_weight use the reference's on-disk format:
 *     one raw fp16 array per diffusers state-dict key; conv [Co,Ci,kh,kw];
 *     norm [C]; every Linear weight TRANSPOSED [in,out] (vk_engine.cpp:497-507).
 *   - One engine per GPU; calls on one engine must be serialised (the
 *     reference serialises on one GpuThread, GenerateViewModel.kt:31).
 */
#ifndef SDG_H_
#define SDG_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SDG_API __attribute__((visibility("default")))

enum {
  SDG_OK = 0,
  SDG_ERR_CUDA = 1,           /* CUDA runtime / launch error */
  SDG_ERR_ARG = 2,            /* bad argument (null, size) */
  SDG_ERR_SHAPE = 3,          /* unsupported shape */
  SDG_ERR_MISSING_WEIGHT = 4, /* a UNet key was never uploaded */
  SDG_ERR_TIMEOUT = 5,        /* host-side wait deadline expired */
  SDG_ERR_IO = 6,             /* weight file missing / short */
  SDG_ERR_NOT_INIT = 7,       /* null or released engine */
  SDG_ERR_DEVICE = 8,         /* a kernel's bounded wait expired (device error word set) */
  SDG_ERR_NCCL = 9,           /* collective failure (multi-GPU gather) */
  SDG_ERR_UNSUPPORTED = 10
};

typedef struct sdg_engine sdg_engine;

typedef struct sdg_profile_row {
  char name[32];   /* op category: GN, LN, CONV3, GEMM, ATTN, GEMV, MISC */
  double ms;       /* summed device time of that category in one forward */
  int launches;
  double flops;    /* algorithmic FLOPs of the category (2*M*N*K; attention 4*Sq*Sk*d per head) */
  double bytes;    /* algorithmic HBM bytes (norms: 1 read + 1 write of the fp16 activation) */
} sdg_profile_row;

/* --- lifecycle --------------------------------------------------------------- */

/* Replaces Java_..._unetInit(shaders, dir) (vk_engine.cpp:796-808): create an
 * engine on CUDA device `device`. When `weights_dir` is non-null every UNet key
 * is read from <weights_dir>/<key>.bin (the reference loads them lazily at
 * vk_engine.cpp:497-507; here they are read once, here). */
SDG_API int sdg_init(int device, const char* weights_dir, sdg_engine** out);

/* One weight in the reference format (see above). `shape` is the PyTorch
 * shape (ndim entries) used to validate the byte count. Replaces the file read
 * inside W(name) (vk_engine.cpp:497-507). */
SDG_API int sdg_upload_weight(sdg_engine* e, const char* key, const uint16_t* fp16, const int64_t* shape, int ndim);

/* Read every UNet key from <dir>/<key>.bin (reference directory format). */
SDG_API int sdg_load_dir(sdg_engine* e, const char* dir);

/* Build device layouts from the uploaded weights (implicit on first forward).
 * Returns SDG_ERR_MISSING_WEIGHT naming the first absent key. */
SDG_API int sdg_prepare(sdg_engine* e);

/* Switch the engine to weight-only int8 before it is prepared (BASELINE
 * config 4; the reference's wo8 model, tools/quantize_wo8.py:42-46 with
 * ai-edge-quantizer's weight_only_wi8_afp32 recipe). At preparation every
 * conv and linear weight is quantized per output channel, symmetric, narrow
 * range: scale = fp16(max|w| / 127) (1 for an all-zero row),
 * q = clamp(round_half_even(w / scale), -127, 127). GEMMs then stream int8
 * tiles and widen them to fp16 in shared memory (dequantised in the
 * mainloop); norms, biases and activations stay as in the fp16 path.
 * SDG_ERR_ARG if the engine is already prepared. */
SDG_API int sdg_quantize_wo8(sdg_engine* e);

/* Replaces Java_..._unetRelease (vk_engine.cpp:915-926): frees everything. */
SDG_API int sdg_release(sdg_engine* e);

/* Message of the last failing call on this thread (empty when none). */
SDG_API int sdg_last_error(char* buf, int n);

/* --- forward ------------------------------------------------------------------- */

/* UNet forward with HOST buffers (north-star unet_forward(latent, timestep,
 * context); replaces Java_..._unetForward, vk_engine.cpp:875-887, whose
 * caller precomputes the 320-d sinusoid — pass timesteps instead).
 *   latent    [B,4,H,W] fp32 (H, W multiples of 8, <= 128)
 *   timesteps [n_t] fp32, n_t == 1 (shared) or B
 *   context   [B,77,768] fp32
 *   out       [B,4,H,W] fp32 (eps prediction)
 * stream may be NULL (engine stream). Synchronous. */
SDG_API int sdg_unet_forward(sdg_engine* e, const float* latent, const float* timesteps, int n_t,
                             const float* context, int B, int H, int W, float* out, void* stream);

/* Same, but with the reference's precomputed 320-d time projection
 * ([n_t,320] fp32, cos first) in place of timesteps — the exact argument list
 * of Java_..._unetForward (vk_engine.cpp:875-887). */
SDG_API int sdg_unet_forward_tproj(sdg_engine* e, const float* latent, const float* temb_proj, int n_t,
                                   const float* context, int B, int H, int W, float* out, void* stream);

/* Device-pointer variant: same layouts, all pointers on the engine's device;
 * asynchronous on `stream` (NULL = the CUDA legacy default stream). */
SDG_API int sdg_unet_forward_device(sdg_engine* e, const float* latent, const float* timesteps, int n_t,
                                    const float* context, int B, int H, int W, float* out, void* stream);

/* Batch-CFG forward, replaces Java_..._unetForward2 (vk_engine.cpp:891-913):
 * one latent [4,H,W], one timestep, cond and uncond contexts [77,768];
 * out2 = [cond eps (4HW) ; uncond eps (4HW)]. Runs one B=2 forward. */
SDG_API int sdg_unet_forward_cfg(sdg_engine* e, const float* latent, float timestep, const float* cond,
                                 const float* uncond, int H, int W, float* out2);

/* 4-step LCM denoise with batch-CFG per image (VulkanUnetPipeline.kt:63-97 +
 * LcmScheduler.kt): n_img latents [n_img,4,H,W] (initial noise), cond/uncond
 * contexts [n_img,77,768] each, step noise [steps-1, n_img,4,H,W] (host
 * generated, used between steps), cfg scale. Writes final latents to out.
 * The CFG combine and the LCM update run on the device. */
SDG_API int sdg_lcm_denoise(sdg_engine* e, const float* latents, const float* cond, const float* uncond,
                            const float* step_noise, int n_img, int H, int W, int steps, float cfg, float* out);

/* sdg_lcm_denoise with classifier-free guidance on the first cfg_steps steps
 * only (TpuUnetPipeline.kt:75-112: the reference's default is 2 of 4); the
 * other steps run one cond-only forward per image (batch n_img) and use its
 * eps directly. cfg <= 1 means no guidance at all (uncond may then be NULL).
 * cfg_steps >= steps is sdg_lcm_denoise. Within one call every step after a
 * forward plan's first run reuses that plan's cross-attention K/V (the
 * context does not change between steps). */
SDG_API int sdg_lcm_denoise_ex(sdg_engine* e, const float* latents, const float* cond, const float* uncond,
                               const float* step_noise, int n_img, int H, int W, int steps, float cfg, int cfg_steps,
                               float* out);

/* Per-category device times of one forward (replaces Java_..._unetProfile,
 * vk_engine.cpp:854-872, which only logs): the forward is captured with a
 * timing event on each side of every launch and replayed as a graph; each
 * launch's time is its event interval (launches serialised against their
 * neighbours). Returns the number of rows written (<= cap) or a negative
 * status. */
SDG_API int sdg_profile(sdg_engine* e, int B, int H, int W, sdg_profile_row* rows, int cap);

/* No reference counterpart (measurement): device time of one op category of the
 * forward at (B,H,W) without per-launch events. The forward's launches are recorded
 * with their arguments; those of the named categories ("GN", "LN", "CONV3", "GEMM",
 * "ATTN", "GEMV", "MISC"; several joined by ',' or '+') are captured alone, in forward
 * order on one stream, as a CUDA graph that is replayed once to warm up and then
 * `reps` times back to back between two CUDA events. *ms = mean time of one replay,
 * i.e. that category's summed kernel time per forward; *launches = launches per
 * replay; *flops / *bytes = the category's algorithmic work per forward. The replays
 * overwrite the plan's intermediate buffers (the next forward recomputes them). */
SDG_API int sdg_profile_category(sdg_engine* e, int B, int H, int W, const char* categories, int reps, double* ms,
                                 int* launches, double* flops, double* bytes);

typedef struct sdg_launch_row {
  char label[128];  /* op, shape and (GEMMs) the tile chooser's plan */
  char category[8]; /* GN, LN, CONV3, GEMM, ATTN, GEMV, MISC */
  double ms;        /* device time of this launch (see sdg_profile_launches) */
  double flops;     /* algorithmic FLOPs of the launch */
  double bytes;     /* algorithmic HBM bytes of the launch (norms) */
} sdg_launch_row;

/* No reference counterpart (measurement): per-launch device times of the forward's
 * launches of the named categories (as for sdg_profile_category), in forward order:
 * each launch is captured `reps` times back to back in a CUDA graph with its recorded
 * arguments, replayed once after a warm-up replay; ms = replay time / reps. Returns
 * the number of rows written (<= cap) or a negative status. */
SDG_API int sdg_profile_launches(sdg_engine* e, int B, int H, int W, const char* categories, int reps,
                                 sdg_launch_row* rows, int cap);

/* Number of kernel launches of one forward at (B,H,W) (after a forward ran). */
SDG_API int sdg_forward_launches(sdg_engine* e, int B, int H, int W);

/* No reference counterpart (introspection for tests and tuning): how the GEMM tile
 * chooser runs an M x N x K product (taps = 9 for a 3x3 convolution, K = 9 * Cin) on
 * the current device: out4 = {tile width, CTA pair (0/1), workspace K splits, cluster
 * K splits}; with_workspace = 0 asks for the choice when no split-K workspace is given. */
SDG_API int sdg_gemm_plan(int M, int N, int K, int taps, int with_workspace, int* out4);

/* No reference counterpart (failure-path test; the reference has no device-side
 * timeouts): runs the tensor-core GEMM y[M,N] = x[M,K] * w[N,K]^T on single-CTA
 * 128x128 tiles with the pipeline stage of k-block iteration `stall_iter` (counted
 * per CTA) never loaded, and every bounded wait limited to `wait_limit_us`. The
 * waits on that stage expire, the kernel records a timeout code in `err_word`,
 * waits for its own copies and MMAs in flight, frees its TMEM and returns. The call
 * synchronises `stream`, clears the word and returns SDG_ERR_DEVICE naming the code
 * (SDG_OK would mean nothing expired). Needs N % 128 == 0, K % 64 == 0 and more than
 * stall_iter pipeline stages of K. No GPU fault, trap or hang is involved. */
SDG_API int sdg_selftest_stalled_gemm(const uint16_t* x, const uint16_t* w, int M, int N, int K, uint16_t* y,
                                      int stall_iter, int wait_limit_us, int* err_word, void* stream);

/* --- operator surface (device pointers, fp16 NHWC, stream may be NULL) -------------
 * Replaces the engine's internal op wrappers conv / matmul / groupnorm(_silu) /
 * layernorm / attention op / addbias / addv / concat / upsample
 * (vk_engine.cpp:546-697). Weights here are in ENGINE layout:
 *   conv weight   [Co][k*k][Ci1+Ci2]   (k = 3 or 1; tap-major, channel-minor)
 *   linear weight [N][K]               (K-major, i.e. PyTorch [out,in])
 * err_word: device int zeroed by the caller; a kernel whose bounded wait
 * expires writes a non-zero code there (NULL: the op uses an internal word). */

/* y = conv(x) (+bias[Co]) (+rowbias[b,Co]) (+residual) (act: 0 none, 1 SiLU).
 * x is [B,H,W,Ci1], x2 (optional, channel concat after x) [B,H,W,Ci2].
 * k = 3 (pad 1, stride 1 or 2; stride 2 needs even H and W) or 1. y is
 * [B,Ho,Wo,Co]. col_scratch is not used (kept for source compatibility; NULL
 * is fine): stride 2 runs as an implicit GEMM too.
 * workspace (optional, fp32-aligned device memory): when the tile chooser
 * splits K across CTAs (small M, large K) it needs up to 32*M*Co*4 bytes; with
 * less (or NULL) the op runs without split-K. */
SDG_API int sdg_conv2d(const uint16_t* x, const uint16_t* x2, int B, int H, int W, int Ci1, int Ci2,
                       const uint16_t* w, const float* bias, int Co, int k, int stride, const float* rowbias,
                       const uint16_t* residual, int act, uint16_t* y, uint16_t* col_scratch, void* workspace,
                       size_t workspace_bytes, int* err_word, void* stream);

/* y[M,N] = x[M,K] * w[N,K]^T (+bias) (+residual) (act: 0 none, 1 SiLU,
 * 2 GEGLU: w rows interleaved in groups of 16, [16 value rows ; the matching 16 gate
 * rows] repeated (bias likewise), y is [M, N/2]; N a multiple of 64). */
SDG_API int sdg_linear(const uint16_t* x, int M, int K, const uint16_t* w, const float* bias, int N,
                       const uint16_t* residual, int act, uint16_t* y, void* workspace, size_t workspace_bytes,
                       int* err_word, void* stream);

/* sdg_linear with weight-only int8 weights: w8 [N,K] int8 and wscale [N] fp32
 * (per output row; the weight is w8[n,k] * wscale[n]). The int8 tile is
 * widened to fp16 in shared memory inside the GEMM mainloop and the scale is
 * applied to the fp32 accumulator in the epilogue. Same act / GEGLU layout /
 * residual / workspace rules as sdg_linear. Replaces the reference's wo8
 * model path (tools/quantize_wo8.py:42-46, weight_only_wi8_afp32), which has
 * no op-level entry of its own. */
SDG_API int sdg_linear_wo8(const uint16_t* x, int M, int K, const int8_t* w8, const float* wscale, const float* bias,
                           int N, const uint16_t* residual, int act, uint16_t* y, void* workspace,
                           size_t workspace_bytes, int* err_word, void* stream);

/* GroupNorm(groups) (+SiLU) over x (optionally channel-concat [x ; x2]),
 * [B,HW,C1+C2] -> y. stats_scratch: device memory of at least
 * sdg_groupnorm_scratch_bytes(B, HW, C1+C2, groups) bytes, any contents.
 * Deterministic: per-image results do not depend on the batch. */
SDG_API int sdg_groupnorm(const uint16_t* x, const uint16_t* x2, int B, int HW, int C1, int C2, int groups,
                          const float* gamma, const float* beta, float eps, int silu, uint16_t* y,
                          float* stats_scratch, void* stream);

/* Bytes of device scratch sdg_groupnorm needs for this shape (0 on bad input). */
SDG_API size_t sdg_groupnorm_scratch_bytes(int B, int HW, int C, int groups);

/* sdg_groupnorm without the stats_scratch argument: it allocates nothing.
 * No counterpart in the reference (whose engine allocates its own buffers).
 * For callers that cannot allocate device memory themselves — e.g. a JNI or
 * other foreign-language front end that reaches this library only through
 * the C ABI and has no CUDA runtime of its own. The scratch is a fixed array
 * of sdg_groupnorm_noalloc_max_scratch_bytes() bytes (64 KiB: batch * groups
 * <= 8192) inside the library, held on every GPU that loads it until the
 * process exits; shapes needing more (see sdg_groupnorm_scratch_bytes) return
 * SDG_ERR_SHAPE.
 * The first call on a device looks up the array's device address; make that
 * first call before any stream capture. All calls share the one array: calls
 * that overlap on the GPU (different streams, or different host threads
 * without ordering) race and must be serialised by the caller. */
SDG_API int sdg_groupnorm_noalloc(const uint16_t* x, const uint16_t* x2, int B, int HW, int C1, int C2, int groups,
                                  const float* gamma, const float* beta, float eps, int silu, uint16_t* y,
                                  void* stream);
SDG_API size_t sdg_groupnorm_noalloc_max_scratch_bytes(void);

SDG_API int sdg_layernorm(const uint16_t* x, int M, int C, const float* gamma, const float* beta, float eps,
                          uint16_t* y, void* stream);

/* Multi-head attention with per-image keys. q [BH,Sq,dp], k [BH,Sk,dp]
 * (dp = d rounded up to 64), v TRANSPOSED [BH,d16,vt_ld] (d16 = d rounded up
 * to 16, vt_ld >= Sk, multiple of 8); all padding zero. o [B,Sq,heads*d]. */
SDG_API int sdg_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int heads, int Sq,
                          int Sk, int d, int vt_ld, uint16_t* o, int* err_word, void* stream);

SDG_API int sdg_add(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* y, void* stream);
SDG_API int sdg_concat(const uint16_t* a, int Ca, const uint16_t* b, int Cb, int rows, uint16_t* y, void* stream);
SDG_API int sdg_upsample2x(const uint16_t* x, int B, int H, int W, int C, uint16_t* y, void* stream);

/* Replaces the reference's upsample() block (vk_engine.cpp:693-697: upsample_f32.comp nearest 2x, then
 * a 3x3 pad-1 conv) with one implicit GEMM that never writes the upsampled tensor: each output phase
 * (py, px) of the 2H x 2W output is a 2x2 convolution of the H x W input with folded weights.
 * Host-only (no GPU): folds a 3x3 kernel w3 [Co][Ci][3][3] (the reference's conv layout, fp16 bits)
 * into wp [4 phases][Co][4 taps][Ci] (ph = 2 py + px, tap = 2 ty + tx): the fp32 sum of the 3x3 taps
 * that land on input pixel (i + ty + py - 1, j + tx + px - 1) of output pixel (2i + py, 2j + px),
 * rounded once to fp16. 16 * Co * Ci values. */
SDG_API int sdg_pack_upsample_conv_weights(const uint16_t* w3, int Co, int Ci, uint16_t* wp);
/* y [B,2H,2W,Co] = conv3x3(upsample2x(x)) + bias, x [B,H,W,Ci] (Ci and Co multiples of 64), wp from
 * sdg_pack_upsample_conv_weights, bias4 the conv bias repeated per phase [4 * Co] (fp32, may be NULL).
 * workspace as in sdg_conv2d. */
SDG_API int sdg_upsample_conv3x3(const uint16_t* x, int B, int H, int W, int Ci, const uint16_t* wp,
                                 const float* bias4, int Co, uint16_t* y, void* workspace, size_t workspace_bytes,
                                 int* err_word, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SDG_H_ */
