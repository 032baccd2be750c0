// api_ops.cu — reference-format weight directory loader and the operator
// surface of the C ABI (include/sdg.h): conv2d / linear / groupnorm /
// layernorm / attention / add / concat / upsample on device tensors, the
// counterparts of the reference engine's op wrappers (vk_engine.cpp:546-697).
#include <dirent.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/sdg.h"
#include "sdg_kernels.h"

namespace sdg {
int op_fail(int code, const std::string& msg);
}

// Load every "<key>.bin" of a reference weight directory (vk_engine.cpp:497-507:
// raw fp16, no header). The engine validates sizes per key when it prepares.
void sdg_internal_mark_file(sdg_engine* e, const char* key, const std::string& path);  // engine.cu

// Reads every <key>.bin of `dir` (the reference's unet_w/ format: raw little-endian fp16, Linear
// weights stored [in,out]; vk_engine.cpp:497-507). An unreadable, empty or odd-sized file is an I/O
// error naming it; a file whose value count does not match its key is reported by sdg_prepare as
// SDG_ERR_IO naming the file and the key (the reference instead substitutes zeros, :500-503).
int sdg_internal_load_dir(sdg_engine* e, const char* dir) {
  DIR* d = opendir(dir);
  if (!d) return sdg::op_fail(SDG_ERR_IO, std::string("cannot open weight dir ") + dir);
  int n = 0;
  std::vector<uint16_t> buf;
  while (struct dirent* ent = readdir(d)) {
    const std::string name = ent->d_name;
    if (name.size() < 5 || name.compare(name.size() - 4, 4, ".bin") != 0) continue;
    const std::string path = std::string(dir) + "/" + name;
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) { closedir(d); return sdg::op_fail(SDG_ERR_IO, "cannot read " + path); }
    fseek(f, 0, SEEK_END);
    const long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (sz <= 0 || sz % 2) {
      fclose(f);
      closedir(d);
      return sdg::op_fail(SDG_ERR_IO, path + ": " + std::to_string(sz) + " bytes is not a whole number of fp16 values");
    }
    buf.resize((size_t)sz / 2);
    const size_t got = fread(buf.data(), 2, buf.size(), f);
    fclose(f);
    if (got != buf.size()) { closedir(d); return sdg::op_fail(SDG_ERR_IO, "short read " + path); }
    const int64_t shape[1] = {(int64_t)buf.size()};
    const std::string key = name.substr(0, name.size() - 4);
    const int st = sdg_upload_weight(e, key.c_str(), buf.data(), shape, 1);
    if (st) { closedir(d); return st; }
    sdg_internal_mark_file(e, key.c_str(), path);
    ++n;
  }
  closedir(d);
  if (n == 0) return sdg::op_fail(SDG_ERR_IO, std::string("no .bin weights in ") + dir);
  return SDG_OK;
}

namespace {

int* internal_err_word() {
  static int* w[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return nullptr;
  if (!w[dev]) {
    if (cudaMalloc(&w[dev], 256) != cudaSuccess) return nullptr;
    cudaMemset(w[dev], 0, 256);
  }
  return w[dev];
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SDG_OK;
  if (e == cudaErrorInvalidValue) return sdg::op_fail(SDG_ERR_SHAPE, std::string(what) + ": unsupported shape or arguments");
  return sdg::op_fail(SDG_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" {

SDG_API int sdg_conv2d(const uint16_t* x, const uint16_t* x2, int B, int H, int W, int Ci1, int Ci2, const uint16_t* w,
                       const float* bias, int Co, int k, int stride, const float* rowbias, const uint16_t* residual,
                       int act, uint16_t* y, uint16_t* col_scratch, void* workspace, size_t workspace_bytes,
                       int* err_word, void* stream) {
  if (!x || !w || !y || B <= 0 || H <= 0 || W <= 0 || Ci1 <= 0 || Co <= 0 || (x2 == nullptr) != (Ci2 == 0))
    return sdg::op_fail(SDG_ERR_ARG, "conv2d: bad arguments");
  if (!(k == 1 || k == 3) || !(stride == 1 || stride == 2) || (k == 1 && stride != 1))
    return sdg::op_fail(SDG_ERR_SHAPE, "conv2d: k must be 1 or 3, stride 1 (or 2 for k=3)");
  int* err = err_word ? err_word : internal_err_word();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int Ci = Ci1 + Ci2;
  sdg::GemmArgs a;
  a.N = Co;
  a.w = reinterpret_cast<const __half*>(w);
  a.bias = bias;
  a.rowbias = rowbias;
  a.rowbias_ld = Co;
  a.residual = reinterpret_cast<const __half*>(residual);
  a.act = act == 1 ? 1 : 0;
  a.out = reinterpret_cast<__half*>(y);
  a.ws = static_cast<float*>(workspace);
  a.ws_bytes = workspace ? workspace_bytes : 0;
  if (k == 3 && stride == 2) {  // implicit GEMM over the input walked with stride 2 (col_scratch unused)
    if (x2) return sdg::op_fail(SDG_ERR_SHAPE, "conv2d: stride 2 takes one source");
    if (H % 2 || W % 2) return sdg::op_fail(SDG_ERR_SHAPE, "conv2d: stride 2 needs even H and W");
    (void)col_scratch;
    const int Ho = H / 2, Wo = W / 2;
    a.M = B * Ho * Wo; a.K = 9 * Ci; a.taps = 9; a.stride = 2;
    a.a0 = reinterpret_cast<const __half*>(x); a.cin0 = Ci;
    a.B = B; a.H = H; a.W = W;
    a.rows_per_image = Ho * Wo;
    return cuda_status(sdg::launch_gemm(a, err, s), "conv2d");
  }
  a.M = B * H * W;
  a.K = k * k * Ci;
  a.taps = k * k;
  a.a0 = reinterpret_cast<const __half*>(x);
  a.a1 = reinterpret_cast<const __half*>(x2);
  a.cin0 = Ci1; a.cin1 = Ci2;
  a.B = B; a.H = H; a.W = W;
  a.rows_per_image = H * W;
  return cuda_status(sdg::launch_gemm(a, err, s), "conv2d");
}

SDG_API int sdg_pack_upsample_conv_weights(const uint16_t* w3, int Co, int Ci, uint16_t* wp) {
  if (!w3 || !wp || Co <= 0 || Ci <= 0) return sdg::op_fail(SDG_ERR_ARG, "pack_upsample_conv_weights: bad arguments");
  sdg::pack_upsample_conv_weights(w3, Co, Ci, wp);
  return SDG_OK;
}

SDG_API int sdg_upsample_conv3x3(const uint16_t* x, int B, int H, int W, int Ci, const uint16_t* wp,
                                 const float* bias4, int Co, uint16_t* y, void* workspace, size_t workspace_bytes,
                                 int* err_word, void* stream) {
  if (!x || !wp || !y || B <= 0 || H <= 0 || W <= 0 || Ci <= 0 || Co <= 0)
    return sdg::op_fail(SDG_ERR_ARG, "upsample_conv3x3: bad arguments");
  if (Ci % 64 || Co % 64) return sdg::op_fail(SDG_ERR_SHAPE, "upsample_conv3x3: Ci and Co must be multiples of 64");
  sdg::GemmArgs a;
  a.M = B * H * W; a.N = 4 * Co; a.K = 4 * Ci; a.taps = 4; a.up_co = Co;
  a.a0 = reinterpret_cast<const __half*>(x); a.cin0 = Ci;
  a.B = B; a.H = H; a.W = W; a.rows_per_image = H * W;
  a.w = reinterpret_cast<const __half*>(wp);
  a.bias = bias4;
  a.out = reinterpret_cast<__half*>(y);
  a.ws = static_cast<float*>(workspace);
  a.ws_bytes = workspace ? workspace_bytes : 0;
  return cuda_status(sdg::launch_gemm(a, err_word ? err_word : internal_err_word(), static_cast<cudaStream_t>(stream)),
                     "upsample_conv3x3");
}

static int linear_common(const char* name, const uint16_t* x, int M, int K, const uint16_t* w, const int8_t* w8,
                         const float* wscale, const float* bias, int N, const uint16_t* residual, int act, uint16_t* y,
                         void* workspace, size_t workspace_bytes, int* err_word, void* stream) {
  if (!x || !(w || (w8 && wscale)) || !y || M <= 0 || K <= 0 || N <= 0)
    return sdg::op_fail(SDG_ERR_ARG, std::string(name) + ": bad arguments");
  sdg::GemmArgs a;
  a.M = M; a.N = N; a.K = K; a.taps = 1;
  a.a0 = reinterpret_cast<const __half*>(x); a.cin0 = K;
  a.w = reinterpret_cast<const __half*>(w);
  a.w8 = w8;
  a.wscale = wscale;
  a.bias = bias;
  a.residual = reinterpret_cast<const __half*>(residual);
  a.out = reinterpret_cast<__half*>(y);
  a.ws = static_cast<float*>(workspace);
  a.ws_bytes = workspace ? workspace_bytes : 0;
  if (act == 2) {
    if (residual) return sdg::op_fail(SDG_ERR_ARG, std::string(name) + ": GEGLU takes no residual");
    a.epi = sdg::kEpiGeglu;
  } else {
    a.act = act == 1 ? 1 : 0;
  }
  int* err = err_word ? err_word : internal_err_word();
  return cuda_status(sdg::launch_gemm(a, err, static_cast<cudaStream_t>(stream)), name);
}

SDG_API int sdg_selftest_stalled_gemm(const uint16_t* x, const uint16_t* w, int M, int N, int K, uint16_t* y,
                                      int stall_iter, int wait_limit_us, int* err_word, void* stream) {
  if (!x || !w || !y || !err_word || M <= 0 || N <= 0 || N % 128 || K <= 0 || K % 64 || stall_iter < 0 ||
      wait_limit_us <= 0 || wait_limit_us > 2000000)
    return sdg::op_fail(SDG_ERR_ARG, "selftest_stalled_gemm: bad arguments");
  sdg::GemmArgs a;
  a.M = M; a.N = N; a.K = K; a.taps = 1;
  a.a0 = reinterpret_cast<const __half*>(x); a.cin0 = K;
  a.w = reinterpret_cast<const __half*>(w);
  a.out = reinterpret_cast<__half*>(y);
  a.bn = 128;  // single-CTA 128x128 tiles, no K split: one pipeline per CTA
  a.test_stall_iter = stall_iter;
  a.wait_limit_ns = 1000ull * (unsigned long long)wait_limit_us;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = cuda_status(sdg::launch_gemm(a, err_word, s), "selftest_stalled_gemm");
  if (st) return st;
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, err_word, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e, "selftest_stalled_gemm");
  if (v != 0) {
    cudaMemsetAsync(err_word, 0, sizeof(int), s);
    cudaStreamSynchronize(s);
    char buf[112];
    snprintf(buf, sizeof buf, "selftest_stalled_gemm: device error word 0x%x (a kernel's bounded wait expired)", v);
    return sdg::op_fail(SDG_ERR_DEVICE, buf);
  }
  return SDG_OK;
}

SDG_API int sdg_gemm_plan(int M, int N, int K, int taps, int with_workspace, int* out4) {
  if (!out4 || M <= 0 || N <= 0 || K <= 0 || K % 64 || !(taps == 1 || taps == 9) || K % (64 * taps))
    return sdg::op_fail(SDG_ERR_ARG, "gemm_plan: bad arguments");
  sdg::GemmArgs a;
  a.M = M; a.N = N; a.K = K; a.taps = taps; a.cin0 = K / taps;
  const sdg::GemmPlan pl = sdg::gemm_plan(a, with_workspace != 0);
  out4[0] = pl.bn; out4[1] = pl.pair; out4[2] = pl.splits; out4[3] = pl.csplit;
  return SDG_OK;
}

SDG_API int sdg_linear(const uint16_t* x, int M, int K, const uint16_t* w, const float* bias, int N,
                       const uint16_t* residual, int act, uint16_t* y, void* workspace, size_t workspace_bytes,
                       int* err_word, void* stream) {
  if (!w) return sdg::op_fail(SDG_ERR_ARG, "linear: bad arguments");
  return linear_common("linear", x, M, K, w, nullptr, nullptr, bias, N, residual, act, y, workspace,
                       workspace_bytes, err_word, stream);
}

SDG_API int sdg_linear_wo8(const uint16_t* x, int M, int K, const int8_t* w8, const float* wscale, const float* bias,
                           int N, const uint16_t* residual, int act, uint16_t* y, void* workspace,
                           size_t workspace_bytes, int* err_word, void* stream) {
  if (!w8 || !wscale) return sdg::op_fail(SDG_ERR_ARG, "linear_wo8: bad arguments");
  return linear_common("linear_wo8", x, M, K, nullptr, w8, wscale, bias, N, residual, act, y, workspace,
                       workspace_bytes, err_word, stream);
}

SDG_API int sdg_groupnorm(const uint16_t* x, const uint16_t* x2, int B, int HW, int C1, int C2, int groups,
                          const float* gamma, const float* beta, float eps, int silu, uint16_t* y,
                          float* stats_scratch, void* stream) {
  if (!x || !y || !gamma || !beta || !stats_scratch || (x2 == nullptr) != (C2 == 0) || B <= 0 || HW <= 0 ||
      C1 <= 0 || C2 < 0 || groups <= 0)
    return sdg::op_fail(SDG_ERR_ARG, "groupnorm: bad arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  sdg::GroupNormArgs a;
  a.x0 = reinterpret_cast<const __half*>(x); a.x1 = reinterpret_cast<const __half*>(x2);
  a.C0 = C1; a.C1 = C2; a.B = B; a.HW = HW; a.groups = groups;
  a.gamma = gamma; a.beta = beta; a.eps = eps; a.silu = silu;
  a.y = reinterpret_cast<__half*>(y);
  a.stats = stats_scratch;
  return cuda_status(sdg::launch_groupnorm(a, s), "groupnorm");
}

SDG_API size_t sdg_groupnorm_scratch_bytes(int B, int HW, int C, int groups) {
  if (B <= 0 || HW <= 0 || C <= 0 || groups <= 0) return 0;
  return sdg::groupnorm_scratch_bytes(B, HW, C, groups);
}

SDG_API int sdg_layernorm(const uint16_t* x, int M, int C, const float* gamma, const float* beta, float eps, uint16_t* y,
                          void* stream) {
  if (!x || !y || !gamma || !beta) return sdg::op_fail(SDG_ERR_ARG, "layernorm: bad arguments");
  return cuda_status(sdg::launch_layernorm(reinterpret_cast<const __half*>(x), M, C, gamma, beta, eps,
                                           reinterpret_cast<__half*>(y), static_cast<cudaStream_t>(stream)),
                     "layernorm");
}

SDG_API int sdg_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int heads, int Sq, int Sk,
                          int d, int vt_ld, uint16_t* o, int* err_word, void* stream) {
  if (!q || !k || !v || !o || B <= 0 || heads <= 0) return sdg::op_fail(SDG_ERR_ARG, "attention: bad arguments");
  sdg::AttnArgs a;
  a.q = reinterpret_cast<const __half*>(q);
  a.k = reinterpret_cast<const __half*>(k);
  a.v = reinterpret_cast<const __half*>(v);
  a.BH = B * heads; a.heads = heads; a.Sq = Sq; a.Sk = Sk; a.d = d;
  a.dp = (d + 63) / 64 * 64; a.d16 = (d + 15) / 16 * 16; a.vt_ld = vt_ld;
  a.o = reinterpret_cast<__half*>(o); a.ld_o = heads * d;
  a.scale = 1.0f / sqrtf((float)d);
  int* err = err_word ? err_word : internal_err_word();
  return cuda_status(sdg::launch_attention(a, err, static_cast<cudaStream_t>(stream)), "attention");
}

SDG_API int sdg_add(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* y, void* stream) {
  if (!a || !b || !y) return sdg::op_fail(SDG_ERR_ARG, "add: bad arguments");
  return cuda_status(sdg::launch_add(reinterpret_cast<const __half*>(a), reinterpret_cast<const __half*>(b), n,
                                     reinterpret_cast<__half*>(y), static_cast<cudaStream_t>(stream)),
                     "add");
}

SDG_API int sdg_concat(const uint16_t* a, int Ca, const uint16_t* b, int Cb, int rows, uint16_t* y, void* stream) {
  if (!a || !b || !y) return sdg::op_fail(SDG_ERR_ARG, "concat: bad arguments");
  return cuda_status(sdg::launch_concat(reinterpret_cast<const __half*>(a), Ca, reinterpret_cast<const __half*>(b), Cb,
                                        rows, reinterpret_cast<__half*>(y), static_cast<cudaStream_t>(stream)),
                     "concat");
}

SDG_API int sdg_upsample2x(const uint16_t* x, int B, int H, int W, int C, uint16_t* y, void* stream) {
  if (!x || !y) return sdg::op_fail(SDG_ERR_ARG, "upsample: bad arguments");
  return cuda_status(sdg::launch_upsample2x(reinterpret_cast<const __half*>(x), B, H, W, C,
                                            reinterpret_cast<__half*>(y), static_cast<cudaStream_t>(stream)),
                     "upsample2x");
}

}  // extern "C"
