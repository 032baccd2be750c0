// misc.cu — small bandwidth kernels around the tensor-core path:
// time embedding (VulkanUnetPipeline.kt:36-46 sinusoid, computed in fp64),
// small-M GEMV (time MLP vk_engine.cpp:716-717, per-ResNet time_emb_proj
// :627-630, batched into one launch), im2col for
// the 4-channel conv_in, nearest 2x upsample (upsample_f32.comp), channel
// concat (vk_engine.cpp:677-688), add, and the fused CFG-combine + LCM step
// (VulkanUnetPipeline.kt:86, LcmScheduler.kt:56-82).
#include <cmath>

#include "sdg_kernels.h"
#include "sdg_launch.h"
#include "sdg_ptx.cuh"

namespace sdg {
namespace {

__global__ void time_embedding_kernel(const float* t, int n_t, int B, const float* tin, float* out) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const int i = threadIdx.x;  // 0..159
  if (i >= 160) return;
  float* o = out + (size_t)b * 320;
  if (tin) {
    const float* src = tin + (size_t)(n_t == 1 ? 0 : b) * 320;
    o[i] = src[i];
    o[160 + i] = src[160 + i];
    return;
  }
  const double tv = (double)t[n_t == 1 ? 0 : b];
  const double freq = exp(-log(10000.0) * (double)i / 160.0);
  const double arg = tv * freq;
  o[i] = (float)cos(arg);
  o[160 + i] = (float)sin(arg);
}

constexpr int kGemvMaxM = 8;
constexpr int kGemvMaxK = 1280;

// Each warp computes kGemvRows outputs n; W8 = weight-only int8 rows [N, K] with
// per-row scale ws[n]. All of a warp's weight loads are issued before any use
// (K <= kGemvMaxK: at most kGemvVecs 8-element vectors per lane and row).
constexpr int kGemvRows = 2;
constexpr int kGemvVecs = kGemvMaxK / 256;
template <bool W8>
__global__ void __launch_bounds__(256) gemv_kernel(const float* __restrict__ x, int M, int K, const __half* __restrict__ w,
                                                   const int8_t* __restrict__ w8, const float* __restrict__ ws,
                                                   const float* __restrict__ bias, int N, int act_in, int act_out,
                                                   float* __restrict__ y, int ldy) {
  pdl_wait();
  pdl_trigger();
  __shared__ __align__(16) float xs[kGemvMaxM * kGemvMaxK];
  for (int i = threadIdx.x; i < M * K; i += blockDim.x) {
    const float v = x[i];
    xs[i] = act_in ? silu_f(v) : v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_first = (blockIdx.x * (blockDim.x >> 5) + warp) * kGemvRows;
  if (n_first >= N) return;
  uint4 wv[kGemvRows][kGemvVecs];
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r) {
    const int n = min(n_first + r, N - 1);
#pragma unroll
    for (int i = 0; i < kGemvVecs; ++i) {
      const int k0 = lane * 8 + i * 256;
      if (k0 < K) {
        if constexpr (W8) {
          const uint2 u = __ldg(reinterpret_cast<const uint2*>(w8 + (size_t)n * K + k0));
          wv[r][i] = make_uint4(u.x, u.y, 0u, 0u);
        } else {
          wv[r][i] = __ldg(reinterpret_cast<const uint4*>(w + (size_t)n * K + k0));
        }
      }
    }
  }
  float acc[kGemvRows][kGemvMaxM];
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
    for (int m = 0; m < kGemvMaxM; ++m) acc[r][m] = 0.f;
#pragma unroll
  for (int i = 0; i < kGemvVecs; ++i) {
    const int k0 = lane * 8 + i * 256;
    if (k0 >= K) break;
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r) {
      float wf[8];
      if constexpr (W8) {
        const uint32_t b4[2] = {wv[r][i].x, wv[r][i].y};
#pragma unroll
        for (int e = 0; e < 8; ++e) wf[e] = (float)(int8_t)((b4[e >> 2] >> (8 * (e & 3))) & 0xff);
      } else {
        const __half2* h = reinterpret_cast<const __half2*>(&wv[r][i]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f = __half22float2(h[e]);
          wf[2 * e] = f.x;
          wf[2 * e + 1] = f.y;
        }
      }
#pragma unroll
      for (int m = 0; m < kGemvMaxM; ++m) {
        if (m < M) {
          // two 16-byte shared loads per 8 weights (scalar loads here were the kernel's bottleneck:
          // lanes 32 bytes apart, several-way bank conflicts per element)
          const float4 xa = *reinterpret_cast<const float4*>(xs + m * K + k0);
          const float4 xb = *reinterpret_cast<const float4*>(xs + m * K + k0 + 4);
          acc[r][m] += wf[0] * xa.x + wf[1] * xa.y + wf[2] * xa.z + wf[3] * xa.w +
                       wf[4] * xb.x + wf[5] * xb.y + wf[6] * xb.z + wf[7] * xb.w;
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r) {
    const int n = n_first + r;
#pragma unroll
    for (int m = 0; m < kGemvMaxM; ++m) {
      float v = acc[r][m];
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && m < M && n < N) {
        if constexpr (W8) v *= ws[n];
        v += bias ? bias[n] : 0.f;
        if (act_out) v = silu_f(v);
        y[(size_t)m * ldy + n] = v;
      }
    }
  }
}

__global__ void latent_im2col_kernel(const float* __restrict__ lat, int B, int Cl, int H, int W, int Kpad,
                                     __half* __restrict__ col) {
  pdl_wait();
  pdl_trigger();
  const size_t total = (size_t)B * H * W * Kpad;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int k = (int)(i % Kpad);
    const size_t pix = i / Kpad;
    float v = 0.f;
    if (k < 9 * Cl) {
      const int tap = k / Cl, c = k % Cl;
      const int x = (int)(pix % W), y = (int)((pix / W) % H), b = (int)(pix / ((size_t)W * H));
      const int iy = y + tap / 3 - 1, ix = x + tap % 3 - 1;
      if (iy >= 0 && iy < H && ix >= 0 && ix < W) v = lat[(((size_t)b * Cl + c) * H + iy) * W + ix];
    }
    col[i] = __float2half_rn(v);
  }
}

__global__ void upsample2x_kernel(const __half* __restrict__ x, int B, int H, int W, int C, __half* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int nvec = C / 8;
  const int Ho = 2 * H, Wo = 2 * W;
  const size_t total = (size_t)B * Ho * Wo * nvec;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int v = (int)(i % nvec);
    const size_t pix = i / nvec;
    const int ox = (int)(pix % Wo), oy = (int)((pix / Wo) % Ho), b = (int)(pix / ((size_t)Wo * Ho));
    const uint4 u = *reinterpret_cast<const uint4*>(x + (((size_t)b * H + oy / 2) * W + ox / 2) * C + v * 8);
    *reinterpret_cast<uint4*>(y + pix * C + v * 8) = u;
  }
}

__global__ void concat_kernel(const __half* __restrict__ a, int Ca, const __half* __restrict__ b, int Cb, int rows,
                              __half* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int C = Ca + Cb, nvec = C / 8;
  const size_t total = (size_t)rows * nvec;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % nvec) * 8;
    const size_t r = i / nvec;
    const uint4 u = c < Ca ? *reinterpret_cast<const uint4*>(a + r * Ca + c) : *reinterpret_cast<const uint4*>(b + r * Cb + (c - Ca));
    *reinterpret_cast<uint4*>(y + r * C + c) = u;
  }
}

__global__ void add_kernel(const __half2* __restrict__ a, const __half2* __restrict__ b, size_t n2, __half2* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n2; i += (size_t)gridDim.x * blockDim.x) {
    const float2 fa = __half22float2(a[i]), fb = __half22float2(b[i]);
    y[i] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
  }
}

__global__ void f32_to_f16_kernel(const float* __restrict__ x, size_t n, __half* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] = __float2half_rn(x[i]);
}

// eps2: [n_img, 2, L] (cond then uncond per image); latents [n_img, L] fp32.
// eps = uncond + cfg*(cond-uncond); LCM step (LcmScheduler.kt:68-80, fp64 math
// like the Kotlin reference); lat_pair[img, 0|1, :] = new latents (input of
// the next batch-CFG forward).
__global__ void cfg_lcm_kernel(const float* __restrict__ eps, int eps_pairs, float* __restrict__ lat,
                               const float* __restrict__ noise, int n_img, int L, float cfg, double c_skip,
                               double c_out, double sa, double sb, double sap, double sbp, int last,
                               float* __restrict__ lat_next, int next_pairs) {
  pdl_wait();
  pdl_trigger();
  const size_t total = (size_t)n_img * L;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t img = i / L, j = i % L;
    float e;
    if (eps_pairs) {
      const float ec = eps[(img * 2 + 0) * L + j];
      const float eu = eps[(img * 2 + 1) * L + j];
      e = eu + cfg * (ec - eu);
    } else {
      e = eps[i];
    }
    const double x = (double)lat[i];
    const double x0 = (x - sb * (double)e) / sa;
    const double den = c_out * x0 + c_skip * x;
    const float nv = last ? (float)den : (float)(sap * den + sbp * (double)noise[i]);
    lat[i] = nv;
    if (lat_next) {
      if (next_pairs) {
        lat_next[(img * 2 + 0) * L + j] = nv;
        lat_next[(img * 2 + 1) * L + j] = nv;
      } else {
        lat_next[i] = nv;
      }
    }
  }
}

inline int grid_for(size_t n, int threads = 256) {
  size_t g = (n + threads - 1) / threads;
  const size_t cap = (size_t)num_sms() * 16;
  if (g > cap) g = cap;
  return (int)(g ? g : 1);
}

}  // namespace

cudaError_t launch_time_embedding(const float* t, int n_t, int B, const float* tin, float* out320, cudaStream_t s) {
  if (B <= 0 || (n_t != 1 && n_t != B)) return cudaErrorInvalidValue;
  return launch_kernel(time_embedding_kernel, dim3(B), dim3(160), 0, s, 0, t, n_t, B, tin, out320);
}

cudaError_t launch_gemv(const float* x, int M, int K, const __half* w, const int8_t* w8, const float* ws,
                        const float* bias, int N, int act_in, int act_out, float* y, int ldy, cudaStream_t s) {
  if (M <= 0 || K <= 0 || K > kGemvMaxK || K % 8) return cudaErrorInvalidValue;
  if ((w8 != nullptr) == (w != nullptr) || (w8 && !ws)) return cudaErrorInvalidValue;
  const int rows_per_block = 8 * kGemvRows;
  const int blocks = (N + rows_per_block - 1) / rows_per_block;
  for (int m0 = 0; m0 < M; m0 += kGemvMaxM) {  // rows in chunks of kGemvMaxM
    const int mc = M - m0 < kGemvMaxM ? M - m0 : kGemvMaxM;
    cudaError_t e;
    if (w8)
      e = launch_kernel(gemv_kernel<true>, dim3(blocks), dim3(256), 0, s, 0, x + (size_t)m0 * K, mc, K,
                        (const __half*)nullptr, w8, ws, bias, N, act_in, act_out, y + (size_t)m0 * ldy, ldy);
    else
      e = launch_kernel(gemv_kernel<false>, dim3(blocks), dim3(256), 0, s, 0, x + (size_t)m0 * K, mc, K, w,
                        (const int8_t*)nullptr, (const float*)nullptr, bias, N, act_in, act_out,
                        y + (size_t)m0 * ldy, ldy);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_latent_im2col(const float* lat, int B, int Cl, int H, int W, int Kpad, __half* col, cudaStream_t s) {
  if (Kpad < 9 * Cl) return cudaErrorInvalidValue;
  const size_t total = (size_t)B * H * W * Kpad;
  return launch_kernel(latent_im2col_kernel, dim3(grid_for(total)), dim3(256), 0, s, 0, lat, B, Cl, H, W, Kpad, col);
}

cudaError_t launch_upsample2x(const __half* x, int B, int H, int W, int C, __half* y, cudaStream_t s) {
  if (C % 8) return cudaErrorInvalidValue;
  const size_t total = (size_t)B * 4 * H * W * (C / 8);
  return launch_kernel(upsample2x_kernel, dim3(grid_for(total)), dim3(256), 0, s, 0, x, B, H, W, C, y);
}

cudaError_t launch_concat(const __half* a, int Ca, const __half* b, int Cb, int rows, __half* y, cudaStream_t s) {
  if (Ca % 8 || Cb % 8) return cudaErrorInvalidValue;
  const size_t total = (size_t)rows * ((Ca + Cb) / 8);
  return launch_kernel(concat_kernel, dim3(grid_for(total)), dim3(256), 0, s, 0, a, Ca, b, Cb, rows, y);
}

cudaError_t launch_add(const __half* a, const __half* b, size_t n, __half* y, cudaStream_t s) {
  if (n % 2) return cudaErrorInvalidValue;
  return launch_kernel(add_kernel, dim3(grid_for(n / 2)), dim3(256), 0, s, 0, reinterpret_cast<const __half2*>(a),
                       reinterpret_cast<const __half2*>(b), n / 2, reinterpret_cast<__half2*>(y));
}

cudaError_t launch_f32_to_f16(const float* x, size_t n, __half* y, cudaStream_t s) {
  return launch_kernel(f32_to_f16_kernel, dim3(grid_for(n)), dim3(256), 0, s, 0, x, n, y);
}

cudaError_t launch_cfg_lcm(const float* eps, int eps_pairs, float* latents, const float* noise, int n_img, int L,
                           float cfg, double c_skip, double c_out, double sa, double sb, double sap, double sbp,
                           int last, float* lat_next, int next_pairs, cudaStream_t s) {
  if (n_img <= 0 || L <= 0 || (!last && !noise)) return cudaErrorInvalidValue;
  const size_t total = (size_t)n_img * L;
  return launch_kernel(cfg_lcm_kernel, dim3(grid_for(total)), dim3(256), 0, s, 0, eps, eps_pairs, latents, noise, n_img,
                       L, cfg, c_skip, c_out, sa, sb, sap, sbp, last, lat_next, next_pairs);
}

}  // namespace sdg
