// norm.cu — GroupNorm(32)(+SiLU) and LayerNorm for NHWC fp16 activations.
//
// GroupNorm replaces groupnorm_f32.comp / groupnorm_silu.comp
// (vk_engine.cpp:548-549): statistics per (image, group), y = (x-mu)*rstd*g+b,
// optional SiLU. The reference reduces one group per workgroup with
// var = E[x^2] - mu^2 (groupnorm_f32.comp:24-25); here the work is split for
// bandwidth instead:
//   pass 1 (stats): blocks of (image, pixel chunk); each thread owns one
//     128-bit vector of 8 channels and accumulates shifted sums
//     S1 = sum(x-K_c), S2 = sum((x-K_c)^2) with K_c = x[img, pixel 0, c]
//     (the shift removes the E[x^2]-mu^2 cancellation); per-channel partials
//     are reduced in shared memory and added to a [B, C, 2] fp32 scratch.
//   pass 2 (apply): each block folds the per-channel sums into per-group
//     (mu, rstd) exactly, then streams its chunk with 128-bit loads/stores.
// The input may be a channel concat [x0 ; x1] (up-block skip connections),
// read in place from both sources.
#include <algorithm>

#include "sdg_kernels.h"
#include "sdg_ptx.cuh"

namespace sdg {
namespace {

constexpr int kGnThreads = 256;
constexpr int kGnMaxC = 2560;

__device__ __forceinline__ const __half* gn_src(const GroupNormArgs& a, int c, size_t pix, int& cl) {
  if (c < a.C0) {
    cl = c;
    return a.x0 + pix * a.C0;
  }
  cl = c - a.C0;
  return a.x1 + pix * a.C1;
}

__global__ void __launch_bounds__(kGnThreads) gn_stats_kernel(GroupNormArgs a, int pix_per_block) {
  const int C = a.C0 + a.C1;
  const int nvec = C / 8;
  const int img = blockIdx.y;
  const int p_begin = blockIdx.x * pix_per_block;
  const int p_end = min(a.HW, p_begin + pix_per_block);
  __shared__ float s1[kGnMaxC];
  __shared__ float s2[kGnMaxC];
  for (int c = threadIdx.x; c < C; c += blockDim.x) { s1[c] = 0.f; s2[c] = 0.f; }
  __syncthreads();
  const size_t img_base = (size_t)img * a.HW;
  // threads cover (vector, pixel-row) pairs; each thread keeps one channel vector fixed
  const int rows = max(1, (int)blockDim.x / nvec);
  const int vecs_per_pass = rows * nvec <= (int)blockDim.x ? nvec : (int)blockDim.x;
  for (int v0 = 0; v0 < nvec; v0 += vecs_per_pass) {
    const int t = threadIdx.x;
    const int v = v0 + t % vecs_per_pass;
    const int r = t / vecs_per_pass;
    const int nrows = (vecs_per_pass == nvec) ? rows : 1;
    if (v < nvec && r < nrows) {
      const int c0 = v * 8;
      int cl;
      const __half* k_ptr = gn_src(a, c0, img_base, cl);
      float K[8], S1[8], S2[8];
      {
        uint4 u = *reinterpret_cast<const uint4*>(k_ptr + cl);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f = __half22float2(h[e]);
          K[2 * e] = f.x;
          K[2 * e + 1] = f.y;
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) { S1[e] = 0.f; S2[e] = 0.f; }
      for (int pix = p_begin + r; pix < p_end; pix += nrows) {
        const __half* src = gn_src(a, c0, img_base + pix, cl);
        uint4 u = *reinterpret_cast<const uint4*>(src + cl);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f = __half22float2(h[e]);
          const float d0 = f.x - K[2 * e], d1 = f.y - K[2 * e + 1];
          S1[2 * e] += d0; S2[2 * e] += d0 * d0;
          S1[2 * e + 1] += d1; S2[2 * e + 1] += d1 * d1;
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        atomicAdd(&s1[c0 + e], S1[e]);
        atomicAdd(&s2[c0 + e], S2[e]);
      }
    }
  }
  __syncthreads();
  float* st = a.stats + (size_t)img * C * 2;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    atomicAdd(st + 2 * c, s1[c]);
    atomicAdd(st + 2 * c + 1, s2[c]);
  }
}

__global__ void __launch_bounds__(kGnThreads) gn_apply_kernel(GroupNormArgs a, int pix_per_block) {
  const int C = a.C0 + a.C1;
  const int G = a.groups;
  const int cpg = C / G;
  const int img = blockIdx.y;
  __shared__ float sc[kGnMaxC];
  __shared__ float sh[kGnMaxC];
  __shared__ float gmu[64];
  __shared__ float grs[64];
  const float* st = a.stats + (size_t)img * C * 2;
  const size_t img_base = (size_t)img * a.HW;
  const float n = (float)a.HW;
  const float Ng = (float)a.HW * cpg;
  // per-group mean / rstd from per-channel shifted sums (one warp per group)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int g = warp; g < G; g += blockDim.x / 32) {
    float sum = 0.f;
    for (int j = lane; j < cpg; j += 32) {
      const int c = g * cpg + j;
      int cl;
      const __half* kp = gn_src(a, c, img_base, cl);
      const float K = __half2float(kp[cl]);
      sum += K * n + st[2 * c];
    }
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mu = sum / Ng;
    float m2 = 0.f;
    for (int j = lane; j < cpg; j += 32) {
      const int c = g * cpg + j;
      int cl;
      const __half* kp = gn_src(a, c, img_base, cl);
      const float dK = __half2float(kp[cl]) - mu;
      m2 += st[2 * c + 1] + 2.f * dK * st[2 * c] + n * dK * dK;
    }
    for (int o = 16; o; o >>= 1) m2 += __shfl_xor_sync(0xffffffffu, m2, o);
    if (lane == 0) {
      gmu[g] = mu;
      grs[g] = rsqrtf(fmaxf(m2 / Ng, 0.f) + a.eps);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const int g = c / cpg;
    const float s = grs[g] * a.gamma[c];
    sc[c] = s;
    sh[c] = a.beta[c] - gmu[g] * s;
  }
  __syncthreads();
  const int nvec = C / 8;
  const int p_begin = blockIdx.x * pix_per_block;
  const int p_end = min(a.HW, p_begin + pix_per_block);
  const size_t total = (size_t)(p_end - p_begin) * nvec;
  for (size_t i = threadIdx.x; i < total; i += blockDim.x) {
    const int pix = p_begin + (int)(i / nvec);
    const int c0 = (int)(i % nvec) * 8;
    int cl;
    const __half* src = gn_src(a, c0, img_base + pix, cl);
    uint4 u = *reinterpret_cast<const uint4*>(src + cl);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __half22float2(h[e]);
      float y0 = f.x * sc[c0 + 2 * e] + sh[c0 + 2 * e];
      float y1 = f.y * sc[c0 + 2 * e + 1] + sh[c0 + 2 * e + 1];
      if (a.silu) { y0 = silu_f(y0); y1 = silu_f(y1); }
      ow[e] = pack_half2(y0, y1);
    }
    *reinterpret_cast<uint4*>(a.y + (img_base + pix) * C + c0) = o;
  }
}

// LayerNorm over C per token: one warp per token, values kept in registers,
// exact centred variance. Replaces layernorm_f32.comp (vk_engine.cpp:652).
template <int VPL>  // 8-channel vectors per lane
__global__ void __launch_bounds__(256) ln_kernel(const __half* __restrict__ x, int M, int C, const float* __restrict__ g,
                                                 const float* __restrict__ b, float eps, __half* __restrict__ y) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= M) return;
  const int nvec = C / 8;
  const __half* xr = x + (size_t)warp * C;
  float v[VPL * 8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      uint4 u = *reinterpret_cast<const uint4*>(xr + vi * 8);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __half22float2(h[e]);
        v[i * 8 + 2 * e] = f.x;
        v[i * 8 + 2 * e + 1] = f.y;
        sum += f.x + f.y;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i * 8 + e] = 0.f;
    }
  }
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mu = sum / C;
  float m2 = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[i * 8 + e] - mu;
        m2 += d * d;
      }
    }
  }
  for (int o = 16; o; o >>= 1) m2 += __shfl_xor_sync(0xffffffffu, m2, o);
  const float rs = rsqrtf(m2 / C + eps);
  __half* yr = y + (size_t)warp * C;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = vi * 8 + 2 * e;
        ow[e] = pack_half2((v[i * 8 + 2 * e] - mu) * rs * g[c] + b[c], (v[i * 8 + 2 * e + 1] - mu) * rs * g[c + 1] + b[c + 1]);
      }
      *reinterpret_cast<uint4*>(yr + vi * 8) = o;
    }
  }
}

}  // namespace

cudaError_t launch_groupnorm(const GroupNormArgs& a, cudaStream_t s) {
  const int C = a.C0 + a.C1;
  if (C <= 0 || C > kGnMaxC || C % 8 || a.C0 % 8 || (a.C1 && a.x1 == nullptr) || a.groups <= 0 || a.groups > 64 ||
      C % a.groups || a.HW <= 0 || a.B <= 0 || !a.stats || !a.y || !a.gamma || !a.beta)
    return cudaErrorInvalidValue;
  // pixel chunk: ~256 KB of input per block, at least 4 pixels, and enough
  // blocks to cover every SM a few times
  const int bytes_per_pix = C * 2;
  int ppb = std::max(4, (256 * 1024) / bytes_per_pix);
  const int want_blocks = num_sms() * 4;
  while (ppb > 4 && (long)a.B * ((a.HW + ppb - 1) / ppb) < want_blocks) ppb /= 2;
  dim3 grid((a.HW + ppb - 1) / ppb, a.B);
  gn_stats_kernel<<<grid, kGnThreads, 0, s>>>(a, ppb);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  gn_apply_kernel<<<grid, kGnThreads, 0, s>>>(a, ppb);
  return cudaGetLastError();
}

cudaError_t launch_layernorm(const __half* x, int M, int C, const float* g, const float* b, float eps, __half* y,
                             cudaStream_t s) {
  if (C % 8 || C > 2048 || M <= 0) return cudaErrorInvalidValue;
  const int nvec = C / 8;
  const int blocks = (M * 32 + 255) / 256;
  if (nvec <= 32) ln_kernel<1><<<blocks, 256, 0, s>>>(x, M, C, g, b, eps, y);
  else if (nvec <= 64) ln_kernel<2><<<blocks, 256, 0, s>>>(x, M, C, g, b, eps, y);
  else if (nvec <= 128) ln_kernel<4><<<blocks, 256, 0, s>>>(x, M, C, g, b, eps, y);
  else ln_kernel<8><<<blocks, 256, 0, s>>>(x, M, C, g, b, eps, y);
  return cudaGetLastError();
}

}  // namespace sdg
