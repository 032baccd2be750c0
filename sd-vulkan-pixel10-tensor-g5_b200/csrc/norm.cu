// norm.cu — GroupNorm(32)(+SiLU) and LayerNorm for NHWC fp16 activations.
//
// GroupNorm replaces groupnorm_f32.comp / groupnorm_silu.comp
// (vk_engine.cpp:548-549): statistics per (image, group), y = (x-mu)*rstd*g+b,
// optional SiLU. The reference reduces one group per workgroup with
// var = E[x^2] - mu^2 (groupnorm_f32.comp:24-25); here the work is split for
// bandwidth and made exact and deterministic (no atomics):
//   pass 1 (stats):   blocks of (pixel chunk, image); each thread owns one
//                     128-bit vector of 8 channels; two passes over the chunk
//                     (the second hits L1/L2) give per-channel chunk mean and
//                     centred M2, reduced across thread rows in fixed order.
//   pass 2 (combine): one block per (image, group) merges the chunk partials
//                     with Chan's formula M2 = sum M2_i + n_i (mu_i - mu)^2
//                     (all terms non-negative: no cancellation).
//   pass 3 (apply):   128-bit loads/stores, per-channel scale/shift, SiLU.
// The chunking depends only on (HW, C), never on the batch, so an image's
// result does not depend on what else is in the batch.
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

__device__ __forceinline__ void load8(const __half* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float2 f = __half22float2(h[e]);
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}

// partials layout: [B][nblk][C] float2 (chunk mean, chunk M2)
__global__ void __launch_bounds__(kGnThreads) gn_stats_kernel(GroupNormArgs a, int ppb, float2* __restrict__ part) {
  const int C = a.C0 + a.C1;
  const int nvec = C / 8;
  const int img = blockIdx.y;
  const int nblk = gridDim.x;
  const int p_begin = blockIdx.x * ppb;
  const int p_end = min(a.HW, p_begin + ppb);
  const float n = (float)(p_end - p_begin);
  __shared__ float red[kGnMaxC];   // [rows][C] partial sums, then M2
  __shared__ float mean_s[kGnMaxC];
  const size_t img_base = (size_t)img * a.HW;
  const int rows = nvec <= kGnThreads ? kGnThreads / nvec : 1;
  const int per_pass = nvec <= kGnThreads ? nvec : kGnThreads;
  const int r = threadIdx.x / per_pass;
  for (int v0 = 0; v0 < nvec; v0 += per_pass) {
    const int v = v0 + threadIdx.x % per_pass;
    const bool active = r < rows && v < nvec;
    const int c0 = v * 8;
    float S[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) S[e] = 0.f;
    if (active) {
      for (int pix = p_begin + r; pix < p_end; pix += rows) {
        int cl;
        const __half* src = gn_src(a, c0, img_base + pix, cl);
        float x[8];
        load8(src + cl, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) S[e] += x[e];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) red[r * (per_pass * 8) + (v - v0) * 8 + e] = S[e];
    }
    __syncthreads();
    for (int c = threadIdx.x; c < per_pass * 8 && v0 * 8 + c < C; c += blockDim.x) {
      float t = 0.f;
      for (int rr = 0; rr < rows; ++rr) t += red[rr * (per_pass * 8) + c];
      mean_s[v0 * 8 + c] = t / n;
    }
    __syncthreads();
    float M[8], m[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) { M[e] = 0.f; m[e] = active ? mean_s[c0 + e] : 0.f; }
    if (active) {
      for (int pix = p_begin + r; pix < p_end; pix += rows) {
        int cl;
        const __half* src = gn_src(a, c0, img_base + pix, cl);
        float x[8];
        load8(src + cl, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = x[e] - m[e];
          M[e] += d * d;
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) red[r * (per_pass * 8) + (v - v0) * 8 + e] = M[e];
    }
    __syncthreads();
    float2* dst = part + ((size_t)img * nblk + blockIdx.x) * C;
    for (int c = threadIdx.x; c < per_pass * 8 && v0 * 8 + c < C; c += blockDim.x) {
      float t = 0.f;
      for (int rr = 0; rr < rows; ++rr) t += red[rr * (per_pass * 8) + c];
      dst[v0 * 8 + c] = make_float2(mean_s[v0 * 8 + c], t);
    }
    __syncthreads();
  }
}

// one block per (group, image): Chan merge of (chunk, channel) partials -> (mu, rstd)
__global__ void __launch_bounds__(256) gn_combine_kernel(GroupNormArgs a, int ppb, int nblk,
                                                         const float2* __restrict__ part, float2* __restrict__ gstat) {
  const int C = a.C0 + a.C1;
  const int g = blockIdx.x, img = blockIdx.y;
  const int cpg = C / a.groups;
  const int items = nblk * cpg;
  __shared__ float red[256];
  const float2* base = part + (size_t)img * nblk * C + g * cpg;
  auto n_of = [&](int blk) { return (float)(min(a.HW, (blk + 1) * ppb) - blk * ppb); };
  // mean = sum n_i mu_i / N
  float s = 0.f;
  for (int i = threadIdx.x; i < items; i += blockDim.x) {
    const int blk = i / cpg, j = i % cpg;
    s += n_of(blk) * base[(size_t)blk * C + j].x;
  }
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = 128; o; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  const float N = (float)a.HW * cpg;
  const float mu = red[0] / N;
  __syncthreads();
  float m2 = 0.f;
  for (int i = threadIdx.x; i < items; i += blockDim.x) {
    const int blk = i / cpg, j = i % cpg;
    const float2 pr = base[(size_t)blk * C + j];
    const float d = pr.x - mu;
    m2 += pr.y + n_of(blk) * d * d;
  }
  red[threadIdx.x] = m2;
  __syncthreads();
  for (int o = 128; o; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) gstat[img * a.groups + g] = make_float2(mu, rsqrtf(red[0] / N + a.eps));
}

__global__ void __launch_bounds__(kGnThreads) gn_apply_kernel(GroupNormArgs a, int ppb, const float2* __restrict__ gstat) {
  const int C = a.C0 + a.C1;
  const int cpg = C / a.groups;
  const int img = blockIdx.y;
  __shared__ float sc[kGnMaxC];
  __shared__ float sh[kGnMaxC];
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float2 st = gstat[img * a.groups + c / cpg];
    const float s = st.y * a.gamma[c];
    sc[c] = s;
    sh[c] = a.beta[c] - st.x * s;
  }
  __syncthreads();
  const size_t img_base = (size_t)img * a.HW;
  const int nvec = C / 8;
  const int p_begin = blockIdx.x * ppb;
  const int p_end = min(a.HW, p_begin + ppb);
  const size_t total = (size_t)(p_end - p_begin) * nvec;
  for (size_t i = threadIdx.x; i < total; i += blockDim.x) {
    const int pix = p_begin + (int)(i / nvec);
    const int c0 = (int)(i % nvec) * 8;
    int cl;
    const __half* src = gn_src(a, c0, img_base + pix, cl);
    float x[8];
    load8(src + cl, x);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float y0 = x[2 * e] * sc[c0 + 2 * e] + sh[c0 + 2 * e];
      float y1 = x[2 * e + 1] * sc[c0 + 2 * e + 1] + sh[c0 + 2 * e + 1];
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

// Pixels per GroupNorm chunk: ~16 KB of input per block (second stats pass
// stays in L1). Depends only on (HW, C) so results are batch-invariant.
static int gn_ppb(int HW, int C) { return std::max(1, std::min(HW, (16 * 1024) / (2 * C))); }

size_t groupnorm_scratch_bytes(int B, int HW, int C, int groups) {
  const int ppb = gn_ppb(HW, C);
  const int nblk = (HW + ppb - 1) / ppb;
  return (size_t)B * nblk * C * sizeof(float2) + (size_t)B * groups * sizeof(float2);
}

cudaError_t launch_groupnorm(const GroupNormArgs& a, cudaStream_t s) {
  const int C = a.C0 + a.C1;
  if (C <= 0 || C > kGnMaxC || C % 8 || a.C0 % 8 || (a.C1 && a.x1 == nullptr) || a.groups <= 0 || a.groups > 64 ||
      C % a.groups || a.HW <= 0 || a.B <= 0 || !a.stats || !a.y || !a.gamma || !a.beta)
    return cudaErrorInvalidValue;
  const int ppb = gn_ppb(a.HW, C);
  const int nblk = (a.HW + ppb - 1) / ppb;
  float2* part = reinterpret_cast<float2*>(a.stats);
  float2* gstat = part + (size_t)a.B * nblk * C;
  gn_stats_kernel<<<dim3(nblk, a.B), kGnThreads, 0, s>>>(a, ppb, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  gn_combine_kernel<<<dim3(a.groups, a.B), 256, 0, s>>>(a, ppb, nblk, part, gstat);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  gn_apply_kernel<<<dim3(nblk, a.B), kGnThreads, 0, s>>>(a, ppb, gstat);
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
