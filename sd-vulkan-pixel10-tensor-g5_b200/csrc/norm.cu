// norm.cu — GroupNorm(32)(+SiLU) and LayerNorm for NHWC fp16 activations.
//
// GroupNorm replaces groupnorm_f32.comp / groupnorm_silu.comp
// (vk_engine.cpp:548-549): statistics per (image, group), y = (x-mu)*rstd*g+b,
// optional SiLU. The reference reduces one group per workgroup with
// var = E[x^2] - mu^2 (groupnorm_f32.comp:24-25). Here:
//   kernel 1 (stats): one block per (group, image), exact two-pass mean and
//                     centred variance over the group's elements read
//                     straight from L2 (the producer just wrote them), fixed
//                     reduction order -> deterministic, no atomics;
//   kernel 2 (apply): 128-bit loads/stores over pixel chunks, per-channel
//                     scale/shift from the group stats, optional SiLU.
// The input may be a channel concat [x0 ; x1] (up-block skip connections),
// read in place from both sources. An image's result never depends on the
// rest of the batch.
#include <cooperative_groups.h>

#include <algorithm>

#include "sdg_kernels.h"
#include "sdg_ptx.cuh"

namespace sdg {
namespace {

constexpr int kGnThreads = 256;
constexpr int kGnStatThreads = 512;
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

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  t = red[32];
  __syncthreads();
  return t;
}

// one block per (group, image): exact mean / centred variance -> (mu, rstd)
__global__ void __launch_bounds__(kGnStatThreads) gn_stats_kernel(GroupNormArgs a, float2* __restrict__ gstat) {
  __shared__ float red[40];
  const int C = a.C0 + a.C1;
  const int g = blockIdx.x, img = blockIdx.y;
  const int cpg = C / a.groups;
  const int pairs = cpg / 2;  // half2 per pixel of this group (C0 and cpg are even)
  const int n_items = a.HW * pairs;
  const size_t img_base = (size_t)img * a.HW;
  auto item = [&](int i) -> float2 {
    const int pix = i / pairs, j = i - (i / pairs) * pairs;
    int cl;
    const __half* src = gn_src(a, g * cpg + 2 * j, img_base + pix, cl);
    return __half22float2(*reinterpret_cast<const __half2*>(src + cl));
  };
  float s = 0.f;
  for (int i = threadIdx.x; i < n_items; i += blockDim.x) {
    const float2 f = item(i);
    s += f.x + f.y;
  }
  const float N = (float)a.HW * cpg;
  const float mu = block_sum(s, red) / N;
  float m2 = 0.f;
  for (int i = threadIdx.x; i < n_items; i += blockDim.x) {
    const float2 f = item(i);
    const float d0 = f.x - mu, d1 = f.y - mu;
    m2 += d0 * d0 + d1 * d1;
  }
  const float var = block_sum(m2, red) / N;
  if (threadIdx.x == 0) gstat[img * a.groups + g] = make_float2(mu, rsqrtf(var + a.eps));
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

// Fused single-launch GroupNorm: a cluster of K CTAs (K = 1..16, chosen per
// launch from the work: ~40 KB of input per CTA) per (channel slice, image).
// Each CTA owns 1/K of the image's pixels for a slice of whole groups. Every
// thread issues all loads of its share of the chunk up front (at most kGnMaxV
// 16-byte vectors, kept in registers: high memory-level parallelism, one
// global read per element). Group sums (pass 1, mean) and centred sums of
// squares (pass 2, variance) are exchanged through distributed shared memory
// and summed in rank order (deterministic, exact two-pass); pass 3 normalises
// from registers. Rank 0 also records (mean, rstd) per group.
constexpr int kGnMaxCluster = 16;  // non-portable size, opted in at launch
constexpr int kGnFusedThreads = 512;
constexpr int kGnMaxV = 8;

__global__ void __launch_bounds__(kGnFusedThreads)
    gn_fused_kernel(GroupNormArgs a, int nslices, float2* __restrict__ gstat) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int kc = (int)cluster.num_blocks();
  const int slice = blockIdx.x / kc;
  const int img = blockIdx.y;
  const int C = a.C0 + a.C1;
  const int cpg = C / a.groups;
  const int Ws = C / nslices;        // channels of this slice (whole groups, multiple of 8)
  const int gps = Ws / cpg;          // groups in the slice
  const int cbeg = slice * Ws;
  const int nv = Ws / 8;
  const int rows = kGnFusedThreads / nv;
  const int chunk = (a.HW + kc - 1) / kc;
  const int p0 = rank * chunk, p1 = min(a.HW, p0 + chunk);
  const size_t img_base = (size_t)img * a.HW;
  __shared__ float red[4096];        // [rows][Ws] per-channel partials (rows * Ws <= 4096)
  __shared__ float red2[kGnFusedThreads];  // [row slice][Ws] (slices * Ws <= threads)
  __shared__ float chan[320];        // per-channel CTA sums
  __shared__ float part[2][32];      // per-group partials of this CTA, read by the whole cluster
  __shared__ float gmu[32], grs[32];
  __shared__ float sc[320], sh[320];
  const int t = threadIdx.x;
  const int v = t % nv, r = t / nv;
  const bool active = r < rows;
  const int c0 = cbeg + v * 8;       // first channel of this thread's vector
  const int cnt = (active && p0 + r < p1) ? (p1 - p0 - r + rows - 1) / rows : 0;
  const float N = (float)a.HW * cpg;

  uint4 xs[kGnMaxV];
  int cl;
  const __half* src0 = gn_src(a, c0, img_base + p0 + r, cl);
  const size_t pstride = (size_t)rows * (c0 < a.C0 ? a.C0 : a.C1);  // elements between a thread's pixels
#pragma unroll
  for (int i = 0; i < kGnMaxV; ++i)
    if (i < cnt) xs[i] = *reinterpret_cast<const uint4*>(src0 + cl + i * pstride);

  auto unpack = [](const uint4& u, float (&x)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __half22float2(h[e]);
      x[2 * e] = f.x;
      x[2 * e + 1] = f.y;
    }
  };
  auto reduce_to_groups = [&](const float (&acc)[8], int which) {
    if (active) {
#pragma unroll
      for (int e = 0; e < 8; ++e) red[r * Ws + v * 8 + e] = acc[e];
    }
    __syncthreads();
    // rows -> row slices (all threads), slices -> channels, channels -> groups (a warp per group);
    // every sum in a fixed order (deterministic)
    const int nslc = kGnFusedThreads / Ws;
    if (t < nslc * Ws) {
      const int c = t % Ws, rs = t / Ws;
      float s = 0.f;
      for (int rr = rs; rr < rows; rr += nslc) s += red[rr * Ws + c];
      red2[rs * Ws + c] = s;
    }
    __syncthreads();
    if (t < Ws) {
      float s = 0.f;
      for (int rs = 0; rs < nslc; ++rs) s += red2[rs * Ws + t];
      chan[t] = s;
    }
    __syncthreads();
    for (int g = t >> 5; g < gps; g += kGnFusedThreads / 32) {
      float s = 0.f;
      for (int j = (t & 31); j < cpg; j += 32) s += chan[g * cpg + j];
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if ((t & 31) == 0) part[which][g] = s;
    }
    cluster.sync();
    if (t < gps) {
      float s = 0.f;
      for (int q = 0; q < kc; ++q) s += cluster.map_shared_rank(&part[which][0], q)[t];
      if (which == 0) gmu[t] = s / N;
      else grs[t] = rsqrtf(s / N + a.eps);
    }
    __syncthreads();
  };

  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
  for (int i = 0; i < kGnMaxV; ++i) {
    if (i < cnt) {
      float x[8];
      unpack(xs[i], x);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += x[e];
    }
  }
  reduce_to_groups(acc, 0);
  float mu[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) { acc[e] = 0.f; mu[e] = active ? gmu[(v * 8 + e) / cpg] : 0.f; }
#pragma unroll
  for (int i = 0; i < kGnMaxV; ++i) {
    if (i < cnt) {
      float x[8];
      unpack(xs[i], x);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = x[e] - mu[e];
        acc[e] += d * d;
      }
    }
  }
  reduce_to_groups(acc, 1);
  if (rank == 0 && t < gps && gstat) gstat[img * a.groups + slice * gps + t] = make_float2(gmu[t], grs[t]);
  for (int c = t; c < Ws; c += blockDim.x) {
    const int g = c / cpg;
    const float s = grs[g] * a.gamma[cbeg + c];
    sc[c] = s;
    sh[c] = a.beta[cbeg + c] - gmu[g] * s;
  }
  __syncthreads();
  if (active) {
    float scl[8], shf[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) { scl[e] = sc[v * 8 + e]; shf[e] = sh[v * 8 + e]; }
    __half* dst0 = a.y + (img_base + p0 + r) * C + c0;
#pragma unroll
    for (int i = 0; i < kGnMaxV; ++i) {
      if (i < cnt) {
        float x[8];
        unpack(xs[i], x);
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float y0 = x[2 * e] * scl[2 * e] + shf[2 * e];
          float y1 = x[2 * e + 1] * scl[2 * e + 1] + shf[2 * e + 1];
          if (a.silu) { y0 = silu_f(y0); y1 = silu_f(y1); }
          ow[e] = pack_half2(y0, y1);
        }
        *reinterpret_cast<uint4*>(dst0 + (size_t)i * rows * C) = o;
      }
    }
  }
  cluster.sync();  // no CTA leaves while another may still read its `part`
}

// Cluster size for a (slice, image): ~40 KB of input per CTA, at most 16, and
// small enough that each thread's share of the chunk fits kGnMaxV vectors.
int gn_cluster_ctas(int HW, int Ws) {
  const int rows = kGnFusedThreads / (Ws / 8);
  const long bytes = (long)HW * Ws * 2;
  int k = (int)std::min<long>(kGnMaxCluster, std::max<long>(1, (bytes + 40959) / 40960));
  int pow2 = 1;
  while (pow2 < k) pow2 *= 2;
  k = pow2;
  while (k <= kGnMaxCluster && ((HW + k - 1) / k + rows - 1) / rows > kGnMaxV) k *= 2;
  return k <= kGnMaxCluster ? k : 0;
}

// Largest slice count (dividing the group count) whose slice keeps whole
// 8-channel vectors and at least 64 channels per pixel row and fits a cluster;
// 0 if none fits.
int gn_fused_slices(int C, int groups, int HW) {
  int best = 0;
  for (int ns = 1; ns <= groups; ns *= 2) {
    if (groups % ns || C % ns) continue;
    const int Ws = C / ns;
    if (Ws % 8 || Ws > 320 || (Ws % (C / groups)) || Ws / (C / groups) > 32) continue;
    if (gn_cluster_ctas(HW, Ws) == 0) continue;
    if (Ws >= 64 || best == 0) best = ns;
  }
  return best;
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

// Pixels per apply block: ~32 KB of input, depends only on (HW, C).
static int gn_ppb(int HW, int C) { return std::max(1, std::min(HW, (32 * 1024) / (2 * C))); }

size_t groupnorm_scratch_bytes(int B, int HW, int C, int groups) {
  (void)HW;
  (void)C;
  return (size_t)B * groups * sizeof(float2);
}

int groupnorm_launch_count(const GroupNormArgs& a) {
  return (a.groups <= 32 && gn_fused_slices(a.C0 + a.C1, a.groups, a.HW) > 0) ? 1 : 2;
}

cudaError_t launch_groupnorm(const GroupNormArgs& a, cudaStream_t s) {
  const int C = a.C0 + a.C1;
  if (C <= 0 || C > kGnMaxC || C % 8 || a.C0 % 8 || (a.C1 && a.x1 == nullptr) || a.groups <= 0 || a.groups > 64 ||
      C % a.groups || (C / a.groups) % 2 || a.HW <= 0 || a.B <= 0 || !a.stats || !a.y || !a.gamma || !a.beta)
    return cudaErrorInvalidValue;
  float2* gstat = reinterpret_cast<float2*>(a.stats);
  const int ns = a.groups <= 32 ? gn_fused_slices(C, a.groups, a.HW) : 0;
  static bool cluster_ok[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (ns > 0 && dev < 64 && !cluster_ok[dev]) {
    if (cudaFuncSetAttribute(gn_fused_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
      return cudaErrorInvalidValue;
    cluster_ok[dev] = true;
  }
  if (ns > 0) {
    const int kc = gn_cluster_ctas(a.HW, C / ns);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ns * kc, a.B);
    cfg.blockDim = dim3(kGnFusedThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kc;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gn_fused_kernel, a, ns, gstat);
  }
  gn_stats_kernel<<<dim3(a.groups, a.B), kGnStatThreads, 0, s>>>(a, gstat);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int ppb = gn_ppb(a.HW, C);
  const int nblk = (a.HW + ppb - 1) / ppb;
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
