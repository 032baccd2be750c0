// norm.cu — GroupNorm(32)(+SiLU) and LayerNorm for NHWC fp16 activations.
//
// GroupNorm replaces groupnorm_f32.comp / groupnorm_silu.comp
// (vk_engine.cpp:548-549): statistics per (image, group), y = (x-mu)*rstd*g+b,
// optional SiLU. The reference reduces one group per workgroup with
// var = E[x^2] - mu^2 (groupnorm_f32.comp:24-25). Here one launch
// (gn_fused_kernel, below) for every shape the UNet has; otherwise two:
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
#include "sdg_launch.h"
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
  pdl_wait();
  pdl_trigger();
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
  pdl_wait();
  pdl_trigger();
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
// launch from the work: ~20 KB of input per CTA) per (channel slice, image).
// Each CTA owns 1/K of the image's pixels for a slice of whole groups; every
// thread owns one 8-channel vector column of it (at most kGnMaxV pixels, all
// loads issued up front and kept in registers: one global read per element).
// The affine parameters do not depend on the previous kernel and are fetched
// before its completion (pdl_wait).
// Statistics in one pass over the registers, as sums of shifted values: every
// group is shifted by one of its own elements (the image's pixel-0 value of
// the group's first channel, the same in every CTA of the cluster), so
// var = S2/n - (S1/n)^2 stays well conditioned whatever the group's mean
// (the shifted-data variance of Chan, Golub and LeVeque). A thread's vector
// spans at most two groups (>= 8 channels per group); its two (S1, S2) pairs
// go through shared memory to one warp per group, which sums them in a fixed
// order and pushes the CTA's pair into slot [rank] of every cluster CTA
// (st.shared::cluster). After one cluster barrier each CTA adds the K slots in
// rank order (deterministic, no atomics) and normalises from registers (fp32
// pairs in f32x2 instructions, rounded to fp16, SiLU on the f16x2 pair: one
// tanh.approx.f16x2 per two values). Rank 0 also records (mean, rstd) per group.
// Clusters of up to 8 CTAs (the portable size) where the shape allows: a
// 16-CTA cluster needs 16 free SMs inside one GPC. 16 (non-portable, opted in
// at launch) only for shapes no smaller cluster can hold.
constexpr int kGnMaxCluster = 16;
constexpr int kGnPreferredCluster = 8;
constexpr int kGnFusedThreads = 256;  // two CTAs per SM
constexpr int kGnMaxV = 16;

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(kGnFusedThreads, 2)
    gn_fused_kernel(GroupNormArgs a, int nslices, float2* __restrict__ gstat) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  // first cluster barrier phase: every CTA of the cluster has started before any CTA stores into its
  // shared memory (the matching wait comes just before the push)
  cluster_arrive_relaxed();
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
  // per thread (r, v), at [v * rows + r]: (S1, S2) of its first / second group
  __shared__ float2 pa[kGnFusedThreads], pb[kGnFusedThreads];
  __shared__ float2 allp[kGnMaxCluster][32];                   // [source rank][group], pushed by the cluster
  __shared__ float gmu[32], grs[32];
  const int t = threadIdx.x;
  const int v = t % nv, r = t / nv;
  const bool active = r < rows;
  const int cl0 = v * 8;             // slice-local first channel of this thread's vector
  const int c0 = cbeg + cl0;
  const int ga = cl0 / cpg;          // slice-local group of channels [0, split) of the vector ...
  const int split = min(8, (ga + 1) * cpg - cl0);  // ... the rest belong to group ga + 1
  const int cnt = (active && p0 + r < p1) ? (p1 - p0 - r + rows - 1) / rows : 0;
  const float inv_n = 1.f / ((float)a.HW * cpg);

  float gam[8], bet[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    gam[e] = active ? a.gamma[c0 + e] : 0.f;
    bet[e] = active ? a.beta[c0 + e] : 0.f;
  }
  pdl_wait();
  pdl_trigger();

  uint4 xs[kGnMaxV];
  int cl;
  const __half* src0 = gn_src(a, c0, img_base + p0 + r, cl);
  const size_t pstride = (size_t)rows * (c0 < a.C0 ? a.C0 : a.C1);  // elements between a thread's pixels
#pragma unroll
  for (int i = 0; i < kGnMaxV; ++i)
    if (i < cnt) xs[i] = *reinterpret_cast<const uint4*>(src0 + cl + i * pstride);
  // the shift of slice-local group gl: pixel 0 of the image, the group's first channel
  auto shift_of = [&](int gl) -> float {
    int c;
    const __half* p = gn_src(a, cbeg + gl * cpg, img_base, c);
    return __half2float(p[c]);
  };
  const float ka = active ? shift_of(ga) : 0.f;
  const float kb = (active && split < 8) ? shift_of(ga + 1) : ka;
  const float kown = t < gps ? shift_of(t) : 0.f;  // merge thread of group t

  // one pass: per-channel sums of shifted values and of their squares (channel pairs in f32x2)
  float2 s1[4], s2[4], kk[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    s1[j] = make_float2(0.f, 0.f);
    s2[j] = make_float2(0.f, 0.f);
    kk[j] = make_float2(2 * j < split ? ka : kb, 2 * j + 1 < split ? ka : kb);
  }
#pragma unroll
  for (int i = 0; i < kGnMaxV; ++i) {
    if (i < cnt) {
      const __half2* h = reinterpret_cast<const __half2*>(&xs[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 d = sub_f32x2(__half22float2(h[j]), kk[j]);
        s1[j] = add_f32x2(s1[j], d);
        s2[j] = fma_f32x2(d, d, s2[j]);
      }
    }
  }
  float2 qa = make_float2(0.f, 0.f), qb = make_float2(0.f, 0.f);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a1 = (e & 1) ? s1[e >> 1].y : s1[e >> 1].x, a2 = (e & 1) ? s2[e >> 1].y : s2[e >> 1].x;
    if (e < split) {
      qa.x += a1;
      qa.y += a2;
    } else {
      qb.x += a1;
      qb.y += a2;
    }
  }
  if (active) {
    pa[v * rows + r] = qa;
    pb[v * rows + r] = qb;
  }
  __syncthreads();
  cluster_wait();  // first phase: the whole cluster is running
  // one warp per group: the group's vector columns [vlo, vhi] (contiguous in pa / pb), strided over
  // the lanes in a fixed order, then a butterfly (every lane ends with the same sum); the CTA's pair is
  // pushed to slot [rank] of every CTA of the cluster. Only column vlo can start in group g - 1 (its
  // second-group sums, pb, belong to g).
  const int w = t >> 5, lane = t & 31;
  for (int g = w; g < gps; g += kGnFusedThreads / 32) {
    const int vlo = (g * cpg) >> 3, vhi = ((g + 1) * cpg - 1) >> 3;
    const int b_end = vlo * 8 < g * cpg ? (vlo + 1) * rows : vlo * rows;
    float S1 = 0.f, S2 = 0.f;
    for (int i = vlo * rows + lane; i < (vhi + 1) * rows; i += 32) {
      const float2 q = i < b_end ? pb[i] : pa[i];
      S1 += q.x;
      S2 += q.y;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      S1 += __shfl_xor_sync(0xffffffffu, S1, o);
      S2 += __shfl_xor_sync(0xffffffffu, S2, o);
    }
    if (lane < kc) *cluster.map_shared_rank(&allp[rank][g], lane) = make_float2(S1, S2);
  }
  cluster_arrive();  // second phase: the pushes are visible to their targets after the wait
  cluster_wait();
  if (t < gps) {
    float S1 = 0.f, S2 = 0.f;
    for (int q = 0; q < kc; ++q) {
      S1 += allp[q][t].x;
      S2 += allp[q][t].y;
    }
    const float m1 = S1 * inv_n;
    const float var = fmaxf(S2 * inv_n - m1 * m1, 0.f);
    const float mu = kown + m1;
    const float rs = rsqrtf(var + a.eps);
    gmu[t] = mu;
    grs[t] = rs;
    if (rank == 0 && gstat) gstat[img * a.groups + slice * gps + t] = make_float2(mu, rs);
  }
  __syncthreads();
  if (cnt > 0) {
    const int gb = split < 8 ? ga + 1 : ga;
    const float mua = gmu[ga], rsa = grs[ga], mub = gmu[gb], rsb = grs[gb];
    float scl[8], shf[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float m = e < split ? mua : mub;
      scl[e] = (e < split ? rsa : rsb) * gam[e];
      shf[e] = bet[e] - m * scl[e];
    }
    float2 scl2[4], shf2[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      scl2[j] = make_float2(scl[2 * j], scl[2 * j + 1]);
      shf2[j] = make_float2(shf[2 * j], shf[2 * j + 1]);
    }
    __half* dst0 = a.y + (img_base + p0 + r) * C + c0;
    // normalise in fp32 (f32x2), round to fp16, SiLU on the f16x2 pair
#pragma unroll
    for (int i = 0; i < kGnMaxV; ++i) {
      if (i < cnt) {
        const __half2* h = reinterpret_cast<const __half2*>(&xs[i]);
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 y = fma_f32x2(__half22float2(h[j]), scl2[j], shf2[j]);
          const uint32_t p = pack_half2(y.x, y.y);
          ow[j] = a.silu ? silu_h2(p) : p;
        }
        *reinterpret_cast<uint4*>(dst0 + (size_t)i * rows * C) = o;
      }
    }
  }
}

// Cluster size for a (slice, image): ~20 KB of input per CTA, at most `maxc`,
// and large enough that each thread's share of the chunk fits kGnMaxV vectors.
int gn_cluster_ctas(int HW, int Ws, int maxc = kGnPreferredCluster) {
  const int rows = kGnFusedThreads / (Ws / 8);
  const long bytes = (long)HW * Ws * 2;
  int k = (int)std::min<long>(maxc, std::max<long>(1, (bytes + 20479) / 20480));
  int pow2 = 1;
  while (pow2 < k) pow2 *= 2;
  k = pow2;
  while (k <= maxc && ((HW + k - 1) / k + rows - 1) / rows > kGnMaxV) k *= 2;
  return k <= maxc ? k : 0;
}

// Slice count (dividing the group count; whole groups and whole 8-channel
// vectors per slice) for the fused kernel: the one giving the most CTAs per
// image up to ~72 (so a batch of 2 stays within one wave of 148 SMs), among
// slices of at least 40 channels when any fits; 0 if none fits or a group has
// fewer than 8 channels (an 8-channel vector would span more than two groups).
int gn_fused_slices(int C, int groups, int HW, int maxc = kGnPreferredCluster) {
  int best = 0, best_ctas = 0;
  bool best_wide = false;
  for (int ns = 1; ns <= groups; ns *= 2) {
    if (groups % ns || C % ns) continue;
    const int Ws = C / ns;
    if (Ws % 8 || Ws > 256 || (Ws % (C / groups)) || Ws / (C / groups) > 32 || C / groups < 8) continue;
    const int k = gn_cluster_ctas(HW, Ws, maxc);
    if (k == 0) continue;
    const int ctas = ns * k;
    const bool wide = Ws >= 40;
    if (best == 0 || (wide && !best_wide) ||
        (wide == best_wide && ((ctas <= 72 && ctas > best_ctas) || (best_ctas > 72 && ctas < best_ctas)))) {
      best = ns;
      best_ctas = ctas;
      best_wide = wide;
    }
  }
  if (best == 0 && maxc < kGnMaxCluster) return gn_fused_slices(C, groups, HW, kGnMaxCluster);
  return best;
}

// Cluster size used with gn_fused_slices' choice.
int gn_fused_cluster(int C, int groups, int HW, int ns) {
  const int k = gn_cluster_ctas(HW, C / ns, kGnPreferredCluster);
  if (k && gn_fused_slices(C, groups, HW, kGnPreferredCluster) == ns) return k;
  return gn_cluster_ctas(HW, C / ns, kGnMaxCluster);
}

// LayerNorm over C per token: one warp per token, values kept in registers,
// exact centred variance. Replaces layernorm_f32.comp (vk_engine.cpp:652).
// Up to five vectors per lane (C <= 1280) the lane's affine parameters are
// fetched into registers before the programmatic-launch wait (they do not
// depend on the previous kernel), off the normalisation's critical path.
template <int VPL>  // 8-channel vectors per lane
__global__ void __launch_bounds__(256) ln_kernel(const __half* __restrict__ x, int M, int C, const float* __restrict__ g,
                                                 const float* __restrict__ b, float eps, __half* __restrict__ y) {
  constexpr bool kPre = VPL <= 5;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = C / 8;
  float4 gpre[kPre ? VPL * 2 : 1], bpre[kPre ? VPL * 2 : 1];
  if constexpr (kPre) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) {
        const float4* g4 = reinterpret_cast<const float4*>(g + vi * 8);
        const float4* b4 = reinterpret_cast<const float4*>(b + vi * 8);
        gpre[2 * i] = __ldg(g4);
        gpre[2 * i + 1] = __ldg(g4 + 1);
        bpre[2 * i] = __ldg(b4);
        bpre[2 * i + 1] = __ldg(b4 + 1);
      }
    }
  }
  pdl_wait();
  pdl_trigger();
  if (warp >= M) return;
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
      float4 ga, gb, ba, bb;
      if constexpr (kPre) {
        ga = gpre[2 * i];
        gb = gpre[2 * i + 1];
        ba = bpre[2 * i];
        bb = bpre[2 * i + 1];
      } else {
        const float4* g4 = reinterpret_cast<const float4*>(g + vi * 8);
        const float4* b4 = reinterpret_cast<const float4*>(b + vi * 8);
        ga = __ldg(g4);
        gb = __ldg(g4 + 1);
        ba = __ldg(b4);
        bb = __ldg(b4 + 1);
      }
      const float gg[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
      const float bt[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        ow[e] = pack_half2((v[i * 8 + 2 * e] - mu) * rs * gg[2 * e] + bt[2 * e],
                           (v[i * 8 + 2 * e + 1] - mu) * rs * gg[2 * e + 1] + bt[2 * e + 1]);
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
    const int kc = gn_fused_cluster(C, a.groups, a.HW, ns);
    return launch_kernel(gn_fused_kernel, dim3(ns * kc, a.B), dim3(kGnFusedThreads), 0, s, kc, a, ns, gstat);
  }
  cudaError_t e = launch_kernel(gn_stats_kernel, dim3(a.groups, a.B), dim3(kGnStatThreads), 0, s, 0, a, gstat);
  if (e != cudaSuccess) return e;
  const int ppb = gn_ppb(a.HW, C);
  const int nblk = (a.HW + ppb - 1) / ppb;
  return launch_kernel(gn_apply_kernel, dim3(nblk, a.B), dim3(kGnThreads), 0, s, 0, a, ppb,
                       (const float2*)gstat);
}

cudaError_t launch_layernorm(const __half* x, int M, int C, const float* g, const float* b, float eps, __half* y,
                             cudaStream_t s) {
  if (C % 8 || C > 2048 || M <= 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(b)) & 15) return cudaErrorInvalidValue;
  const int nvec = C / 8;
  const int blocks = (M * 32 + 255) / 256;
  auto k = nvec <= 32    ? ln_kernel<1>
           : nvec <= 64  ? ln_kernel<2>
           : nvec <= 96  ? ln_kernel<3>
           : nvec <= 160 ? ln_kernel<5>
                         : ln_kernel<8>;
  return launch_kernel(k, dim3(blocks), dim3(256), 0, s, 0, x, M, C, g, b, eps, y);
}

}  // namespace sdg
