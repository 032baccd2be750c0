// gemm_tc.cu — tcgen05 GEMM / implicit-GEMM 3x3 convolution for sm_100a.
//
// Replaces the reference's conv/matmul family (vk_engine.cpp:578-613;
// matmul_f32.comp, im2col_f32.comp, winograd_*.comp, addbias*_f32.comp,
// add_f32.comp, geglu_f32.comp) with one persistent, warp-specialised kernel:
//   warp 0      TMA producer: A tile 128x64 + W tile BNx64 per k-block (SW128);
//               a pipeline stage holds one or two k-blocks
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128,K=16)
//   warps 2..9  epilogue (two warps per TMEM lane quadrant): tcgen05.ld rows
//               from TMEM, fused bias / per-image bias / residual / SiLU /
//               GEGLU / head scatter, fp16 stores
// Accumulators are double-buffered in TMEM so the epilogue of tile i overlaps
// the main loop of tile i+1. No TMA load uses multicast (the only
// .multicast::cluster is the tcgen05.commit that signals an mbarrier in both
// CTAs of a pair). A CTA pair (cluster of 2, tcgen05.mma.cta_group::2)
// computes 256-row tiles.
//
// Weight-only int8 (wo8): W arrives as int8 by TMA into a staging tile;
// 4 converter warps (warps 6..9, leaving warps 2..5 to the epilogue) rewrite
// it as fp16 (exact) in the swizzled B layout while the MMA runs, and the
// per-output-channel scale is applied in the epilogue (sum_k a*(q*s) = s * sum_k a*q).
//
// Split-K (deep UNet levels, small M): the K range is divided either among the
// 2..8 CTAs of a cluster working on one tile, whose fp32 partial rows are summed
// through distributed shared memory, or among independent CTAs writing fp32
// partials to a workspace that a reduce kernel sums. Both sum in a fixed order
// and apply the same fused epilogue, so results are deterministic.
#include <algorithm>
#include <cmath>
#include <cstdio>

#include <cooperative_groups.h>

#include "sdg_kernels.h"
#include "sdg_launch.h"
#include "sdg_ptx.cuh"
#include "sdg_tma.h"

namespace sdg {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
// cluster K split: up to 10 CTAs (a non-portable cluster size above 8). Measured on B200 for the 8x8-level
// 128 x 1280 x 11520 conv: 16.4 us with a 14-way workspace split, 14.35 / 13.9 / 13.5 us over clusters of
// 8 / 9 / 10 CTAs, 24 us and more over clusters of 12 to 16 (too few of them co-resident)
constexpr int kMaxCsplitCtas = 10;
// epilogue kinds of the kernel instantiations (gemm_tc_kernel's EK)
constexpr int kEkGeneric = 0, kEkPlain = 1, kEkHeads = 3;
// Epilogue warps: two per TMEM lane quadrant (10 warps in all: at most three per SM sub-partition,
// 168 registers a thread); wo8 four epilogue and four int8 converter warps. (Three per quadrant, 14
// warps at 128 registers, measured no faster on B200.)
constexpr int gemm_epi_warps(bool w8, int ek) { return (void)ek, w8 ? 4 : 8; }
constexpr int gemm_threads(bool w8, int ek) { return 64 + 32 * (gemm_epi_warps(w8, ek) + (w8 ? 4 : 0)); }
constexpr uint32_t kATileBytes = BM * BK * 2;  // 16 KB

struct GemmDev {
  int M, N, K;
  int taps, cin0, cin1;
  int H, W;                // conv geometry (input image)
  int cs;                  // conv stride (1 or 2): output Ho = H / cs, Wo = W / cs
  int up_w, up_co;         // taps == 4 (upsample conv): input width, output channels per phase; else 0
  int epi, act;
  const float* bias;
  const float* rowbias;
  int rowbias_ld;
  int rows_per_image;
  const __half* residual;
  int ld_res;
  __half* out;
  int ld_out;
  float* out_f32;
  __half* head_out0;
  __half* head_out1;
  __half* head_out2;
  int head_C, heads, head_d, head_dp;
  int head_vt, head_d16, head_spad;
  int splits, kb_per_split;  // split-K
  int csplit;                // > 1: K split over the CTAs of a cluster, reduced through DSMEM
  float* ws;                 // [splits][M][N] fp32 partials when splits > 1
  const float* wscale;       // wo8: per-output-channel weight scale [N]
  int* err;
  // LayerNorm folded into the GEMMs around it. Producer (plain single-pass epilogue): per output row,
  // each epilogue warp's (sum, sum of squares) over its column chunks of the tile goes to
  // stat_out[m * stat_ld + kSplit * n_blk + warp half]. Consumer (attention-head epilogue): A is the raw
  // row x, W already carries gamma; per row mean / rstd come from the stat_parts partials at
  // stat_in[m * stat_parts ..], and the epilogue computes rstd * (acc - mean * colsum[n]) + bias[n]
  // (bias = b + W beta).
  float2* stat_out;
  int stat_ld;
  const float2* stat_in;
  int stat_parts;
  float ln_inv_c, ln_eps;
  const float* colsum;
  int stall_it;              // failure-path test: k-block iteration whose stage is never loaded (-1: none)
  unsigned long long wait_ns;  // limit of every bounded wait
};

// PAIR: a CTA pair (cluster of 2) computes a 256 x BN tile with
// tcgen05.mma.cta_group::2: each CTA loads its own 128 A rows and half of the
// BN W rows, the even CTA issues the MMAs, and each CTA's TMEM receives its
// 128 rows of the accumulator. Per CTA this halves the W bytes moved per MMA.
template <int BN, bool W8, bool PAIR = false>
struct Cfg {
  static_assert(!(W8 && PAIR), "weight-only int8 tiles use single-CTA kernels");
  // warps: 0 TMA, 1 MMA, then 8 epilogue warps (two per TMEM lane quadrant, alternating
  // column chunks), or for wo8 4 epilogue warps + 4 int8 converter warps
  static constexpr int kThreads = gemm_threads(W8, kEkGeneric);  // of the generic instantiation
  static constexpr int kEpiWarps = gemm_epi_warps(W8, kEkGeneric);
  static constexpr int kBRows = PAIR ? BN / 2 : BN;  // W rows held by this CTA
  static constexpr uint32_t kBTileBytes = kBRows * BK * 2;
  static constexpr uint32_t kB8Bytes = W8 ? BN * BK : 0;  // int8 staging tile
  static constexpr uint32_t kSubBytes = kATileBytes + kBTileBytes + kB8Bytes;  // one 64-deep k-block
  // bytes TMA delivers per k-block (PAIR: counted on the even CTA's barrier for both CTAs)
  static constexpr uint32_t kTxBytes =
      PAIR ? 2 * (kATileBytes + kBTileBytes) : kATileBytes + (W8 ? kB8Bytes : kBTileBytes);
  // k-blocks per pipeline stage. Every mbarrier wait in the MMA-issuing thread leaves the tensor
  // pipe a bubble (measured on B200: a 64-deep stage costs >= ~500 cycles with a wait per stage,
  // ~340 per k-block with one wait per two k-blocks, against 256/320 cycles of MMA work at
  // N = 128/160), so a stage holds two k-blocks (8 MMAs per wait) wherever three such stages
  // fit in shared memory.
  static constexpr int kG = (!W8 && (232448 - 1024 - 512) / (2 * kSubBytes) >= 3) ? 2 : 1;
  static constexpr uint32_t kStageBytes = kG * kSubBytes;
  // as many stages as shared memory holds: TMA latency from L2 needs deep pipelines
  static constexpr int kStages = (232448 - 1024 - 512) / kStageBytes > 12 ? 12 : (232448 - 1024 - 512) / kStageBytes;
  static constexpr int kAccStride = BN <= 16 ? 16 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
  static constexpr uint32_t kTmemCols = (2 * kAccStride) < 32 ? 32 : 2 * kAccStride;
  static constexpr int kChunk = BN >= 32 ? 32 : 16;
  static constexpr size_t kSmem = 1024 + (size_t)kStages * kStageBytes + 512;  // tail: barriers + TMEM slot
  static_assert(kSmem <= 232448, "GEMM tile configuration exceeds 227 KB of shared memory");
};

__device__ __forceinline__ void load8h(const __half* src, float (&v)[8]) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float2 f = __half22float2(h[e]);
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 u;
  u.x = pack_half2(v[0], v[1]);
  u.y = pack_half2(v[2], v[3]);
  u.z = pack_half2(v[4], v[5]);
  u.w = pack_half2(v[6], v[7]);
  return u;
}

__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// Pull the lines the epilogue will read for columns [n, n+CH) of row m into L1 ahead of use.
template <int CH>
__device__ __forceinline__ void epi_prefetch(const GemmDev& p, int m, int img, int n, bool mvalid) {
  if (n >= p.N) return;
  if (p.bias) prefetch_l1(p.bias + n);
  if (p.rowbias && mvalid) prefetch_l1(p.rowbias + (size_t)img * p.rowbias_ld + n);
  if (p.residual && mvalid) prefetch_l1(p.residual + (size_t)m * p.ld_res + n);
  (void)CH;
}

__device__ __forceinline__ void add8_f32(const float* src, float (&v)[8]) {  // src 16-byte aligned
  const float4 a = __ldg(reinterpret_cast<const float4*>(src));
  const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
  v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
  v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
}

// Address of output element (m, n) of a plain fp16 output. For the taps == 4 upsample convolution,
// GEMM row m is input pixel (I, j) (I = m / W counting rows of all images, j = m % W) and column n is
// channel c of phase ph = 2 py + px (n = ph * up_co + c); it lands on output pixel (2I + py, 2j + px)
// of the NHWC output (rows of 2W pixels, all images stacked), i.e. output row 2 m + 2 W I + 2 W py + px.
__device__ __forceinline__ __half* out_at(const GemmDev& p, int m, int n) {
  if (p.up_w) {
    const int ph = n / p.up_co;
    const int orow = 2 * m + 2 * p.up_w * (m / p.up_w + (ph >> 1)) + (ph & 1);
    return p.out + (size_t)orow * p.ld_out + (n - ph * p.up_co);
  }
  return p.out + (size_t)m * p.ld_out + n;
}

// Fused epilogue for 8 consecutive output columns [n, n+8) of row m (m < M) of
// image img = m / rows_per_image. Not used for GEGLU (which pairs two column ranges).
__device__ __forceinline__ void epilogue8(const GemmDev& p, int m, int img, int n, float (&v)[8]) {
  if (p.wscale) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] *= __ldg(p.wscale + min(n + j, p.N - 1));
  }
  if (p.epi == kEpiNchwF32) {
    const int pix = m - img * p.rows_per_image;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (n + j < p.N)
        p.out_f32[((size_t)img * p.N + n + j) * p.rows_per_image + pix] = v[j] + (p.bias ? __ldg(p.bias + n + j) : 0.f);
    return;
  }
  if (p.bias) add8_f32(p.bias + n, v);
  if (p.rowbias) add8_f32(p.rowbias + (size_t)img * p.rowbias_ld + n, v);
  if (p.residual) {
    float rv[8];
    load8h(p.residual + (size_t)m * p.ld_res + n, rv);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] += rv[j];
  }
  if (p.act == 1) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = silu_f(v[j]);
  }
  if (p.epi == kEpiHeads) {
    const int s_idx = m - img * p.rows_per_image;
    const int which = n / p.head_C;
    const int cc = n - which * p.head_C;
    const int h = cc / p.head_d;
    const int jj = cc - h * p.head_d;
    __half* base = which == 0 ? p.head_out0 : (which == 1 ? p.head_out1 : p.head_out2);
    if (which == p.head_vt) {
      // transposed V: [BH, d16, spad]; consecutive rows of a warp are consecutive keys
      __half* dst = base + (((size_t)img * p.heads + h) * p.head_d16 + jj) * p.head_spad + s_idx;
#pragma unroll
      for (int e = 0; e < 8; ++e) dst[(size_t)e * p.head_spad] = __float2half_rn(v[e]);
      return;
    }
    __half* dst = base + (((size_t)img * p.heads + h) * p.rows_per_image + s_idx) * p.head_dp + jj;
    *reinterpret_cast<uint4*>(dst) = pack8(v);
    return;
  }
  *reinterpret_cast<uint4*>(out_at(p, m, n)) = pack8(v);
}

// Epilogue operands of one CH-column chunk of row m, fetched before the accumulator is read so
// the global-load latencies overlap each other and the TMEM load (loading them per 8-column
// group, after each group's store, serialises one L2 round trip per group).
template <int CH>
struct EpiIn {
  float4 b[CH / 4];   // bias + per-image row bias
  uint4 res[CH / 8];  // residual (fp16)
};

// Residual of one CH-column chunk of row m (zero where absent): issued a chunk ahead of its use,
// and for a tile's first chunk before the accumulator wait, so its L2 latency overlaps the main
// loop or the previous chunk instead of adding to each chunk.
template <int CH>
__device__ __forceinline__ void res_load(const GemmDev& p, int m, int n, bool mvalid, uint4 (&res)[CH / 8]) {
#pragma unroll
  for (int g = 0; g < CH / 8; ++g)
    res[g] = (mvalid && p.residual && n + 8 * g < p.N)
                 ? __ldg(reinterpret_cast<const uint4*>(p.residual + (size_t)m * p.ld_res + n) + g)
                 : make_uint4(0u, 0u, 0u, 0u);
}

// Bias and per-image row bias of one chunk (the residual comes from res_load).
template <int CH>
__device__ __forceinline__ void epi_load(const GemmDev& p, int m, int img, int n, bool mvalid, EpiIn<CH>& in) {
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int q = 0; q < CH / 4; ++q) {
    const bool ok = n + 4 * q < p.N;
    in.b[q] = (ok && p.bias) ? __ldg(reinterpret_cast<const float4*>(p.bias + n) + q) : z;
  }
  if (p.rowbias) {  // resnet conv1: the time-embedding projection per image
    const int im = mvalid ? img : 0;  // rows past M (last partial tile) must not index past the last image
#pragma unroll
    for (int q = 0; q < CH / 4; ++q) {
      if (n + 4 * q >= p.N) break;
      const float4 t = __ldg(reinterpret_cast<const float4*>(p.rowbias + (size_t)im * p.rowbias_ld + n) + q);
      in.b[q].x += t.x; in.b[q].y += t.y; in.b[q].z += t.z; in.b[q].w += t.w;
    }
  }
  (void)m;
}

// Fused epilogue of one chunk (plain or attention-head outputs) from the accumulator words r and
// the prefetched operands; same arithmetic as epilogue8.
template <int CH>
__device__ __forceinline__ void epi_apply(const GemmDev& p, int m, int img, int n, const uint32_t* r, const EpiIn<CH>& in) {
#pragma unroll
  for (int g = 0; g < CH / 8; ++g) {
    const int ng = n + g * 8;
    if (ng >= p.N) break;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[g * 8 + j]);
    if (p.wscale) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] *= __ldg(p.wscale + min(ng + j, p.N - 1));
    }
    const float4 b0 = in.b[2 * g], b1 = in.b[2 * g + 1];
    v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
    v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
    if (p.residual) {
      const __half2* h = reinterpret_cast<const __half2*>(&in.res[g]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h[e]);
        v[2 * e] += f.x;
        v[2 * e + 1] += f.y;
      }
    }
    if (p.act == 1) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = silu_f(v[j]);
    }
    if (p.epi == kEpiHeads) {
      const int s_idx = m - img * p.rows_per_image;
      const int which = ng / p.head_C;
      const int cc = ng - which * p.head_C;
      const int h = cc / p.head_d;
      const int jj = cc - h * p.head_d;
      __half* base = which == 0 ? p.head_out0 : (which == 1 ? p.head_out1 : p.head_out2);
      if (which == p.head_vt) {
        __half* dst = base + (((size_t)img * p.heads + h) * p.head_d16 + jj) * p.head_spad + s_idx;
#pragma unroll
        for (int e = 0; e < 8; ++e) dst[(size_t)e * p.head_spad] = __float2half_rn(v[e]);
        continue;
      }
      __half* dst = base + (((size_t)img * p.heads + h) * p.rows_per_image + s_idx) * p.head_dp + jj;
      *reinterpret_cast<uint4*>(dst) = pack8(v);
      continue;
    }
    *reinterpret_cast<uint4*>(out_at(p, m, ng)) = pack8(v);
  }
}

// 4x4 transpose of 16-byte blocks within each quad of lanes: on return, lane 4g + j holds in b[i]
// what lane 4g + i held in b[j]. Two pairwise exchanges (lane ^ 1, then lane ^ 2), each swapping the
// two blocks whose index bit differs from the lane's bit; register-only (selects, no local memory).
__device__ __forceinline__ uint4 sel4(bool c, const uint4& a, const uint4& b) {
  return make_uint4(c ? a.x : b.x, c ? a.y : b.y, c ? a.z : b.z, c ? a.w : b.w);
}
__device__ __forceinline__ uint4 shfl_xor4(const uint4& v, int m) {
  return make_uint4(__shfl_xor_sync(0xffffffffu, v.x, m), __shfl_xor_sync(0xffffffffu, v.y, m),
                    __shfl_xor_sync(0xffffffffu, v.z, m), __shfl_xor_sync(0xffffffffu, v.w, m));
}
__device__ __forceinline__ void quad_transpose(uint4 (&b)[4], int lane) {
  {  // stage 1 (partner lane ^ 1): blocks {0,1} and {2,3}; a lane with bit 0 set swaps out 0 and 2
    const bool hi = lane & 1;
    const uint4 w0 = shfl_xor4(sel4(hi, b[0], b[1]), 1);
    const uint4 w1 = shfl_xor4(sel4(hi, b[2], b[3]), 1);
    b[0] = sel4(hi, w0, b[0]); b[1] = sel4(hi, b[1], w0);
    b[2] = sel4(hi, w1, b[2]); b[3] = sel4(hi, b[3], w1);
  }
  {  // stage 2 (partner lane ^ 2): blocks {0,2} and {1,3}; a lane with bit 1 set swaps out 0 and 1
    const bool hi = lane & 2;
    const uint4 w0 = shfl_xor4(sel4(hi, b[0], b[2]), 2);
    const uint4 w1 = shfl_xor4(sel4(hi, b[1], b[3]), 2);
    b[0] = sel4(hi, w0, b[0]); b[2] = sel4(hi, b[2], w0);
    b[1] = sel4(hi, w1, b[1]); b[3] = sel4(hi, b[3], w1);
  }
}

// Plain fused epilogue of one 32-column chunk with coalesced stores: each thread computes its own
// row's 32 outputs (four 16-byte blocks), a quad transpose hands lane 4g + j block j of rows
// 4g .. 4g + 3, and each of four stores writes eight rows x 64 contiguous bytes (instead of 32 rows x
// 16 bytes). Called by all 32 lanes of the warp (rows >= M compute on zero residual, store nothing).
__device__ __forceinline__ void epi_apply_rows(const GemmDev& p, int m, int img, int n, const uint32_t* r,
                                               const EpiIn<32>& in, int lane) {
  uint4 b[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[g * 8 + j]);
    if (p.wscale) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] *= __ldg(p.wscale + n + g * 8 + j);
    }
    const float4 b0 = in.b[2 * g], b1 = in.b[2 * g + 1];
    v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
    v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
    if (p.residual) {
      const __half2* h = reinterpret_cast<const __half2*>(&in.res[g]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h[e]);
        v[2 * e] += f.x;
        v[2 * e + 1] += f.y;
      }
    }
    if (p.act == 1) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = silu_f(v[j]);
    }
    b[g] = pack8(v);
  }
  quad_transpose(b, lane);
  const int row0 = m - lane + (lane & ~3);  // first row of this lane's quad
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int mr = row0 + i;
    if (mr < p.M) *reinterpret_cast<uint4*>(out_at(p, mr, n + 8 * (lane & 3))) = b[i];
  }
  (void)img;
}

// Plain fused epilogue of a tile's 32-column chunks owned by one warp, specialised on the operands
// present (residual, per-image row bias, SiLU, int8 weight scales), so the chunk loop runs
// straight-line code without per-group branches on the launch arguments. res_next holds the
// first chunk's residual on entry (loaded before the accumulator wait). Same arithmetic, order of
// operations and stores as epi_apply_rows.
template <int BN, int kSplit, bool W8, bool RES, bool ROWB, bool SILU, bool STATS = false>
__device__ __forceinline__ void epi_plain_chunks(const GemmDev& p, uint32_t t_row, int m, int img, int n0, bool mvalid,
                                                 int eh, int lane, uint4 (&res_next)[4], float& s1, float& s2) {
  const int im = mvalid ? img : 0;  // rows past M (last partial tile) must not index past the last image
  const float* rb_row = ROWB ? p.rowbias + (size_t)im * p.rowbias_ld : nullptr;
  const __half* res_row = RES ? p.residual + (size_t)m * p.ld_res : nullptr;
  const int row0 = m - lane + (lane & ~3);  // first row of this lane's quad
#pragma unroll 1
  for (int c = eh * 32; c < BN; c += kSplit * 32) {
    const int n = n0 + c;
    const int nn = n + kSplit * 32;  // this warp's next chunk
    if (nn < p.N) {                  // its lines into L1
      if (p.bias) prefetch_l1(p.bias + nn);
      if (ROWB) prefetch_l1(rb_row + nn);
      if (RES && mvalid) prefetch_l1(res_row + nn);
    }
    uint32_t r[32];
    tmem_ld32(t_row + c, r);
    float4 b[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const bool ok = n + 4 * q < p.N;
      b[q] = (ok && p.bias) ? __ldg(reinterpret_cast<const float4*>(p.bias + n) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      if (ROWB && ok) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(rb_row + n) + q);
        b[q].x += t.x; b[q].y += t.y; b[q].z += t.z; b[q].w += t.w;
      }
    }
    uint4 res[4];
    if constexpr (RES) {
#pragma unroll
      for (int g = 0; g < 4; ++g) res[g] = res_next[g];
      if (c + kSplit * 32 < BN) {
#pragma unroll
        for (int g = 0; g < 4; ++g)
          res_next[g] = (mvalid && nn + 8 * g < p.N) ? __ldg(reinterpret_cast<const uint4*>(res_row + nn) + g)
                                                    : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    tmem_wait_ld();
    if (n >= p.N) continue;  // (the same for every lane of the warp)
    uint4 o[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[g * 8 + j]);
      if constexpr (W8) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] *= __ldg(p.wscale + n + g * 8 + j);
      }
      const float4 b0 = b[2 * g], b1 = b[2 * g + 1];
      v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
      v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
      if constexpr (RES) {
        const __half2* h = reinterpret_cast<const __half2*>(&res[g]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(h[e]);
          v[2 * e] += f.x;
          v[2 * e + 1] += f.y;
        }
      }
      if constexpr (SILU) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = silu_f(v[j]);
      }
      if constexpr (STATS) {  // LayerNorm partials of this row (fp32 values before the fp16 rounding)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          s1 += v[j];
          s2 = fmaf(v[j], v[j], s2);
        }
      }
      o[g] = pack8(v);
    }
    quad_transpose(o, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int mr = row0 + i;
      if (mr < p.M) *reinterpret_cast<uint4*>(out_at(p, mr, n + 8 * (lane & 3))) = o[i];
    }
  }
}

template <int BN, int kSplit, bool W8>
__device__ __forceinline__ void epi_plain_dispatch(const GemmDev& p, uint32_t t_row, int m, int img, int n0, bool mvalid,
                                                   int eh, int lane, uint4 (&res_next)[4], float& s1, float& s2) {
  // (LayerNorm statistics come only with a plain output: no row bias, no activation; checked on the host)
  const int sel = (p.residual ? 1 : 0) | (p.rowbias ? 2 : 0) | (p.act == 1 ? 4 : 0) | (p.stat_out ? 8 : 0);
  switch (sel) {
    case 0: epi_plain_chunks<BN, kSplit, W8, false, false, false>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2); break;
    case 1: epi_plain_chunks<BN, kSplit, W8, true, false, false>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2); break;
    case 2: epi_plain_chunks<BN, kSplit, W8, false, true, false>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2); break;
    case 3: epi_plain_chunks<BN, kSplit, W8, true, true, false>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2); break;
    case 4: epi_plain_chunks<BN, kSplit, W8, false, false, true>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2); break;
    case 5: epi_plain_chunks<BN, kSplit, W8, true, false, true>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2); break;
    case 6: epi_plain_chunks<BN, kSplit, W8, false, true, true>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2); break;
    case 7: epi_plain_chunks<BN, kSplit, W8, true, true, true>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2); break;
    default:  // the statistics variants exist for fp16 weights only (the wo8 engine keeps its LayerNorm launches)
      if constexpr (!W8) {
        if (sel == 8)
          epi_plain_chunks<BN, kSplit, W8, false, false, false, true>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2);
        else
          epi_plain_chunks<BN, kSplit, W8, true, false, false, true>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2);
      }
      break;
  }
}

// Per-row LayerNorm factors of a consumer GEMM tile row m: rstd and rstd * mean from the producer's
// stat_parts (sum, sum of squares) partials (an even count, 16-byte aligned rows), summed in order
// (deterministic); var = E[x^2] - mean^2.
__device__ __forceinline__ void ln_row_factors(const GemmDev& p, int m, bool mvalid, float& rstd, float& mr) {
  float s1 = 0.f, s2 = 0.f;
  if (mvalid) {
    const float4* src = reinterpret_cast<const float4*>(p.stat_in + (size_t)m * p.stat_parts);
#pragma unroll 4
    for (int i = 0; i < p.stat_parts / 2; ++i) {
      const float4 v = __ldg(src + i);
      s1 += v.x + v.z;
      s2 += v.y + v.w;
    }
  }
  const float mean = s1 * p.ln_inv_c;
  const float var = fmaxf(fmaf(s2, p.ln_inv_c, -mean * mean), 0.f);
  rstd = rsqrtf(var + p.ln_eps);
  mr = rstd * mean;
}

// Attention-head epilogue (Q / K / V projections: bias, no residual, no activation) of a warp's
// 32-column chunks: scatter into the padded per-head layouts, V (head_vt) transposed.
template <int BN, int kSplit, bool W8, bool LN = false>
__device__ __forceinline__ void epi_heads_chunks(const GemmDev& p, uint32_t t_row, int m, int img, int n0, bool mvalid,
                                                 int eh, float rstd = 1.f, float mr = 0.f) {
  const int s_idx = m - img * p.rows_per_image;
#pragma unroll 1
  for (int c = eh * 32; c < BN; c += kSplit * 32) {
    const int n = n0 + c;
    if (p.bias && n + kSplit * 32 < p.N) prefetch_l1(p.bias + n + kSplit * 32);
    if (LN && n + kSplit * 32 < p.N) prefetch_l1(p.colsum + n + kSplit * 32);
    uint32_t r[32];
    tmem_ld32(t_row + c, r);
    float4 b[8];
#pragma unroll
    for (int q = 0; q < 8; ++q)
      b[q] = (p.bias && n + 4 * q < p.N) ? __ldg(reinterpret_cast<const float4*>(p.bias + n) + q)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 cs[LN ? 8 : 1];
    if constexpr (LN) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        cs[q] = n + 4 * q < p.N ? __ldg(reinterpret_cast<const float4*>(p.colsum + n) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    tmem_wait_ld();
    if (!mvalid || n >= p.N) continue;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int ng = n + g * 8;
      if (ng >= p.N) break;
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[g * 8 + j]);
      if constexpr (W8) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] *= __ldg(p.wscale + ng + j);
      }
      if constexpr (LN) {  // LayerNorm of the A row, folded: rstd * acc - rstd * mean * colsum
        const float* c8 = reinterpret_cast<const float*>(&cs[2 * g]);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = fmaf(rstd, v[j], -mr * c8[j]);
      }
      const float4 b0 = b[2 * g], b1 = b[2 * g + 1];
      v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
      v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
      const int which = ng / p.head_C;
      const int cc = ng - which * p.head_C;
      const int h = cc / p.head_d;
      const int jj = cc - h * p.head_d;
      __half* base = which == 0 ? p.head_out0 : (which == 1 ? p.head_out1 : p.head_out2);
      if (which == p.head_vt) {  // consecutive rows of the warp are consecutive keys
        __half* dst = base + (((size_t)img * p.heads + h) * p.head_d16 + jj) * p.head_spad + s_idx;
#pragma unroll
        for (int e = 0; e < 8; ++e) dst[(size_t)e * p.head_spad] = __float2half_rn(v[e]);
        continue;
      }
      __half* dst = base + (((size_t)img * p.heads + h) * p.rows_per_image + s_idx) * p.head_dp + jj;
      *reinterpret_cast<uint4*>(dst) = pack8(v);
    }
  }
}

// int8 x4 (one 32-bit word) -> two fp16x2, exact: bias the bytes to unsigned,
// splice each under the fp16 exponent of 1024 (0x64), subtract 1024 + 128.
__device__ __forceinline__ void i8x4_to_h4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;
  uint32_t a = __byte_perm(x, 0x64646464u, 0x4140);
  uint32_t b = __byte_perm(x, 0x64646464u, 0x4342);
  const __half2 k = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152.0
  __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), k);
  __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), k);
  lo = *reinterpret_cast<uint32_t*>(&ha);
  hi = *reinterpret_cast<uint32_t*>(&hb);
}

// EK: the epilogue this instantiation carries. Single-pass launches (no K split) with a plain fp16
// output or attention-head outputs (no residual, no activation) run an instantiation with that
// epilogue alone (kEkPlain / kEkHeads); kEkGeneric carries every epilogue (GEGLU included: its
// own instantiation measured slower on B200) and both K-split forms. Keeping them apart keeps each
// path free of the others' register pressure, code and branches.
template <int BN, bool W8, bool PAIR, int EK>
__global__ void __launch_bounds__(gemm_threads(W8, EK), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_a1,
                   const __grid_constant__ CUtensorMap map_w, const GemmDev p) {
  using C = Cfg<BN, W8, PAIR>;
  constexpr int kEpiW = gemm_epi_warps(W8, EK);
  constexpr int TM = PAIR ? 2 * BM : BM;  // output rows per unit
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  // cluster K split (1-CTA tiles only): the csp CTAs of a cluster share one output tile, CTA krank
  // computes the k-blocks [krank * kb_per_split, ...) and the partial tiles are summed through
  // distributed shared memory; one tile per cluster (no persistent loop)
  const int csp = (PAIR || EK != kEkGeneric) ? 1 : p.csplit;
  const int krank = csp > 1 ? (int)cluster_ctarank() : 0;
  const int team = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x / csp;  // pair / cluster / CTA index
  const int nteams = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x / csp;
  constexpr int S = C::kStages;
  constexpr int kRedStride = BN + 4;  // floats per partial row in the cluster K-split reduction
  static_assert((size_t)(BM + kMaxCsplitCtas - 1) * kRedStride * 4 <= (size_t)S * C::kStageBytes,
                "cluster K-split slots exceed stage memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int G = C::kG;  // k-blocks per stage; k-block g of stage s lives in slot s * G + g
  static_assert(!W8 || G == 1, "wo8 converters walk one k-block per stage");
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * G * kATileBytes;
  uint8_t* sB8 = sB + S * G * C::kBTileBytes;  // int8 staging (wo8 only)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB8 + S * C::kB8Bytes);
  // bars: full[S], empty[S], tfull[2], tempty[2], drain, conv[S] (wo8: fp16 B tile ready)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 5);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (S + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * S + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * S + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * S + 4);
  auto conv_bar = [&](int s) { return bar0 + 8u * (2 * S + 5 + s); };

  const int num_m = (p.M + TM - 1) / TM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_mn = num_m * num_n;
  const int num_units = csp > 1 ? num_mn : num_mn * p.splits;
  const int kb_per_tap = (p.cin0 + p.cin1) / BK;
  const int KB = p.K / BK;
  // unit -> (m block, n block, k range); m fastest so co-resident CTAs share W tiles
  auto decode = [&](int unit, int& m_blk, int& n_blk, int& kb0, int& kb1) {
    const int ks = csp > 1 ? krank : unit / num_mn;
    const int r = csp > 1 ? unit : unit - ks * num_mn;
    m_blk = r % num_m;
    n_blk = r / num_m;
    kb0 = ks * p.kb_per_split;
    kb1 = min(KB, kb0 + p.kb_per_split);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), kEpiW * (PAIR ? 2 : 1));  // epilogue warps of both CTAs arrive on the even CTA's
    }
    mbar_init(drain_bar, 1);
    if constexpr (W8)
      for (int s = 0; s < S; ++s) mbar_init(conv_bar(s), 128);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a0);
    tma_prefetch_desc(&map_w);
    if (p.cin1 > 0) tma_prefetch_desc(&map_a1);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc2(smem_u32(tmem_slot), C::kTmemCols);
      tmem_relinquish2();
    } else {
      tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncwarp();
  if constexpr (PAIR)
    cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA signal
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic launch: the next kernel may be scheduled now (its own wait orders its accesses).
  // The roles that touch global memory wait for the previous kernel themselves, as late as they
  // can: the producer just before its first copy (its setup overlaps the previous kernel's tail),
  // the epilogue warps before their first load. The MMA issuer and the wo8 converters work on
  // shared memory and TMEM only, ordered after the producer's copies by the mbarriers.
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      int last_phase[S];
      bool issued[S];
      for (int s = 0; s < S; ++s) { issued[s] = false; last_phase[s] = 0; }
      bool ok = true, waited = false;
      for (int unit = team; unit < num_units && ok; unit += nteams) {
        int m_blk, n_blk, kb0, kb1;
        decode(unit, m_blk, n_blk, kb0, kb1);
        const int m0 = m_blk * TM + (int)rank * BM;          // this CTA's A rows
        const int n0 = n_blk * BN + (int)rank * C::kBRows;   // this CTA's W rows
        int img0 = 0, y0 = 0;
        if (p.taps != 1) {  // output geometry; the tensor map walks the input with stride cs
          const int wo = p.W / p.cs, hwo = (p.H / p.cs) * wo;
          img0 = m0 / hwo;
          y0 = (m0 % hwo) / wo;
        }
        // taps == 4: the output phase of this tile's columns (a tile never straddles two phases)
        const int oph = p.taps == 4 ? (n_blk * BN) / p.up_co : 0;
        for (int kb = kb0; kb < kb1; kb += G, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          const int nsub = min(G, kb1 - kb);  // k-blocks in this stage (the unit's last may be short)
          if (!mbar_wait(empty_bar(s), ph ^ 1u, p.err, kDevTimeoutEmpty, p.wait_ns)) { ok = false; break; }
          if ((int)it == p.stall_it) continue;  // failure-path test: this stage is never loaded
          if (!waited) {
            pdl_wait();  // the previous kernel's outputs are visible from here on
            waited = true;
          }
          if (rank == 0) mbar_arrive_expect_tx(full_bar(s), (uint32_t)nsub * C::kTxBytes);
          issued[s] = true;
          last_phase[s] = ph;
          const uint32_t fb = PAIR ? mapa_shared(full_bar(s), 0) : full_bar(s);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            if (g >= nsub) break;
            const int k = kb + g;
            const int slot = s * G + g;
            const uint32_t dA = smem_u32(sA + slot * kATileBytes);
            const uint32_t dB = W8 ? smem_u32(sB8 + slot * C::kB8Bytes) : smem_u32(sB + slot * C::kBTileBytes);
            const int tap = k / kb_per_tap;
            const int cc = (k % kb_per_tap) * BK;
            const bool second = cc >= p.cin0;
            const CUtensorMap* ma = second ? &map_a1 : &map_a0;
            const int ch = second ? cc - p.cin0 : cc;
            if constexpr (PAIR) {
              if (p.taps == 9) {
                const int dy = tap / 3 - 1, dx = tap % 3 - 1;
                tma_load_4d_pair(dA, ma, fb, ch, dx, p.cs * y0 + dy, img0);
              } else if (p.taps == 4) {  // 2x2 tap (ty, tx) of phase (py, px): input offset (ty + py - 1, tx + px - 1)
                tma_load_4d_pair(dA, ma, fb, ch, (tap & 1) + (oph & 1) - 1, y0 + (tap >> 1) + (oph >> 1) - 1, img0);
              } else {
                tma_load_2d_pair(dA, ma, fb, ch, m0);
              }
              tma_load_2d_pair(dB, &map_w, fb, k * BK, n0);
            } else {
              if (p.taps == 9) {
                const int dy = tap / 3 - 1, dx = tap % 3 - 1;
                tma_load_4d(dA, ma, fb, ch, dx, p.cs * y0 + dy, img0);
              } else if (p.taps == 4) {
                tma_load_4d(dA, ma, fb, ch, (tap & 1) + (oph & 1) - 1, y0 + (tap >> 1) + (oph >> 1) - 1, img0);
              } else {
                tma_load_2d(dA, ma, fb, ch, m0);
              }
              tma_load_2d(dB, &map_w, fb, k * BK, n0);
            }
          }
        }
      }
      if (!ok) {
        // abort path: wait (bounded) for every copy this thread put in flight; the odd
        // CTA of a pair cannot observe the even CTA's barrier and waits out a fixed time
        if (rank == 0) {
          for (int s = 0; s < S; ++s)
            if (issued[s]) mbar_drain(full_bar(s), (uint32_t)last_phase[s], p.err, kDevTimeoutDrain, p.wait_ns);
        } else {
          spin_ns(200000);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (the even CTA of a pair)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_f16(TM, BN, false);
      uint32_t it = 0, tl = 0;
      bool ok = true;
      for (int unit = team; unit < num_units && ok; unit += nteams, ++tl) {
        int m_blk, n_blk, kb0, kb1;
        decode(unit, m_blk, n_blk, kb0, kb1);
        const uint32_t acc = tl & 1u, acc_ph = (tl >> 1) & 1u;
        const bool got = PAIR ? mbar_wait_cluster(tempty_bar(acc), acc_ph ^ 1u, p.err, kDevTimeoutAcc, p.wait_ns)
                              : mbar_wait(tempty_bar(acc), acc_ph ^ 1u, p.err, kDevTimeoutAcc, p.wait_ns);
        if (!got) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::kAccStride;
        for (int kb = kb0; kb < kb1; kb += G, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          const int nsub = min(G, kb1 - kb);
          if (!mbar_wait(full_bar(s), ph, p.err, kDevTimeoutFull, p.wait_ns)) { ok = false; break; }
          if (W8 && !mbar_wait(conv_bar(s), ph, p.err, kDevTimeoutFull, p.wait_ns)) { ok = false; break; }
          // No tcgen05 fence here: the stage's operands are shared memory written by TMA (or by the
          // converter warps, fenced to the async proxy before their arrive), ordered by the mbarrier
          // itself; the accumulator (TMEM) hazard was fenced once per tile after the tempty wait.
#pragma unroll
          for (int g = 0; g < G; ++g) {
            if (g >= nsub) break;
            const int slot = s * G + g;
            const uint64_t da = sdesc_sw128(smem_u32(sA + slot * kATileBytes), 16, 1024);
            const uint64_t db = sdesc_sw128(smem_u32(sB + slot * C::kBTileBytes), 16, 1024);
            const uint32_t first = (kb == kb0 && g == 0) ? 1u : 0u;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint32_t accum = (first && k == 0) ? 0u : 1u;
              if constexpr (PAIR)
                mma_f16_ss2(d_tmem, da + 2ull * k, db + 2ull * k, idesc, accum);
              else
                mma_f16_ss(d_tmem, da + 2ull * k, db + 2ull * k, idesc, accum);
            }
          }
          if constexpr (PAIR)
            mma_commit2_mc(empty_bar(s), 0x3);  // frees stage s in both CTAs
          else
            mma_commit(empty_bar(s));
        }
        if (!ok) break;
        if constexpr (PAIR)
          mma_commit2_mc(tfull_bar(acc), 0x3);
        else
          mma_commit(tfull_bar(acc));
      }
      // every issued MMA has retired before TMEM is released
      if constexpr (PAIR)
        mma_commit2_mc(drain_bar, 0x1);
      else
        mma_commit(drain_bar);
      mbar_drain(drain_bar, 0, p.err, kDevTimeoutDrain, p.wait_ns);
    }
  } else if (W8 && warp >= 6) {
    // ------------------------------------------------------------ int8 -> fp16 converters (wo8)
    const int ct = threadIdx.x - 192;  // 0..127
    uint32_t it = 0;
    for (int unit = team; unit < num_units; unit += nteams) {
      int m_blk, n_blk, kb0, kb1;
      decode(unit, m_blk, n_blk, kb0, kb1);
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1u;
        ok = mbar_wait(full_bar(s), ph, p.err, kDevTimeoutFull, p.wait_ns);
        if (!ok) break;
        const uint8_t* src = sB8 + s * C::kB8Bytes;
        uint8_t* dst = sB + s * C::kBTileBytes;
#pragma unroll 2
        for (int i = ct; i < BN * 4; i += 128) {  // 16 int8 of row i/4 -> two 16-byte fp16 chunks
          const int row = i >> 2, c = i & 3;
          const uint4 q = *reinterpret_cast<const uint4*>(src + row * 64 + c * 16);
          uint4 h0, h1;
          i8x4_to_h4(q.x, h0.x, h0.y);
          i8x4_to_h4(q.y, h0.z, h0.w);
          i8x4_to_h4(q.z, h1.x, h1.y);
          i8x4_to_h4(q.w, h1.z, h1.w);
          const int r7 = row & 7;
          *reinterpret_cast<uint4*>(dst + row * 128 + (((2 * c) ^ r7) << 4)) = h0;
          *reinterpret_cast<uint4*>(dst + row * 128 + (((2 * c + 1) ^ r7) << 4)) = h1;
        }
        fence_proxy_async_smem();
        mbar_arrive(conv_bar(s));
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();  // residual / bias reads and the output stores come after the previous kernel
    const int lg = warp & 3;  // TMEM lane group this warp may access
    const int row = lg * 32 + lane;
    constexpr int kSplit = kEpiW / 4;  // warps sharing a lane quadrant split its column chunks
    const int eh = (warp - 2) >> 2;
    uint32_t tl = 0;
    for (int unit = team; unit < num_units; unit += nteams, ++tl) {
      int m_blk, n_blk, kb0, kb1;
      decode(unit, m_blk, n_blk, kb0, kb1);
      const uint32_t acc = tl & 1u, acc_ph = (tl >> 1) & 1u;
      const int m = m_blk * TM + (int)rank * BM + row;
      const int img = m / p.rows_per_image;
      const int n0 = n_blk * BN;
      const bool mvalid = m < p.M;
      if (p.splits == 1 && csp == 1 && p.epi != kEpiGeglu) epi_prefetch<C::kChunk>(p, m, img, n0 + eh * C::kChunk, mvalid);
      // the first chunk's residual, in flight while the main loop finishes
      uint4 res_next[C::kChunk / 8];
      const bool fused_res = csp == 1 && p.splits == 1 && p.epi != kEpiNchwF32 && p.epi != kEpiGeglu && p.residual;
      if (fused_res) res_load<C::kChunk>(p, m, n0 + eh * C::kChunk, mvalid, res_next);
      // LayerNorm consumer (attention-head epilogue): the row's factors, read while the main loop runs
      float ln_rstd = 1.f, ln_mr = 0.f;
      const bool ln_in = EK == kEkHeads && p.stat_in != nullptr;
      if (ln_in) ln_row_factors(p, m, mvalid, ln_rstd, ln_mr);
      bool ok = mbar_wait(tfull_bar(acc), acc_ph, p.err, kDevTimeoutAcc, p.wait_ns);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + acc * C::kAccStride + (static_cast<uint32_t>(lg * 32) << 16);
      constexpr int CH = C::kChunk;
      if constexpr (EK != kEkGeneric) static_assert(CH == 32, "the specialised epilogues walk 32-column chunks");
      if constexpr (EK == kEkPlain) {
        float s1 = 0.f, s2 = 0.f;
        epi_plain_dispatch<BN, kSplit, W8>(p, t_row, m, img, n0, mvalid, eh, lane, res_next, s1, s2);
        // LayerNorm producer: each epilogue warp's partial over its column chunks of the row (the kSplit
        // warps of a lane quadrant hold disjoint chunks; no barrier between them)
        if (p.stat_out && mvalid) p.stat_out[(size_t)m * p.stat_ld + n_blk * kSplit + eh] = make_float2(s1, s2);
      } else if constexpr (EK == kEkHeads) {
        if (ln_in)
          epi_heads_chunks<BN, kSplit, W8, true>(p, t_row, m, img, n0, mvalid, eh, ln_rstd, ln_mr);
        else
          epi_heads_chunks<BN, kSplit, W8>(p, t_row, m, img, n0, mvalid, eh);
      } else if (csp > 1) {
        // cluster K split: the partial tile stays in TMEM until every CTA of the cluster is
        // past its main loop (reduction below)
      } else if (p.epi == kEpiGeglu) {
        // GEGLU: W rows interleave 16 value rows and 16 gate rows, so each 32-column chunk of the
        // accumulator holds 16 value columns then their 16 gate columns, and yields 16 outputs
        // (output column = packed column / 2) -- any tile width that is a multiple of 32 works.
        if constexpr (CH == 32) {  // (tiles narrower than 32 columns never take GEGLU)
#pragma unroll 1
        for (int c = eh * CH; c < BN; c += kSplit * CH) {
          uint32_t r[32];
          tmem_ld32(t_row + c, r);
          const int nb = n0 + c;  // packed column of the chunk
          float4 b[8];
          const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int q = 0; q < 8; ++q) b[q] = p.bias ? __ldg(reinterpret_cast<const float4*>(p.bias + nb) + q) : z;
          tmem_wait_ld();
          const int nc = nb / 2;
          if (mvalid && nc < p.N / 2) {
            const float* bf = reinterpret_cast<const float*>(b);
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float a = __uint_as_float(r[j]), gt = __uint_as_float(r[16 + j]);
              if (p.wscale) {
                a *= __ldg(p.wscale + nb + j);
                gt *= __ldg(p.wscale + nb + 16 + j);
              }
              v[j] = (a + bf[j]) * gelu_as(gt + bf[16 + j]);
            }
            float lo[8], hi[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) { lo[j] = v[j]; hi[j] = v[8 + j]; }
            uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)m * p.ld_out + nc);
            dst[0] = pack8(lo);
            dst[1] = pack8(hi);
          }
        }
        }
      } else {
#pragma unroll 1
        for (int c = eh * CH; c < BN; c += kSplit * CH) {
          if (p.splits == 1) epi_prefetch<CH>(p, m, img, n0 + c + kSplit * CH, mvalid);  // next chunk's lines
          uint32_t r[32];
          if constexpr (CH == 32) {
            tmem_ld32(t_row + c, r);
          } else {
            uint32_t t16[16];
            tmem_ld16(t_row + c, t16);
#pragma unroll
            for (int j = 0; j < 16; ++j) r[j] = t16[j];
          }
          const int n = n0 + c;
          const bool fused = p.splits == 1 && p.epi != kEpiNchwF32;
          EpiIn<CH> in;
          if (fused) epi_load<CH>(p, m, img, n, mvalid, in);  // in flight with the TMEM load
          if (fused_res) {
#pragma unroll
            for (int g = 0; g < CH / 8; ++g) in.res[g] = res_next[g];
            if (c + kSplit * CH < BN) res_load<CH>(p, m, n + kSplit * CH, mvalid, res_next);  // next chunk's
          }
          tmem_wait_ld();
          if (n >= p.N) continue;  // (the same for every lane of the warp)
          if constexpr (CH == 32) {
            if (fused && p.epi == kEpiPlain) {  // all 32 lanes: the stores are transposed across the warp
              epi_apply_rows(p, m, img, n, r, in, lane);
              continue;
            }
          }
          if (!mvalid) continue;
          if (fused) {
            epi_apply<CH>(p, m, img, n, r, in);
            continue;
          }
          if (p.splits > 1) {
            // raw fp32 partials; the reduce kernel applies the epilogue
            const int ks = kb0 / p.kb_per_split;
            float4* dst = reinterpret_cast<float4*>(p.ws + ((size_t)ks * p.M + m) * p.N + n);
#pragma unroll
            for (int q = 0; q < CH / 4; ++q)
              dst[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                                   __uint_as_float(r[4 * q + 3]));
            continue;
          }
#pragma unroll
          for (int g = 0; g < CH / 8; ++g) {
            if (n + g * 8 >= p.N) break;
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[g * 8 + j]);
            epilogue8(p, m, img, n + g * 8, v);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && rank != 0)
          mbar_arrive_cluster(mapa_shared(tempty_bar(acc), 0));
        else
          mbar_arrive(tempty_bar(acc));
      }
    }
  }

  if (csp > 1) {
    // Cluster K split. CTA q of the cluster owns rows [q * rpc, (q + 1) * rpc) of the tile
    // (rpc = ceil(128 / csp)); every CTA pushes each partial row to its owner's stage memory,
    // slot [krank], and the owner sums the slots in rank order (deterministic) and applies
    // the fused epilogue. Stage memory is reused, so the pushes start only once every CTA of
    // the cluster is past its main loop.
    const int rpc = (BM + csp - 1) / csp;
    const bool epi_warp = warp >= 2 && warp < 2 + kEpiW && team < num_units;
    tc_fence_before();
    cluster_sync_all();
    if (epi_warp) {
      tc_fence_after();
      const int lg = warp & 3;
      const int row = lg * 32 + lane;
      constexpr int kSplit = kEpiW / 4;
      const int eh = (warp - 2) >> 2;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(lg * 32) << 16);
      const int owner = row / rpc;
      const uint32_t dst_row = mapa_shared(
          smem_u32(smem) + (uint32_t)(((krank * rpc) + (row - owner * rpc)) * kRedStride) * 4u, (uint32_t)owner);
      constexpr int CH = C::kChunk;
#pragma unroll 1
      for (int c = eh * CH; c < BN; c += kSplit * CH) {
        uint32_t r[32];
        if constexpr (CH == 32) {
          tmem_ld32(t_row + c, r);
        } else {
          uint32_t t16[16];
          tmem_ld16(t_row + c, t16);
#pragma unroll
          for (int j = 0; j < 16; ++j) r[j] = t16[j];
        }
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < CH / 4; ++q)
          st_cluster_v4(dst_row + (uint32_t)(c + 4 * q) * 4u, r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
      }
    }
    cluster_sync_all();  // every partial row is in its owner's shared memory
    if (epi_warp) {
      int m_blk, n_blk, kb0, kb1;
      decode(team, m_blk, n_blk, kb0, kb1);
      const int r0 = krank * rpc, nrows = min(rpc, BM - r0);
      const int ngrp = BN / 8;
      const float* buf = reinterpret_cast<const float*>(smem);
      for (int i = threadIdx.x - 64; i < nrows * ngrp; i += kEpiW * 32) {
        const int rl = i / ngrp;
        const int c = (i % ngrp) * 8;
        const int m = m_blk * BM + r0 + rl;
        const int n = n_blk * BN + c;
        if (m >= p.M || n >= p.N) continue;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int q = 0; q < csp; ++q) {
          const float4* src = reinterpret_cast<const float4*>(buf + (size_t)(q * rpc + rl) * kRedStride + c);
          const float4 a = src[0], b = src[1];
          v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w; v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
        }
        epilogue8(p, m, m / p.rows_per_image, n, v);
      }
    }
  }
  tc_fence_before();
  __syncwarp();
  if constexpr (PAIR)
    cluster_sync_all();  // neither CTA frees TMEM or shared memory the pair still uses
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc2(tmem_base, C::kTmemCols);
    else
      tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// Sum split-K partials in split order and apply the fused epilogue; one
// thread per 8 output columns.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const GemmDev p) {
  pdl_wait();
  pdl_trigger();
  const int ngrp = (p.N + 7) / 8;
  const size_t total = (size_t)p.M * ngrp;
  const size_t plane = (size_t)p.M * p.N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / ngrp);
    const int n = (int)(i % ngrp) * 8;
    const float* src = p.ws + (size_t)m * p.N + n;
    float v[8];
    {
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 b = *reinterpret_cast<const float4*>(src + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    for (int s = 1; s < p.splits; ++s) {
      const float4 a = *reinterpret_cast<const float4*>(src + s * plane);
      const float4 b = *reinterpret_cast<const float4*>(src + s * plane + 4);
      v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w; v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
    }
    epilogue8(p, m, m / p.rows_per_image, n, v);
  }
}

template <int BN, bool W8, bool PAIR, int EK>
cudaError_t set_gemm_smem() {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, W8, PAIR, EK>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg<BN, W8, PAIR>::kSmem);
    if (e != cudaSuccess) return e;
    if (EK == kEkGeneric && !PAIR) {  // cluster K splits of up to kMaxCsplitCtas (> 8) CTAs
      e = cudaFuncSetAttribute(gemm_tc_kernel<BN, W8, PAIR, EK>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
    }
    attr_set[dev] = true;
  }
  return cudaSuccess;
}

template <int BN, bool W8, bool PAIR>
cudaError_t launch_bn(const GemmDev& d, const CUtensorMap& ma0, const CUtensorMap& ma1, const CUtensorMap& mw,
                      cudaStream_t s) {
  using C = Cfg<BN, W8, PAIR>;
  constexpr int TM = PAIR ? 2 * BM : BM;
  const int tiles = ((d.M + TM - 1) / TM) * ((d.N + BN - 1) / BN);
  if (!PAIR && d.csplit > 1) {  // one cluster of csplit CTAs per output tile
    cudaError_t e = set_gemm_smem<BN, W8, PAIR, kEkGeneric>();
    if (e != cudaSuccess) return e;
    return launch_kernel(gemm_tc_kernel<BN, W8, PAIR, kEkGeneric>, dim3(tiles * d.csplit), dim3(C::kThreads), C::kSmem,
                         s, d.csplit, ma0, ma1, mw, d);
  }
  const int units = tiles * d.splits;
  const int teams = std::max(1, std::min(units, PAIR ? num_sms() / 2 : num_sms()));
  // the epilogue-specialised instantiations exist for 32-column chunks (every width but 16)
  constexpr bool kSpec = C::kChunk == 32;
  int ek = kEkGeneric;
  if (kSpec && d.splits == 1) {
    if (d.epi == kEpiPlain) ek = kEkPlain;
    else if (d.epi == kEpiHeads && !d.residual && d.act == 0) ek = kEkHeads;
  }
  constexpr int kP = kSpec ? kEkPlain : kEkGeneric, kH = kSpec ? kEkHeads : kEkGeneric;
  auto kern = ek == kEkPlain   ? gemm_tc_kernel<BN, W8, PAIR, kP>
              : ek == kEkHeads ? gemm_tc_kernel<BN, W8, PAIR, kH>
                               : gemm_tc_kernel<BN, W8, PAIR, kEkGeneric>;
  cudaError_t e = ek == kEkPlain   ? set_gemm_smem<BN, W8, PAIR, kP>()
                  : ek == kEkHeads ? set_gemm_smem<BN, W8, PAIR, kH>()
                                   : set_gemm_smem<BN, W8, PAIR, kEkGeneric>();
  if (e != cudaSuccess) return e;
  const int kern_ek = ek == kEkPlain ? kP : ek == kEkHeads ? kH : kEkGeneric;
  e = launch_kernel(kern, dim3(PAIR ? 2 * teams : teams), dim3(gemm_threads(W8, kern_ek)), C::kSmem, s, PAIR ? 2 : 0,
                    ma0, ma1, mw, d);
  if (e != cudaSuccess || d.splits == 1) return e;
  const size_t total = (size_t)d.M * ((d.N + 7) / 8);
  const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)num_sms() * 8);
  return launch_kernel(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, s, 0, d);
}

struct TileChoice {
  int bn = 64, splits = 1, kb_per_split = 1;
  bool pair = false;  // 256-row tiles on a CTA pair (cta_group::2)
  int csplit = 1;     // > 1: K split over a cluster of csplit CTAs per tile, reduced through DSMEM
};

// Cost model, fitted to launch times measured on B200 over the SD1.5 UNet's GEMM and conv shapes
// (graph replay, 1-CTA and CTA-pair tiles of width 64..256, 1..32 K splits; median error 5 %):
//   t = waves * (k-blocks per unit * t_kb + t_unit) + (splits > 1 ? 8.5 us + 0.181 us per MB of partials : 0)
// (the workspace-split constant was refitted from 5.5 us: the forward's three workspace-split shapes,
// 128 x 1280 x 11520 / 23040 and 512 x 1280 x 23040 on CTA pairs, measured 3.0-3.2 us above the model)
// Tiles whose stages hold two k-blocks (1-CTA widths <= 160, every CTA-pair width) cost ~0.26-0.29 us
// per 64-deep k-block and CTA; the 1-CTA 192/256 tiles, one k-block per stage, 0.33-0.38. t_unit
// (pipeline fill + epilogue) grows with the tile width.
struct TileCost {
  int bn;
  bool pair;
  double us_per_kb, us_per_unit;
};
constexpr TileCost kTileCosts[] = {
    {256, false, 0.334, 6.52}, {192, false, 0.383, 4.23}, {160, false, 0.269, 3.99}, {128, false, 0.265, 2.79},
    {64, false, 0.267, 1.35},  {256, true, 0.293, 6.92},  {192, true, 0.276, 5.20},  {160, true, 0.269, 4.42},
    {128, true, 0.260, 3.32},
};

// K split inside a cluster: partial tiles summed through distributed shared memory (no workspace,
// no second launch). Its cost over the shortened main loop, fitted on B200 like the tile costs
// (median error 1 us): 0.92 us + 0.62 us per CTA of the cluster + 0.61 us per 128 tile columns.
constexpr double kCsplitUs = 0.92, kCsplitUsPerCta = 0.62, kCsplitUsPer128Cols = 0.61;

// Clusters of `cs` GEMM CTAs (one CTA per SM) that can be resident at once: a cluster must fit in
// one GPC, so this is below num_sms() / cs for the larger sizes. 0 when the device answers that no
// such cluster fits (the chooser then skips that split). Without a device (plan queries on a host
// with no GPU) the estimate is num_sms() / cs.
int cluster_capacity(int cs) {
  static int cap[64][kMaxCsplitCtas + 1] = {};
  static bool known[64][kMaxCsplitCtas + 1] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = 0;
  }
  if (dev >= 64 || cs < 2 || cs > kMaxCsplitCtas) return std::max(1, num_sms() / std::max(1, cs));
  if (!known[dev][cs]) {
    using C = Cfg<160, false, false>;
    auto k = gemm_tc_kernel<160, false, false, kEkGeneric>;
    int n = 0;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem) == cudaSuccess &&
        cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(cs * 64);
      cfg.blockDim = dim3(C::kThreads);
      cfg.dynamicSmemBytes = C::kSmem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = cs;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, (const void*)k, &cfg) != cudaSuccess) n = -1;
    } else {
      n = -1;  // no device to ask
    }
    cudaGetLastError();
    cap[dev][cs] = n >= 0 ? n : std::max(1, num_sms() / cs);
    known[dev][cs] = true;
  }
  return cap[dev][cs];
}

TileChoice choose_tiles(const GemmArgs& a, bool allow_ws = true) {
  TileChoice best;
  const int KB = a.K / BK;
  const int sms = num_sms();
  best.kb_per_split = KB;
  if (a.bn) {
    best.bn = a.bn;
    return best;
  }
  if (a.N <= 16) {
    best.bn = 16;
    return best;
  }
  const bool w8 = a.w8 != nullptr;
  const bool pair_ok = !w8 && a.M > BM;
  double best_t = 1e30;
  for (const TileCost& tcst : kTileCosts) {
    const int bn = tcst.bn;
    if (a.N % bn != 0 || (tcst.pair && !pair_ok)) continue;
    if (a.taps == 4 && a.up_co % bn != 0) continue;  // upsample conv: a tile covers one output phase
    if (w8 && bn == 192) continue;                  // wo8 tiles: 64 / 128 / 160 / 256
    if (a.epi == kEpiGeglu && bn % 32) continue;  // whole 16 value + 16 gate row groups per tile
    const int tiles = (tcst.pair ? (a.M + 2 * BM - 1) / (2 * BM) : (a.M + BM - 1) / BM) * (a.N / bn);
    const int teams = tcst.pair ? sms / 2 : sms;
    const int max_split = (a.epi == kEpiNchwF32 || a.epi == kEpiGeglu) ? 1 : std::max(1, std::min(32, KB / 3));
    for (int sp = 1; sp <= max_split; ++sp) {
      const int kbs = (KB + sp - 1) / sp;
      const int real_sp = (KB + kbs - 1) / kbs;
      if (real_sp != sp) continue;
      if (sp > 1 && allow_ws) {  // workspace split-K + reduce launch
        const int waves = (tiles * sp + teams - 1) / teams;
        const double t = waves * (kbs * tcst.us_per_kb + tcst.us_per_unit) + 8.5 +
                         0.181 * ((double)sp * a.M * a.N * 4.0 / 1e6);
        if (t < best_t) {
          best_t = t;
          best = TileChoice{bn, sp, kbs, tcst.pair, 1};
        }
      }
      // single pass, or cluster split-K (not on 1-CTA 256-wide tiles: measured 1.8x slower than the
      // workspace split of the 512 x 1280 x 23040 conv and never the fastest plan of a UNet shape)
      if (sp == 1 || (!tcst.pair && bn != 256 && sp <= kMaxCsplitCtas)) {
        const int cap = sp > 1 ? cluster_capacity(sp) : teams;  // resident clusters (sp > 1) or CTAs
        if (cap <= 0) continue;                                  // no cluster of this size fits
        const int waves = (tiles + cap - 1) / cap;
        double t = waves * (kbs * tcst.us_per_kb + tcst.us_per_unit);
        if (sp > 1) t += kCsplitUs + kCsplitUsPerCta * sp + kCsplitUsPer128Cols * bn / 128.0;
        if (t < best_t) {
          best_t = t;
          best = TileChoice{bn, 1, sp > 1 ? kbs : KB, tcst.pair, sp};
        }
      }
    }
  }
  if (best_t == 1e30) best.bn = 64;  // N not a multiple of any tile: ragged 64-wide tiles
  return best;
}

}  // namespace

size_t gemm_workspace_bytes(const GemmArgs& a) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.K % BK) return 0;
  const TileChoice t = choose_tiles(a);
  return t.splits > 1 ? (size_t)t.splits * a.M * a.N * sizeof(float) : 0;
}

GemmPlan gemm_plan(const GemmArgs& a, bool with_workspace) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.K % BK) return GemmPlan{0, 0, 0, 0};
  const TileChoice t = choose_tiles(a, with_workspace);
  return GemmPlan{t.bn, t.pair ? 1 : 0, t.splits, t.csplit};
}

void pack_upsample_conv_weights(const uint16_t* w3, int Co, int Ci, uint16_t* wp) {
  // taps (ky or kx) of the 3x3 kernel that fold into 2x2 tap t of output phase q: R(q, t)
  static const int kLo[2][2] = {{0, 1}, {0, 2}}, kHi[2][2] = {{0, 2}, {1, 2}};  // [q][t]: ky in [lo, hi]
  for (int ph = 0; ph < 4; ++ph) {
    const int py = ph >> 1, px = ph & 1;
    for (int co = 0; co < Co; ++co)
      for (int tap = 0; tap < 4; ++tap) {
        const int ty = tap >> 1, tx = tap & 1;
        uint16_t* dst = wp + ((size_t)(ph * Co + co) * 4 + tap) * Ci;
        for (int ci = 0; ci < Ci; ++ci) {
          const uint16_t* k3 = w3 + ((size_t)co * Ci + ci) * 9;
          float acc = 0.f;
          for (int ky = kLo[py][ty]; ky <= kHi[py][ty]; ++ky)
            for (int kx = kLo[px][tx]; kx <= kHi[px][tx]; ++kx) {
              __half_raw r;
              r.x = k3[ky * 3 + kx];
              acc += __half2float(__half(r));
            }
          const __half h = __float2half_rn(acc);
          dst[ci] = static_cast<__half_raw>(h).x;
        }
      }
  }
}

int gemm_launch_count(const GemmArgs& a) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.K % BK) return 1;
  const TileChoice t = choose_tiles(a);
  return (t.splits > 1 && a.ws != nullptr && a.ws_bytes >= (size_t)t.splits * a.M * a.N * sizeof(float)) ? 2 : 1;
}

cudaError_t launch_gemm(const GemmArgs& a, int* dev_err, cudaStream_t s) {
  const int cin = a.cin0 + a.cin1;
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.K % BK != 0 || cin % BK != 0 || a.cin0 % BK != 0 ||
      a.K != a.taps * cin || !(a.taps == 1 || a.taps == 4 || a.taps == 9) || (a.w == nullptr && a.w8 == nullptr) ||
      a.a0 == nullptr || (a.cin1 > 0 && a.a1 == nullptr))
    return cudaErrorInvalidValue;
  // upsample conv: fp16 weights, N = 4 phases x up_co (a multiple of 64, so every tile width the chooser
  // may take -- 64 at least -- divides it), plain output [B, 2H, 2W, up_co]
  if (a.taps == 4 && (a.up_co <= 0 || a.up_co % 64 != 0 || a.N != 4 * a.up_co || a.w8 != nullptr ||
                      a.epi != kEpiPlain || a.residual != nullptr || a.rowbias != nullptr || a.out == nullptr ||
                      (a.ld_out != 0 && a.ld_out != a.up_co) || a.bn != 0))
    return cudaErrorInvalidValue;
  if (a.epi != kEpiNchwF32 && a.epi != kEpiGeglu && a.N % 16 != 0) return cudaErrorInvalidValue;
  if ((a.epi == kEpiPlain || a.epi == kEpiHeads) && a.N > 16 && a.N % 32 != 0) return cudaErrorInvalidValue;
  TileChoice tc = choose_tiles(a);
  if (tc.splits > 1 && (a.ws == nullptr || a.ws_bytes < (size_t)tc.splits * a.M * a.N * sizeof(float)))
    tc = choose_tiles(a, false);  // no workspace: single pass or cluster split
  const int bn = tc.bn;
  if (a.epi == kEpiGeglu && (a.N % bn != 0 || bn % 32 != 0 || (a.ld_out ? a.ld_out : a.N / 2) % 8))
    return cudaErrorInvalidValue;
  if (a.epi == kEpiHeads && (a.head_d % 8 != 0 || a.head_C % 8 != 0 || a.head_dp < a.head_d ||
                             (a.head_vt >= 0 && (a.head_d16 < a.head_d || a.head_spad < a.rows_per_image))))
    return cudaErrorInvalidValue;

  GemmDev d{};
  d.M = a.M; d.N = a.N; d.K = a.K;
  d.taps = a.taps; d.cin0 = a.cin0; d.cin1 = a.cin1;
  d.H = a.H; d.W = a.W; d.cs = a.taps == 9 ? a.stride : 1;
  d.up_w = a.taps == 4 ? a.W : 0;
  d.up_co = a.taps == 4 ? a.up_co : 0;
  d.epi = a.epi; d.act = a.act;
  d.bias = a.bias; d.rowbias = a.rowbias; d.rowbias_ld = a.rowbias_ld;
  d.rows_per_image = a.rows_per_image > 0 ? a.rows_per_image : 1;
  d.residual = a.residual; d.ld_res = a.ld_res ? a.ld_res : a.N;
  d.out = a.out;
  d.ld_out = a.taps == 4 ? a.up_co : (a.ld_out ? a.ld_out : (a.epi == kEpiGeglu ? a.N / 2 : a.N));
  d.out_f32 = a.out_f32;
  d.head_out0 = a.head_out[0]; d.head_out1 = a.head_out[1]; d.head_out2 = a.head_out[2];
  d.head_C = a.head_C; d.heads = a.heads; d.head_d = a.head_d; d.head_dp = a.head_dp;
  d.head_vt = a.head_vt; d.head_d16 = a.head_d16; d.head_spad = a.head_spad;
  d.splits = tc.splits; d.kb_per_split = tc.kb_per_split; d.ws = a.ws;
  d.csplit = tc.csplit;
  d.wscale = a.w8 ? a.wscale : nullptr;
  d.err = dev_err;
  d.stat_out = a.ln_stat_out; d.stat_ld = a.ln_stat_ld;
  d.stat_in = a.ln_stat_in; d.stat_parts = a.ln_stat_parts;
  d.ln_inv_c = a.ln_C > 0 ? 1.f / (float)a.ln_C : 0.f; d.ln_eps = a.ln_eps;
  d.colsum = a.ln_colsum;
  if (a.ln_stat_out || a.ln_stat_in) {  // LayerNorm folding: single-pass 1-CTA fp16 plans only
    const bool single = tc.splits == 1 && tc.csplit == 1 && !tc.pair && bn >= 32 && a.w8 == nullptr;
    if (!single) return cudaErrorInvalidValue;
    if (a.ln_stat_out && (a.epi != kEpiPlain || a.rowbias || a.act != 0 || a.N % bn || a.ln_stat_ld < 2 * (a.N / bn) ||
                          a.taps == 4))
      return cudaErrorInvalidValue;
    if (a.ln_stat_in && (!(a.epi == kEpiHeads && !a.residual && a.act == 0) || a.ln_stat_parts <= 0 ||
         a.ln_stat_parts % 2 || a.ln_C <= 0 || !a.ln_colsum ||
         ((reinterpret_cast<uintptr_t>(a.ln_colsum) | reinterpret_cast<uintptr_t>(a.ln_stat_in)) & 15)))
      return cudaErrorInvalidValue;
  }
  d.stall_it = a.test_stall_iter;
  d.wait_ns = a.wait_limit_ns ? a.wait_limit_ns : kWaitTimeoutNs;
  if (a.w8 && !a.wscale) return cudaErrorInvalidValue;
  // the epilogue reads bias / per-image bias 8 columns at a time as two float4
  if ((reinterpret_cast<uintptr_t>(a.bias) | reinterpret_cast<uintptr_t>(a.rowbias)) & 15) return cudaErrorInvalidValue;
  if (a.rowbias && a.rowbias_ld % 4) return cudaErrorInvalidValue;

  CUtensorMap ma0{}, ma1{}, mw{};
  if (a.taps == 9 || a.taps == 4) {
    // Box over the input {64 channels, row, rows, images}, shifted per tap; with stride 2 the box spans
    // twice the output extent in x and y and TMA loads every second element (element strides 2), so
    // the tile still lands as 128 output pixels x 64 channels. Out-of-range rows / columns read zero.
    // (taps == 4: the 2x2 phase convolutions walk the input like a stride-1 conv of its own size)
    const int st = a.taps == 9 ? a.stride : 1;
    if (!(st == 1 || st == 2) || a.H % st || a.W % st) return cudaErrorInvalidValue;
    const int ho = a.H / st, wo = a.W / st, hw = a.H * a.W, hwo = ho * wo;
    int box_h, box_b;
    if (wo > 128 || (BM % wo) != 0) return cudaErrorInvalidValue;
    if (hwo >= BM) {
      box_h = BM / wo; box_b = 1;
      if (ho % box_h) return cudaErrorInvalidValue;
    } else {
      if (BM % hwo) return cudaErrorInvalidValue;
      box_h = ho; box_b = BM / hwo;
    }
    auto mk4 = [&](CUtensorMap* m, const __half* base, int c) {
      uint64_t dims[4] = {(uint64_t)c, (uint64_t)a.W, (uint64_t)a.H, (uint64_t)a.B};
      uint64_t str[3] = {(uint64_t)c * 2, (uint64_t)a.W * c * 2, (uint64_t)hw * c * 2};
      uint32_t box[4] = {BK, (uint32_t)(st * wo), (uint32_t)(st * box_h), (uint32_t)box_b};
      const uint32_t estr[4] = {1u, (uint32_t)st, (uint32_t)st, 1u};
      return make_tmap(m, base, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, estr);
    };
    if (a.M != a.B * hwo) return cudaErrorInvalidValue;
    if (!mk4(&ma0, a.a0, a.cin0)) return cudaErrorInvalidValue;
    if (a.cin1 > 0 && !mk4(&ma1, a.a1, a.cin1)) return cudaErrorInvalidValue;
  } else {
    const int ld0 = a.lda0 ? a.lda0 : a.cin0;
    if (!make_tmap_2d(&ma0, a.a0, a.M, a.cin0, ld0, BM, BK)) return cudaErrorInvalidValue;
    if (a.cin1 > 0) {
      const int ld1 = a.lda1 ? a.lda1 : a.cin1;
      if (!make_tmap_2d(&ma1, a.a1, a.M, a.cin1, ld1, BM, BK)) return cudaErrorInvalidValue;
    }
  }
  if (a.cin1 == 0) ma1 = ma0;
  if (a.w8) {
    // int8 weights: 64-byte rows of [N, K], no swizzle (the converters re-lay them out)
    uint64_t dims[2] = {(uint64_t)a.K, (uint64_t)a.N};
    uint64_t str[1] = {(uint64_t)a.K};
    uint32_t box[2] = {BK, (uint32_t)bn};
    if (!make_tmap(&mw, a.w8, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_DATA_TYPE_UINT8))
      return cudaErrorInvalidValue;
    switch (bn) {
      case 16: return launch_bn<16, true, false>(d, ma0, ma1, mw, s);
      case 64: return launch_bn<64, true, false>(d, ma0, ma1, mw, s);
      case 128: return launch_bn<128, true, false>(d, ma0, ma1, mw, s);
      case 160: return launch_bn<160, true, false>(d, ma0, ma1, mw, s);
      case 256: return launch_bn<256, true, false>(d, ma0, ma1, mw, s);
      default: return cudaErrorInvalidValue;
    }
  }
  // W box: the rows one CTA loads (half the tile's N on a CTA pair)
  if (!make_tmap_2d(&mw, a.w, a.N, a.K, a.K, tc.pair ? bn / 2 : bn, BK)) return cudaErrorInvalidValue;
  if (tc.pair) {
    switch (bn) {
      case 192: return launch_bn<192, false, true>(d, ma0, ma1, mw, s);
      case 128: return launch_bn<128, false, true>(d, ma0, ma1, mw, s);
      case 160: return launch_bn<160, false, true>(d, ma0, ma1, mw, s);
      case 256: return launch_bn<256, false, true>(d, ma0, ma1, mw, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (bn) {
    case 192: return launch_bn<192, false, false>(d, ma0, ma1, mw, s);
    case 16: return launch_bn<16, false, false>(d, ma0, ma1, mw, s);
    case 64: return launch_bn<64, false, false>(d, ma0, ma1, mw, s);
    case 128: return launch_bn<128, false, false>(d, ma0, ma1, mw, s);
    case 160: return launch_bn<160, false, false>(d, ma0, ma1, mw, s);
    case 256: return launch_bn<256, false, false>(d, ma0, ma1, mw, s);
    default: return cudaErrorInvalidValue;
  }
}

int num_sms() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) dev = 63;
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

}  // namespace sdg
