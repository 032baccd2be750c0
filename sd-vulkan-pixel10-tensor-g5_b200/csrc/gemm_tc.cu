// gemm_tc.cu — tcgen05 GEMM / implicit-GEMM 3x3 convolution for sm_100a.
//
// Replaces the reference's conv/matmul family (vk_engine.cpp:578-613;
// matmul_f32.comp, im2col_f32.comp, winograd_*.comp, addbias*_f32.comp,
// add_f32.comp, geglu_f32.comp) with one persistent, warp-specialised kernel:
//   warp 0      TMA producer: A tile 128x64 + W tile BNx64 per stage (SW128)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128,K=16)
//   warps 2..5  epilogue: tcgen05.ld rows from TMEM, fused bias / per-image
//               bias / residual / SiLU / GEGLU / head scatter, fp16 stores
// Accumulators are double-buffered in TMEM so the epilogue of tile i overlaps
// the main loop of tile i+1. No cluster multicast is used anywhere.
#include <algorithm>
#include <cstdio>

#include "sdg_kernels.h"
#include "sdg_ptx.cuh"
#include "sdg_tma.h"

namespace sdg {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr uint32_t kATileBytes = BM * BK * 2;  // 16 KB

struct GemmDev {
  int M, N, K;
  int taps, cin0, cin1;
  int H, W, box_h, box_b;  // conv geometry
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
  int* err;
};

template <int BN>
struct Cfg {
  static constexpr int kStages = BN >= 256 ? 4 : (BN >= 160 ? 5 : (BN >= 128 ? 6 : 8));
  static constexpr uint32_t kBTileBytes = BN * BK * 2;
  static constexpr uint32_t kStageBytes = kATileBytes + kBTileBytes;
  static constexpr int kAccStride = BN <= 16 ? 16 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
  static constexpr uint32_t kTmemCols = (2 * kAccStride) < 32 ? 32 : 2 * kAccStride;
  static constexpr int kChunk = BN >= 32 ? 32 : 16;
  static constexpr size_t kSmem = 1024 + (size_t)kStages * kStageBytes + 256;
  static_assert(kSmem <= 232448, "GEMM tile configuration exceeds 227 KB of shared memory");
};

__device__ __forceinline__ void store_row_chunk(__half* dst, const float* v, int n) {
  // n is 16 or 32 consecutive fp16 (16-byte aligned destination)
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (q * 8 < n) {
      uint4 u;
      u.x = pack_half2(v[q * 8 + 0], v[q * 8 + 1]);
      u.y = pack_half2(v[q * 8 + 2], v[q * 8 + 3]);
      u.z = pack_half2(v[q * 8 + 4], v[q * 8 + 5]);
      u.w = pack_half2(v[q * 8 + 6], v[q * 8 + 7]);
      d4[q] = u;
    }
  }
}

__device__ __forceinline__ void load_half_chunk(const __half* src, float* v, int n) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (q * 8 < n) {
      uint4 u = __ldg(s4 + q);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __half22float2(h[e]);
        v[q * 8 + 2 * e] = f.x;
        v[q * 8 + 2 * e + 1] = f.y;
      }
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_a1,
                   const __grid_constant__ CUtensorMap map_w, const GemmDev p) {
  using C = Cfg<BN>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kATileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * C::kBTileBytes);
  // bars: full[S], empty[S], tfull[2], tempty[2], drain
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (S + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * S + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * S + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * S + 4);

  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int kb_per_tap = (p.cin0 + p.cin1) / BK;
  const int KB = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(drain_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a0);
    tma_prefetch_desc(&map_w);
    if (p.cin1 > 0) tma_prefetch_desc(&map_a1);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      int last_phase[S];
      bool issued[S];
      for (int s = 0; s < S; ++s) { issued[s] = false; last_phase[s] = 0; }
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_blk = tile % num_m, n_blk = tile / num_m;
        const int m0 = m_blk * BM, n0 = n_blk * BN;
        int img0 = 0, y0 = 0;
        if (p.taps == 9) {
          const int hw = p.H * p.W;
          img0 = m0 / hw;
          y0 = (m0 % hw) / p.W;
        }
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait(empty_bar(s), ph ^ 1u, p.err, kDevTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(full_bar(s), C::kStageBytes);
          issued[s] = true;
          last_phase[s] = ph;
          const uint32_t dA = smem_u32(sA + s * kATileBytes);
          const uint32_t dB = smem_u32(sB + s * C::kBTileBytes);
          const int tap = kb / kb_per_tap;
          const int cc = (kb % kb_per_tap) * BK;
          const bool second = cc >= p.cin0;
          const CUtensorMap* ma = second ? &map_a1 : &map_a0;
          const int ch = second ? cc - p.cin0 : cc;
          if (p.taps == 9) {
            const int dy = tap / 3 - 1, dx = tap % 3 - 1;
            tma_load_4d(dA, ma, full_bar(s), ch, dx, y0 + dy, img0);
          } else {
            tma_load_2d(dA, ma, full_bar(s), ch, m0);
          }
          tma_load_2d(dB, &map_w, full_bar(s), kb * BK, n0);
        }
      }
      if (!ok) {
        // abort path: wait (bounded) for every copy this thread put in flight
        for (int s = 0; s < S; ++s)
          if (issued[s]) mbar_wait(full_bar(s), (uint32_t)last_phase[s], p.err, kDevTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BM, BN, false);
      uint32_t it = 0, tl = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++tl) {
        const uint32_t acc = tl & 1u, acc_ph = (tl >> 1) & 1u;
        if (!mbar_wait(tempty_bar(acc), acc_ph ^ 1u, p.err, kDevTimeoutAcc)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::kAccStride;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait(full_bar(s), ph, p.err, kDevTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = sdesc_sw128(smem_u32(sA + s * kATileBytes), 16, 1024);
          const uint64_t db = sdesc_sw128(smem_u32(sB + s * C::kBTileBytes), 16, 1024);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_ss(d_tmem, da + 2ull * k, db + 2ull * k, idesc, (kb | k) != 0 ? 1u : 0u);
          mma_commit(empty_bar(s));
        }
        if (!ok) break;
        mma_commit(tfull_bar(acc));
      }
      // every issued MMA has retired before TMEM is released
      mma_commit(drain_bar);
      mbar_wait(drain_bar, 0, p.err, kDevTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int lg = warp & 3;  // TMEM lane group this warp may access
    const int row = lg * 32 + lane;
    uint32_t tl = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tl) {
      const uint32_t acc = tl & 1u, acc_ph = (tl >> 1) & 1u;
      bool ok = mbar_wait(tfull_bar(acc), acc_ph, p.err, kDevTimeoutAcc);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int m_blk = tile % num_m, n_blk = tile / num_m;
      const int m = m_blk * BM + row;
      const int n0 = n_blk * BN;
      const bool mvalid = m < p.M;
      const int img = mvalid ? m / p.rows_per_image : 0;
      const uint32_t t_row = tmem_base + acc * C::kAccStride + (static_cast<uint32_t>(lg * 32) << 16);
      constexpr int CH = C::kChunk;
      if (p.epi == kEpiGeglu) {
        constexpr int HALF = BN / 2;
        const int nout0 = n_blk * HALF;
#pragma unroll 1
        for (int c = 0; c < HALF; c += CH) {
          uint32_t ra[32], rg[32];
          if constexpr (CH == 32) {
            tmem_ld32(t_row + c, ra);
            tmem_ld32(t_row + HALF + c, rg);
          } else {
            uint32_t t16a[16], t16g[16];
            tmem_ld16(t_row + c, t16a);
            tmem_ld16(t_row + HALF + c, t16g);
#pragma unroll
            for (int j = 0; j < 16; ++j) { ra[j] = t16a[j]; rg[j] = t16g[j]; }
          }
          tmem_wait_ld();
          const int nc = nout0 + c;
          if (mvalid && nc < p.N / 2) {
            float v[32];
#pragma unroll
            for (int j = 0; j < CH; ++j) {
              const float a = __uint_as_float(ra[j]) + (p.bias ? __ldg(p.bias + n0 + c + j) : 0.f);
              const float g = __uint_as_float(rg[j]) + (p.bias ? __ldg(p.bias + n0 + HALF + c + j) : 0.f);
              v[j] = a * gelu_erf(g);
            }
            store_row_chunk(p.out + (size_t)m * p.ld_out + nc, v, CH);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += CH) {
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
          const int n = n0 + c;
          if (!mvalid || n >= p.N) continue;
          float v[32];
#pragma unroll
          for (int j = 0; j < CH; ++j) v[j] = __uint_as_float(r[j]);
          if (p.epi == kEpiNchwF32) {
            const int pix = m % p.rows_per_image;
            for (int j = 0; j < CH && n + j < p.N; ++j) {
              float x = v[j] + (p.bias ? __ldg(p.bias + n + j) : 0.f);
              p.out_f32[((size_t)img * p.N + n + j) * p.rows_per_image + pix] = x;
            }
            continue;
          }
          if (p.bias) {
#pragma unroll
            for (int j = 0; j < CH; ++j) v[j] += __ldg(p.bias + n + j);
          }
          if (p.rowbias) {
            const float* rb = p.rowbias + (size_t)img * p.rowbias_ld + n;
#pragma unroll
            for (int j = 0; j < CH; ++j) v[j] += __ldg(rb + j);
          }
          if (p.residual) {
            float rv[32];
            load_half_chunk(p.residual + (size_t)m * p.ld_res + n, rv, CH);
#pragma unroll
            for (int j = 0; j < CH; ++j) v[j] += rv[j];
          }
          if (p.act == 1) {
#pragma unroll
            for (int j = 0; j < CH; ++j) v[j] = silu_f(v[j]);
          }
          if (p.epi == kEpiHeads) {
            const int s_idx = m % p.rows_per_image;
#pragma unroll
            for (int g = 0; g < CH / 8; ++g) {
              const int nn = n + g * 8;
              const int which = nn / p.head_C;
              const int cc = nn - which * p.head_C;
              const int h = cc / p.head_d;
              const int jj = cc - h * p.head_d;
              __half* base = which == 0 ? p.head_out0 : (which == 1 ? p.head_out1 : p.head_out2);
              if (which == p.head_vt) {
                // transposed V: [BH, d16, spad]; consecutive rows of the warp are consecutive keys
                __half* dst = base + (((size_t)img * p.heads + h) * p.head_d16 + jj) * p.head_spad + s_idx;
#pragma unroll
                for (int e = 0; e < 8; ++e) dst[(size_t)e * p.head_spad] = __float2half_rn(v[g * 8 + e]);
                continue;
              }
              __half* dst = base + (((size_t)img * p.heads + h) * p.rows_per_image + s_idx) * p.head_dp + jj;
              uint4 u;
              u.x = pack_half2(v[g * 8 + 0], v[g * 8 + 1]);
              u.y = pack_half2(v[g * 8 + 2], v[g * 8 + 3]);
              u.z = pack_half2(v[g * 8 + 4], v[g * 8 + 5]);
              u.w = pack_half2(v[g * 8 + 6], v[g * 8 + 7]);
              *reinterpret_cast<uint4*>(dst) = u;
            }
          } else {
            store_row_chunk(p.out + (size_t)m * p.ld_out + n, v, CH);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

template <int BN>
cudaError_t launch_bn(const GemmArgs& a, const GemmDev& d, const CUtensorMap& ma0, const CUtensorMap& ma1,
                      const CUtensorMap& mw, cudaStream_t s) {
  using C = Cfg<BN>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, num_sms()));
  gemm_tc_kernel<BN><<<grid, kThreads, C::kSmem, s>>>(ma0, ma1, mw, d);
  return cudaGetLastError();
}

int choose_bn(const GemmArgs& a) {
  if (a.bn) return a.bn;
  if (a.N <= 16) return 16;
  if (a.epi == kEpiGeglu) return 256;
  // prefer the widest tile that divides N and still gives >= ~1 wave of tiles
  const int num_m = (a.M + BM - 1) / BM;
  const int cands[4] = {256, 160, 128, 64};
  for (int bn : cands) {
    if (a.N % bn) continue;
    if (num_m * (a.N / bn) >= num_sms() * 3 / 4 || bn == 64) return bn;
  }
  return a.N % 64 == 0 ? 64 : 128;
}

}  // namespace

cudaError_t launch_gemm(const GemmArgs& a, int* dev_err, cudaStream_t s) {
  const int cin = a.cin0 + a.cin1;
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.K % BK != 0 || cin % BK != 0 || a.cin0 % BK != 0 ||
      a.K != a.taps * cin || !(a.taps == 1 || a.taps == 9) || a.w == nullptr || a.a0 == nullptr ||
      (a.cin1 > 0 && a.a1 == nullptr))
    return cudaErrorInvalidValue;
  if (a.epi != kEpiNchwF32 && a.epi != kEpiGeglu && a.N % 16 != 0) return cudaErrorInvalidValue;
  const int bn = choose_bn(a);
  if (a.epi == kEpiGeglu && (a.N % bn != 0)) return cudaErrorInvalidValue;
  if (a.epi == kEpiHeads && (a.head_d % 8 != 0 || a.head_C % 8 != 0 || a.head_dp < a.head_d ||
                             (a.head_vt >= 0 && (a.head_d16 < a.head_d || a.head_spad < a.rows_per_image))))
    return cudaErrorInvalidValue;
  if ((a.epi == kEpiPlain || a.epi == kEpiHeads) && a.N > 16 && a.N % 32 != 0) return cudaErrorInvalidValue;

  GemmDev d{};
  d.M = a.M; d.N = a.N; d.K = a.K;
  d.taps = a.taps; d.cin0 = a.cin0; d.cin1 = a.cin1;
  d.H = a.H; d.W = a.W;
  d.epi = a.epi; d.act = a.act;
  d.bias = a.bias; d.rowbias = a.rowbias; d.rowbias_ld = a.rowbias_ld;
  d.rows_per_image = a.rows_per_image > 0 ? a.rows_per_image : 1;
  d.residual = a.residual; d.ld_res = a.ld_res ? a.ld_res : a.N;
  d.out = a.out; d.ld_out = a.ld_out ? a.ld_out : (a.epi == kEpiGeglu ? a.N / 2 : a.N);
  d.out_f32 = a.out_f32;
  d.head_out0 = a.head_out[0]; d.head_out1 = a.head_out[1]; d.head_out2 = a.head_out[2];
  d.head_C = a.head_C; d.heads = a.heads; d.head_d = a.head_d; d.head_dp = a.head_dp;
  d.head_vt = a.head_vt; d.head_d16 = a.head_d16; d.head_spad = a.head_spad;
  d.err = dev_err;

  CUtensorMap ma0{}, ma1{}, mw{};
  if (a.taps == 9) {
    const int hw = a.H * a.W;
    if (a.W > 128 || (BM % a.W) != 0) return cudaErrorInvalidValue;
    if (hw >= BM) {
      d.box_h = BM / a.W; d.box_b = 1;
      if (a.H % d.box_h) return cudaErrorInvalidValue;
    } else {
      if (BM % hw) return cudaErrorInvalidValue;
      d.box_h = a.H; d.box_b = BM / hw;
    }
    auto mk4 = [&](CUtensorMap* m, const __half* base, int c) {
      uint64_t dims[4] = {(uint64_t)c, (uint64_t)a.W, (uint64_t)a.H, (uint64_t)a.B};
      uint64_t str[3] = {(uint64_t)c * 2, (uint64_t)a.W * c * 2, (uint64_t)hw * c * 2};
      uint32_t box[4] = {BK, (uint32_t)a.W, (uint32_t)d.box_h, (uint32_t)d.box_b};
      return make_tmap(m, base, 4, dims, str, box);
    };
    if (a.M != a.B * hw) return cudaErrorInvalidValue;
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
  if (!make_tmap_2d(&mw, a.w, a.N, a.K, a.K, bn, BK)) return cudaErrorInvalidValue;

  switch (bn) {
    case 16: return launch_bn<16>(a, d, ma0, ma1, mw, s);
    case 64: return launch_bn<64>(a, d, ma0, ma1, mw, s);
    case 128: return launch_bn<128>(a, d, ma0, ma1, mw, s);
    case 160: return launch_bn<160>(a, d, ma0, ma1, mw, s);
    case 256: return launch_bn<256>(a, d, ma0, ma1, mw, s);
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
