// attention_tc.cu — fused flash attention for sm_100a (tcgen05 + TMA).
//
// Replaces attention_f32.comp / attention_big_f32.comp and the split/merge
// head shaders (vk_engine.cpp:649-663): softmax(Q K^T / sqrt(d)) V per head,
// keys restricted to the query's own image, online softmax in fp32.
//
// Layout: Q and K arrive in a padded per-head layout [B*heads, S, DP]
// (DP = d rounded up to 64) and V transposed, [B*heads, D16, S_pad]
// (D16 = d rounded up to 16), all written by the projection GEMM's epilogue
// with zero padding. Every operand tile is then a plain 3D TMA box with
// 128-byte swizzle and both MMAs take K-major operands.
// CTA = NQT query tiles of 128 rows of one (image, head):
//   warp 0        TMA producer (Q once, K/V ring of NKV stages)
//   warp 1        MMA issuer: S_t = Q_t K^T (TMEM), then PV_t = P_t V (TMEM)
//   warps 2..     NQT softmax warpgroups, one TMEM row per thread: max,
//                 exp2, fp16 P into swizzled smem (A operand of PV); O stays
//                 in TMEM (PV accumulates), rescaled lazily per row.
// When d < D16 (d = 40) row d of the V^T tile is set to ones in shared memory
// (the TMA box loads only d rows), so PV column d is the row sum of the fp16
// P actually used — the tensor core does the softmax denominators.
// Keys beyond Sk (cross-attention: 77 keys) are masked in the last tile only.
#include <algorithm>

#include "sdg_kernels.h"
#include "sdg_launch.h"
#include "sdg_ptx.cuh"
#include "sdg_tma.h"

namespace sdg {
namespace {

// TPV: PV computed transposed, O^T[d][q] += V^T[d][keys] * P^T — one M=64 MMA per 16 keys covers
// both query tiles (N = 256), half the PV instructions of the per-tile form (M=128, N=D16).
// POLY: of every 16 exponential pairs of a 32-key chunk, how many the softmax evaluates with ex2_poly
// on the FMA pipe instead of ex2.approx.f16x2 on the MUFU pipe (balances the two pipes).
template <int DP_, int BKV_, int NQT_, int D16_, bool ONES_, bool TPV_ = false, int POLY_ = 0>
struct AttnCfg {
  static constexpr int DP = DP_, BKV = BKV_, NQT = NQT_, D16 = D16_;
  static constexpr bool ONES = ONES_;
  static constexpr bool TPV = TPV_;
  static constexpr int POLY = POLY_;
  static_assert(POLY >= 0 && POLY <= 16 && (POLY == 0 || 16 % POLY == 0), "POLY pairs spread evenly over 16");
  static_assert(!TPV || (NQT == 2 && BKV == 128 && ONES && D16 <= 64), "transposed PV: two 128-row query tiles");
  static constexpr int DV = TPV ? 64 : D16;                   // rows of a V^T atom
  static constexpr int NATOM = DP / 64;                       // 128B swizzle atoms along d
  static constexpr int NKATOM = BKV / 64;                     // 128B swizzle atoms along keys
  static constexpr int NKV = BKV > 64 ? 2 : (DP == 64 ? (NQT >= 4 ? 2 : 4) : (DP == 128 ? 3 : 2));  // K/V pipeline depth
  static constexpr uint32_t kQTile = 128 * 128 * NATOM;       // bytes per 128-row Q tile
  static constexpr uint32_t kKTile = BKV * 128 * NATOM;       // bytes of K per stage
  static constexpr uint32_t kVAtom = DV * 128;                // bytes of one 64-key V^T atom
  static constexpr uint32_t kVTile = NKATOM * kVAtom;         // bytes of V^T per stage
  static constexpr uint32_t kPTile = 128 * BKV * 2;           // fp16 P per query tile
  static constexpr int PVS = (D16 + 31) / 32 * 32;            // TMEM column stride of PV buffers
  static constexpr int kTmemNeed = NQT * BKV + (TPV ? NQT * 128 : NQT * PVS);
  static constexpr uint32_t kTmemCols = kTmemNeed <= 32 ? 32 : kTmemNeed <= 64 ? 64 : kTmemNeed <= 128 ? 128 : kTmemNeed <= 256 ? 256 : 512;
  static constexpr int kThreads = 64 + 128 * NQT;
  static constexpr size_t kSmem = 1024 + (size_t)NQT * kQTile + (size_t)NKV * (kKTile + kVTile) + (size_t)2 * NQT * kPTile + 1024 +
                                  (TPV ? 1024 : 0);  // TPV: per-row O^T correction factors
  static_assert(kSmem <= 232448, "attention tile configuration exceeds 227 KB of shared memory");
  static_assert(kTmemNeed <= 512, "attention tile configuration exceeds TMEM");
  static_assert(kVAtom % 1024 == 0, "V^T atoms must stay 1024-byte aligned");
};

// Named barrier over `n` threads with an AND / OR reduction of a predicate.
__device__ __forceinline__ bool bar_and(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.and.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ bool bar_or(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.or.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void bar_sync_n(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

struct AttnDev {
  int heads, Sq, Sk, d;
  __half* o;
  int ld_o;
  float sl2;  // scale * log2(e)
  int* err;
};


// Maximum of a score row held as NCH x 32 words: eight independent partial maxima, then a
// tree, so the dependency chain is 4 * NCH + 3 deep instead of 32 * NCH.
template <int NCH>
__device__ __forceinline__ float row_max(const uint32_t (&sv)[NCH][32]) {
  float pm[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) pm[k] = -INFINITY;
#pragma unroll
  for (int h = 0; h < NCH; ++h)
#pragma unroll
    for (int e = 0; e < 32; ++e) pm[e & 7] = fmaxf(pm[e & 7], __uint_as_float(sv[h][e]));
#pragma unroll
  for (int k = 4; k; k >>= 1)
#pragma unroll
    for (int i = 0; i < k; ++i) pm[i] = fmaxf(pm[i], pm[i + k]);
  return pm[0];
}

template <class CF>
__global__ void __launch_bounds__(CF::kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                   const __grid_constant__ CUtensorMap map_v, const AttnDev p) {
  constexpr int BKV = CF::BKV, NQT = CF::NQT, NKV = CF::NKV, NATOM = CF::NATOM, D16 = CF::D16;
  constexpr bool ONES = CF::ONES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + NQT * CF::kQTile;
  uint8_t* sV = sK + NKV * CF::kKTile;
  uint8_t* sP = sV + NKV * CF::kVTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * NQT * CF::kPTile);  // P double-buffered per tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 96);
  const uint32_t b0 = smem_u32(bars);
  // barrier indices
  const uint32_t q_full = b0;
  auto kv_full = [&](int s) { return b0 + 8u * (1 + s); };
  auto kv_empty = [&](int s) { return b0 + 8u * (1 + NKV + s); };
  auto s_full = [&](int t) { return b0 + 8u * (1 + 2 * NKV + t); };
  auto s_free = [&](int t) { return b0 + 8u * (1 + 2 * NKV + NQT + t); };
  // one P-ready barrier per (tile, P buffer): P(j) and P(j+2) share a barrier and P(j+2)
  // cannot be written before PV(j) ran, so a barrier never runs two phases ahead
  auto p_full = [&](int t, int buf) { return b0 + 8u * (1 + 2 * NKV + 2 * NQT + 2 * t + buf); };
  // likewise one PV-done barrier per P buffer: PV(j) commits to pv_full(t, j & 1), so a
  // waiter on PV(j-2) or PV(j-1) never finds its barrier two phases ahead
  auto pv_full = [&](int t, int buf) { return b0 + 8u * (1 + 2 * NKV + 4 * NQT + 2 * t + buf); };
  const uint32_t drain = b0 + 8u * (1 + 2 * NKV + 6 * NQT);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int q0 = blockIdx.x * 128 * NQT;
  const int nkv = (p.Sk + BKV - 1) / BKV;
  const int vrows = ONES ? p.d : D16;  // rows of each V^T atom written by TMA

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NKV; ++s) { mbar_init(kv_full(s), 1); mbar_init(kv_empty(s), 1); }
    for (int t = 0; t < NQT; ++t) {
      mbar_init(s_full(t), 1);
      mbar_init(s_free(t), 4);
      mbar_init(p_full(t, 0), 128);
      mbar_init(p_full(t, 1), 128);
      mbar_init(pv_full(t, 0), 1);
      mbar_init(pv_full(t, 1), 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if constexpr (ONES) {
    // rows d..D16-1 of every V^T atom: row d = 1.0 (row-sum column of PV), the rest 0.
    // TMA never writes these rows; the generic-proxy writes are fenced before any MMA.
    const int extra = CF::DV - p.d;
    const int per_stage = CF::NKATOM * extra * 8;  // 16-byte chunks
    for (int i = threadIdx.x; i < NKV * per_stage; i += blockDim.x) {
      const int s = i / per_stage, rem = i % per_stage;
      const int a = rem / (extra * 8), rr = (rem / 8) % extra, ch = rem % 8;
      const uint32_t v = (rr == 0) ? 0x3C003C00u : 0u;
      *reinterpret_cast<uint4*>(sV + s * CF::kVTile + a * CF::kVAtom + (p.d + rr) * 128 + ch * 16) = make_uint4(v, v, v, v);
    }
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), CF::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic launch: the next kernel may be scheduled now. The producer waits for the previous
  // kernel's outputs (Q/K/V) just before its first copy, the softmax warps before their stores; the
  // MMA issuer works on shared memory and TMEM only, ordered by the mbarriers.
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      pdl_wait();  // the previous kernel's outputs are visible from here on
      mbar_arrive_expect_tx(q_full, NQT * CF::kQTile);
      for (int t = 0; t < NQT; ++t)
        for (int a = 0; a < NATOM; ++a)
          tma_load_3d(smem_u32(sQ + t * CF::kQTile + a * 16384), &map_q, q_full, 64 * a, q0 + 128 * t, bh);
      bool issued[NKV];
      int last_ph[NKV];
      for (int s = 0; s < NKV; ++s) { issued[s] = false; last_ph[s] = 0; }
      bool ok = true;
      const uint32_t kv_bytes = CF::kKTile + CF::NKATOM * vrows * 128;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % NKV;
        const uint32_t ph = (j / NKV) & 1;
        if (!mbar_wait(kv_empty(s), ph ^ 1u, p.err, kDevTimeoutAttn)) { ok = false; break; }
        mbar_arrive_expect_tx(kv_full(s), kv_bytes);
        issued[s] = true;
        last_ph[s] = ph;
        for (int a = 0; a < NATOM; ++a)
          tma_load_3d(smem_u32(sK + s * CF::kKTile + a * BKV * 128), &map_k, kv_full(s), 64 * a, j * BKV, bh);
        for (int a = 0; a < CF::NKATOM; ++a)
          tma_load_3d(smem_u32(sV + s * CF::kVTile + a * CF::kVAtom), &map_v, kv_full(s), j * BKV + 64 * a, 0, bh);
      }
      if (!ok) {
        mbar_drain(q_full, 0, p.err, kDevTimeoutDrain);
        for (int s = 0; s < NKV; ++s)
          if (issued[s]) mbar_drain(kv_full(s), (uint32_t)last_ph[s], p.err, kDevTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // Event-driven issue: each query tile advances on its own barriers, so one slow
      // softmax warpgroup never delays the tensor-core work of the others.
      const uint32_t idesc_s = idesc_f16(128, BKV, false);
      const uint32_t idesc_o = idesc_f16(128, D16, false);
      const int ksteps = (p.d + 15) / 16;  // QK^T depth: d rounded up to 16 (pads are zero)
      auto issue_qk = [&](int t, int s) {
        const uint32_t d_s = tmem + t * BKV;
        for (int kk = 0; kk < ksteps; ++kk) {
          const int a = kk >> 2;
          const uint64_t da = sdesc_sw128(smem_u32(sQ + t * CF::kQTile + a * 16384) + (kk & 3) * 32, 16, 1024);
          const uint64_t db = sdesc_sw128(smem_u32(sK + s * CF::kKTile + a * BKV * 128) + (kk & 3) * 32, 16, 1024);
          mma_f16_ss(d_s, da, db, idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(s_full(t));
      };
      // TPV: both tiles' P_j side by side (rows 0..255 of each 64-key atom) are the B operand
      auto issue_pv_both = [&](int s, int j) {
        const uint32_t d_o = tmem + NQT * BKV;
        constexpr uint32_t idesc_t = idesc_f16(64, NQT * 128, false);
        const uint8_t* pbuf = sP + (j & 1) * NQT * CF::kPTile;
        for (int kk = 0; kk < BKV / 16; ++kk) {
          const int a = kk >> 2;
          const uint64_t da = sdesc_sw128(smem_u32(sV + s * CF::kVTile + a * CF::kVAtom) + (kk & 3) * 32, 16, 1024);
          const uint64_t db = sdesc_sw128(smem_u32(pbuf + a * NQT * 16384) + (kk & 3) * 32, 16, 1024);
          mma_f16_ss(d_o, da, db, idesc_t, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(pv_full(0, j & 1));
      };
      auto issue_pv = [&](int t, int s, int j) {
        const uint32_t d_o = tmem + NQT * BKV + t * CF::PVS;
        const uint8_t* pbuf = sP + (2 * t + (j & 1)) * CF::kPTile;
        for (int kk = 0; kk < BKV / 16; ++kk) {
          const int a = kk >> 2;
          const uint64_t da = sdesc_sw128(smem_u32(pbuf + a * 16384) + (kk & 3) * 32, 16, 1024);
          const uint64_t db = sdesc_sw128(smem_u32(sV + s * CF::kVTile + a * CF::kVAtom) + (kk & 3) * 32, 16, 1024);
          mma_f16_ss(d_o, da, db, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(pv_full(t, j & 1));
      };
      bool ok = mbar_wait(q_full, 0, p.err, kDevTimeoutAttn);
      int nq[NQT], np[NQT];
      for (int t = 0; t < NQT; ++t) { nq[t] = 0; np[t] = 0; }
      int kv_loaded = 0, kv_released = 0;
      uint64_t t_last = globaltimer();
      uint32_t spins = 0;
      while (ok) {
        bool progress = false;
        if (kv_loaded < nkv && mbar_test(kv_full(kv_loaded % NKV), (kv_loaded / NKV) & 1)) {
          ++kv_loaded;
          progress = true;
          tc_fence_after();
        }
        int min_np = nkv;
#pragma unroll
        for (int t = 0; t < NQT; ++t) {
          // S buffer of tile t is free once the softmax released S(nq-1)
          if (nq[t] < kv_loaded && (nq[t] == 0 || mbar_test(s_free(t), (nq[t] - 1) & 1))) {
            tc_fence_after();
            issue_qk(t, nq[t] % NKV);
            ++nq[t];
            progress = true;
          }
          if constexpr (!CF::TPV) {
            if (np[t] < nq[t] && mbar_test(p_full(t, np[t] & 1), (np[t] >> 1) & 1)) {
              tc_fence_after();
              issue_pv(t, np[t] % NKV, np[t]);
              ++np[t];
              progress = true;
            }
            min_np = min(min_np, np[t]);
          }
        }
        if constexpr (CF::TPV) {  // np[0] counts the joint PVs
          const int k = np[0];
          if (k < nq[0] && k < nq[1] && mbar_test(p_full(0, k & 1), (k >> 1) & 1) &&
              mbar_test(p_full(1, k & 1), (k >> 1) & 1)) {
            tc_fence_after();
            issue_pv_both(k % NKV, k);
            ++np[0];
            progress = true;
          }
          min_np = np[0];
        }
        while (kv_released < min_np) {  // every tile's QK and PV of this K/V stage issued
          mma_commit(kv_empty(kv_released % NKV));
          ++kv_released;
        }
        if (kv_released == nkv) break;
        // back off while nothing is ready: mbarrier polls from the issuing thread slow the
        // tensor pipe (d=40 self-attention 136 -> 131 us with a 100 ns pause)
        if (!progress) __nanosleep(100);
        if (progress) {
          t_last = globaltimer();
          spins = 0;
        } else if ((++spins & 255u) == 0u) {
          if (*reinterpret_cast<volatile int*>(p.err) != 0) ok = false;
          else if (globaltimer() - t_last > kWaitTimeoutNs) {
            atomicCAS(p.err, 0, kDevTimeoutAttn);
            ok = false;
          }
        }
      }
      mma_commit(drain);
      mbar_drain(drain, 0, p.err, kDevTimeoutDrain);
    }
  } else if constexpr (CF::TPV) {
    // ---------------------------------------------------------------- softmax, transposed PV
    pdl_wait();
    // As the per-tile path below, but O^T accumulates in TMEM for both tiles: d row r of the
    // M=64 accumulator sits in lane (r % 16) + 32 (r / 16), query row `row` of tile t in column
    // 128 t + row. A row-max raise rescales that row's O^T column across all 64 lanes, so the
    // four warps of a tile decide rescales and aborts together (named-barrier reductions) and
    // each warp rescales the lanes of its own quadrant.
    constexpr int NCH = BKV / 32;
    constexpr float kRescale = 8.f;
    const int sw = warp - 2;
    const int t = sw >> 2;
    const int lg = warp & 3;
    const int row = lg * 32 + lane;
    const int bar_id = 1 + t;  // named barrier of this tile's 128 softmax threads
    const uint32_t lane_off = static_cast<uint32_t>(lg * 32) << 16;
    const uint32_t t_s = tmem + t * BKV + lane_off;
    const uint32_t t_ot = tmem + NQT * BKV + t * 128 + lane_off;
    float* corr_s = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 1024) + t * 128;
    const int r7 = row & 7;
    float m_used = -INFINITY;
    bool ok = true;
    auto wait_pv = [&](int k) -> bool {  // joint PV(k) complete
      return mbar_wait(pv_full(0, k & 1), (k >> 1) & 1, p.err, kDevTimeoutAttn);
    };
    for (int j = 0; j < nkv; ++j) {
      bool mine = mbar_wait(s_full(t), j & 1, p.err, kDevTimeoutAttn);
      mine = __all_sync(0xffffffffu, mine);
      uint32_t sv[NCH][32];
      float m_new = m_used, corr = 1.f;
      bool need = false;
      if (mine) {
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < NCH; ++h) tmem_ld32(t_s + 32 * h, sv[h]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free(t));
        const int kbase = j * BKV;
        if (kbase + BKV > p.Sk) {
#pragma unroll
          for (int h = 0; h < NCH; ++h)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (kbase + 32 * h + e >= p.Sk) sv[h][e] = __float_as_uint(-INFINITY);
        }
        const float m_cand = row_max<NCH>(sv) * p.sl2;
        need = m_cand > m_used + kRescale;
        m_new = need ? m_cand : m_used;
        corr = need ? ex2_approx(m_used - m_new) : 1.f;
        corr_s[row] = corr;
      }
      // a failed wait takes the rescale branch too; the barrier below then ends the loop
      const bool rescale = bar_or(bar_id, 128, need || !mine) && j > 0;
      // P buffer j%2 was read by PV(j-2); a rescale needs PV(j-1) retired as well
      bool waited = true;
      if (rescale || j >= 2) waited = wait_pv(rescale ? j - 1 : j - 2);
      waited = __all_sync(0xffffffffu, waited);
      if (waited && rescale) {
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 128; c += 16) {
          uint32_t r[16];
          tmem_ld16(t_ot + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * corr_s[c + e]);
          tmem_st16(t_ot + c, r);
        }
        tmem_wait_st();
      }
      if (!bar_and(bar_id, 128, waited && mine)) { ok = false; break; }  // also: every read of corr_s is done
      uint8_t* prow = sP + (j & 1) * NQT * CF::kPTile + (t * 128 + row) * 128;
      auto emit_chunk = [&](const uint32_t (&c32)[32], int h) {
        uint8_t* arow = prow + (h >> 1) * (NQT * 16384);
        const int q0c = (h & 1) * 4;
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float x0 = fmaf(__uint_as_float(c32[e]), p.sl2, -m_new);
          const float x1 = fmaf(__uint_as_float(c32[e + 1]), p.sl2, -m_new);
          if (CF::POLY > 0 && (e >> 1) % (16 / (CF::POLY > 0 ? CF::POLY : 1)) == 0)
            pk[e >> 1] = pack_half2(ex2_poly(x0), ex2_poly(x1));  // FMA pipe
          else
            pk[e >> 1] = ex2_f16x2(pack_half2(x0, x1));  // exponent in fp16, one MUFU op per pair
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 u = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          *reinterpret_cast<uint4*>(arow + (((q0c + q) ^ r7) << 4)) = u;
        }
      };
#pragma unroll
      for (int h = 0; h < NCH; ++h) emit_chunk(sv[h], h);
      m_used = m_new;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full(t, j & 1));
    }
    if (ok && nkv > 0) ok = bar_and(bar_id, 128, __all_sync(0xffffffffu, wait_pv(nkv - 1)));
    if (ok) {
      // O^T columns of this tile -> shared memory as [row][d] (P buffers are free now), then each
      // thread normalises its row by the ones-row sum (d row p.d) and stores it
      tc_fence_after();
      float* ob = reinterpret_cast<float*>(sP) + t * (128 * 65);
#pragma unroll 1
      for (int c = 0; c < 128; c += 16) {
        uint32_t r[16];
        tmem_ld16(t_ot + c, r);
        tmem_wait_ld();
        if (lane < 16) {
          const int d = lg * 16 + lane;
#pragma unroll
          for (int e = 0; e < 16; ++e) ob[(c + e) * 65 + d] = __uint_as_float(r[e]);
        }
      }
      bar_sync_n(bar_id, 128);
      const int qi = q0 + t * 128 + row;
      if (qi < p.Sq) {
        const float inv = 1.f / ob[row * 65 + p.d];
        const int b = bh / p.heads, h = bh % p.heads;
        __half* dst = p.o + ((size_t)b * p.Sq + qi) * p.ld_o + (size_t)h * p.d;
        for (int c = 0; c < p.d; c += 8) {
          const float* src = ob + row * 65 + c;
          uint4 u;
          u.x = pack_half2(src[0] * inv, src[1] * inv);
          u.y = pack_half2(src[2] * inv, src[3] * inv);
          u.z = pack_half2(src[4] * inv, src[5] * inv);
          u.w = pack_half2(src[6] * inv, src[7] * inv);
          *reinterpret_cast<uint4*>(dst + c) = u;
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    pdl_wait();
    // O accumulates in TMEM (PV with accumulate); a row's running max is only
    // raised when a new score exceeds it by more than 2^8 (then that O row and l
    // are rescaled through tcgen05.ld/st), so P <= 256 always fits fp16 and the
    // per-tile path is: load S, max, exp2, store P.
    static_assert(BKV % 64 == 0, "softmax path works on whole 64-key swizzle atoms");
    constexpr int NCH = BKV / 32;   // 32-key chunks of a score row
    constexpr float kRescale = 8.f;
    const int sw = warp - 2;        // 0 .. 4*NQT-1
    const int t = sw >> 2;          // query tile of this warpgroup
    const int lg = warp & 3;        // TMEM lane group
    const int row = lg * 32 + lane; // row within the query tile
    const uint32_t lane_off = static_cast<uint32_t>(lg * 32) << 16;
    const uint32_t t_s = tmem + t * BKV + lane_off;
    const uint32_t t_o = tmem + NQT * BKV + t * CF::PVS + lane_off;
    const int r7 = row & 7;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    auto wait_pv = [&](int k) -> bool {  // PV(k) complete: phase k>>1 of barrier k&1
      return mbar_wait(pv_full(t, k & 1), (k >> 1) & 1, p.err, kDevTimeoutAttn);
    };
    for (int j = 0; j < nkv; ++j) {
      ok = mbar_wait(s_full(t), j & 1, p.err, kDevTimeoutAttn);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[NCH][32];
#pragma unroll
      for (int h = 0; h < NCH; ++h) tmem_ld32(t_s + 32 * h, sv[h]);
      tmem_wait_ld();
      // S is in registers: release its TMEM so QK^T of the next tile can start
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free(t));
      const int kbase = j * BKV;
      if (kbase + BKV > p.Sk) {  // ragged last tile: masked keys score -inf (exp2 -> 0)
#pragma unroll
        for (int h = 0; h < NCH; ++h)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (kbase + 32 * h + e >= p.Sk) sv[h][e] = __float_as_uint(-INFINITY);
      }
      const float m_cand = row_max<NCH>(sv) * p.sl2;
      const bool need = m_cand > m_used + kRescale;
      const float m_new = need ? m_cand : m_used;
      const float corr = need ? ex2_approx(m_used - m_new) : 1.f;
      const bool rescale = j > 0 && __any_sync(0xffffffffu, need);
      if (rescale || j >= 2) {
        // P buffer j%2 was read by PV(j-2); an O rescale needs PV(j-1) retired as well
        ok = wait_pv(rescale ? j - 1 : j - 2);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (rescale) {
#pragma unroll
          for (int c = 0; c < D16; c += 16) {
            uint32_t r[16];
            tmem_ld16(t_o + c, r);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * corr);
            tmem_st16(t_o + c, r);
          }
          tmem_wait_st();
        }
      }
      float rs = 0.f;
      // P row in 64-key swizzle atoms of 128 rows x 128 B each
      uint8_t* prow = sP + (2 * t + (j & 1)) * CF::kPTile + row * 128;
      auto emit_chunk = [&](const uint32_t (&c32)[32], int h) {
        // keys 32h..32h+31 -> four 16-byte chunks of the 128B-swizzled K-major row of atom h/2
        uint8_t* arow = prow + (h >> 1) * 16384;
        const int q0c = (h & 1) * 4;
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          if constexpr (ONES) {
            // the ones row of V^T sums the fp16 P itself: exponent in fp16, 2^x two at a time
            pk[e >> 1] = ex2_f16x2(pack_half2(fmaf(__uint_as_float(c32[e]), p.sl2, -m_new),
                                              fmaf(__uint_as_float(c32[e + 1]), p.sl2, -m_new)));
          } else {
            const float x0 = ex2_approx(fmaf(__uint_as_float(c32[e]), p.sl2, -m_new));
            const float x1 = ex2_approx(fmaf(__uint_as_float(c32[e + 1]), p.sl2, -m_new));
            rs += x0 + x1;
            pk[e >> 1] = pack_half2(x0, x1);
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 u = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          *reinterpret_cast<uint4*>(arow + (((q0c + q) ^ r7) << 4)) = u;
        }
      };
#pragma unroll
      for (int h = 0; h < NCH; ++h) emit_chunk(sv[h], h);
      if constexpr (!ONES) l = l * corr + rs;
      m_used = m_new;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full(t, j & 1));
    }
    if (ok && nkv > 0) {
      ok = wait_pv(nkv - 1);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      float O[D16];
#pragma unroll
      for (int c = 0; c < D16; c += 16) {
        uint32_t r[16];
        tmem_ld16(t_o + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) O[c + e] = __uint_as_float(r[e]);
      }
      if constexpr (ONES) {
        // column d of the PV accumulator is the row sum of the fp16 P (same rescaling as O)
#pragma unroll
        for (int c = 0; c < D16; ++c)
          if (c == p.d) l = O[c];
      }
      const int qi = q0 + t * 128 + row;
      if (qi < p.Sq) {
        const float inv = 1.f / l;
        const int b = bh / p.heads, h = bh % p.heads;
        __half* dst = p.o + ((size_t)b * p.Sq + qi) * p.ld_o + (size_t)h * p.d;
#pragma unroll
        for (int c = 0; c < D16; c += 8) {
          if (c >= p.d) break;
          uint4 u;
          u.x = pack_half2(O[c + 0] * inv, O[c + 1] * inv);
          u.y = pack_half2(O[c + 2] * inv, O[c + 3] * inv);
          u.z = pack_half2(O[c + 4] * inv, O[c + 5] * inv);
          u.w = pack_half2(O[c + 6] * inv, O[c + 7] * inv);
          *reinterpret_cast<uint4*>(dst + c) = u;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, CF::kTmemCols);
  }
}

template <class CF>
cudaError_t launch_cfg(const AttnArgs& a, int* err, cudaStream_t s) {
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<CF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)CF::kSmem);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  if (CF::ONES && a.d >= CF::D16) return cudaErrorInvalidValue;
  CUtensorMap mq{}, mk{}, mv{};
  auto mk3 = [&](CUtensorMap* m, const __half* base, uint64_t inner, uint64_t rows, uint32_t box_rows) {
    uint64_t dims[3] = {inner, rows, (uint64_t)a.BH};
    uint64_t str[2] = {inner * 2, rows * inner * 2};
    uint32_t box[3] = {64, box_rows, 1};
    return make_tmap(m, base, 3, dims, str, box);
  };
  const uint32_t vrows = CF::ONES ? (uint32_t)a.d : (uint32_t)CF::D16;
  if (!mk3(&mq, a.q, CF::DP, a.Sq, 128) || !mk3(&mk, a.k, CF::DP, a.Sk, CF::BKV) ||
      !mk3(&mv, a.v, a.vt_ld, CF::D16, vrows))
    return cudaErrorInvalidValue;
  AttnDev d{a.heads, a.Sq, a.Sk, a.d, a.o, a.ld_o, a.scale * 1.4426950408889634f, err};
  dim3 grid((a.Sq + 128 * CF::NQT - 1) / (128 * CF::NQT), a.BH);
  return launch_kernel(attn_tc_kernel<CF>, grid, dim3(CF::kThreads), CF::kSmem, s, 0, mq, mk, mv, d);
}

}  // namespace

cudaError_t launch_attention(const AttnArgs& a, int* err, cudaStream_t s) {
  if (a.BH <= 0 || a.heads <= 0 || a.Sq <= 0 || a.Sk <= 0 || a.d % 8 || !a.q || !a.k || !a.v || !a.o)
    return cudaErrorInvalidValue;
  const int dp = (a.d + 63) / 64 * 64;
  if (a.dp != dp || a.vt_ld < a.Sk || a.vt_ld % 8 || a.d16 != (a.d + 15) / 16 * 16) return cudaErrorInvalidValue;
  // few query tiles: fewer tiles per CTA keep more SMs busy
  const bool small_q = (long)((a.Sq + 127) / 128) * a.BH < 2 * num_sms();
  switch (a.d16) {
    case 48:
      if (small_q) return launch_cfg<AttnCfg<64, 64, 2, 48, true>>(a, err, s);
      // wide QK^T, transposed PV; every exponential on the MUFU pipe (POLY = 0): moving 2 / 4 / 8 of every
      // 16 pairs to ex2_poly measured 130.2 -> 132.2 / 134.7 / 145.4 us at S = 4096 on B200 -- the softmax
      // warps are bound by issue and dependent latency, not by the MUFU pipe
      if (a.Sk >= 1024) return launch_cfg<AttnCfg<64, 128, 2, 48, true, true>>(a, err, s);
      return launch_cfg<AttnCfg<64, 64, 4, 48, true>>(a, err, s);  // short key sets (cross-attention)
    case 64: return launch_cfg<AttnCfg<64, 64, 3, 64, false>>(a, err, s);
    case 80:  // 128-key tiles; 64-key tiles for the 77 context keys (cross-attention 6.44 -> 5.65 us on B200)
      if (a.Sk <= 128) return launch_cfg<AttnCfg<128, 64, 1, 80, false>>(a, err, s);
      return launch_cfg<AttnCfg<128, 128, 1, 80, false>>(a, err, s);
    case 160: return launch_cfg<AttnCfg<192, 64, 1, 160, false>>(a, err, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace sdg
