// FlashAttention-2 backward for fp16 on sm_100a: the dQ kernel (one CTA per 128-row query tile) and
// the atomic-free dK/dV kernel (one CTA per 128-row key tile), with TMA-fed shared memory, tcgen05
// MMAs into TMEM and warp-specialised roles.
//
// Algorithm (reference src/tattn/kernels.py): P is rebuilt from the saved base-2 log-sum-exp,
// P = exp2(S * sm_scale * log2(e) - M); dS = P * (dP - D) with D = rowsum(dO * O);
//   dQ kernel    (kernels.py:242-321): S = Q K^T, dP = dO V^T, dQ += dS K, dQ *= sm_scale
//   dK/dV kernel (kernels.py:151-239): S^T = K Q^T, dP^T = V dO^T, dV += P^T dO, dK += dS^T Q, dK *= sm_scale
// No atomics: every output row is owned by exactly one CTA.
//
// All kernels run 384 threads. Warps 0-7 are two compute warpgroups; thread t of a warpgroup owns TMEM
// lane t (a query row in the dQ kernels, a key row in the dK/dV kernel). Warp 8 is the TMA producer (in
// the dK/dV kernel it also stages -M and -delta), warp 9 issues the S/dP MMAs, warp 10 the accumulating
// MMAs (dQ, or dV and dK), warp 11 allocates TMEM (and, in the D = 128 dQ kernel, issues the S/dP MMAs
// of the second warpgroup). setmaxnreg moves registers from the last warpgroup to the compute warps.
//
// TMEM holds S and dP, the fp16 operand of the accumulating MMAs (P^T and dS^T, or dS) in buffers of
// their own, and the fp32 accumulators. Because nothing is overwritten in place, the S/dP MMAs of the
// next block are issued as soon as the compute warps have loaded the current S and dP into registers,
// and run on the tensor core while the compute warps turn them into P and dS.
//   dQ, D <= 64:   128-key blocks, the warpgroups split each block's columns (64 each); persistent
//                  (one CTA per SM looping over query tiles) when not causal
//   dQ, D = 128:   64-key blocks, the warpgroups take alternate blocks and ping-pong (the 128-key
//                  layout leaves room for only two K/V ring stages at this head dim)
//   dK/dV:         128-query blocks (64 at D = 128), the warpgroups split each block's columns;
//                  persistent when not causal and D <= 64
// Persistent kernels write their outputs through shared-memory staging and TMA stores; causal grids
// keep one tile per CTA, because their tiles differ in cost and the hardware's dynamic CTA scheduling
// balances them (static round-robin was measured 6-12% slower there).
// 128-wide blocks keep every S/dP MMA at N = 128, where the tensor core, not shared-memory bandwidth,
// sets the rate (an N = 64 MMA with both operands in shared memory is bandwidth-bound at 2/3 rate).
//
// Separate issuer warps for S/dP and for the accumulating MMAs, because the tensor core accepts only a
// handful of queued MMAs: a warp that issues a longer run stalls until the earlier ones have executed,
// and each barrier wait or commit costs it a hundred cycles or more, so one issuer would serialise the
// S/dP MMAs of one block behind the accumulating MMAs of another. A ring slot is released when both
// commits for it (S/dP and accumulation) have landed.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"
#include "tiles.h"

namespace tattn {
namespace {

// Swizzled K-major fp16 tile geometry for rows of D elements: chunks of CW columns, each chunk
// [rows, CW] stored with a SWB-byte swizzle (TMA box = one chunk).
template <int D>
struct Geo {
  static constexpr int CW = D < 64 ? D : 64;
  static constexpr int NCH = D / CW;
  static constexpr int SWB = CW * 2;
  static constexpr uint32_t LAYOUT = SWB == 128 ? 2u : (SWB == 64 ? 4u : 6u);
  static constexpr int chunk(int rows) { return rows * SWB; }
  static constexpr int tile(int rows) { return rows * SWB * NCH; }
};

constexpr int kThreads = 384;
// Register split: launch = 384 x 168 = 64512; compute warps take 216, the last warpgroup keeps 72:
// 8*32*216 + 4*32*72 = 64512. (With 56 the issuer and staging warps spill.)
constexpr int kComputeRegs = 216;
constexpr int kProducerRegs = 72;
// The fused backward's issuer warps hold more descriptors (dS^T as two operands, K for dQ) and need
// more than 72 registers; its compute warps fit in 208. Both splits use the whole 384 x 168 pool.
constexpr int kFusedComputeRegs = 208;
constexpr int kFusedProducerRegs = 88;
static_assert(256 * kFusedComputeRegs + 128 * kFusedProducerRegs == 384 * 168, "register split");

constexpr int kTmaWarp = 8, kMmaSWarp = 9, kMmaAccWarp = 10, kAllocWarp = 11;
constexpr unsigned long long kDrainNs = 100ull * 1000ull * 1000ull;

// D[tmem] = A x B^T over K = D. A: 128-row K-major tile (chunk stride A_CH bytes), B: K-major tile of
// N rows (chunk stride B_CH bytes); `a`/`b` are the tiles' base descriptors.
template <int D, int A_CH, int B_CH>
__device__ __forceinline__ void mma_kmajor(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc) {
  using G = Geo<D>;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int ch = kk * 16 / G::CW, inner = ((kk * 16) % G::CW) * 2;
    mma_f16_ss_elect(d_tmem, a + uint64_t((ch * A_CH + inner) >> 4), b + uint64_t((ch * B_CH + inner) >> 4),
                     idesc, kk > 0 ? 1u : 0u);
  }
}

// D[tmem] (+)= A x B with A from TMEM (128 lanes x KSTEPS*16 fp16, 8 columns per K step) and B a
// [KSTEPS*16, D] tile read MN-major (base descriptor `b_mn`).
template <int D, int KSTEPS>
__device__ __forceinline__ void mma_tmem_mn(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_mn, uint32_t idesc,
                                            uint32_t accumulate) {
  using G = Geo<D>;
#pragma unroll
  for (int kk = 0; kk < KSTEPS; ++kk)
    mma_f16_ts_elect(d_tmem, a_tmem + kk * 8, b_mn + uint64_t((kk * 16 * G::SWB) >> 4), idesc,
                     kk > 0 ? 1u : accumulate);
}

// CTA position of a one-tile-per-CTA grid: head-major when every tile costs the same; causal grids run
// longest first within groups of heads (causal_cta_rank; 0 = the longest tile of its head).
__device__ __forceinline__ int cta_order(int nct, int zh, bool longest_first, int N, int D, int* bh) {
  if (longest_first) return causal_cta_rank(nct, zh, N, D, bh);
  *bh = blockIdx.x / nct;
  return blockIdx.x % nct;
}

__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// exp2 of a pair: on MUFU, or (EMU) on the FMA pipe.
template <bool EMU>
__device__ __forceinline__ float2 exp2_pair(uint64_t x) {
  if (EMU) return f2_unpack(exp2_poly4_x2(x));  // degree 4: gradients sum P over many rows
  const float2 v = f2_unpack(x);
  return make_float2(ex2_approx(v.x), ex2_approx(v.y));
}
// Of every 8 column pairs, this many take exp2 on the FMA pipe (degree-4 polynomial), the rest on MUFU.
// Measured on the fused backward: 2 of 8 is 1.4-1.7 % faster than all on MUFU at configs 2, 3 and a
// config-5 slice, with the same worst-case errors at full size (the polynomial's 2.7e-6 relative error
// is below the fp16 output rounding); the degree-3 polynomial at 3 of 8 was faster too but took the
// config-3 dK/dV error past 2e-3 (2.4e-3).
constexpr int kDqEmuPairs = 2;
constexpr int kDkvEmuPairs = 2;

// Write a [128, D] fp32 TMEM accumulator slice (this thread's lane, columns [c_begin, c_begin + W))
// times `mul` as fp16 to dst[c_begin .. c_begin + W).
template <int W>
__device__ __forceinline__ void store_rows(uint32_t t_acc, __half* dst, float mul, bool in_range) {
#pragma unroll
  for (int c0 = 0; c0 < W; c0 += 32) {
    constexpr int V = W < 32 ? W : 32;
    uint32_t o[V];
    tmem_load_cols<V>(t_acc + c0, o);
    tmem_wait_ld();
    reg_fence<V>(o);
    uint32_t h[V / 2];
#pragma unroll
    for (int c = 0; c < V; c += 2)
      h[c / 2] = pack_half2(__uint_as_float(o[c]) * mul, __uint_as_float(o[c + 1]) * mul);
    if (in_range) {
      uint4* p = reinterpret_cast<uint4*>(dst + c0);
#pragma unroll
      for (int v = 0; v < V / 8; ++v) p[v] = make_uint4(h[4 * v], h[4 * v + 1], h[4 * v + 2], h[4 * v + 3]);
    }
  }
}

// =============================================================================================== dQ
// dS = P * (dP - D_r) for 64 columns of one row; P = exp2(S * scale - M_r). MASK zeroes columns >= lim.
template <bool MASK>
__device__ __forceinline__ void ds_row64(const uint32_t* s, const uint32_t* dp, uint32_t* ds, uint64_t scale2,
                                         uint64_t negm2, uint64_t negd2, int lim) {
#pragma unroll
  for (int c = 0; c < 64; c += 2) {
    const uint64_t x = ffma2(f2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), scale2, negm2);
    float2 e = (((c / 2) & 7) < kDqEmuPairs) ? exp2_pair<true>(x) : exp2_pair<false>(x);
    if (MASK) {
      e.x = c < lim ? e.x : 0.f;
      e.y = c + 1 < lim ? e.y : 0.f;
    }
    const uint64_t d = fadd2(f2(__uint_as_float(dp[c]), __uint_as_float(dp[c + 1])), negd2);
    const float2 v = f2_unpack(fmul2(f2(e.x, e.y), d));
    ds[c / 2] = pack_half2(v.x, v.y);
  }
}

// ------------------------------------------------------------ dQ, D <= 64: split columns, 128 keys
// One CTA per 128-row query tile; key blocks of 128 whose columns the two compute warpgroups split
// (warpgroup w takes key columns [64w, 64w + 64) of every block). TMEM: S [128] | dP [128] | dS [64] | dQ [D].
template <int D>
struct DqSplitCfg {
  using G = Geo<D>;
  static constexpr int BK = 128;                    // key rows per block
  static constexpr int H = BK / 2;                  // key columns per compute warpgroup
  static constexpr int NS = 4;                      // K/V ring stages
  static constexpr int T_ROW = G::tile(128);
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = T_ROW;
  static constexpr int OFF_K = 2 * T_ROW;           // NS key blocks
  static constexpr int OFF_V = OFF_K + NS * T_ROW;  // NS value blocks
  static constexpr int OFF_BAR = OFF_V + NS * T_ROW;
  // q_full, kv_full[NS], kv_empty[NS], s_full, s_free, ds_full, ds_free, dq_done, fin[2]
  static constexpr int NBARS = 1 + 2 * NS + 7;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  // > 113.5 KB keeps one CTA per SM, so the 512-column TMEM allocation never waits on a neighbour.
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  static constexpr uint32_t T_S = 0, T_DP = 128, T_DS = 256, T_DQ = 320;
  static_assert(T_DQ + D <= 512, "TMEM budget");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BK, false);
  static constexpr uint32_t IDESC_DQ = idesc_f16_f32(128, D, true);
};

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dq_split_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  const BwdArgs args) {
  using C = DqSplitCfg<D>;
  using G = Geo<D>;
  constexpr int H = C::H;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q = bars;
  uint64_t* bar_kv_full = bars + 1;           // [NS]
  uint64_t* bar_kv_empty = bars + 1 + C::NS;  // [NS]
  uint64_t* bar_s_full = bars + 1 + 2 * C::NS;
  uint64_t* bar_s_free = bar_s_full + 1;
  uint64_t* bar_ds_full = bar_s_full + 2;
  uint64_t* bar_ds_free = bar_s_full + 3;
  uint64_t* bar_dq_done = bar_s_full + 4;
  uint64_t* bar_fin = bar_s_full + 5;               // [2]: one per issuer warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status, args.wait_limit_ns};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int zh = args.Z * args.H;
  const int nct = (N + 127) / 128;
  int bh;
  int cta = cta_order(nct, zh, CAUSAL, N, D, &bh);
  if (CAUSAL) cta = nct - 1 - cta;  // longest-first: the highest query tiles see the most keys
  const int zi = bh / args.H, hi = bh % args.H;
  const int NBk = (N + C::BK - 1) / C::BK;
  const int q0 = 128 * cta;
  const int n = CAUSAL ? min(q0 / C::BK + 1, NBk) : NBk;  // key blocks; q0 is a multiple of BK

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 2);  // S/dP issuer + dQ issuer
    }
    mbar_init(bar_s_full, 1);
    mbar_init(bar_s_free, 256);
    mbar_init(bar_ds_full, 256);
    mbar_init(bar_ds_free, 1);
    mbar_init(bar_dq_done, 1);
    mbar_init(&bar_fin[0], 1);
    mbar_init(&bar_fin[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kAllocWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = base_u32 + C::OFF_Q, sDO = base_u32 + C::OFF_DO;
  const uint32_t sK = base_u32 + C::OFF_K, sV = base_u32 + C::OFF_V;

  if (warp >= kTmaWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == kTmaWarp && lane == 0) {
      // -------------------------------------------------------------- TMA producer
      mbar_arrive_expect_tx(bar_q, 2 * C::T_ROW);
      for (int ch = 0; ch < G::NCH; ++ch) {
        tma_load_4d(sQ + ch * G::chunk(128), &tm_q, ch * G::CW, q0, hi, zi, bar_q);
        tma_load_4d(sDO + ch * G::chunk(128), &tm_do, ch * G::CW, q0, hi, zi, bar_q);
      }
      int c = 0;
      for (; c < n; ++c) {
        const int st = c % C::NS;
        if (c >= C::NS && !mbar_wait(&bar_kv_empty[st], ((c / C::NS) - 1) & 1, ab)) break;
        mbar_arrive_expect_tx(&bar_kv_full[st], 2 * C::T_ROW);
        for (int ch = 0; ch < G::NCH; ++ch) {
          tma_load_4d(sK + st * C::T_ROW + ch * G::chunk(128), &tm_k, ch * G::CW, c * C::BK, hi, zi, &bar_kv_full[st]);
          tma_load_4d(sV + st * C::T_ROW + ch * G::chunk(128), &tm_v, ch * G::CW, c * C::BK, hi, zi, &bar_kv_full[st]);
        }
      }
      mbar_drain(bar_q, 0, kDrainNs);
      for (int cc = max(0, c - C::NS); cc < c; ++cc) mbar_drain(&bar_kv_full[cc % C::NS], (cc / C::NS) & 1, kDrainNs);
    } else if (warp == kMmaSWarp) {
      // -------------------------------------------------------------- S/dP issuer
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      const uint64_t dQ = smem_desc(sQ, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dDO = smem_desc(sDO, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dK = smem_desc(sK, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dV = smem_desc(sV, 16, 8 * G::SWB, G::LAYOUT);
      auto issue_s_dp = [&](int c) {
        const uint64_t so = uint64_t(((c % C::NS) * C::T_ROW) >> 4);
        mma_kmajor<D, G::chunk(128), G::chunk(128)>(tmem + C::T_S, dQ, dK + so, idesc_s);
        mma_kmajor<D, G::chunk(128), G::chunk(128)>(tmem + C::T_DP, dDO, dV + so, C::IDESC_S);
        mma_commit_elect(bar_s_full);
        mma_commit_elect(&bar_kv_empty[c % C::NS]);
      };
      bool ok = n > 0 && warp_wait(bar_q, 0, ab) && warp_wait(&bar_kv_full[0], 0, ab);
      if (ok) {
        tc_fence_after();
        issue_s_dp(0);
      }
      for (int c = 0; ok && c + 1 < n; ++c) {
        const int b = c + 1;
        if (!warp_wait(bar_s_free, c & 1, ab) || !warp_wait(&bar_kv_full[b % C::NS], (b / C::NS) & 1, ab)) break;
        tc_fence_after();
        issue_s_dp(b);
      }
      mma_commit_elect(&bar_fin[0]);
      mbar_drain(&bar_fin[0], 0, kDrainNs);
    } else if (warp == kMmaAccWarp) {
      // -------------------------------------------------------------- dQ issuer
      const uint64_t dKmn = smem_desc(sK, G::chunk(128), 8 * G::SWB, G::LAYOUT);
      for (int c = 0; c < n; ++c) {
        // kv_full is complete already (the S MMA of block c needed it); waiting on it orders the K reads.
        if (!warp_wait(bar_ds_full, c & 1, ab) || !warp_wait(&bar_kv_full[c % C::NS], (c / C::NS) & 1, ab)) break;
        tc_fence_after();
        mma_tmem_mn<D, C::BK / 16>(tmem + C::T_DQ, tmem + C::T_DS,
                                   dKmn + uint64_t(((c % C::NS) * C::T_ROW) >> 4), C::IDESC_DQ, c > 0 ? 1u : 0u);
        mma_commit_elect(bar_ds_free);
        mma_commit_elect(&bar_kv_empty[c % C::NS]);
      }
      mma_commit_elect(bar_dq_done);
      mma_commit_elect(&bar_fin[1]);
      mbar_drain(&bar_fin[1], 0, kDrainNs);
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kComputeRegs));
    const int w = warp / 4;              // column half of every key block
    const int r = threadIdx.x % 128;     // query row within the tile = TMEM lane
    const int row = q0 + r;
    const uint32_t tl = tmem + (uint32_t((warp % 4) * 32) << 16);
    const int64_t rowidx = int64_t(bh) * N + row;
    const float m_r = row < N ? args.m[rowidx] : 0.f;
    const float d_r = row < N ? args.delta[rowidx] : 0.f;
    const uint64_t scale2 = f2(args.qk_scale, args.qk_scale), negm2 = f2(-m_r, -m_r), negd2 = f2(-d_r, -d_r);
    const int row_lim = CAUSAL ? min(N, row + 1) : N;  // valid key columns: key < row_lim
    bool ok = true;
    for (int c = 0; c < n; ++c) {
      if (!warp_wait(bar_s_full, c & 1, ab)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[H], dp[H];
      tmem_load_cols<H>(tl + C::T_S + w * H, s);
      tmem_load_cols<H>(tl + C::T_DP + w * H, dp);
      tmem_wait_ld();
      reg_fence<H>(s);
      reg_fence<H>(dp);
      tc_fence_before();
      mbar_arrive(bar_s_free);  // the tensor core may now write S/dP of the next block
      const int k0 = c * C::BK + w * H;
      const bool masked = (k0 + H > N) || (CAUSAL && k0 + H - 1 > q0);
      uint32_t ds[H / 2];
      if (masked)
        ds_row64<true>(s, dp, ds, scale2, negm2, negd2, row_lim - k0);
      else
        ds_row64<false>(s, dp, ds, scale2, negm2, negd2, 0);
      if (c > 0) {  // the dQ MMA of the previous block has read dS
        if (!warp_wait(bar_ds_free, (c - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
      }
      tmem_store_cols<H / 2>(tl + C::T_DS + w * (H / 2), ds);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_ds_full);
    }
    if (ok && n > 0 && warp_wait(bar_dq_done, 0, ab)) {
      tc_fence_after();
      constexpr int W = D / 2;  // each warpgroup writes half of the columns
      store_rows<W>(tl + C::T_DQ + w * W, reinterpret_cast<__half*>(args.dq) + rowidx * D + w * W, args.sm_scale,
                    row < N);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kAllocWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------- dQ, D <= 64: persistent
// One CTA per SM looping over 128-row query tiles (static round-robin over the same order as the
// one-tile-per-CTA grid: longest-first when causal). Q/dO tiles are double-buffered, the K/V ring and
// every barrier phase run on across tiles (g = global key-block index, it = tile iteration), the next
// tile's first S/dP MMAs go out while the current tile finishes, each compute warp writes its 32 rows
// of its warpgroup's dQ columns through shared-memory staging and a TMA store, and M/delta of the next
// tile are fetched before the current tile's epilogue. The first dQ MMA of a tile waits until the
// compute warps have read the previous tile's accumulator (dq_read).
template <int D>
struct DqPersistCfg {
  using G = Geo<D>;
  static_assert(D <= 64, "persistent dQ: 128-key blocks");
  static constexpr int BK = 128, H = 64;
  static constexpr int NS = 3;                          // K/V ring stages
  static constexpr int T_ROW = G::tile(128);            // [128, D] tile
  static constexpr int HW = D / 2;                      // dQ columns per compute warpgroup
  static constexpr int SWB_O = HW * 2;                  // staging row bytes (swizzle span of the store map)
  static constexpr int STG = 32 * SWB_O;                // per-warp staging: 32 rows x D/2 fp16
  static constexpr int OFF_Q = 0;                       // [2 buffers]
  static constexpr int OFF_DO = 2 * T_ROW;              // [2 buffers]
  static constexpr int OFF_K = 4 * T_ROW;               // NS key blocks
  static constexpr int OFF_V = OFF_K + NS * T_ROW;      // NS value blocks
  static constexpr int OFF_STG = OFF_V + NS * T_ROW;    // 8 compute warps x STG
  static constexpr int OFF_BAR = OFF_STG + 8 * (STG < 1024 ? 1024 : STG);
  // q_full[2], q_empty[2], kv_full[NS], kv_empty[NS], s_full, s_free, ds_full, ds_free, dq_done,
  // dq_read, fin[3]
  static constexpr int NBARS = 4 + 2 * NS + 9;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  static constexpr uint32_t T_S = 0, T_DP = 128, T_DS = 256, T_DQ = 320;
  static_assert(T_DQ + D <= 512, "TMEM budget");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(OFF_STG % 1024 == 0, "staging alignment");
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BK, false);
  static constexpr uint32_t IDESC_DQ = idesc_f16_f32(128, D, true);
};

// Query tile `tile` of the one-tile-per-CTA order: (b*h index, query tile), longest first when causal.
__device__ __forceinline__ void dq_tile(int tile, int nct, int zh, bool causal, int* bh, int* qt) {
  if (causal) {
    *bh = tile % zh;
    *qt = nct - 1 - tile / zh;
  } else {
    *bh = tile / nct;
    *qt = tile % nct;
  }
}

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dq_persist_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                          const __grid_constant__ CUtensorMap tm_dq, const BwdArgs args) {
  using C = DqPersistCfg<D>;
  using G = Geo<D>;
  constexpr int H = C::H, NS = C::NS, HW = C::HW;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q_full = bars;                  // [2] Q/dO buffer landed
  uint64_t* bar_q_empty = bars + 2;             // [2] every S/dP MMA of the buffer's tile has completed
  uint64_t* bar_kv_full = bars + 4;             // [NS]
  uint64_t* bar_kv_empty = bars + 4 + NS;       // [NS]
  uint64_t* bar_s_full = bars + 4 + 2 * NS;
  uint64_t* bar_s_free = bar_s_full + 1;
  uint64_t* bar_ds_full = bar_s_full + 2;
  uint64_t* bar_ds_free = bar_s_full + 3;
  uint64_t* bar_dq_done = bar_s_full + 4;
  uint64_t* bar_dq_read = bar_s_full + 5;       // the compute warps hold the tile's dQ in registers
  uint64_t* bar_fin = bar_s_full + 6;           // [3]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status, args.wait_limit_ns};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int zh = args.Z * args.H;
  const int nct = (N + 127) / 128;
  const int ntiles = nct * zh;
  const int NBk = (N + C::BK - 1) / C::BK;
  auto tile_n = [&](int qt) { return CAUSAL ? min(qt + 1, NBk) : NBk; };  // key blocks of query tile qt

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_q_full[b], 1);
      mbar_init(&bar_q_empty[b], 1);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 2);  // S/dP issuer + dQ issuer
    }
    mbar_init(bar_s_full, 1);
    mbar_init(bar_s_free, 256);
    mbar_init(bar_ds_full, 256);
    mbar_init(bar_ds_free, 1);
    mbar_init(bar_dq_done, 1);
    mbar_init(bar_dq_read, 256);
    for (int i = 0; i < 3; ++i) mbar_init(&bar_fin[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kAllocWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = base_u32 + C::OFF_Q, sDO = base_u32 + C::OFF_DO;
  const uint32_t sK = base_u32 + C::OFF_K, sV = base_u32 + C::OFF_V;

  if (warp >= kTmaWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == kTmaWarp && lane == 0) {
      // -------------------------------------------------------------- TMA producer
      int g = 0, it = 0, q_issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
        int bh, qt;
        dq_tile(tile, nct, zh, CAUSAL, &bh, &qt);
        const int zi = bh / args.H, hi = bh % args.H, n = tile_n(qt);
        const int qb = it & 1;
        if (it >= 2 && !mbar_wait(&bar_q_empty[qb], ((it >> 1) - 1) & 1, ab)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar_q_full[qb], 2 * C::T_ROW);
        for (int ch = 0; ch < G::NCH; ++ch) {
          tma_load_4d(sQ + qb * C::T_ROW + ch * G::chunk(128), &tm_q, ch * G::CW, 128 * qt, hi, zi, &bar_q_full[qb]);
          tma_load_4d(sDO + qb * C::T_ROW + ch * G::chunk(128), &tm_do, ch * G::CW, 128 * qt, hi, zi, &bar_q_full[qb]);
        }
        ++q_issued;
        for (int c = 0; c < n; ++c, ++g) {
          const int st = g % NS;
          if (g >= NS && !mbar_wait(&bar_kv_empty[st], ((g / NS) - 1) & 1, ab)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar_kv_full[st], 2 * C::T_ROW);
          for (int ch = 0; ch < G::NCH; ++ch) {
            tma_load_4d(sK + st * C::T_ROW + ch * G::chunk(128), &tm_k, ch * G::CW, c * C::BK, hi, zi, &bar_kv_full[st]);
            tma_load_4d(sV + st * C::T_ROW + ch * G::chunk(128), &tm_v, ch * G::CW, c * C::BK, hi, zi, &bar_kv_full[st]);
          }
        }
      }
      for (int ii = max(0, q_issued - 2); ii < q_issued; ++ii) mbar_drain(&bar_q_full[ii & 1], (ii >> 1) & 1, kDrainNs);
      for (int gg = max(0, g - NS); gg < g; ++gg) mbar_drain(&bar_kv_full[gg % NS], (gg / NS) & 1, kDrainNs);
    } else if (warp == kMmaSWarp) {
      // -------------------------------------------------------------- S/dP issuer
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      const uint64_t dQ = smem_desc(sQ, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dDO = smem_desc(sDO, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dK = smem_desc(sK, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dV = smem_desc(sV, 16, 8 * G::SWB, G::LAYOUT);
      int g = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
        int bh, qt;
        dq_tile(tile, nct, zh, CAUSAL, &bh, &qt);
        const int n = tile_n(qt);
        const int qb = it & 1;
        if (!warp_wait(&bar_q_full[qb], (it >> 1) & 1, ab)) { ok = false; break; }
        const uint64_t qo = uint64_t((qb * C::T_ROW) >> 4);
        for (int c = 0; c < n; ++c, ++g) {
          if (g > 0 && !warp_wait(bar_s_free, (g - 1) & 1, ab)) { ok = false; break; }
          if (!warp_wait(&bar_kv_full[g % NS], (g / NS) & 1, ab)) { ok = false; break; }
          tc_fence_after();
          const uint64_t so = uint64_t(((g % NS) * C::T_ROW) >> 4);
          mma_kmajor<D, G::chunk(128), G::chunk(128)>(tmem + C::T_S, dQ + qo, dK + so, idesc_s);
          mma_kmajor<D, G::chunk(128), G::chunk(128)>(tmem + C::T_DP, dDO + qo, dV + so, C::IDESC_S);
          mma_commit_elect(bar_s_full);
          mma_commit_elect(&bar_kv_empty[g % NS]);
        }
        mma_commit_elect(&bar_q_empty[qb]);  // the buffer's Q/dO have been read by every MMA of this tile
      }
      mma_commit_elect(&bar_fin[0]);
      mbar_drain(&bar_fin[0], 0, kDrainNs);
    } else if (warp == kMmaAccWarp) {
      // -------------------------------------------------------------- dQ issuer
      const uint64_t dKmn = smem_desc(sK, G::chunk(128), 8 * G::SWB, G::LAYOUT);
      int g = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
        int bh, qt;
        dq_tile(tile, nct, zh, CAUSAL, &bh, &qt);
        const int n = tile_n(qt);
        // This tile's first MMA overwrites the accumulator: the previous epilogue must have read it.
        if (it > 0 && !warp_wait(bar_dq_read, (it - 1) & 1, ab)) { ok = false; break; }
        for (int c = 0; c < n; ++c, ++g) {
          // kv_full is complete already (the S MMA of block g needed it); waiting on it orders the K reads.
          if (!warp_wait(bar_ds_full, g & 1, ab) || !warp_wait(&bar_kv_full[g % NS], (g / NS) & 1, ab)) {
            ok = false;
            break;
          }
          tc_fence_after();
          mma_tmem_mn<D, C::BK / 16>(tmem + C::T_DQ, tmem + C::T_DS, dKmn + uint64_t(((g % NS) * C::T_ROW) >> 4),
                                     C::IDESC_DQ, c > 0 ? 1u : 0u);
          mma_commit_elect(bar_ds_free);
          mma_commit_elect(&bar_kv_empty[g % NS]);
        }
        if (ok) mma_commit_elect(bar_dq_done);
      }
      mma_commit_elect(&bar_fin[2]);
      mbar_drain(&bar_fin[2], 0, kDrainNs);
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kComputeRegs));
    const int w = warp / 4;            // column half of every key block, and of dQ
    const int r = threadIdx.x % 128;   // query row within the tile = TMEM lane
    const int q4 = warp % 4;
    const uint32_t tl = tmem + (uint32_t(q4 * 32) << 16);
    const uint32_t stg = base_u32 + C::OFF_STG + warp * (C::STG < 1024 ? 1024 : C::STG);
    const uint64_t scale2 = f2(args.qk_scale, args.qk_scale);
    int g = 0, it = 0;
    bool ok = true;
    // M and delta of this thread's row in the first tile; later tiles' are fetched one tile ahead.
    float m_nx = 0.f, d_nx = 0.f;
    if (blockIdx.x < ntiles) {
      int bh, qt;
      dq_tile(blockIdx.x, nct, zh, CAUSAL, &bh, &qt);
      const int row = 128 * qt + r;
      if (row < N) {
        m_nx = args.m[int64_t(bh) * N + row];
        d_nx = args.delta[int64_t(bh) * N + row];
      }
    }
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
      int bh, qt;
      dq_tile(tile, nct, zh, CAUSAL, &bh, &qt);
      const int zi = bh / args.H, hi = bh % args.H, q0 = 128 * qt, n = tile_n(qt);
      const int row = q0 + r;
      const uint64_t negm2 = f2(-m_nx, -m_nx), negd2 = f2(-d_nx, -d_nx);
      const int row_lim = CAUSAL ? min(N, row + 1) : N;  // valid key columns: key < row_lim
      for (int c = 0; c < n; ++c, ++g) {
        if (!warp_wait(bar_s_full, g & 1, ab)) { ok = false; break; }
        tc_fence_after();
        uint32_t s[H], dp[H];
        tmem_load_cols<H>(tl + C::T_S + w * H, s);
        tmem_load_cols<H>(tl + C::T_DP + w * H, dp);
        tmem_wait_ld();
        reg_fence<H>(s);
        reg_fence<H>(dp);
        tc_fence_before();
        mbar_arrive(bar_s_free);  // the tensor core may now write S/dP of the next block
        const int k0 = c * C::BK + w * H;
        const bool masked = (k0 + H > N) || (CAUSAL && k0 + H - 1 > q0);
        uint32_t ds[H / 2];
        if (masked)
          ds_row64<true>(s, dp, ds, scale2, negm2, negd2, row_lim - k0);
        else
          ds_row64<false>(s, dp, ds, scale2, negm2, negd2, 0);
        if (g > 0) {  // the dQ MMA of the previous block has read dS
          if (!warp_wait(bar_ds_free, (g - 1) & 1, ab)) { ok = false; break; }
          tc_fence_after();
        }
        tmem_store_cols<H / 2>(tl + C::T_DS + w * (H / 2), ds);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_ds_full);
      }
      if (!ok) break;
      // M and delta of the next tile's row, in flight during this epilogue.
      if (tile + int(gridDim.x) < ntiles) {
        int bh2, qt2;
        dq_tile(tile + gridDim.x, nct, zh, CAUSAL, &bh2, &qt2);
        const int row2 = 128 * qt2 + r;
        m_nx = row2 < N ? args.m[int64_t(bh2) * N + row2] : 0.f;
        d_nx = row2 < N ? args.delta[int64_t(bh2) * N + row2] : 0.f;
      }
      if (!warp_wait(bar_dq_done, it & 1, ab)) { ok = false; break; }
      // ---- epilogue: this warpgroup's dQ columns [w*HW, w*HW + HW) * sm_scale, 32 rows per warp
      tc_fence_after();
      uint32_t o[HW];
      tmem_load_cols<HW>(tl + C::T_DQ + w * HW, o);
      tmem_wait_ld();
      reg_fence<HW>(o);
      tc_fence_before();
      mbar_arrive(bar_dq_read);  // the next tile's first dQ MMA may overwrite the accumulator
      if (lane == 0) tma_store_wait_read_all();  // this warp's previous store has left the staging area
      __syncwarp();
      const float mul = args.sm_scale;
#pragma unroll
      for (int u = 0; u < C::SWB_O / 16; ++u) {
        const int c = u * 8;
        const uint32_t addr = stg + swizzle_offset<C::SWB_O>(uint32_t(lane * C::SWB_O + u * 16));
        const uint32_t h0 = pack_half2(__uint_as_float(o[c + 0]) * mul, __uint_as_float(o[c + 1]) * mul);
        const uint32_t h1 = pack_half2(__uint_as_float(o[c + 2]) * mul, __uint_as_float(o[c + 3]) * mul);
        const uint32_t h2 = pack_half2(__uint_as_float(o[c + 4]) * mul, __uint_as_float(o[c + 5]) * mul);
        const uint32_t h3 = pack_half2(__uint_as_float(o[c + 6]) * mul, __uint_as_float(o[c + 7]) * mul);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(h0), "r"(h1), "r"(h2), "r"(h3)
                     : "memory");
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {  // rows past N are clipped by the tensor map
        tma_store_4d(&tm_dq, stg, w * HW, q0 + 32 * q4, hi, zi);
        tma_store_commit();
      }
    }
    if (lane == 0) tma_store_wait_all();  // the staging area must stay valid until the stores are done
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kAllocWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------- dQ, D = 128: alternating 64-key blocks
// One CTA per 128-row query tile; key blocks of 64 rows. (128-key blocks as above would leave room for
// only two K/V ring stages at D = 128.) Compute warpgroup w takes the blocks c with c % 2 == w, each
// into its own S/dP/dS TMEM buffers, and the warpgroups ping-pong: the exponentials of block c start
// when the other warpgroup has finished those of block c-1, so one warpgroup's waits and TMEM traffic
// overlap the other's exponentials.
template <int D>
struct DqAltCfg {
  using G = Geo<D>;
  static constexpr int BK = 64;                      // key rows per block
  static constexpr int NS = 4;                       // K/V ring stages
  static constexpr int T_ROW = G::tile(128);         // [128, D] Q or dO tile
  static constexpr int T_BLK = G::tile(BK);          // [64, D] key or value block
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = T_ROW;
  static constexpr int OFF_K = 2 * T_ROW;            // NS key blocks
  static constexpr int OFF_V = OFF_K + NS * T_BLK;   // NS value blocks
  static constexpr int OFF_BAR = OFF_V + NS * T_BLK;
  // q_ready, kv_full[NS], kv_empty[NS], s_full[2], s_free[2], ds_full[2][2], ds_free[2][2], dq_done,
  // fin[3], tok[2]
  static constexpr int NBARS = 1 + 2 * NS + 18;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  // > 113.5 KB keeps one CTA per SM, so the 512-column TMEM allocation never waits on a neighbour.
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  // TMEM columns: S0 dP0 S1 dP1 [64 each] | dS [2 warpgroups x 2 buffers, 32 each] | dQ [D]. Two dS
  // buffers per warpgroup: storing block c's dS waits only for the dQ MMA of block c-4.
  static constexpr uint32_t T_DQ = 384;
  static __device__ __forceinline__ uint32_t t_s(int w) { return 128 * w; }
  static __device__ __forceinline__ uint32_t t_dp(int w) { return 128 * w + 64; }
  static __device__ __forceinline__ uint32_t t_ds(int w, int b) { return 256 + 64 * w + 32 * b; }
  static_assert(T_DQ + D <= 512, "TMEM budget");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BK, false);
  static constexpr uint32_t IDESC_DQ = idesc_f16_f32(128, D, true);
};

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dq_alt_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  const BwdArgs args) {
  using C = DqAltCfg<D>;
  using G = Geo<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q = bars;                      // Q and dO landed
  uint64_t* bar_kv_full = bars + 1;            // [NS]
  uint64_t* bar_kv_empty = bars + 1 + C::NS;   // [NS]
  uint64_t* bar_s_full = bars + 1 + 2 * C::NS; // [2] per warpgroup
  uint64_t* bar_s_free = bar_s_full + 2;       // [2]
  uint64_t* bar_ds_full = bar_s_full + 4;      // [2 warpgroups][2 buffers]
  uint64_t* bar_ds_free = bar_s_full + 8;      // [2 warpgroups][2 buffers]
  uint64_t* bar_dq_done = bar_s_full + 12;
  uint64_t* bar_fin = bar_s_full + 13;         // [3]: one per issuer warp
  uint64_t* bar_tok = bar_s_full + 16;         // [2]: warpgroup w may start its exponentials
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status, args.wait_limit_ns};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int zh = args.Z * args.H;
  const int nct = (N + 127) / 128;
  int bh;
  int cta = cta_order(nct, zh, CAUSAL, N, D, &bh);
  if (CAUSAL) cta = nct - 1 - cta;  // longest-first: the highest query tiles see the most keys
  const int zi = bh / args.H, hi = bh % args.H;
  const int NBk = (N + C::BK - 1) / C::BK;
  const int q0 = 128 * cta;
  const int n = CAUSAL ? min(q0 / C::BK + 128 / C::BK, NBk) : NBk;  // key blocks; q0 is a multiple of BK

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 2);  // S/dP issuer + dQ issuer
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&bar_s_full[w], 1);
      mbar_init(&bar_s_free[w], 128);
      mbar_init(&bar_ds_full[2 * w], 128);
      mbar_init(&bar_ds_full[2 * w + 1], 128);
      mbar_init(&bar_ds_free[2 * w], 1);
      mbar_init(&bar_ds_free[2 * w + 1], 1);
      mbar_init(&bar_fin[w], 1);
      mbar_init(&bar_tok[w], 128);
    }
    mbar_init(&bar_fin[2], 1);
    mbar_init(bar_dq_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kAllocWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = base_u32 + C::OFF_Q, sDO = base_u32 + C::OFF_DO;
  const uint32_t sK = base_u32 + C::OFF_K, sV = base_u32 + C::OFF_V;

  if (warp >= kTmaWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == kTmaWarp && lane == 0) {
      // -------------------------------------------------------------- TMA producer
      mbar_arrive_expect_tx(bar_q, 2 * C::T_ROW);
      for (int ch = 0; ch < G::NCH; ++ch) {
        tma_load_4d(sQ + ch * G::chunk(128), &tm_q, ch * G::CW, q0, hi, zi, bar_q);
        tma_load_4d(sDO + ch * G::chunk(128), &tm_do, ch * G::CW, q0, hi, zi, bar_q);
      }
      int c = 0;
      for (; c < n; ++c) {
        const int st = c % C::NS;
        if (c >= C::NS && !mbar_wait(&bar_kv_empty[st], ((c / C::NS) - 1) & 1, ab)) break;
        mbar_arrive_expect_tx(&bar_kv_full[st], 2 * C::T_BLK);
        for (int ch = 0; ch < G::NCH; ++ch) {
          tma_load_4d(sK + st * C::T_BLK + ch * G::chunk(C::BK), &tm_k, ch * G::CW, c * C::BK, hi, zi, &bar_kv_full[st]);
          tma_load_4d(sV + st * C::T_BLK + ch * G::chunk(C::BK), &tm_v, ch * G::CW, c * C::BK, hi, zi, &bar_kv_full[st]);
        }
      }
      mbar_drain(bar_q, 0, kDrainNs);
      for (int cc = max(0, c - C::NS); cc < c; ++cc) mbar_drain(&bar_kv_full[cc % C::NS], (cc / C::NS) & 1, kDrainNs);
    } else if (warp == kMmaSWarp || warp == kAllocWarp) {
      // -------------------------------------------------------------- S/dP issuer of warpgroup w
      const int w = warp == kMmaSWarp ? 0 : 1;
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      const uint64_t dQ = smem_desc(sQ, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dDO = smem_desc(sDO, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dK = smem_desc(sK, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dV = smem_desc(sV, 16, 8 * G::SWB, G::LAYOUT);
      if (w < n && warp_wait(bar_q, 0, ab)) {
        for (int i = 0, c = w; c < n; ++i, c += 2) {
          if (i > 0 && !warp_wait(&bar_s_free[w], (i - 1) & 1, ab)) break;
          if (!warp_wait(&bar_kv_full[c % C::NS], (c / C::NS) & 1, ab)) break;
          tc_fence_after();
          const uint64_t so = uint64_t(((c % C::NS) * C::T_BLK) >> 4);
          mma_kmajor<D, G::chunk(128), G::chunk(C::BK)>(tmem + C::t_s(w), dQ, dK + so, idesc_s);
          mma_kmajor<D, G::chunk(128), G::chunk(C::BK)>(tmem + C::t_dp(w), dDO, dV + so, C::IDESC_S);
          mma_commit_elect(&bar_s_full[w]);
          mma_commit_elect(&bar_kv_empty[c % C::NS]);
        }
      }
      mma_commit_elect(&bar_fin[w]);
      mbar_drain(&bar_fin[w], 0, kDrainNs);
    } else if (warp == kMmaAccWarp) {
      // -------------------------------------------------------------- dQ issuer
      const uint64_t dKmn = smem_desc(sK, G::chunk(C::BK), 8 * G::SWB, G::LAYOUT);
      for (int c = 0; c < n; ++c) {
        const int w = c & 1, i = c >> 1;
        // kv_full is complete already (the S MMA of block c needed it); waiting on it orders the K reads.
        if (!warp_wait(&bar_ds_full[2 * w + (i & 1)], (i >> 1) & 1, ab) ||
            !warp_wait(&bar_kv_full[c % C::NS], (c / C::NS) & 1, ab))
          break;
        tc_fence_after();
        mma_tmem_mn<D, C::BK / 16>(tmem + C::T_DQ, tmem + C::t_ds(w, i & 1),
                                   dKmn + uint64_t(((c % C::NS) * C::T_BLK) >> 4), C::IDESC_DQ, c > 0 ? 1u : 0u);
        mma_commit_elect(&bar_ds_free[2 * w + (i & 1)]);
        mma_commit_elect(&bar_kv_empty[c % C::NS]);
      }
      mma_commit_elect(bar_dq_done);
      mma_commit_elect(&bar_fin[2]);
      mbar_drain(&bar_fin[2], 0, kDrainNs);
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kComputeRegs));
    const int w = warp / 4;              // takes key blocks c = w, w + 2, ...
    const int r = threadIdx.x % 128;     // query row within the tile = TMEM lane
    const int row = q0 + r;
    const uint32_t tl = tmem + (uint32_t((warp % 4) * 32) << 16);
    const int64_t rowidx = int64_t(bh) * N + row;
    const float m_r = row < N ? args.m[rowidx] : 0.f;
    const float d_r = row < N ? args.delta[rowidx] : 0.f;
    const uint64_t scale2 = f2(args.qk_scale, args.qk_scale), negm2 = f2(-m_r, -m_r), negd2 = f2(-d_r, -d_r);
    const int row_lim = CAUSAL ? min(N, row + 1) : N;  // valid key columns: key < row_lim
    bool ok = true;
    for (int i = 0, c = w; c < n; ++i, c += 2) {
      if (!warp_wait(&bar_s_full[w], i & 1, ab)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[64], dp[64];
      tmem_load_cols<64>(tl + C::t_s(w), s);
      tmem_load_cols<64>(tl + C::t_dp(w), dp);
      tmem_wait_ld();
      reg_fence<64>(s);
      reg_fence<64>(dp);
      tc_fence_before();
      mbar_arrive(&bar_s_free[w]);  // the tensor core may now write this warpgroup's S/dP of block c+2
      // Ping-pong: the exponentials of block c start after the other warpgroup's of block c-1 ended.
      if (c > 0) {
        if (!warp_wait(&bar_tok[w], (w ? i : i - 1) & 1, ab)) { ok = false; break; }
      }
      const int k0 = c * C::BK;
      const bool masked = (k0 + C::BK > N) || (CAUSAL && k0 + C::BK - 1 > q0);
      uint32_t ds[32];
      if (masked)
        ds_row64<true>(s, dp, ds, scale2, negm2, negd2, row_lim - k0);
      else
        ds_row64<false>(s, dp, ds, scale2, negm2, negd2, 0);
      mbar_arrive(&bar_tok[w ^ 1]);
      if (i > 1) {  // the dQ MMA of block c-4 has read this dS buffer
        if (!warp_wait(&bar_ds_free[2 * w + (i & 1)], ((i >> 1) - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
      }
      tmem_store_cols<32>(tl + C::t_ds(w, i & 1), ds);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_ds_full[2 * w + (i & 1)]);
    }
    if (ok && n > 0 && warp_wait(bar_dq_done, 0, ab)) {
      tc_fence_after();
      constexpr int W = D / 2;  // each warpgroup writes half of the columns
      store_rows<W>(tl + C::T_DQ + w * W, reinterpret_cast<__half*>(args.dq) + rowidx * D + w * W, args.sm_scale,
                    row < N);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kAllocWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================================ dK/dV
// P^T and dS^T for H query columns of one key row, from the staged -M and -delta of those columns.
// MASK keeps only columns c_lo <= c < c_hi.
template <int H, bool MASK>
__device__ __forceinline__ void pds_row(const uint32_t* s, const uint32_t* dp, const float* negm_q,
                                        const float* negd_q, uint32_t* pt, uint32_t* dst, uint64_t scale2, int c_lo,
                                        int c_hi) {
#pragma unroll
  for (int c = 0; c < H; c += 4) {
    const float4 mv = *reinterpret_cast<const float4*>(negm_q + c);
    const float4 dv = *reinterpret_cast<const float4*>(negd_q + c);
#pragma unroll
    for (int h = 0; h < 4; h += 2) {
      const int cc = c + h;
      const uint64_t negm = f2(h ? mv.z : mv.x, h ? mv.w : mv.y);
      const uint64_t negd = f2(h ? dv.z : dv.x, h ? dv.w : dv.y);
      const uint64_t x = ffma2(f2(__uint_as_float(s[cc]), __uint_as_float(s[cc + 1])), scale2, negm);
      float2 e = (((cc / 2) & 7) < kDkvEmuPairs) ? exp2_pair<true>(x) : exp2_pair<false>(x);
      if (MASK) {
        e.x = (cc >= c_lo && cc < c_hi) ? e.x : 0.f;
        e.y = (cc + 1 >= c_lo && cc + 1 < c_hi) ? e.y : 0.f;
      }
      pt[cc / 2] = pack_half2(e.x, e.y);
      const uint64_t d = fadd2(f2(__uint_as_float(dp[cc]), __uint_as_float(dp[cc + 1])), negd);
      const float2 v = f2_unpack(fmul2(f2(e.x, e.y), d));
      dst[cc / 2] = pack_half2(v.x, v.y);
    }
  }
}

// The scale the folded -M step divides by: qk_scale, but at least 2^-60, so that sm_scale = 0 (or any
// tinier one) still folds: x = s_eff * (S - M / s_eff) = -M + s_eff * S, and s_eff * S < 2^-60 * |S| is
// far below an fp32 ulp of M whenever qk_scale is below s_eff. Staging and compute use the same value.
__device__ __forceinline__ float fold_scale(float qk_scale) { return fmaxf(qk_scale, 0x1p-60f); }

// v as the sum of three bf16 values (exact: each step leaves at most 8 fewer significant bits).
__device__ __forceinline__ void split_bf16x3(float v, uint32_t* h) {
  const __nv_bfloat16 a = __float2bfloat16_rn(v);
  const float r1 = v - __bfloat162float(a);
  const __nv_bfloat16 b = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(b);
  const __nv_bfloat16 c = __float2bfloat16_rn(r2);
  h[0] = __bfloat16_as_ushort(a);
  h[1] = __bfloat16_as_ushort(b);
  h[2] = __bfloat16_as_ushort(c);
}

// P^T and dS^T for H query columns of one key row of the fused backward, whose S^T and dP^T already hold
// S^T - M/qk_scale and dP^T - delta (folded into the MMAs): P = exp2(S'^T * qk_scale), dS = P * dP'^T.
// MASK keeps only columns c_lo <= c < c_hi.
template <int H, bool MASK>
__device__ __forceinline__ void pds_row_folded(const uint32_t* s, const uint32_t* dp, uint32_t* pt, uint32_t* dst,
                                               uint64_t scale2, int c_lo, int c_hi) {
#pragma unroll
  for (int c = 0; c < H; c += 2) {
    const uint64_t x = fmul2(f2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), scale2);
    float2 e = (((c / 2) & 7) < kDkvEmuPairs) ? exp2_pair<true>(x) : exp2_pair<false>(x);
    if (MASK) {
      e.x = (c >= c_lo && c < c_hi) ? e.x : 0.f;
      e.y = (c + 1 >= c_lo && c + 1 < c_hi) ? e.y : 0.f;
    }
    pt[c / 2] = pack_half2(e.x, e.y);
    const float2 v = f2_unpack(fmul2(f2(e.x, e.y), f2(__uint_as_float(dp[c]), __uint_as_float(dp[c + 1]))));
    dst[c / 2] = pack_half2(v.x, v.y);
  }
}

// TMA producer of the split dK/dV kernel (whole warp; lane 0 issues the copies): the CTA's key and value
// tiles once, then per query block its Q and dO blocks (ring slot c % NS) and, staged by all lanes, the
// -M / -delta values of its BQ queries: FOLD, the bf16 parts of -M/qk_scale and -delta (16 bytes a query,
// the B operand of the folded K step of the S^T / dP^T MMAs, as in the fused kernel); otherwise -M and
// -delta as fp32 (BQ of each) for the compute warps to read.
template <int D, int BQ, int NS, bool FOLD>
__device__ __forceinline__ void dkdv_producer(const CUtensorMap* tm_q, const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                                              const CUtensorMap* tm_do, const BwdArgs& args, uint32_t sK, uint32_t sV,
                                              uint32_t sQ, uint32_t sDO, uint8_t* md, uint64_t* bar_kv,
                                              uint64_t* bar_q_full, uint64_t* bar_md_full, uint64_t* bar_q_empty,
                                              int bh, int zi, int hi, int k0, int lo, int n, const CtaAbort& ab) {
  using G = Geo<D>;
  constexpr int T_KEY = G::tile(128), T_Q = G::tile(BQ);
  const int lane = threadIdx.x % 32;
  const int N = args.N;
  if (lane == 0) {
    mbar_arrive_expect_tx(bar_kv, 2 * T_KEY);
    for (int ch = 0; ch < G::NCH; ++ch) {
      tma_load_4d(sK + ch * G::chunk(128), tm_k, ch * G::CW, k0, hi, zi, bar_kv);
      tma_load_4d(sV + ch * G::chunk(128), tm_v, ch * G::CW, k0, hi, zi, bar_kv);
    }
  }
  const float* mrow = args.m + int64_t(bh) * N;
  const float* drow = args.delta + int64_t(bh) * N;
  int c = 0;
  for (; c < n; ++c) {
    const int st = c % NS;
    if (c >= NS && !warp_wait(&bar_q_empty[st], ((c / NS) - 1) & 1, ab)) break;
    const int qr = (lo + c) * BQ;
    if (lane == 0) {
      mbar_arrive_expect_tx(&bar_q_full[st], 2 * T_Q);
      for (int ch = 0; ch < G::NCH; ++ch) {
        tma_load_4d(sQ + st * T_Q + ch * G::chunk(BQ), tm_q, ch * G::CW, qr, hi, zi, &bar_q_full[st]);
        tma_load_4d(sDO + st * T_Q + ch * G::chunk(BQ), tm_do, ch * G::CW, qr, hi, zi, &bar_q_full[st]);
      }
    }
    if constexpr (FOLD) {
      uint8_t* slot = md + st * BQ * 16;
      const float inv_scale = 1.f / fold_scale(args.qk_scale);
#pragma unroll
      for (int j = lane; j < BQ; j += 32) {
        const int q = qr + j;
        uint32_t hm[3], hd[3];
        split_bf16x3(q < N ? -mrow[q] * inv_scale : 0.f, hm);
        split_bf16x3(q < N ? -drow[q] : 0.f, hd);
        *reinterpret_cast<uint4*>(slot + j * 16) =
            make_uint4(hm[0] | (hm[1] << 16), hm[2] | (hd[0] << 16), hd[1] | (hd[2] << 16), 0u);
      }
      fence_proxy_async_smem();  // read by the S^T / dP^T MMAs through the async proxy
    } else {
      float* slot = reinterpret_cast<float*>(md) + st * 2 * BQ;
#pragma unroll
      for (int j = lane; j < BQ; j += 32) {
        const int q = qr + j;
        slot[j] = q < N ? -mrow[q] : 0.f;
        slot[BQ + j] = q < N ? -drow[q] : 0.f;
      }
    }
    mbar_arrive(&bar_md_full[st]);
  }
  if (lane == 0) {
    mbar_drain(bar_kv, 0, kDrainNs);
    for (int cc = max(0, c - NS); cc < c; ++cc) mbar_drain(&bar_q_full[cc % NS], (cc / NS) & 1, kDrainNs);
  }
}

// ------------------------------------------------------------------- dK/dV, D <= 64: persistent
// One CTA per SM looping over 128-row key tiles (static round-robin over the same longest-first tile
// order as the one-tile-per-CTA grid), so a tile's setup, first loads and epilogue overlap its
// neighbours' work: K/V tiles are double-buffered (the next tile's are loaded during the current one),
// the Q/dO ring and every barrier phase run on across tiles (counters g = global block index and
// it = tile iteration), the next tile's first S^T/dP^T MMAs are issued as soon as the current tile's
// last ones are in registers, and dV/dK leave through per-warp shared-memory staging and TMA stores
// instead of per-thread row stores. The first dV/dK MMA of a tile waits until the compute warps have
// read the previous tile's accumulators (acc_read).
template <int D>
struct DkvPersistCfg {
  using G = Geo<D>;
  static_assert(D <= 64, "persistent dK/dV: 128-query blocks");
  static constexpr int BQ = 128, H = 64;
  static constexpr int NS = 4;                            // Q/dO ring stages
  static constexpr int T_KEY = G::tile(128);
  static constexpr int T_Q = G::tile(BQ);
  static constexpr int HW = D / 2;                        // columns per store round (two rounds)
  static constexpr int SWB_O = HW * 2;                    // staging row bytes (swizzle span of the store map)
  static constexpr int STG = 32 * SWB_O < 1024 ? 1024 : 32 * SWB_O;  // per-warp staging: 32 rows x D/2 fp16
  static constexpr int OFF_K = 0;                         // [2 buffers] key tiles
  static constexpr int OFF_V = 2 * T_KEY;                 // [2 buffers] value tiles
  static constexpr int OFF_Q = 4 * T_KEY;                 // NS query blocks
  static constexpr int OFF_DO = OFF_Q + NS * T_Q;         // NS dO blocks
  static constexpr int OFF_STG = OFF_DO + NS * T_Q;       // 8 compute warps x STG (1024-aligned)
  static constexpr int OFF_MD = OFF_STG + 8 * STG;        // NS x (BQ -M | BQ -delta) fp32
  static constexpr int OFF_BAR = OFF_MD + NS * 2 * BQ * 4;
  // kv_full[2], kv_empty[2], q_full[NS], md_full[NS], q_empty[NS], s_full, s_free, p_full, acc_free,
  // acc_done, acc_read, fin[3]
  static constexpr int NBARS = 4 + 3 * NS + 9;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  static constexpr uint32_t T_ST = 0, T_DPT = BQ, T_PT = 2 * BQ, T_DST = 2 * BQ + BQ / 2;
  static constexpr uint32_t T_DV = 3 * BQ, T_DK = 3 * BQ + D;
  static_assert(3 * BQ + 2 * D <= 512, "TMEM budget");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(OFF_STG % 1024 == 0 && STG % 1024 == 0, "staging alignment");
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BQ, false);
  static constexpr uint32_t IDESC_ACC = idesc_f16_f32(128, D, true);
};

// Tile `tile` of the longest-first order (as cta_order over the same grid): (b*h index, key tile).
__device__ __forceinline__ void dkdv_tile(int tile, int nct, int zh, bool causal, int* bh, int* kt) {
  if (causal) {
    *bh = tile % zh;
    *kt = tile / zh;
  } else {
    *bh = tile / nct;
    *kt = tile % nct;
  }
}

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dkdv_persist_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                            const __grid_constant__ CUtensorMap tm_dk, const __grid_constant__ CUtensorMap tm_dv,
                            const BwdArgs args) {
  using C = DkvPersistCfg<D>;
  using G = Geo<D>;
  constexpr int H = C::H, BQ = C::BQ, NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_kv_full = bars;                 // [2] key/value buffer landed
  uint64_t* bar_kv_empty = bars + 2;            // [2] every S^T/dP^T MMA of the buffer's tile has completed
  uint64_t* bar_q_full = bars + 4;              // [NS]
  uint64_t* bar_md_full = bars + 4 + NS;        // [NS]
  uint64_t* bar_q_empty = bars + 4 + 2 * NS;    // [NS]
  uint64_t* bar_s_full = bars + 4 + 3 * NS;
  uint64_t* bar_s_free = bar_s_full + 1;
  uint64_t* bar_p_full = bar_s_full + 2;
  uint64_t* bar_acc_free = bar_s_full + 3;
  uint64_t* bar_acc_done = bar_s_full + 4;
  uint64_t* bar_acc_read = bar_s_full + 5;      // the compute warps hold the tile's dV/dK in registers
  uint64_t* bar_fin = bar_s_full + 6;           // [3]
  float* md = reinterpret_cast<float*>(smem + C::OFF_MD);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status, args.wait_limit_ns};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int zh = args.Z * args.H;
  const int nct = (N + 127) / 128;
  const int ntiles = nct * zh;
  const int NBq = (N + BQ - 1) / BQ;
  // Query blocks of a key tile kt: [lo, NBq).
  auto tile_lo = [&](int kt) { return CAUSAL ? (128 * kt) / BQ : 0; };

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_kv_full[b], 1);
      mbar_init(&bar_kv_empty[b], 1);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bar_q_full[s], 1);
      mbar_init(&bar_md_full[s], 32);
      mbar_init(&bar_q_empty[s], 2);  // S^T/dP^T issuer + dV/dK issuer
    }
    mbar_init(bar_s_full, 1);
    mbar_init(bar_s_free, 256);
    mbar_init(bar_p_full, 256);
    mbar_init(bar_acc_free, 1);
    mbar_init(bar_acc_done, 1);
    mbar_init(bar_acc_read, 256);
    for (int i = 0; i < 3; ++i) mbar_init(&bar_fin[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kAllocWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sK = base_u32 + C::OFF_K, sV = base_u32 + C::OFF_V;
  const uint32_t sQ = base_u32 + C::OFF_Q, sDO = base_u32 + C::OFF_DO;

  if (warp >= kTmaWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == kTmaWarp) {
      // -------------------------------------------------------------- TMA producer + -M/-delta staging
      int g = 0, it = 0, kv_issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
        int bh, kt;
        dkdv_tile(tile, nct, zh, CAUSAL, &bh, &kt);
        const int zi = bh / args.H, hi = bh % args.H, k0 = 128 * kt, lo = tile_lo(kt), n = NBq - lo;
        const int kb = it & 1;
        if (it >= 2 && !warp_wait(&bar_kv_empty[kb], ((it >> 1) - 1) & 1, ab)) { ok = false; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(&bar_kv_full[kb], 2 * C::T_KEY);
          for (int ch = 0; ch < G::NCH; ++ch) {
            tma_load_4d(sK + kb * C::T_KEY + ch * G::chunk(128), &tm_k, ch * G::CW, k0, hi, zi, &bar_kv_full[kb]);
            tma_load_4d(sV + kb * C::T_KEY + ch * G::chunk(128), &tm_v, ch * G::CW, k0, hi, zi, &bar_kv_full[kb]);
          }
        }
        ++kv_issued;
        const float* mrow = args.m + int64_t(bh) * N;
        const float* drow = args.delta + int64_t(bh) * N;
        for (int c = 0; c < n; ++c, ++g) {
          const int st = g % NS;
          if (g >= NS && !warp_wait(&bar_q_empty[st], ((g / NS) - 1) & 1, ab)) { ok = false; break; }
          const int qr = (lo + c) * BQ;
          if (lane == 0) {
            mbar_arrive_expect_tx(&bar_q_full[st], 2 * C::T_Q);
            for (int ch = 0; ch < G::NCH; ++ch) {
              tma_load_4d(sQ + st * C::T_Q + ch * G::chunk(BQ), &tm_q, ch * G::CW, qr, hi, zi, &bar_q_full[st]);
              tma_load_4d(sDO + st * C::T_Q + ch * G::chunk(BQ), &tm_do, ch * G::CW, qr, hi, zi, &bar_q_full[st]);
            }
          }
          float* slot = md + st * 2 * BQ;
#pragma unroll
          for (int j = lane; j < BQ; j += 32) {
            const int q = qr + j;
            slot[j] = q < N ? -mrow[q] : 0.f;
            slot[BQ + j] = q < N ? -drow[q] : 0.f;
          }
          mbar_arrive(&bar_md_full[st]);
        }
      }
      // Every copy issued must land before the CTA exits (instant on the normal path).
      if (lane == 0) {
        for (int ii = max(0, kv_issued - 2); ii < kv_issued; ++ii) mbar_drain(&bar_kv_full[ii & 1], (ii >> 1) & 1, kDrainNs);
        for (int gg = max(0, g - NS); gg < g; ++gg) mbar_drain(&bar_q_full[gg % NS], (gg / NS) & 1, kDrainNs);
      }
    } else if (warp == kMmaSWarp) {
      // -------------------------------------------------------------- S^T/dP^T issuer
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      const uint64_t dK = smem_desc(sK, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dV = smem_desc(sV, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dQ = smem_desc(sQ, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dDO = smem_desc(sDO, 16, 8 * G::SWB, G::LAYOUT);
      int g = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
        int bh, kt;
        dkdv_tile(tile, nct, zh, CAUSAL, &bh, &kt);
        const int n = NBq - tile_lo(kt);
        const int kb = it & 1;
        if (!warp_wait(&bar_kv_full[kb], (it >> 1) & 1, ab)) { ok = false; break; }
        const uint64_t ko = uint64_t((kb * C::T_KEY) >> 4);
        for (int c = 0; c < n; ++c, ++g) {
          if (g > 0 && !warp_wait(bar_s_free, (g - 1) & 1, ab)) { ok = false; break; }
          if (!warp_wait(&bar_q_full[g % NS], (g / NS) & 1, ab)) { ok = false; break; }
          tc_fence_after();
          const uint64_t so = uint64_t(((g % NS) * C::T_Q) >> 4);
          mma_kmajor<D, G::chunk(128), G::chunk(BQ)>(tmem + C::T_ST, dK + ko, dQ + so, idesc_s);
          mma_kmajor<D, G::chunk(128), G::chunk(BQ)>(tmem + C::T_DPT, dV + ko, dDO + so, C::IDESC_S);
          mma_commit_elect(bar_s_full);
          mma_commit_elect(&bar_q_empty[g % NS]);
        }
        mma_commit_elect(&bar_kv_empty[kb]);  // the buffer's K/V have been read by every MMA of this tile
      }
      mma_commit_elect(&bar_fin[0]);
      mbar_drain(&bar_fin[0], 0, kDrainNs);
    } else if (warp == kMmaAccWarp) {
      // -------------------------------------------------------------- dV/dK issuer
      const uint64_t dQmn = smem_desc(sQ, G::chunk(BQ), 8 * G::SWB, G::LAYOUT);
      const uint64_t dDOmn = smem_desc(sDO, G::chunk(BQ), 8 * G::SWB, G::LAYOUT);
      int g = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
        int bh, kt;
        dkdv_tile(tile, nct, zh, CAUSAL, &bh, &kt);
        const int n = NBq - tile_lo(kt);
        // The accumulators are overwritten by this tile's first MMAs: the previous tile's epilogue
        // must have read them.
        if (it > 0 && !warp_wait(bar_acc_read, (it - 1) & 1, ab)) { ok = false; break; }
        for (int c = 0; c < n; ++c, ++g) {
          // q_full is complete already (the S^T MMA of block g needed it); waiting on it orders the reads.
          if (!warp_wait(bar_p_full, g & 1, ab) || !warp_wait(&bar_q_full[g % NS], (g / NS) & 1, ab)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t so = uint64_t(((g % NS) * C::T_Q) >> 4);
          mma_tmem_mn<D, BQ / 16>(tmem + C::T_DV, tmem + C::T_PT, dDOmn + so, C::IDESC_ACC, c > 0 ? 1u : 0u);
          mma_tmem_mn<D, BQ / 16>(tmem + C::T_DK, tmem + C::T_DST, dQmn + so, C::IDESC_ACC, c > 0 ? 1u : 0u);
          mma_commit_elect(bar_acc_free);
          mma_commit_elect(&bar_q_empty[g % NS]);
        }
        if (ok) mma_commit_elect(bar_acc_done);
      }
      mma_commit_elect(&bar_fin[2]);
      mbar_drain(&bar_fin[2], 0, kDrainNs);
    } else {
      // warp 11: allocated TMEM above; nothing else until the teardown
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kComputeRegs));
    const int w = warp / 4;            // column half of every query block; 0 writes dV, 1 writes dK
    const int r = threadIdx.x % 128;   // key row within the tile = TMEM lane
    const int q4 = warp % 4;           // TMEM lane quadrant: rows [32 q4, 32 q4 + 32)
    const uint32_t tl = tmem + (uint32_t(q4 * 32) << 16);
    const uint32_t stg = base_u32 + C::OFF_STG + warp * C::STG;
    const uint64_t scale2 = f2(args.qk_scale, args.qk_scale);
    const CUtensorMap* tm_out = w ? &tm_dk : &tm_dv;
    const float mul = w ? args.sm_scale : 1.f;
    int g = 0, it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
      int bh, kt;
      dkdv_tile(tile, nct, zh, CAUSAL, &bh, &kt);
      const int zi = bh / args.H, hi = bh % args.H, k0 = 128 * kt, lo = tile_lo(kt), n = NBq - lo;
      const int key = k0 + r;
      for (int c = 0; c < n; ++c, ++g) {
        const int st = g % NS;
        if (!warp_wait(bar_s_full, g & 1, ab)) { ok = false; break; }
        tc_fence_after();
        uint32_t s[H], dp[H];
        tmem_load_cols<H>(tl + C::T_ST + w * H, s);
        tmem_load_cols<H>(tl + C::T_DPT + w * H, dp);
        tmem_wait_ld();
        reg_fence<H>(s);
        reg_fence<H>(dp);
        tc_fence_before();
        mbar_arrive(bar_s_free);  // the tensor core may now write S^T/dP^T of the next block
        if (!warp_wait(&bar_md_full[st], (g / NS) & 1, ab)) { ok = false; break; }
        const float* mq = md + st * 2 * BQ + w * H;
        const int q0 = (lo + c) * BQ + w * H;  // first query column of this warpgroup's half
        const bool masked = (q0 + H > N) || (k0 + 128 > N) || (CAUSAL && q0 < k0 + 127);
        const int c_lo = CAUSAL ? max(0, key - q0) : 0;  // valid query columns: c_lo <= c < c_hi
        const int c_hi = key < N ? N - q0 : 0;
        uint32_t pt[H / 2], dst[H / 2];
        if (masked)
          pds_row<H, true>(s, dp, mq, mq + BQ, pt, dst, scale2, c_lo, c_hi);
        else
          pds_row<H, false>(s, dp, mq, mq + BQ, pt, dst, scale2, c_lo, c_hi);
        if (g > 0) {  // the dV/dK MMAs of the previous block have read P^T/dS^T
          if (!warp_wait(bar_acc_free, (g - 1) & 1, ab)) { ok = false; break; }
          tc_fence_after();
        }
        tmem_store_cols<H / 2>(tl + C::T_PT + w * (H / 2), pt);
        tmem_store_cols<H / 2>(tl + C::T_DST + w * (H / 2), dst);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_p_full);
      }
      if (!ok || !warp_wait(bar_acc_done, it & 1, ab)) { ok = false; break; }
      // ---- epilogue: dV (warpgroup 0) or dK * sm_scale (warpgroup 1), 32 rows per warp via TMA stores
      tc_fence_after();
      uint32_t o[D];
      tmem_load_cols<D>(tl + (w ? C::T_DK : C::T_DV), o);
      tmem_wait_ld();
      reg_fence<D>(o);
      tc_fence_before();
      mbar_arrive(bar_acc_read);  // the next tile's first dV/dK MMAs may overwrite the accumulators
#pragma unroll
      for (int half = 0; half < 2; ++half) {  // columns [half * HW, half * HW + HW)
        if (lane == 0) tma_store_wait_read_all();  // this warp's previous store has left the staging area
        __syncwarp();
#pragma unroll
        for (int u = 0; u < C::SWB_O / 16; ++u) {
          const int c = half * C::HW + u * 8;
          const uint32_t addr = stg + swizzle_offset<C::SWB_O>(uint32_t(lane * C::SWB_O + u * 16));
          const uint32_t h0 = pack_half2(__uint_as_float(o[c + 0]) * mul, __uint_as_float(o[c + 1]) * mul);
          const uint32_t h1 = pack_half2(__uint_as_float(o[c + 2]) * mul, __uint_as_float(o[c + 3]) * mul);
          const uint32_t h2 = pack_half2(__uint_as_float(o[c + 4]) * mul, __uint_as_float(o[c + 5]) * mul);
          const uint32_t h3 = pack_half2(__uint_as_float(o[c + 6]) * mul, __uint_as_float(o[c + 7]) * mul);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(h0), "r"(h1), "r"(h2), "r"(h3)
                       : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {  // rows past N are clipped by the tensor map
          tma_store_4d(tm_out, stg, half * C::HW, k0 + 32 * q4, hi, zi);
          tma_store_commit();
        }
      }
    }
    if (lane == 0) tma_store_wait_all();  // the staging area must stay valid until the stores are done
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kAllocWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------- dK/dV: split columns
// One CTA per 128-row key tile; query blocks of BQ rows (the tile variant's block_n: 128, which fits
// TMEM only for D <= 64, or 64) whose columns the two compute warpgroups split (warpgroup w takes
// columns [w*H, w*H + H), H = BQ/2).
// TMEM: S^T [BQ] | dP^T [BQ] | P^T [BQ/2] | dS^T [BQ/2] | dV [D] | dK [D].
template <int D, int BQ_>
struct DkvSplitCfg {
  using G = Geo<D>;
  static constexpr int BQ = BQ_;                 // query rows per block
  static constexpr int H = BQ / 2;               // query columns per compute warpgroup
  static constexpr int NS = 4;                   // Q/dO ring stages
  static constexpr int T_KEY = G::tile(128);
  static constexpr int T_Q = G::tile(BQ);
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = T_KEY;
  static constexpr int OFF_Q = 2 * T_KEY;            // NS query blocks
  static constexpr int OFF_DO = OFF_Q + NS * T_Q;    // NS dO blocks
  // -M and -delta reach S^T and dP^T through one more MMA K step when D <= 64 (see the fused kernel). At
  // D = 128 every block already carries twice the MMA work per exponential and the extra step costs
  // more than the shared-memory loads it saves (measured: -10 % non-causal), so there the compute warps
  // read fp32 -M / -delta from shared memory.
  static constexpr bool FOLD = D <= 64;
  static constexpr int MD_SLOT = FOLD ? BQ * 16 : 2 * BQ * 4;
  static constexpr int OFF_MD = OFF_DO + NS * T_Q;   // NS x MD_SLOT
  static constexpr int ONES_TILE = FOLD ? 128 * 32 : 0;  // constant A of the folded K step
  static constexpr int OFF_ONES = OFF_MD + NS * MD_SLOT;  // 2 x ONES_TILE
  static constexpr int OFF_BAR = OFF_ONES + 2 * ONES_TILE;
  // kv_full, q_full[NS], md_full[NS], q_empty[NS], s_full, s_free, p_full, acc_free, acc_done, fin[2]
  static constexpr int NBARS = 1 + 3 * NS + 7;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  static constexpr uint32_t T_ST = 0, T_DPT = BQ, T_PT = 2 * BQ, T_DST = 2 * BQ + BQ / 2;
  static constexpr uint32_t T_DV = 3 * BQ, T_DK = 3 * BQ + D;
  static_assert(3 * BQ + 2 * D <= 512, "TMEM budget");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(OFF_MD % 128 == 0 && OFF_ONES % 128 == 0, "alignment");
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BQ, false);
  static constexpr uint32_t IDESC_ACC = idesc_f16_f32(128, D, true);
  static constexpr uint32_t IDESC_MD = idesc_f16_f32(128, BQ, false) | (1u << 7) | (1u << 10);  // bf16 A, B
};

template <int D, bool CAUSAL, int BQ>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dkdv_split_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const BwdArgs args) {
  using C = DkvSplitCfg<D, BQ>;
  using G = Geo<D>;
  constexpr int H = C::H;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_kv = bars;
  uint64_t* bar_q_full = bars + 1;              // [NS] Q and dO landed
  uint64_t* bar_md_full = bars + 1 + C::NS;     // [NS] M and delta staged
  uint64_t* bar_q_empty = bars + 1 + 2 * C::NS; // [NS] every MMA reading the slot has completed
  uint64_t* bar_s_full = bars + 1 + 3 * C::NS;
  uint64_t* bar_s_free = bar_s_full + 1;
  uint64_t* bar_p_full = bar_s_full + 2;
  uint64_t* bar_acc_free = bar_s_full + 3;
  uint64_t* bar_acc_done = bar_s_full + 4;
  uint64_t* bar_fin = bar_s_full + 5;           // [2]: one per issuer warp
  uint8_t* md = smem + C::OFF_MD;  // per ring slot: [BQ queries x 16 B] bf16 parts of -M/qk_scale, -delta
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status, args.wait_limit_ns};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int zh = args.Z * args.H;
  const int nct = (N + 127) / 128;
  int bh;
  // Causal: low key tiles see the most query blocks, so they go first.
  const int cta = cta_order(nct, zh, CAUSAL, N, D, &bh);
  const int zi = bh / args.H, hi = bh % args.H;
  const int NBq = (N + BQ - 1) / BQ;
  const int k0 = 128 * cta;                 // keys [k0, k0 + 128)
  const int lo = CAUSAL ? k0 / BQ : 0;      // first query block that sees any of them
  const int n = NBq - lo;

  if (threadIdx.x == 0) {
    mbar_init(bar_kv, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&bar_q_full[s], 1);
      mbar_init(&bar_md_full[s], 32);
      mbar_init(&bar_q_empty[s], 2);  // S^T/dP^T issuer + dV/dK issuer
    }
    mbar_init(bar_s_full, 1);
    mbar_init(bar_s_free, 256);
    mbar_init(bar_p_full, 256);
    mbar_init(bar_acc_free, 1);
    mbar_init(bar_acc_done, 1);
    mbar_init(&bar_fin[0], 1);
    mbar_init(&bar_fin[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kAllocWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
  }
  // Constant A operands of the folded -M / -delta K step (as in the fused kernel; bf16 1.0 = 0x3F80).
  if constexpr (C::FOLD) {
    for (int idx = threadIdx.x; idx < 2 * C::ONES_TILE / 16; idx += blockDim.x) {
      const int t = idx / (C::ONES_TILE / 16), byte = (idx % (C::ONES_TILE / 16)) * 16;
      const uint4 row = t == 0 ? make_uint4(0x3F803F80u, 0x00003F80u, 0u, 0u) : make_uint4(0u, 0x3F800000u, 0x3F803F80u, 0u);
      *reinterpret_cast<uint4*>(smem + C::OFF_ONES + t * C::ONES_TILE + byte) =
          (byte % 256) < 128 ? row : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sK = base_u32 + C::OFF_K, sV = base_u32 + C::OFF_V;
  const uint32_t sQ = base_u32 + C::OFF_Q, sDO = base_u32 + C::OFF_DO;

  if (warp >= kTmaWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == kTmaWarp) {
      dkdv_producer<D, BQ, C::NS, C::FOLD>(&tm_q, &tm_k, &tm_v, &tm_do, args, sK, sV, sQ, sDO, md, bar_kv, bar_q_full,
                                  bar_md_full, bar_q_empty, bh, zi, hi, k0, lo, n, ab);
    } else if (warp == kMmaSWarp) {
      // -------------------------------------------------------------- S^T/dP^T issuer
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      const uint64_t dK = smem_desc(sK, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dV = smem_desc(sV, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dQ = smem_desc(sQ, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dDO = smem_desc(sDO, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dOnesM = smem_desc(base_u32 + C::OFF_ONES, 128, 256, 0u);
      const uint64_t dOnesD = smem_desc(base_u32 + C::OFF_ONES + C::ONES_TILE, 128, 256, 0u);
      const uint64_t dMD = smem_desc(base_u32 + C::OFF_MD, 0, 128, 0u);
      // S'^T = S^T - M/qk_scale, dP'^T = dP^T - delta: the K = D steps, then one folded bf16 K step each.
      auto issue_s = [&](int c) {
        const uint64_t so = uint64_t(((c % C::NS) * C::T_Q) >> 4);
        const uint64_t mo = uint64_t(((c % C::NS) * C::MD_SLOT) >> 4);
        mma_kmajor<D, G::chunk(128), G::chunk(BQ)>(tmem + C::T_ST, dK, dQ + so, idesc_s);
        if constexpr (C::FOLD) mma_f16_ss_elect(tmem + C::T_ST, dOnesM, dMD + mo, C::IDESC_MD, 1u);
        mma_kmajor<D, G::chunk(128), G::chunk(BQ)>(tmem + C::T_DPT, dV, dDO + so, C::IDESC_S);
        if constexpr (C::FOLD) mma_f16_ss_elect(tmem + C::T_DPT, dOnesD, dMD + mo, C::IDESC_MD, 1u);
        mma_commit_elect(bar_s_full);
        mma_commit_elect(&bar_q_empty[c % C::NS]);
      };
      bool ok = n > 0 && warp_wait(bar_kv, 0, ab) && warp_wait(&bar_q_full[0], 0, ab) &&
                (!C::FOLD || warp_wait(&bar_md_full[0], 0, ab));
      if (ok) {
        tc_fence_after();
        issue_s(0);
      }
      for (int c = 0; ok && c + 1 < n; ++c) {
        const int b = c + 1;
        if (!warp_wait(bar_s_free, c & 1, ab) || !warp_wait(&bar_q_full[b % C::NS], (b / C::NS) & 1, ab) ||
            (C::FOLD && !warp_wait(&bar_md_full[b % C::NS], (b / C::NS) & 1, ab)))
          break;
        tc_fence_after();
        issue_s(b);
      }
      mma_commit_elect(&bar_fin[0]);
      mbar_drain(&bar_fin[0], 0, kDrainNs);
    } else if (warp == kMmaAccWarp) {
      // -------------------------------------------------------------- dV/dK issuer
      const uint64_t dQmn = smem_desc(sQ, G::chunk(BQ), 8 * G::SWB, G::LAYOUT);
      const uint64_t dDOmn = smem_desc(sDO, G::chunk(BQ), 8 * G::SWB, G::LAYOUT);
      for (int c = 0; c < n; ++c) {
        // q_full is complete already (the S^T MMA of block c needed it); waiting on it orders the reads.
        if (!warp_wait(bar_p_full, c & 1, ab) || !warp_wait(&bar_q_full[c % C::NS], (c / C::NS) & 1, ab)) break;
        tc_fence_after();
        const uint64_t so = uint64_t(((c % C::NS) * C::T_Q) >> 4);
        mma_tmem_mn<D, BQ / 16>(tmem + C::T_DV, tmem + C::T_PT, dDOmn + so, C::IDESC_ACC, c > 0 ? 1u : 0u);  // dV += P^T dO
        mma_tmem_mn<D, BQ / 16>(tmem + C::T_DK, tmem + C::T_DST, dQmn + so, C::IDESC_ACC, c > 0 ? 1u : 0u);  // dK += dS^T Q
        mma_commit_elect(bar_acc_free);
        mma_commit_elect(&bar_q_empty[c % C::NS]);
      }
      mma_commit_elect(bar_acc_done);
      mma_commit_elect(&bar_fin[1]);
      mbar_drain(&bar_fin[1], 0, kDrainNs);
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kComputeRegs));
    const int w = warp / 4;            // column half of every query block
    const int r = threadIdx.x % 128;   // key row within the tile = TMEM lane
    const int key = k0 + r;
    const uint32_t tl = tmem + (uint32_t((warp % 4) * 32) << 16);
    const float sc = C::FOLD ? fold_scale(args.qk_scale) : args.qk_scale;
    const uint64_t scale2 = f2(sc, sc);
    bool ok = true;
    for (int c = 0; c < n; ++c) {
      const int st = c % C::NS;
      if (!warp_wait(bar_s_full, c & 1, ab)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[H], dp[H];
      tmem_load_cols<H>(tl + C::T_ST + w * H, s);
      tmem_load_cols<H>(tl + C::T_DPT + w * H, dp);
      tmem_wait_ld();
      reg_fence<H>(s);
      reg_fence<H>(dp);
      tc_fence_before();
      mbar_arrive(bar_s_free);  // the tensor core may now write S^T/dP^T of the next block
      const float* mq = reinterpret_cast<const float*>(md) + st * 2 * BQ + w * H;  // unfolded -M | -delta
      if (!C::FOLD && !warp_wait(&bar_md_full[st], (c / C::NS) & 1, ab)) { ok = false; break; }
      const int q0 = (lo + c) * BQ + w * H;  // first query column of this warpgroup's half
      const bool masked = (q0 + H > N) || (k0 + 128 > N) || (CAUSAL && q0 < k0 + 127);
      const int c_lo = CAUSAL ? max(0, key - q0) : 0;  // valid query columns: c_lo <= c < c_hi
      const int c_hi = key < N ? N - q0 : 0;
      uint32_t pt[H / 2], dst[H / 2];
      if constexpr (C::FOLD) {
        if (masked)
          pds_row_folded<H, true>(s, dp, pt, dst, scale2, c_lo, c_hi);
        else
          pds_row_folded<H, false>(s, dp, pt, dst, scale2, c_lo, c_hi);
      } else {
        if (masked)
          pds_row<H, true>(s, dp, mq, mq + BQ, pt, dst, scale2, c_lo, c_hi);
        else
          pds_row<H, false>(s, dp, mq, mq + BQ, pt, dst, scale2, c_lo, c_hi);
      }
      if (c > 0) {  // the dV/dK MMAs of the previous block have read P^T/dS^T
        if (!warp_wait(bar_acc_free, (c - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
      }
      tmem_store_cols<H / 2>(tl + C::T_PT + w * (H / 2), pt);
      tmem_store_cols<H / 2>(tl + C::T_DST + w * (H / 2), dst);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_p_full);
    }
    if (ok && n > 0 && warp_wait(bar_acc_done, 0, ab)) {
      tc_fence_after();
      // warpgroup 0 writes dV, warpgroup 1 writes dK * sm_scale
      const int64_t rowidx = int64_t(bh) * N + key;
      __half* out = reinterpret_cast<__half*>(w ? args.dk : args.dv) + rowidx * D;
      store_rows<D>(tl + (w ? C::T_DK : C::T_DV), out, w ? args.sm_scale : 1.f, key < N);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kAllocWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <typename Kern>
cudaError_t launch_common(Kern kern, int smem, long long grid, const CUtensorMap& tq, const CUtensorMap& tk,
                          const CUtensorMap& tv, const CUtensorMap& tdo, const BwdArgs& a, cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  if (grid <= 0) return cudaSuccess;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  kern<<<dim3(unsigned(grid)), dim3(kThreads), smem, s>>>(tq, tk, tv, tdo, a);
  return cudaGetLastError();
}

int sm_count();

// dQ pass of the split backward, tile variant with BK-row key blocks: 128 (D <= 64; persistent when every
// tile costs the same, i.e. not causal) or 64 (the ping-pong kernel with alternating blocks).
template <int D, bool CAUSAL, int BK>
cudaError_t dq_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                    const CUtensorMap& tdq, const BwdArgs& a, cudaStream_t s) {
  const long long tiles = (long long)((a.N + 127) / 128) * a.Z * a.H;
  if constexpr (BK == 128 && D <= 64 && !CAUSAL) {  // persistent only when every tile costs the same (as dK/dV)
    auto kern = bwd_dq_persist_kernel<D, CAUSAL>;
    constexpr int smem = DqPersistCfg<D>::SMEM_BYTES;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (tiles <= 0) return cudaSuccess;
    if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const unsigned grid = unsigned(tiles < sm_count() ? tiles : sm_count());
    kern<<<dim3(grid), dim3(kThreads), smem, s>>>(tq, tk, tv, tdo, tdq, a);
    return cudaGetLastError();
  } else if constexpr (BK == 128 && D <= 64) {
    (void)tdq;
    return launch_common(bwd_dq_split_kernel<D, CAUSAL>, DqSplitCfg<D>::SMEM_BYTES, tiles, tq, tk, tv, tdo, a, s);
  } else if constexpr (BK == 64) {
    (void)tdq;
    return launch_common(bwd_dq_alt_kernel<D, CAUSAL>, DqAltCfg<D>::SMEM_BYTES, tiles, tq, tk, tv, tdo, a, s);
  } else {
    return cudaErrorNotSupported;
  }
}

// Streaming multiprocessors of the current device (cached per device).
int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cache[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
  }
  return cache[dev];
}

// dK/dV pass of the split backward, tile variant with BQ-row query blocks: 128 (D <= 64; persistent
// with static round-robin when every tile costs the same -- causal tiles differ, and the hardware's
// dynamic CTA scheduling balances them better) or 64.
template <int D, bool CAUSAL, int BQ>
cudaError_t dkdv_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                      const CUtensorMap& tdk, const CUtensorMap& tdv, const BwdArgs& a, cudaStream_t s) {
  const long long tiles = (long long)((a.N + 127) / 128) * a.Z * a.H;
  if constexpr (BQ == 128 && D <= 64 && !CAUSAL) {
    auto kern = bwd_dkdv_persist_kernel<D, CAUSAL>;
    constexpr int smem = DkvPersistCfg<D>::SMEM_BYTES;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (tiles <= 0) return cudaSuccess;
    if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const unsigned grid = unsigned(tiles < sm_count() ? tiles : sm_count());
    kern<<<dim3(grid), dim3(kThreads), smem, s>>>(tq, tk, tv, tdo, tdk, tdv, a);
    return cudaGetLastError();
  } else if constexpr (BQ == 64 || D <= 64) {
    (void)tdk;
    (void)tdv;
    return launch_common(bwd_dkdv_split_kernel<D, CAUSAL, BQ>, DkvSplitCfg<D, BQ>::SMEM_BYTES, tiles, tq, tk, tv,
                         tdo, a, s);
  } else {
    return cudaErrorNotSupported;
  }
}

// ------------------------------------------------------------------- fused backward, every D
// dK, dV and dQ in one pass (non-causal, or causal with each key tile's query blocks starting at the
// diagonal block; causal tiles are taken longest first) over each (key tile, query block) pair, so S^T,
// dP^T and the exponentials are computed once instead of once per output kernel (the reference's split,
// kernels.py:151-321, recomputes QK^T and dO V^T for dQ). The persistent dK/dV structure (one CTA per
// SM, 128-key tiles, static round-robin, ring of Q/dO blocks; K double-buffered because the dQ MMAs
// read it to the end of a tile, V single-buffered and loaded by warp 11 once the tile's last dP^T MMA
// has read it) plus:
//   * -M and -delta are folded into the S^T and dP^T MMAs (one more K = 16 step each against a
//     constant tile of ones), so the compute warps read S^T - M / qk_scale and dP^T - delta directly.
//   * dS^T goes to shared memory ([128 keys, BQ queries] fp16, 128-byte swizzle, 64-query chunks).
//     The same bytes are the K-major A operand of dK += dS^T Q and the MN-major operand of the dQ MMA
//     (rows = keys, 128 contiguous bytes = 64 queries); at D = 128 dS^T also goes to TMEM as the A
//     operand of the dK MMA.
//   * dQ_part of a block (fp32; D <= 64: 128 queries x D, D = 128: transposed, D x 64 queries) is
//     accumulated in TMEM by its own MMAs; the compute warps read it one block later, right after
//     handing over the next block's P^T/dS^T (the dQ MMAs of that block wait for the read: dq_read),
//     and add it into a dense fp32 workspace through TMA tensor reduce-adds (one 32 x 32 box per warp).
//   * After its last tile every CTA (a cooperative launch of at most one CTA per SM) waits at a grid
//     barrier for all reduce-adds, then its compute warps scale a share of the workspace by sm_scale
//     into the fp16 dQ.
// TMEM (D <= 64): S^T [128] | dP^T [128] | P^T [64] | dV [D] | dK [D] | dQ_part [D]; D = 128: FusedCfg.
template <int D>
struct FusedCfg {
  using G = Geo<D>;
  // D = 128: 64-query blocks, and the dQ part computed transposed (dQ^T = K^T dS^T: 128 head-dim lanes x
  // 64 query columns), so that S^T, dP^T, P^T, dV, dK, the dQ part and dS^T fit TMEM's 512 columns
  // (64 + 64 + 32 + 128 + 128 + 64 + 32); with 128-query blocks and dQ = dS K they would need 704.
  static constexpr bool DQT = D == 128;
  static constexpr int BQ = DQT ? 64 : 128, H = BQ / 2;  // query rows per block, columns per warpgroup
  static constexpr int NS = DQT ? 2 : 3;                  // Q/dO ring stages (shared memory)
  static constexpr int T_KEY = G::tile(128);
  static constexpr int T_Q = G::tile(BQ);
  static constexpr int T_DS = 128 * BQ * 2;               // dS^T [128 keys, BQ queries] fp16
  static constexpr int DS_CHUNK = Geo<128>::chunk(128);   // 64 queries of every key row
  static constexpr int HW = D / 2;                        // dK/dV output columns per warpgroup
  static constexpr int QW = DQT ? 32 : D / 2;             // dQ-part columns per warpgroup (queries if DQT)
  static constexpr int SWB_O = HW * 2;                    // dK/dV staging row bytes (fp16)
  static constexpr int SWB_Q = DQT ? 128 : HW * 4;        // dQ staging row bytes (fp32; 32 head dims if DQT)
  static constexpr int STG_ROW = SWB_O > SWB_Q ? SWB_O : SWB_Q;
  static constexpr int STG = 32 * STG_ROW < 1024 ? 1024 : 32 * STG_ROW;  // per-warp staging, both uses
  static constexpr int OFF_K = 0;                         // [2 buffers] key tiles
  static constexpr int OFF_V = 2 * T_KEY;                 // value tile
  static constexpr int OFF_Q = 3 * T_KEY;                 // NS query blocks
  static constexpr int OFF_DO = OFF_Q + NS * T_Q;         // NS dO blocks
  static constexpr int OFF_DS = OFF_DO + NS * T_Q;        // dS^T of the current block
  static constexpr int OFF_STG = OFF_DS + T_DS;           // 8 compute warps x STG
  // -M/qk_scale and -delta of each query of a ring slot, each as an exact sum of three bf16 parts, as
  // the B operand [128 queries x 16 K] (no swizzle; K columns 0-2 = the -M parts, 3-5 = the -delta
  // parts, 6-7 zero) of one extra K = 16 step of the S^T and dP^T MMAs. Only 8 K columns are stored: the
  // step's upper 8 read the same bytes (LBO = 0), against zeros in the A operand.
  static constexpr int MD_SLOT = BQ * 16;
  static constexpr int OFF_MD = OFF_STG + 8 * STG;        // NS x MD_SLOT
  // The A operands of that step, [128 keys x 16 K] bf16 (no swizzle): ones in K columns 0-2 (S^T) or
  // 3-5 (dP^T), zeros elsewhere, so the step adds -M/qk_scale to S^T and -delta to dP^T.
  static constexpr int ONES_TILE = 128 * 32;
  static constexpr int OFF_ONES = OFF_MD + NS * MD_SLOT;  // 2 x ONES_TILE
  static constexpr int OFF_BAR = OFF_ONES + 2 * ONES_TILE;
  // k_full[2], k_empty[2], q_full[NS], md_full[NS], q_empty[NS], s_full, s_free, p_full, acc_free,
  // acc_done, acc_read, fin[3], dq_read, v_full, v_empty
  static constexpr int NBARS = 4 + 3 * NS + 12;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  // TMEM columns: S^T [BQ], dP^T [BQ], P^T [BQ / 2, fp16 pairs], dV [D], dK [D], the dQ part [DQC].
  static constexpr int DQC = DQT ? BQ : D;
  static constexpr uint32_t T_ST = 0, T_DPT = BQ;
  static constexpr uint32_t T_DV = DQT ? 128 : 320, T_DK = T_DV + D, T_DQ = T_DK + D;
  static constexpr uint32_t T_PT = DQT ? T_DQ + DQC : 256;
  // D = 128: dS^T also in TMEM (fp16 pairs, after P^T), the A operand of the dK MMA, which then reads only
  // Q from shared memory (measured +2% over reading dS^T back from shared memory).
  static constexpr uint32_t T_DST = T_PT + BQ / 2;
  static_assert(T_DQ + DQC <= 512 && T_PT + BQ / 2 <= 512 && (DQT || T_PT + BQ / 2 <= T_DV), "TMEM budget");
  static_assert(!DQT || T_DST + BQ / 2 <= 512, "TMEM budget");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(OFF_DS % 1024 == 0 && OFF_STG % 1024 == 0 && OFF_MD % 128 == 0 && OFF_ONES % 128 == 0,
                "alignment");
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BQ, false);
  static constexpr uint32_t IDESC_ACC = idesc_f16_f32(128, D, true);     // A K-major, B MN-major
  // A and B MN-major: dQ = dS K (A = dS, B = K) or, DQT, dQ^T = K^T dS^T (A = K^T, B = dS^T).
  static constexpr uint32_t IDESC_DQ = idesc_f16_f32_amn(128, DQC, true);
  static constexpr uint32_t IDESC_MD = idesc_f16_f32(128, BQ, false) | (1u << 7) | (1u << 10);  // bf16 A, B
};

// Add the warp's part of a block's dQ partial (32 query rows x D/2 fp32 columns, in registers) into the
// fp32 workspace at (col, row) through the warp's staging area.
template <int D>
__device__ __forceinline__ void fused_dq_out(const uint32_t* o, uint32_t stg, const CUtensorMap* tm, int col, int row,
                                             int hi, int zi, int lane) {
  using C = FusedCfg<D>;
  if (lane == 0) tma_store_wait_read_all();  // the warp's previous reduce / store has read its staging
  __syncwarp();
#pragma unroll
  for (int u = 0; u < C::SWB_Q / 16; ++u) {
    const uint32_t addr = stg + swizzle_offset<C::SWB_Q>(uint32_t(lane * C::SWB_Q + u * 16));
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(o[4 * u]), "r"(o[4 * u + 1]),
                 "r"(o[4 * u + 2]), "r"(o[4 * u + 3]) : "memory");
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {  // rows past N are clipped by the tensor map
    tma_reduce_add_4d(tm, stg, col, row, hi, zi);
    tma_store_commit();
  }
}

// D = 128: the warp holds a transposed dQ part (lane = one of 32 head dims, o[j] = query j of 32), written
// transposed into the staging tile (32 query rows x 32 head-dim fp32, 128-byte swizzle; for each query
// the 32 lanes store one 128-byte row, so the stores are conflict-free), then added like fused_dq_out.
__device__ __forceinline__ void fused_dqt_out(const uint32_t* o, uint32_t stg, const CUtensorMap* tm, int col,
                                              int row, int hi, int zi, int lane) {
  if (lane == 0) tma_store_wait_read_all();
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const uint32_t addr = stg + swizzle_offset<128>(uint32_t(j * 128 + lane * 4));
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(o[j]) : "memory");
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_reduce_add_4d(tm, stg, col, row, hi, zi);
    tma_store_commit();
  }
}

// Barrier over all CTAs of a cooperative launch (all CTAs are resident, so every arrival comes), called
// by the `nthreads` threads of the CTA that take part (named barrier `bar_id`; thread 0 of them first).
// Thread 0 publishes the writes the participants made before the call (release), counts the CTA in and
// waits (acquire) until `target` arrivals are counted, for at most ab.limit_ns: after that it records
// kStatusWaitTimeout, raises the CTA's abort flag and stops waiting. A CTA whose abort flag is already up
// still arrives (so that no other CTA waits for it) but does not wait. Returns whether the CTA may go on.
__device__ __forceinline__ bool grid_barrier(unsigned* ctr, unsigned target, const CtaAbort& ab, int bar_id,
                                             int nthreads, bool first) {
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
  if (first) {
    __threadfence();
    atomicAdd(ctr, 1u);
    const unsigned long long t0 = globaltimer_ns();
    while (*ab.flag == 0) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= target) break;
      if (globaltimer_ns() - t0 > ab.limit_ns) {
        *ab.flag = 1;
        atomicOr(ab.status, kStatusWaitTimeout);
        break;
      }
      __nanosleep(128);
    }
  }
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
  return *ab.flag == 0;
}

// Last phase of the fused backward, grid-stride over threads [0, nthreads) of every CTA: dq = sm_scale *
// dq_acc as fp16, 8 elements a thread. The thread and CTA indices are read here again: otherwise the
// compiler keeps them in registers through the whole main loop, and the compute warps spill.
template <int D>
__device__ __forceinline__ void fused_dq_epilogue(const BwdArgs& a, int nthreads) {
  unsigned t, cta;
  asm volatile("mov.u32 %0, %%tid.x;" : "=r"(t));
  asm volatile("mov.u32 %0, %%ctaid.x;" : "=r"(cta));
  const int64_t n8 = int64_t(a.Z) * a.H * a.N * (D / 8);
  const float4* acc = reinterpret_cast<const float4*>(a.dq_acc);
  uint4* dq = static_cast<uint4*>(a.dq);
  const float sc = a.sm_scale;
  // U groups of 8 a thread per step, all loads issued before any store (the compiler may not move the
  // loads past the stores itself): enough bytes in flight per SM to run at HBM speed.
  constexpr int U = 8;
  const int64_t stride = int64_t(gridDim.x) * nthreads;
  for (int64_t i0 = int64_t(cta) * nthreads + t; i0 < n8; i0 += stride * U) {
    float4 x[U], y[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < n8) {
        x[u] = __ldcg(acc + 2 * i);
        y[u] = __ldcg(acc + 2 * i + 1);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < n8)
        dq[i] = make_uint4(pack_half2(x[u].x * sc, x[u].y * sc), pack_half2(x[u].z * sc, x[u].w * sc),
                           pack_half2(y[u].x * sc, y[u].y * sc), pack_half2(y[u].z * sc, y[u].w * sc));
    }
  }
}

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_fused_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_dk, const __grid_constant__ CUtensorMap tm_dv,
                     const __grid_constant__ CUtensorMap tm_dqacc, const BwdArgs args) {
  using C = FusedCfg<D>;
  using G = Geo<D>;
  constexpr int H = C::H, BQ = C::BQ, NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_kv_full = bars;                 // [2] key buffer landed
  uint64_t* bar_kv_empty = bars + 2;            // [2] every S^T and dQ MMA of the buffer's tile has completed
  uint64_t* bar_q_full = bars + 4;              // [NS]
  uint64_t* bar_md_full = bars + 4 + NS;        // [NS]
  uint64_t* bar_q_empty = bars + 4 + 2 * NS;    // [NS]
  uint64_t* bar_s_full = bars + 4 + 3 * NS;
  uint64_t* bar_s_free = bar_s_full + 1;
  uint64_t* bar_p_full = bar_s_full + 2;        // P^T in TMEM and dS^T in shared memory
  uint64_t* bar_acc_free = bar_s_full + 3;      // the block's dV, dK and dQ MMAs completed
  uint64_t* bar_acc_done = bar_s_full + 4;
  uint64_t* bar_acc_read = bar_s_full + 5;      // the compute warps hold the tile's dV/dK and last dQ part
  uint64_t* bar_fin = bar_s_full + 6;           // [3]
  uint64_t* bar_dq_read = bar_s_full + 9;       // the compute warps hold the previous block's dQ part
  uint64_t* bar_v_full = bar_s_full + 10;       // value tile landed
  uint64_t* bar_v_empty = bar_s_full + 11;      // every dP^T MMA of the value tile's tile has completed
  uint8_t* md = smem + C::OFF_MD;  // per ring slot: [BQ queries x 16 B] bf16 parts of -M/qk_scale, -delta
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status, args.wait_limit_ns};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int zh = args.Z * args.H;
  const int nct = (N + 127) / 128;
  const int ntiles = nct * zh;
  const int NBq = (N + BQ - 1) / BQ;
  // Query blocks of key tile kt: [lo, NBq) (causal: from the diagonal block on).
  auto tile_lo = [&](int kt) { return CAUSAL ? (128 * kt) / BQ : 0; };
  // The CTA's key tiles, in processing order (every role walks the same sequence). Not causal: the
  // head-major tile list round-robin (CTA b: tiles b, b + G, ...). Causal: key tiles kt and nct-1-kt of a
  // head together cost nct + 1 query blocks whatever kt is, so they form one unit of work (a middle tile
  // of odd nct is a unit alone); units are taken round-robin in head-major order, the longer tile of a
  // unit first. Equal units balance the CTAs, and the tiles running at any time belong to a few
  // neighbouring heads, so their fp32 dQ workspace rows and Q/dO blocks are shared in L2 (ordering the
  // tiles longest-first across all heads instead spreads 148 CTAs over ~148 heads, whose workspaces miss
  // L2: ~10x the algorithmic DRAM traffic at N = 8192 with 1,024 heads).
  const int n_units = CAUSAL ? zh * ((nct + 1) / 2) : ntiles;
  auto next_tile = [&](int2& seq, int* bh, int* kt) -> bool {  // seq = (unit, second tile of the unit)
    if (seq.x >= n_units) return false;
    if (!CAUSAL) {
      *bh = seq.x / nct;
      *kt = seq.x % nct;
      seq.x += int(gridDim.x);
      return true;
    }
    const int U = (nct + 1) / 2, p = seq.x % U;
    *bh = seq.x / U;
    *kt = seq.y ? nct - 1 - p : p;
    if (seq.y || nct - 1 - p == p) {
      seq = make_int2(seq.x + int(gridDim.x), 0);
    } else {
      seq.y = 1;
    }
    return true;
  };

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_kv_full[b], 1);
      mbar_init(&bar_kv_empty[b], 2);  // S^T/dP^T issuer + dV/dK/dQ issuer (which reads K for dQ)
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bar_q_full[s], 1);
      mbar_init(&bar_md_full[s], 32);
      mbar_init(&bar_q_empty[s], 2);
    }
    mbar_init(bar_s_full, 1);
    mbar_init(bar_s_free, 256);
    mbar_init(bar_p_full, 256);
    mbar_init(bar_acc_free, 1);
    mbar_init(bar_acc_done, 1);
    mbar_init(bar_acc_read, 256);
    for (int i = 0; i < 3; ++i) mbar_init(&bar_fin[i], 1);
    mbar_init(bar_dq_read, 256);
    mbar_init(bar_v_full, 1);
    mbar_init(bar_v_empty, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kAllocWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
  }
  // The constant A operands of the folded -M / -delta step (bf16 1.0 = 0x3F80): in every 8-row group,
  // bytes [0, 128) hold K columns 0-7 of the 8 rows (16 bytes a row), bytes [128, 256) columns 8-15.
  for (int idx = threadIdx.x; idx < 2 * C::ONES_TILE / 16; idx += blockDim.x) {
    const int t = idx / (C::ONES_TILE / 16), byte = (idx % (C::ONES_TILE / 16)) * 16;
    const bool low_k = (byte % 256) < 128;
    const uint4 row = t == 0 ? make_uint4(0x3F803F80u, 0x00003F80u, 0u, 0u)   // K 0-2: the -M parts
                             : make_uint4(0u, 0x3F800000u, 0x3F803F80u, 0u);  // K 3-5: the -delta parts
    *reinterpret_cast<uint4*>(smem + C::OFF_ONES + t * C::ONES_TILE + byte) = low_k ? row : make_uint4(0u, 0u, 0u, 0u);
  }
  fence_proxy_async_smem();  // the tensor core reads them through the async proxy
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sK = base_u32 + C::OFF_K, sV = base_u32 + C::OFF_V;
  const uint32_t sQ = base_u32 + C::OFF_Q, sDO = base_u32 + C::OFF_DO;
  const uint32_t sDS = base_u32 + C::OFF_DS;

  if (warp >= kTmaWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kFusedProducerRegs));
    if (warp == kTmaWarp) {
      // -------------------------------------------------------------- TMA producer + -M/-delta staging
      int g = 0, it = 0, kv_issued = 0;
      bool ok = true;
      int2 seq = make_int2(int(blockIdx.x), 0);
      for (int bh, kt; ok && next_tile(seq, &bh, &kt); ++it) {
        const int zi = bh / args.H, hi = bh % args.H, k0 = 128 * kt, lo = tile_lo(kt), n = NBq - lo;
        const int kb = it & 1;
        if (it >= 2 && !warp_wait(&bar_kv_empty[kb], ((it >> 1) - 1) & 1, ab)) { ok = false; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(&bar_kv_full[kb], C::T_KEY);
          for (int ch = 0; ch < G::NCH; ++ch)
            tma_load_4d(sK + kb * C::T_KEY + ch * G::chunk(128), &tm_k, ch * G::CW, k0, hi, zi, &bar_kv_full[kb]);
        }
        ++kv_issued;
        const float* mrow = args.m + int64_t(bh) * N;
        const float* drow = args.delta + int64_t(bh) * N;
        const float inv_scale = 1.f / fold_scale(args.qk_scale);
        for (int c = 0; c < n; ++c, ++g) {
          const int st = g % NS;
          if (g >= NS && !warp_wait(&bar_q_empty[st], ((g / NS) - 1) & 1, ab)) { ok = false; break; }
          const int qr = (lo + c) * BQ;
          if (lane == 0) {
            mbar_arrive_expect_tx(&bar_q_full[st], 2 * C::T_Q);
            for (int ch = 0; ch < G::NCH; ++ch) {
              tma_load_4d(sQ + st * C::T_Q + ch * G::chunk(BQ), &tm_q, ch * G::CW, qr, hi, zi, &bar_q_full[st]);
              tma_load_4d(sDO + st * C::T_Q + ch * G::chunk(BQ), &tm_do, ch * G::CW, qr, hi, zi, &bar_q_full[st]);
            }
          }
          // Query j's 16 bytes: bf16 parts of -M/qk_scale (K 0-2) and of -delta (K 3-5), zeros (K 6-7).
          uint8_t* slot = md + st * C::MD_SLOT;
#pragma unroll
          for (int j = lane; j < BQ; j += 32) {
            const int q = qr + j;
            uint32_t hm[3], hd[3];
            split_bf16x3(q < N ? -mrow[q] * inv_scale : 0.f, hm);
            split_bf16x3(q < N ? -drow[q] : 0.f, hd);
            *reinterpret_cast<uint4*>(slot + j * 16) =
                make_uint4(hm[0] | (hm[1] << 16), hm[2] | (hd[0] << 16), hd[1] | (hd[2] << 16), 0u);
          }
          fence_proxy_async_smem();  // read by the S^T / dP^T MMAs through the async proxy
          mbar_arrive(&bar_md_full[st]);
        }
      }
      // Every copy issued must land before the CTA exits (instant on the normal path).
      if (lane == 0) {
        for (int ii = max(0, kv_issued - 2); ii < kv_issued; ++ii) mbar_drain(&bar_kv_full[ii & 1], (ii >> 1) & 1, kDrainNs);
        for (int gg = max(0, g - NS); gg < g; ++gg) mbar_drain(&bar_q_full[gg % NS], (gg / NS) & 1, kDrainNs);
      }
    } else if (warp == kMmaSWarp) {
      // -------------------------------------------------------------- S^T/dP^T issuer
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      const uint64_t dK = smem_desc(sK, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dV = smem_desc(sV, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dQ = smem_desc(sQ, 16, 8 * G::SWB, G::LAYOUT);
      const uint64_t dDO = smem_desc(sDO, 16, 8 * G::SWB, G::LAYOUT);
      // The folded step: A = constant ones tiles (K-major, no swizzle: K core matrices 128 bytes apart,
      // 8-row groups 256), B = the slot's parts (no swizzle: 8-query groups 128 bytes apart, the upper
      // K core matrix the same bytes).
      const uint64_t dOnesM = smem_desc(base_u32 + C::OFF_ONES, 128, 256, 0u);
      const uint64_t dOnesD = smem_desc(base_u32 + C::OFF_ONES + C::ONES_TILE, 128, 256, 0u);
      const uint64_t dMD = smem_desc(base_u32 + C::OFF_MD, 0, 128, 0u);
      int g = 0, it = 0;
      bool ok = true;
      int2 seq = make_int2(int(blockIdx.x), 0);
      for (int bh, kt; ok && next_tile(seq, &bh, &kt); ++it) {
        const int n = NBq - tile_lo(kt);
        const int kb = it & 1;
        if (!warp_wait(&bar_kv_full[kb], (it >> 1) & 1, ab) || !warp_wait(bar_v_full, it & 1, ab)) {
          ok = false;
          break;
        }
        const uint64_t ko = uint64_t((kb * C::T_KEY) >> 4);
        for (int c = 0; c < n; ++c, ++g) {
          if (g > 0 && !warp_wait(bar_s_free, (g - 1) & 1, ab)) { ok = false; break; }
          if (!warp_wait(&bar_q_full[g % NS], (g / NS) & 1, ab) || !warp_wait(&bar_md_full[g % NS], (g / NS) & 1, ab)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t so = uint64_t(((g % NS) * C::T_Q) >> 4);
          const uint64_t mo = uint64_t(((g % NS) * C::MD_SLOT) >> 4);
          // S'^T = S^T - M/qk_scale and dP'^T = dP^T - delta: one more K = 16 step each (bf16, no negation)
          mma_kmajor<D, G::chunk(128), G::chunk(BQ)>(tmem + C::T_ST, dK + ko, dQ + so, idesc_s);
          mma_f16_ss_elect(tmem + C::T_ST, dOnesM, dMD + mo, C::IDESC_MD, 1u);
          mma_kmajor<D, G::chunk(128), G::chunk(BQ)>(tmem + C::T_DPT, dV, dDO + so, C::IDESC_S);
          mma_f16_ss_elect(tmem + C::T_DPT, dOnesD, dMD + mo, C::IDESC_MD, 1u);
          mma_commit_elect(bar_s_full);
          mma_commit_elect(&bar_q_empty[g % NS]);
        }
        mma_commit_elect(&bar_kv_empty[kb]);
        mma_commit_elect(bar_v_empty);
      }
      mma_commit_elect(&bar_fin[0]);
      mbar_drain(&bar_fin[0], 0, kDrainNs);
    } else if (warp == kMmaAccWarp) {
      // -------------------------------------------------------------- dV / dK / dQ issuer
      const uint64_t dQmn = smem_desc(sQ, G::chunk(BQ), 8 * G::SWB, G::LAYOUT);
      const uint64_t dDOmn = smem_desc(sDO, G::chunk(BQ), 8 * G::SWB, G::LAYOUT);
      const uint64_t dKmn = smem_desc(sK, G::chunk(128), 8 * G::SWB, G::LAYOUT);
      const uint64_t dDSk = smem_desc(sDS, 16, 1024, 2u);                // dS^T as K-major A (dK)
      const uint64_t dDSmn = smem_desc(sDS, C::DS_CHUNK, 1024, 2u);      // dS (A) or dS^T (B), MN-major (dQ)
      int g = 0, it = 0;
      bool ok = true;
      int2 seq = make_int2(int(blockIdx.x), 0);
      for (int bh, kt; ok && next_tile(seq, &bh, &kt); ++it) {
        const int n = NBq - tile_lo(kt);
        const int kb = it & 1;
        const uint64_t ko = uint64_t((kb * C::T_KEY) >> 4);
        // The accumulators are overwritten by this tile's first MMAs: the previous tile's epilogue
        // must have read them (and the previous tile's last dQ part).
        if (it > 0 && !warp_wait(bar_acc_read, (it - 1) & 1, ab)) { ok = false; break; }
        if (!warp_wait(&bar_kv_full[kb], (it >> 1) & 1, ab)) { ok = false; break; }  // K for the dQ MMAs
        for (int c = 0; c < n; ++c, ++g) {
          if (!warp_wait(bar_p_full, g & 1, ab) || !warp_wait(&bar_q_full[g % NS], (g / NS) & 1, ab)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t so = uint64_t(((g % NS) * C::T_Q) >> 4);
          const uint32_t acc = c > 0 ? 1u : 0u;
          // dV += P^T dO (A = P^T from TMEM)
          mma_tmem_mn<D, BQ / 16>(tmem + C::T_DV, tmem + C::T_PT, dDOmn + so, C::IDESC_ACC, acc);
          // dK += dS^T Q (A = dS^T from TMEM at D = 128; otherwise from shared memory, K-major over
          // queries: 64-query chunks, 32 bytes per K step)
          if constexpr (C::DQT) {
            mma_tmem_mn<D, BQ / 16>(tmem + C::T_DK, tmem + C::T_DST, dQmn + so, C::IDESC_ACC, acc);
          } else {
#pragma unroll
            for (int kk = 0; kk < BQ / 16; ++kk)
              mma_f16_ss_elect(tmem + C::T_DK, dDSk + uint64_t(((kk / 4) * C::DS_CHUNK + (kk % 4) * 32) >> 4),
                               dQmn + so + uint64_t((kk * 16 * G::SWB) >> 4), C::IDESC_ACC, kk > 0 ? 1u : acc);
          }
          // dQ_part = dS K (A = dS, MN-major: 16 key rows of 128 bytes per K step; B = K, MN-major) or, D =
          // 128, dQ_part^T = K^T dS^T (the same two tiles as A = K^T and B = dS^T), once the compute warps
          // hold the previous block's dQ part.
          if (!warp_wait(bar_dq_read, g & 1, ab)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 128 / 16; ++kk) {
            const uint64_t ds_k = dDSmn + uint64_t((kk * 16 * 128) >> 4);
            const uint64_t k_k = dKmn + ko + uint64_t((kk * 16 * G::SWB) >> 4);
            if constexpr (C::DQT)
              mma_f16_ss_elect(tmem + C::T_DQ, k_k, ds_k, C::IDESC_DQ, kk > 0 ? 1u : 0u);
            else
              mma_f16_ss_elect(tmem + C::T_DQ, ds_k, k_k, C::IDESC_DQ, kk > 0 ? 1u : 0u);
          }
          mma_commit_elect(bar_acc_free);
          mma_commit_elect(&bar_q_empty[g % NS]);
        }
        if (ok) {
          mma_commit_elect(bar_acc_done);
          mma_commit_elect(&bar_kv_empty[kb]);  // the tile's dQ MMAs have read its K buffer
        }
      }
      mma_commit_elect(&bar_fin[2]);
      mbar_drain(&bar_fin[2], 0, kDrainNs);
    } else {
      // -------------------------------------------------------------- value tiles (warp 11)
      int it = 0, v_issued = 0;
      bool ok = true;
      int2 seq = make_int2(int(blockIdx.x), 0);
      for (int bh, kt; ok && next_tile(seq, &bh, &kt); ++it) {
        if (it >= 1 && !warp_wait(bar_v_empty, (it - 1) & 1, ab)) { ok = false; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(bar_v_full, C::T_KEY);
          for (int ch = 0; ch < G::NCH; ++ch)
            tma_load_4d(sV + ch * G::chunk(128), &tm_v, ch * G::CW, 128 * kt, bh % args.H, bh / args.H, bar_v_full);
        }
        ++v_issued;
      }
      if (lane == 0 && v_issued > 0) mbar_drain(bar_v_full, (v_issued - 1) & 1, kDrainNs);
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kFusedComputeRegs));
    const int w = warp / 4;            // query half of every block; writes dV (0) or dK (1)
    const int r = threadIdx.x % 128;   // key row within the tile = TMEM lane
    const int q4 = warp % 4;           // TMEM lane quadrant: rows [32 q4, 32 q4 + 32)
    const uint32_t tl = tmem + (uint32_t(q4 * 32) << 16);
    const uint32_t stg = base_u32 + C::OFF_STG + warp * C::STG;
    // This thread's row of dS^T: key r, queries [H w, H w + H): one 128-byte row of chunk w (H = 64), or
    // 16-byte units [4 w, 4 w + 4) of the single chunk's row r (H = 32).
    const uint32_t ds_row = sDS + (C::DQT ? 0 : w * C::DS_CHUNK) + r * 128;
    constexpr int DS_U = H / 8;                 // 16-byte units of dS^T a thread writes per block
    const int ds_u0 = C::DQT ? 4 * w : 0;
    const uint64_t scale2 = f2(fold_scale(args.qk_scale), fold_scale(args.qk_scale));
    const CUtensorMap* tm_out = w ? &tm_dk : &tm_dv;
    const float mul = w ? args.sm_scale : 1.f;
    int g = 0, it = 0;
    bool ok = true;
    int2 seq = make_int2(int(blockIdx.x), 0);
    for (int bh, kt; ok && next_tile(seq, &bh, &kt); ++it) {
      const int zi = bh / args.H, hi = bh % args.H, k0 = 128 * kt, lo = tile_lo(kt), n = NBq - lo;
      const int key = k0 + r;
      for (int c = 0; c < n; ++c, ++g) {
        if (!warp_wait(bar_s_full, g & 1, ab)) { ok = false; break; }
        tc_fence_after();
        uint32_t s[H], dp[H];
        tmem_load_cols<H>(tl + C::T_ST + w * H, s);
        tmem_load_cols<H>(tl + C::T_DPT + w * H, dp);
        tmem_wait_ld();
        reg_fence<H>(s);
        reg_fence<H>(dp);
        tc_fence_before();
        mbar_arrive(bar_s_free);  // the tensor core may now write S^T/dP^T of the next block
        const int q0 = (lo + c) * BQ + w * H;  // first query column of this warpgroup's half
        const bool masked = (q0 + H > N) || (k0 + 128 > N) || (CAUSAL && q0 < k0 + 127);
        const int c_lo = CAUSAL ? max(0, key - q0) : 0;  // valid query columns: c_lo <= c < c_hi
        const int c_hi = key < N ? N - q0 : 0;
        uint32_t pt[H / 2], dst[H / 2];
        if (masked)
          pds_row_folded<H, true>(s, dp, pt, dst, scale2, c_lo, c_hi);
        else
          pds_row_folded<H, false>(s, dp, pt, dst, scale2, c_lo, c_hi);
        if (g > 0) {  // the previous block's dV/dK/dQ MMAs have read P^T and dS^T and written dQ_part
          if (!warp_wait(bar_acc_free, (g - 1) & 1, ab)) { ok = false; break; }
          tc_fence_after();
        }
        tmem_store_cols<H / 2>(tl + C::T_PT + w * (H / 2), pt);
        if constexpr (C::DQT) tmem_store_cols<H / 2>(tl + C::T_DST + w * (H / 2), dst);
#pragma unroll
        for (int u = 0; u < DS_U; ++u) {
          const uint32_t addr = ds_row + uint32_t(((ds_u0 + u) ^ (r & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(dst[4 * u]), "r"(dst[4 * u + 1]),
                       "r"(dst[4 * u + 2]), "r"(dst[4 * u + 3]) : "memory");
        }
        fence_proxy_async_smem();  // the tensor core reads dS^T through the async proxy
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_p_full);
        // The previous block's dQ part (the last block of a tile leaves in the epilogue): into registers,
        // release the accumulator to this block's dQ MMAs, then add it into the workspace.
        if (c > 0) {
          uint32_t oq[C::QW];
          tmem_load_cols<C::QW>(tl + C::T_DQ + w * C::QW, oq);
          tmem_wait_ld();
          reg_fence<C::QW>(oq);
          tc_fence_before();
          mbar_arrive(bar_dq_read);
          if constexpr (C::DQT)
            fused_dqt_out(oq, stg, &tm_dqacc, 32 * q4, (lo + c - 1) * BQ + 32 * w, hi, zi, lane);
          else
            fused_dq_out<D>(oq, stg, &tm_dqacc, w * C::HW, (lo + c - 1) * BQ + 32 * q4, hi, zi, lane);
        } else {
          mbar_arrive(bar_dq_read);
        }
      }
      if (!ok || !warp_wait(bar_acc_done, it & 1, ab)) { ok = false; break; }
      // ---- epilogue: the last block's dQ part, then dV (warpgroup 0) or dK * sm_scale (warpgroup 1)
      tc_fence_after();
      // D = 128 reads dV / dK one half at a time (64 registers, not 128), releasing the accumulators after
      // the second half.
      constexpr int OR = C::DQT ? C::HW : D;  // accumulator columns held in registers at a time
      uint32_t o[OR];
      tmem_load_cols<OR>(tl + (w ? C::T_DK : C::T_DV), o);
      uint32_t oq[C::QW];
      tmem_load_cols<C::QW>(tl + C::T_DQ + w * C::QW, oq);
      tmem_wait_ld();
      reg_fence<OR>(o);
      reg_fence<C::QW>(oq);
      if constexpr (!C::DQT) {
        tc_fence_before();
        mbar_arrive(bar_acc_read);  // the next tile's first MMAs may overwrite the accumulators
        fused_dq_out<D>(oq, stg, &tm_dqacc, w * C::HW, (lo + n - 1) * BQ + 32 * q4, hi, zi, lane);
      } else {
        fused_dqt_out(oq, stg, &tm_dqacc, 32 * q4, (lo + n - 1) * BQ + 32 * w, hi, zi, lane);
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {  // columns [half * HW, half * HW + HW)
        if constexpr (C::DQT) {
          if (half == 1) {
            tmem_load_cols<OR>(tl + (w ? C::T_DK : C::T_DV) + C::HW, o);
            tmem_wait_ld();
            reg_fence<OR>(o);
            tc_fence_before();
            mbar_arrive(bar_acc_read);
          }
        }
        if (lane == 0) tma_store_wait_read_all();  // this warp's previous store has left the staging area
        __syncwarp();
#pragma unroll
        for (int u = 0; u < C::SWB_O / 16; ++u) {
          const int cc = (C::DQT ? 0 : half * C::HW) + u * 8;
          const uint32_t addr = stg + swizzle_offset<C::SWB_O>(uint32_t(lane * C::SWB_O + u * 16));
          const uint32_t h0 = pack_half2(__uint_as_float(o[cc + 0]) * mul, __uint_as_float(o[cc + 1]) * mul);
          const uint32_t h1 = pack_half2(__uint_as_float(o[cc + 2]) * mul, __uint_as_float(o[cc + 3]) * mul);
          const uint32_t h2 = pack_half2(__uint_as_float(o[cc + 4]) * mul, __uint_as_float(o[cc + 5]) * mul);
          const uint32_t h3 = pack_half2(__uint_as_float(o[cc + 6]) * mul, __uint_as_float(o[cc + 7]) * mul);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(h0), "r"(h1), "r"(h2), "r"(h3)
                       : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {  // rows past N are clipped by the tensor map
          tma_store_4d(tm_out, stg, half * C::HW, k0 + 32 * q4, hi, zi);
          tma_store_commit();
        }
      }
    }
    if (lane == 0) {
      tma_store_wait_all();  // staging must stay valid until the stores and reduces are done
      asm volatile("fence.proxy.async.global;" ::: "memory");  // the completed reduce-adds before the barrier
    }
    __syncwarp();
    // Last phase, once every CTA's dQ additions have completed: dq = sm_scale * dq_acc, by the compute
    // warps of all CTAs (named barrier 1 over their 256 threads).
    if (grid_barrier(args.grid_sync, gridDim.x, ab, 1, 256, threadIdx.x == 0))
      fused_dq_epilogue<D>(args, 256);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kAllocWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool CAUSAL>
cudaError_t fused_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                       const CUtensorMap& tdk, const CUtensorMap& tdv, const CUtensorMap& tdqacc, const BwdArgs& a,
                       cudaStream_t s) {
  auto kern = bwd_fused_kernel<D, CAUSAL>;
  constexpr int smem = FusedCfg<D>::SMEM_BYTES;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const long long nct = (a.N + 127) / 128;
  const long long tiles = nct * a.Z * a.H;
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  const long long units = CAUSAL ? (nct + 1) / 2 * a.Z * a.H : tiles;  // the kernel's next_tile units
  // One CTA per SM at most (shared memory), so a cooperative launch keeps every CTA resident: the grid
  // barrier before the kernel's last phase needs that (its counter is zeroed by the preprocess).
  const unsigned grid = unsigned(units < sm_count() ? units : sm_count());
  BwdArgs args = a;
  CUtensorMap m[7] = {tq, tk, tv, tdo, tdk, tdv, tdqacc};
  void* params[8] = {&m[0], &m[1], &m[2], &m[3], &m[4], &m[5], &m[6], &args};
  e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(kThreads), params, smem, s);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace

void bwd_f16_box_rows(int D, bool dq_pass, int variant, int* q_rows, int* kv_rows) {
  // dQ: 128-row query tiles; key blocks of the variant's block_n rows (the kernels' BK).
  // dK/dV: 128-row key tiles; query blocks of block_n rows (DkvPersistCfg::BQ or DkvSplitCfg::BQ).
  static_assert(DqSplitCfg<64>::BK == 128 && DqPersistCfg<64>::BK == 128 && DqAltCfg<64>::BK == 64, "dQ blocks");
  static_assert(DkvPersistCfg<64>::BQ == 128 && DkvSplitCfg<64, 64>::BQ == 64, "dK/dV blocks");
  const int bn = tile_supported(1, variant, D) ? kBwdTiles[variant].block_n : 0;
  *q_rows = dq_pass ? 128 : bn;
  *kv_rows = dq_pass ? bn : 128;
}

namespace {
template <bool DQ, int D, bool CAUSAL>
cudaError_t split_variant(int variant, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          const CUtensorMap& tdo, const CUtensorMap& t0, const CUtensorMap& t1, const BwdArgs& a,
                          cudaStream_t s) {
  static_assert(kNumBwdTiles == 2 && kBwdTiles[0].block_n == 128 && kBwdTiles[1].block_n == 64, "variant dispatch");
  if (variant == 0) {
    if constexpr (D <= 64) {
      if constexpr (DQ) return dq_impl<D, CAUSAL, 128>(tq, tk, tv, tdo, t0, a, s);
      else return dkdv_impl<D, CAUSAL, 128>(tq, tk, tv, tdo, t0, t1, a, s);
    }
    return cudaErrorNotSupported;
  }
  if constexpr (DQ) return dq_impl<D, CAUSAL, 64>(tq, tk, tv, tdo, t0, a, s);
  else return dkdv_impl<D, CAUSAL, 64>(tq, tk, tv, tdo, t0, t1, a, s);
}

template <bool DQ>
cudaError_t split_dispatch(int D, bool causal, int variant, const CUtensorMap& tq, const CUtensorMap& tk,
                           const CUtensorMap& tv, const CUtensorMap& tdo, const CUtensorMap& t0,
                           const CUtensorMap& t1, const BwdArgs& a, cudaStream_t s) {
  if (!tile_supported(1, variant, D)) return cudaErrorNotSupported;
#define TATTN_SPLIT_CASE(DD)                                                                      \
  case DD:                                                                                        \
    return causal ? split_variant<DQ, DD, true>(variant, tq, tk, tv, tdo, t0, t1, a, s)           \
                  : split_variant<DQ, DD, false>(variant, tq, tk, tv, tdo, t0, t1, a, s);
  switch (D) {
    TATTN_SPLIT_CASE(16)
    TATTN_SPLIT_CASE(32)
    TATTN_SPLIT_CASE(64)
    TATTN_SPLIT_CASE(128)
    default:
      return cudaErrorInvalidValue;
  }
#undef TATTN_SPLIT_CASE
}
}  // namespace

cudaError_t launch_bwd_dq_f16(int D, bool causal, int variant, const CUtensorMap& tq, const CUtensorMap& tk,
                              const CUtensorMap& tv, const CUtensorMap& tdo, const CUtensorMap& tdq, const BwdArgs& a,
                              cudaStream_t s) {
  return split_dispatch<true>(D, causal, variant, tq, tk, tv, tdo, tdq, tdq, a, s);
}

cudaError_t launch_bwd_dkdv_f16(int D, bool causal, int variant, const CUtensorMap& tq, const CUtensorMap& tk,
                                const CUtensorMap& tv, const CUtensorMap& tdo, const CUtensorMap& tdk,
                                const CUtensorMap& tdv, const BwdArgs& a, cudaStream_t s) {
  return split_dispatch<false>(D, causal, variant, tq, tk, tv, tdo, tdk, tdv, a, s);
}

static_assert(FusedCfg<64>::BQ == bwd_fused_query_rows(64) && FusedCfg<128>::BQ == bwd_fused_query_rows(128),
              "fused backward query blocks");

cudaError_t launch_bwd_fused_f16(int D, bool causal, const CUtensorMap& tq, const CUtensorMap& tk,
                                 const CUtensorMap& tv, const CUtensorMap& tdo, const CUtensorMap& tdk,
                                 const CUtensorMap& tdv, const CUtensorMap& tdqacc, const BwdArgs& a, cudaStream_t s) {
  switch (D) {
    case 16: return causal ? fused_impl<16, true>(tq, tk, tv, tdo, tdk, tdv, tdqacc, a, s)
                           : fused_impl<16, false>(tq, tk, tv, tdo, tdk, tdv, tdqacc, a, s);
    case 32: return causal ? fused_impl<32, true>(tq, tk, tv, tdo, tdk, tdv, tdqacc, a, s)
                           : fused_impl<32, false>(tq, tk, tv, tdo, tdk, tdv, tdqacc, a, s);
    case 64: return causal ? fused_impl<64, true>(tq, tk, tv, tdo, tdk, tdv, tdqacc, a, s)
                           : fused_impl<64, false>(tq, tk, tv, tdo, tdk, tdv, tdqacc, a, s);
    case 128: return causal ? fused_impl<128, true>(tq, tk, tv, tdo, tdk, tdv, tdqacc, a, s)
                            : fused_impl<128, false>(tq, tk, tv, tdo, tdk, tdv, tdqacc, a, s);
    default: return cudaErrorNotSupported;
  }
}


}  // namespace tattn
