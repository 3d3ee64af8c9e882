// FlashAttention-2 backward for fp16 on sm_100a: the dQ kernel (one CTA per query block) and the
// atomic-free dK/dV kernel (one CTA per key block), with TMA-fed shared memory, tcgen05 MMAs into TMEM
// and warp-specialised roles (compute warpgroups, a TMA producer warp, an MMA-issuer warp).
//
// Algorithm (reference src/tattn/kernels.py): P is rebuilt from the saved base-2 log-sum-exp,
// P = exp2(S * sm_scale * log2(e) - M); dS = P * (dP - D) with D = rowsum(dO * O);
//   dQ kernel   (kernels.py:242-321): S = Q K^T, dP = dO V^T, dQ += dS K, dQ *= sm_scale
//   dK/dV kernel (kernels.py:151-239): S^T = K Q^T, dP^T = V dO^T, dV += P^T dO, dK += dS^T Q, dK *= sm_scale
// No atomics: every output row is owned by exactly one CTA.
//
// dQ kernel: CTA = 2 query tiles x 128 rows, key blocks of 64. TMEM per tile: S [64] dP [64] dQ [D];
//   dS (fp16) overwrites the first 32 columns of S and is the A operand of the dQ MMA.
// dK/dV kernel: CTA = TPC key tiles x 128 keys (TPC = 2, or 1 for D = 128), query blocks of 64.
//   TMEM per tile: S^T [64] dP^T [64] dV [D] dK [D]; P^T and dS^T (fp16) overwrite the first 32
//   columns of S^T and dP^T and are the A operands of the dV and dK MMAs.
// In both, thread t of a compute warpgroup owns TMEM lane t (one query row, resp. one key row), and
// the two tiles of a CTA ping-pong between the tensor core and their compute warpgroups.
#include "common.cuh"
#include "kernels.h"

namespace tattn {
namespace {

template <int D>
struct BwdLayout {
  static constexpr int CW = D < 64 ? D : 64;  // columns per swizzle chunk
  static constexpr int NCH = D / CW;
  static constexpr int SWB = CW * 2;          // swizzle span, bytes
  static constexpr uint32_t LAYOUT = SWB == 128 ? 2u : (SWB == 64 ? 4u : 6u);
  static constexpr int CH128 = 128 * SWB;     // one 128-row chunk
  static constexpr int CH64 = 64 * SWB;       // one 64-row chunk
  static constexpr int T128 = CH128 * NCH;    // [128, D] fp16 tile
  static constexpr int T64 = CH64 * NCH;      // [64, D] fp16 tile
};

// A (M = 128 rows, K-major) x B (N rows, K-major) over K = D: both operands are [rows, D] tiles.
template <int D>
__device__ __forceinline__ void mma_rows_by_rows(uint32_t d_tmem, uint32_t a_base, int a_chunk, uint32_t b_base,
                                                 int b_chunk, uint32_t idesc) {
  using L = BwdLayout<D>;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t col = (kk * 16 / L::CW), inner = ((kk * 16) % L::CW) * 2;
    const uint64_t a = smem_desc(a_base + col * a_chunk + inner, 16, 8 * L::SWB, L::LAYOUT);
    const uint64_t b = smem_desc(b_base + col * b_chunk + inner, 16, 8 * L::SWB, L::LAYOUT);
    mma_f16_ss(d_tmem, a, b, idesc, kk > 0 ? 1u : 0u);
  }
}

// A from TMEM (M = 128, K = 64 fp16 = 32 columns) x B = a [64, D] tile read MN-major (N = D).
template <int D>
__device__ __forceinline__ void mma_tmem_by_tile64(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_base,
                                                   uint32_t idesc, bool accumulate) {
  using L = BwdLayout<D>;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint64_t b = smem_desc(b_base + kk * 16 * L::SWB, L::CH64, 8 * L::SWB, L::LAYOUT);
    mma_f16_ts(d_tmem, a_tmem + kk * 8, b, idesc, (accumulate || kk > 0) ? 1u : 0u);
  }
}

__device__ __forceinline__ int cta_order(int nct, int zh, bool longest_first, int* bh) {
  if (longest_first) {
    *bh = blockIdx.x % zh;
    return blockIdx.x / zh;
  }
  *bh = blockIdx.x / nct;
  return blockIdx.x % nct;
}

// =============================================================================================== dQ
template <int D>
struct DqCfg {
  using L = BwdLayout<D>;
  static constexpr int BN = 64;
  static constexpr int NS = D <= 64 ? 4 : 2;
  static constexpr int OFF_Q = 0;                         // 2 query tiles
  static constexpr int OFF_DO = 2 * L::T128;              // 2 dO tiles
  static constexpr int OFF_K = 4 * L::T128;               // NS key blocks
  static constexpr int OFF_V = OFF_K + NS * L::T64;       // NS value blocks
  static constexpr int OFF_BAR = OFF_V + NS * L::T64;
  // q_full, kv_full[NS], kv_empty[NS], s_full[2], ds_full[2], dq_done[2], fin
  static constexpr int NBARS = 1 + 2 * NS + 7;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  static constexpr uint32_t TILE_COLS = (128 + D + 31) / 32 * 32;  // S, dP, dQ (32-column aligned)
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BN, false);
  static constexpr uint32_t IDESC_DQ = idesc_f16_f32(128, D, true);
};

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(320, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  const BwdArgs args) {
  using C = DqCfg<D>;
  using L = BwdLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q = bars;
  uint64_t* bar_kv_full = bars + 1;
  uint64_t* bar_kv_empty = bars + 1 + C::NS;
  uint64_t* bar_s_full = bars + 1 + 2 * C::NS;
  uint64_t* bar_ds_full = bar_s_full + 2;
  uint64_t* bar_dq_done = bar_s_full + 4;
  uint64_t* bar_fin = bar_s_full + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int zh = args.Z * args.H;
  const int nct = (N + 255) / 256;
  int bh;
  int cta = cta_order(nct, zh, CAUSAL, &bh);
  if (CAUSAL) cta = nct - 1 - cta;
  const int zi = bh / args.H, hi = bh % args.H;
  const int NBk = (N + C::BN - 1) / C::BN;
  const int row0_0 = 256 * cta, row0_1 = 256 * cta + 128;
  const int n0 = row0_0 >= N ? 0 : (CAUSAL ? min((row0_0 + 128) / 64, NBk) : NBk);
  const int n1 = row0_1 >= N ? 0 : (CAUSAL ? min((row0_1 + 128) / 64, NBk) : NBk);
  const int nmax = max(n0, n1);

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_s_full[i], 1);
      mbar_init(&bar_ds_full[i], 128);
      mbar_init(&bar_dq_done[i], 1);
    }
    mbar_init(bar_fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
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

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t qbytes = ((n0 > 0) + (n1 > 0)) * 2 * L::T128;
      mbar_arrive_expect_tx(bar_q, qbytes);
      for (int t = 0; t < 2; ++t) {
        if ((t ? n1 : n0) == 0) continue;
        const int r0 = t ? row0_1 : row0_0;
        for (int ch = 0; ch < L::NCH; ++ch) {
          tma_load_4d(sQ + t * L::T128 + ch * L::CH128, &tm_q, ch * L::CW, r0, hi, zi, bar_q);
          tma_load_4d(sDO + t * L::T128 + ch * L::CH128, &tm_do, ch * L::CW, r0, hi, zi, bar_q);
        }
      }
      int j = 0;
      for (; j < nmax; ++j) {
        const int st = j % C::NS;
        if (j >= C::NS && !mbar_wait(&bar_kv_empty[st], ((j / C::NS) - 1) & 1, ab)) break;
        mbar_arrive_expect_tx(&bar_kv_full[st], 2 * L::T64);
        for (int ch = 0; ch < L::NCH; ++ch) {
          tma_load_4d(sK + st * L::T64 + ch * L::CH64, &tm_k, ch * L::CW, j * C::BN, hi, zi, &bar_kv_full[st]);
          tma_load_4d(sV + st * L::T64 + ch * L::CH64, &tm_v, ch * L::CW, j * C::BN, hi, zi, &bar_kv_full[st]);
        }
      }
      const unsigned long long lim = 100ull * 1000ull * 1000ull;
      mbar_drain(bar_q, 0, lim);
      for (int jj = max(0, j - C::NS); jj < j; ++jj) mbar_drain(&bar_kv_full[jj % C::NS], (jj / C::NS) & 1, lim);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      bool ok = mbar_wait(bar_q, 0, ab);
      if (ok && nmax > 0) ok = mbar_wait(&bar_kv_full[0], 0, ab);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t) {
          if ((t ? n1 : n0) == 0) continue;
          const uint32_t tb = tmem + t * C::TILE_COLS;
          mma_rows_by_rows<D>(tb, sQ + t * L::T128, L::CH128, sK, L::CH64, idesc_s);
          mma_rows_by_rows<D>(tb + 64, sDO + t * L::T128, L::CH128, sV, L::CH64, C::IDESC_S);
          mma_commit(&bar_s_full[t]);
        }
      }
      for (int j = 0; ok && j < nmax; ++j) {
        const int st = j % C::NS;
        for (int t = 0; t < 2 && ok; ++t) {
          const int n = t ? n1 : n0;
          if (j >= n) continue;
          const uint32_t tb = tmem + t * C::TILE_COLS;
          if (!mbar_wait(&bar_ds_full[t], j & 1, ab)) { ok = false; break; }
          tc_fence_after();
          mma_tmem_by_tile64<D>(tb + 128, tb, sK + st * L::T64, C::IDESC_DQ, j > 0);
          mma_commit(&bar_dq_done[t]);
          if (j + 1 < n) {
            const int st1 = (j + 1) % C::NS;
            if (!mbar_wait(&bar_kv_full[st1], ((j + 1) / C::NS) & 1, ab)) { ok = false; break; }
            tc_fence_after();
            mma_rows_by_rows<D>(tb, sQ + t * L::T128, L::CH128, sK + st1 * L::T64, L::CH64, idesc_s);
            mma_rows_by_rows<D>(tb + 64, sDO + t * L::T128, L::CH128, sV + st1 * L::T64, L::CH64, C::IDESC_S);
            mma_commit(&bar_s_full[t]);
          }
        }
        if (!ok) break;
        mma_commit(&bar_kv_empty[st]);
      }
      mma_commit(bar_fin);
      mbar_drain(bar_fin, 0, 100ull * 1000ull * 1000ull);
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    const int t = warp / 4;
    const int r = threadIdx.x % 128;
    const int row0 = t ? row0_1 : row0_0;
    const int n = t ? n1 : n0;
    const int row = row0 + r;
    const uint32_t tb = tmem + (uint32_t((warp % 4) * 32) << 16) + t * C::TILE_COLS;
    const float scale = args.qk_scale;
    const int64_t rowidx = int64_t(bh) * N + row;
    const float m_r = row < N ? args.m[rowidx] : 0.f;
    const float d_r = row < N ? args.delta[rowidx] : 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!warp_wait(&bar_s_full[t], j & 1, ab)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[64], dp[64];
      tmem_load_cols<64>(tb, s);
      tmem_load_cols<64>(tb + 64, dp);
      tmem_wait_ld();
      reg_fence<64>(s);
      reg_fence<64>(dp);
      const int col0 = j * C::BN;
      const bool masked = (col0 + C::BN > N) || (CAUSAL && col0 + C::BN - 1 > row0);
      const int lim = (CAUSAL ? min(N, row + 1) : N) - col0;  // valid columns: c < lim
      uint32_t ds[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        float p0 = ex2_approx(fmaf(__uint_as_float(s[c]), scale, -m_r));
        float p1 = ex2_approx(fmaf(__uint_as_float(s[c + 1]), scale, -m_r));
        if (masked) {
          p0 = c < lim ? p0 : 0.f;
          p1 = c + 1 < lim ? p1 : 0.f;
        }
        ds[c / 2] = pack_half2(p0 * (__uint_as_float(dp[c]) - d_r), p1 * (__uint_as_float(dp[c + 1]) - d_r));
      }
      tmem_store_cols<32>(tb, ds);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_ds_full[t]);
    }
    if (ok && n > 0 && warp_wait(&bar_dq_done[t], (n - 1) & 1, ab)) {
      tc_fence_after();
      __half* dst = reinterpret_cast<__half*>(args.dq) + rowidx * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        constexpr int W = D < 32 ? D : 32;
        uint32_t o[W];
        tmem_load_cols<W>(tb + 128 + c0, o);
        tmem_wait_ld();
        reg_fence<W>(o);
        uint32_t h[W / 2];
#pragma unroll
        for (int c = 0; c < W; c += 2)
          h[c / 2] = pack_half2(__uint_as_float(o[c]) * args.sm_scale, __uint_as_float(o[c + 1]) * args.sm_scale);
        if (row < N) {
          uint4* p = reinterpret_cast<uint4*>(dst + c0);
#pragma unroll
          for (int v = 0; v < W / 8; ++v) p[v] = make_uint4(h[4 * v], h[4 * v + 1], h[4 * v + 2], h[4 * v + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================================ dK/dV
template <int D>
struct DkvCfg {
  using L = BwdLayout<D>;
  static constexpr int TPC = D <= 64 ? 2 : 1;             // key tiles per CTA
  static constexpr int THREADS = TPC * 128 + 64;
  static constexpr int BQ = 64;                           // query rows per block
  static constexpr int NS = 4;
  static constexpr int OFF_K = 0;                         // TPC key tiles
  static constexpr int OFF_V = TPC * L::T128;             // TPC value tiles
  static constexpr int OFF_Q = 2 * TPC * L::T128;         // NS query blocks
  static constexpr int OFF_DO = OFF_Q + NS * L::T64;      // NS dO blocks
  static constexpr int OFF_MD = OFF_DO + NS * L::T64;     // per tile: 2 buffers x (64 M + 64 delta) fp32
  static constexpr int OFF_BAR = OFF_MD + TPC * 2 * 128 * 4;
  // kv_full, q_full[NS], q_empty[NS], s_full[TPC], p_full[TPC], acc_done[TPC], fin
  static constexpr int NBARS = 1 + 2 * NS + 3 * TPC + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  static constexpr uint32_t TILE_COLS = 128 + 2 * D;      // S^T, dP^T, dV, dK
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BQ, false);
  static constexpr uint32_t IDESC_ACC = idesc_f16_f32(128, D, true);
};

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(DkvCfg<D>::THREADS, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const BwdArgs args) {
  using C = DkvCfg<D>;
  using L = BwdLayout<D>;
  constexpr int TPC = C::TPC;
  constexpr int LOAD_WARP = 4 * TPC, MMA_WARP = 4 * TPC + 1;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_kv = bars;
  uint64_t* bar_q_full = bars + 1;
  uint64_t* bar_q_empty = bars + 1 + C::NS;
  uint64_t* bar_s_full = bars + 1 + 2 * C::NS;
  uint64_t* bar_p_full = bar_s_full + TPC;
  uint64_t* bar_acc = bar_s_full + 2 * TPC;
  uint64_t* bar_fin = bar_s_full + 3 * TPC;
  float* md = reinterpret_cast<float*>(smem + C::OFF_MD);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int zh = args.Z * args.H;
  const int nct = (N + 128 * TPC - 1) / (128 * TPC);
  int bh;
  // Causal: low key blocks see the most query blocks, so they go first.
  const int cta = cta_order(nct, zh, CAUSAL, &bh);
  const int zi = bh / args.H, hi = bh % args.H;
  const int NBq = (N + C::BQ - 1) / C::BQ;
  int k0[TPC], lo[TPC];
  bool valid[TPC];
#pragma unroll
  for (int t = 0; t < TPC; ++t) {
    k0[t] = 128 * (TPC * cta + t);
    valid[t] = k0[t] < N;
    lo[t] = CAUSAL ? k0[t] / C::BQ : 0;
  }
  const int i_begin = lo[0];
  const int nq = NBq - i_begin;  // query blocks this CTA walks (tile 0 is always valid)

  if (threadIdx.x == 0) {
    mbar_init(bar_kv, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&bar_q_full[s], 1);
      mbar_init(&bar_q_empty[s], 1);
    }
    for (int t = 0; t < TPC; ++t) {
      mbar_init(&bar_s_full[t], 1);
      mbar_init(&bar_p_full[t], 128);
      mbar_init(&bar_acc[t], 1);
    }
    mbar_init(bar_fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == LOAD_WARP && lane == 0) {
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

  if (warp == LOAD_WARP) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t kvbytes = 0;
      for (int t = 0; t < TPC; ++t) kvbytes += valid[t] ? 2 * L::T128 : 0;
      mbar_arrive_expect_tx(bar_kv, kvbytes);
      for (int t = 0; t < TPC; ++t) {
        if (!valid[t]) continue;
        for (int ch = 0; ch < L::NCH; ++ch) {
          tma_load_4d(sK + t * L::T128 + ch * L::CH128, &tm_k, ch * L::CW, k0[t], hi, zi, bar_kv);
          tma_load_4d(sV + t * L::T128 + ch * L::CH128, &tm_v, ch * L::CW, k0[t], hi, zi, bar_kv);
        }
      }
      int it = 0;
      for (; it < nq; ++it) {
        const int st = it % C::NS;
        const int i = i_begin + it;
        if (it >= C::NS && !mbar_wait(&bar_q_empty[st], ((it / C::NS) - 1) & 1, ab)) break;
        mbar_arrive_expect_tx(&bar_q_full[st], 2 * L::T64);
        for (int ch = 0; ch < L::NCH; ++ch) {
          tma_load_4d(sQ + st * L::T64 + ch * L::CH64, &tm_q, ch * L::CW, i * C::BQ, hi, zi, &bar_q_full[st]);
          tma_load_4d(sDO + st * L::T64 + ch * L::CH64, &tm_do, ch * L::CW, i * C::BQ, hi, zi, &bar_q_full[st]);
        }
      }
      const unsigned long long lim = 100ull * 1000ull * 1000ull;
      mbar_drain(bar_kv, 0, lim);
      for (int jj = max(0, it - C::NS); jj < it; ++jj) mbar_drain(&bar_q_full[jj % C::NS], (jj / C::NS) & 1, lim);
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      bool ok = mbar_wait(bar_kv, 0, ab);
      if (ok) ok = mbar_wait(&bar_q_full[0], 0, ab);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < TPC; ++t) {
          if (!valid[t] || i_begin < lo[t]) continue;
          const uint32_t tb = tmem + t * C::TILE_COLS;
          mma_rows_by_rows<D>(tb, sK + t * L::T128, L::CH128, sQ, L::CH64, idesc_s);
          mma_rows_by_rows<D>(tb + 64, sV + t * L::T128, L::CH128, sDO, L::CH64, C::IDESC_S);
          mma_commit(&bar_s_full[t]);
        }
      }
      for (int it = 0; ok && it < nq; ++it) {
        const int i = i_begin + it;
        const int st = it % C::NS;
#pragma unroll
        for (int t = 0; t < TPC; ++t) {
          if (!ok || !valid[t]) continue;
          const uint32_t tb = tmem + t * C::TILE_COLS;
          if (i >= lo[t]) {
            const int cnt = i - lo[t];
            if (!mbar_wait(&bar_p_full[t], cnt & 1, ab)) { ok = false; continue; }
            tc_fence_after();
            mma_tmem_by_tile64<D>(tb + 128, tb, sDO + st * L::T64, C::IDESC_ACC, cnt > 0);
            mma_tmem_by_tile64<D>(tb + 128 + D, tb + 64, sQ + st * L::T64, C::IDESC_ACC, cnt > 0);
            mma_commit(&bar_acc[t]);
          }
          if (i + 1 < NBq && i + 1 >= lo[t]) {
            const int st1 = (it + 1) % C::NS;
            if (!mbar_wait(&bar_q_full[st1], ((it + 1) / C::NS) & 1, ab)) { ok = false; continue; }
            tc_fence_after();
            mma_rows_by_rows<D>(tb, sK + t * L::T128, L::CH128, sQ + st1 * L::T64, L::CH64, idesc_s);
            mma_rows_by_rows<D>(tb + 64, sV + t * L::T128, L::CH128, sDO + st1 * L::T64, L::CH64, C::IDESC_S);
            mma_commit(&bar_s_full[t]);
          }
        }
        if (!ok) break;
        mma_commit(&bar_q_empty[st]);
      }
      mma_commit(bar_fin);
      mbar_drain(bar_fin, 0, 100ull * 1000ull * 1000ull);
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    const int t = warp / 4;
    const int r = threadIdx.x % 128;
    const int key = k0[t] + r;
    const int n = valid[t] ? NBq - lo[t] : 0;
    const uint32_t tb = tmem + (uint32_t((warp % 4) * 32) << 16) + t * C::TILE_COLS;
    const float scale = args.qk_scale;
    float* mdt = md + t * 256;  // [2 buffers][64 M | 64 delta]
    const float* mrow = args.m + int64_t(bh) * N;
    const float* drow = args.delta + int64_t(bh) * N;
    // Prefetch M (threads 0-63) or delta (64-127) of the first query block into a register.
    float pre = 0.f;
    if (n > 0) {
      const int q = lo[t] * C::BQ + (r & 63);
      pre = q < N ? (r < 64 ? mrow[q] : drow[q]) : 0.f;
    }
    bool ok = true;
    for (int cnt = 0; cnt < n; ++cnt) {
      const int i = lo[t] + cnt;
      const int buf = cnt & 1;
      mdt[buf * 128 + r] = pre;
      named_barrier_sync(1 + t, 128);
      if (cnt + 1 < n) {
        const int q = (i + 1) * C::BQ + (r & 63);
        pre = q < N ? (r < 64 ? mrow[q] : drow[q]) : 0.f;
      }
      // After a failed wait keep stepping through the named barriers (uniform trip count across the
      // warpgroup), so sibling warps never block on a barrier this warp no longer reaches.
      if (!ok) continue;
      if (!warp_wait(&bar_s_full[t], cnt & 1, ab)) { ok = false; continue; }
      tc_fence_after();
      uint32_t s[64], dp[64];
      tmem_load_cols<64>(tb, s);
      tmem_load_cols<64>(tb + 64, dp);
      tmem_wait_ld();
      reg_fence<64>(s);
      reg_fence<64>(dp);
      const float* mq = mdt + buf * 128;
      const float* dq = mq + 64;
      const int q0 = i * C::BQ;
      const bool masked = (q0 + C::BQ > N) || (CAUSAL && q0 < k0[t] + 127) || (k0[t] + 128 > N);
      // valid query columns c: c_lo <= c < c_hi
      const int c_lo = CAUSAL ? max(0, key - q0) : 0;
      const int c_hi = key < N ? N - q0 : 0;
      uint32_t pt[32], dst[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float4 mv = *reinterpret_cast<const float4*>(mq + (c & ~3));
        const float4 dv4 = *reinterpret_cast<const float4*>(dq + (c & ~3));
        const float m0 = (c & 2) ? mv.z : mv.x, m1 = (c & 2) ? mv.w : mv.y;
        const float d0 = (c & 2) ? dv4.z : dv4.x, d1 = (c & 2) ? dv4.w : dv4.y;
        float p0 = ex2_approx(fmaf(__uint_as_float(s[c]), scale, -m0));
        float p1 = ex2_approx(fmaf(__uint_as_float(s[c + 1]), scale, -m1));
        if (masked) {
          p0 = (c >= c_lo && c < c_hi) ? p0 : 0.f;
          p1 = (c + 1 >= c_lo && c + 1 < c_hi) ? p1 : 0.f;
        }
        pt[c / 2] = pack_half2(p0, p1);
        dst[c / 2] = pack_half2(p0 * (__uint_as_float(dp[c]) - d0), p1 * (__uint_as_float(dp[c + 1]) - d1));
      }
      tmem_store_cols<32>(tb, pt);
      tmem_store_cols<32>(tb + 64, dst);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_p_full[t]);
    }
    if (ok && n > 0 && warp_wait(&bar_acc[t], (n - 1) & 1, ab)) {
      tc_fence_after();
      const int64_t rowidx = int64_t(bh) * N + key;
#pragma unroll
      for (int which = 0; which < 2; ++which) {  // 0: dV, 1: dK * sm_scale
        __half* out = reinterpret_cast<__half*>(which ? args.dk : args.dv) + rowidx * D;
        const float mul = which ? args.sm_scale : 1.f;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          constexpr int W = D < 32 ? D : 32;
          uint32_t o[W];
          tmem_load_cols<W>(tb + 128 + which * D + c0, o);
          tmem_wait_ld();
          reg_fence<W>(o);
          uint32_t h[W / 2];
#pragma unroll
          for (int c = 0; c < W; c += 2)
            h[c / 2] = pack_half2(__uint_as_float(o[c]) * mul, __uint_as_float(o[c + 1]) * mul);
          if (key < N) {
            uint4* p = reinterpret_cast<uint4*>(out + c0);
#pragma unroll
            for (int v = 0; v < W / 8; ++v) p[v] = make_uint4(h[4 * v], h[4 * v + 1], h[4 * v + 2], h[4 * v + 3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <typename Kern>
cudaError_t launch_common(Kern kern, int smem, int threads, long long grid, const CUtensorMap& tq,
                          const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo, const BwdArgs& a,
                          cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  if (grid <= 0) return cudaSuccess;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  kern<<<dim3(unsigned(grid)), dim3(threads), smem, s>>>(tq, tk, tv, tdo, a);
  return cudaGetLastError();
}

template <int D, bool CAUSAL>
cudaError_t dq_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                    const BwdArgs& a, cudaStream_t s) {
  const long long grid = (long long)((a.N + 255) / 256) * a.Z * a.H;
  return launch_common(bwd_dq_kernel<D, CAUSAL>, DqCfg<D>::SMEM_BYTES, 320, grid, tq, tk, tv, tdo, a, s);
}

template <int D, bool CAUSAL>
cudaError_t dkdv_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                      const BwdArgs& a, cudaStream_t s) {
  using C = DkvCfg<D>;
  const long long grid = (long long)((a.N + 128 * C::TPC - 1) / (128 * C::TPC)) * a.Z * a.H;
  return launch_common(bwd_dkdv_kernel<D, CAUSAL>, C::SMEM_BYTES, C::THREADS, grid, tq, tk, tv, tdo, a, s);
}

}  // namespace

void bwd_f16_box_rows(bool dq_pass, int* q_rows, int* kv_rows) {
  // dQ: 128-row query tiles, DqCfg::BN-row key blocks; dK/dV: 128-row key tiles, DkvCfg::BQ-row query
  // blocks (the same for every head dim).
  *q_rows = dq_pass ? 128 : DkvCfg<64>::BQ;
  *kv_rows = dq_pass ? DqCfg<64>::BN : 128;
}

#define TATTN_BWD_SWITCH(FN)                                                                  \
  switch (D) {                                                                                \
    case 16: return causal ? FN<16, true>(tq, tk, tv, tdo, a, s) : FN<16, false>(tq, tk, tv, tdo, a, s);   \
    case 32: return causal ? FN<32, true>(tq, tk, tv, tdo, a, s) : FN<32, false>(tq, tk, tv, tdo, a, s);   \
    case 64: return causal ? FN<64, true>(tq, tk, tv, tdo, a, s) : FN<64, false>(tq, tk, tv, tdo, a, s);   \
    case 128: return causal ? FN<128, true>(tq, tk, tv, tdo, a, s) : FN<128, false>(tq, tk, tv, tdo, a, s); \
    default: return cudaErrorInvalidValue;                                                    \
  }

cudaError_t launch_bwd_dq_f16(int D, bool causal, int tile_cfg, const CUtensorMap& tq, const CUtensorMap& tk,
                              const CUtensorMap& tv, const CUtensorMap& tdo, const BwdArgs& a, cudaStream_t s) {
  (void)tile_cfg;
  TATTN_BWD_SWITCH(dq_impl)
}

cudaError_t launch_bwd_dkdv_f16(int D, bool causal, int tile_cfg, const CUtensorMap& tq, const CUtensorMap& tk,
                                const CUtensorMap& tv, const CUtensorMap& tdo, const BwdArgs& a, cudaStream_t s) {
  (void)tile_cfg;
  TATTN_BWD_SWITCH(dkdv_impl)
}

#undef TATTN_BWD_SWITCH

}  // namespace tattn
