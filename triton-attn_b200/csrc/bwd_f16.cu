// FlashAttention-2 backward for fp16 on sm_100a: the dQ kernel (one CTA per query block) and the
// atomic-free dK/dV kernel (one CTA per key block), with TMA-fed shared memory, tcgen05 MMAs into TMEM
// and warp-specialised roles.
//
// Algorithm (reference src/tattn/kernels.py): P is rebuilt from the saved base-2 log-sum-exp,
// P = exp2(S * sm_scale * log2(e) - M); dS = P * (dP - D) with D = rowsum(dO * O);
//   dQ kernel    (kernels.py:242-321): S = Q K^T, dP = dO V^T, dQ += dS K, dQ *= sm_scale
//   dK/dV kernel (kernels.py:151-239): S^T = K Q^T, dP^T = V dO^T, dV += P^T dO, dK += dS^T Q, dK *= sm_scale
// No atomics: every output row is owned by exactly one CTA.
//
// Both kernels: TPC tiles of 128 rows per CTA (2, or 1 at D = 128), blocks of 64 along the other
// sequence axis. Warps 0 .. 4*TPC-1 are compute warpgroups (thread t owns TMEM lane t: one query row in
// the dQ kernel, one key row in the dK/dV kernel); the last warpgroup holds the TMA producer, one MMA
// issuer warp per tile (warp-converged, elect.sync issues, loop-invariant descriptors) and the TMEM
// allocator. With two tiles, setmaxnreg moves registers from that warpgroup to the compute warps.
//
// dQ TMEM per tile: S [64] | dP [64] | dS [32, fp16 pairs] | dQ [D]. dS has its own buffer, so the next
//   block's S and dP MMAs start as soon as the compute warps hold the current ones (s_free).
// dK/dV TMEM per tile: S^T [64] | dP^T [64] | dV [D] | dK [D]; P^T and dS^T (fp16) overwrite the first
//   32 columns of S^T and dP^T. The next block's S^T/dP^T MMAs are issued after this block's dV/dK
//   MMAs, and tcgen05 MMAs of one thread execute in order, so the overwrite never races the reads.
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
  static constexpr int TPC = D <= 64 ? 2 : 1; // tiles per CTA
  static constexpr int THREADS = TPC * 128 + 128;
};

// Register split for two tiles: launch = 384 x 168 = 64512; compute warps take 216, the producer
// warpgroup keeps 56: 8*32*216 + 4*32*56 = 62464 <= 64512.
constexpr int kComputeRegs = 216;
constexpr int kProducerRegs = 56;

// D[tmem] = A x B^T over K = D, A = 128 rows of a [rows, D] tile (K-major, chunk stride A_CHUNK), B =
// 64 rows of a [64, D] tile (K-major). `a`/`b` are the tiles' base descriptors.
template <int D, int A_CHUNK>
__device__ __forceinline__ void mma_rows_x_rows64(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc) {
  using L = BwdLayout<D>;
  asm volatile("" : "+l"(a), "+l"(b));  // opaque bases: offsets below stay compile-time constants
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int col = kk * 16 / L::CW, inner = ((kk * 16) % L::CW) * 2;
    mma_f16_ss_elect(d_tmem, a + uint64_t((col * A_CHUNK + inner) >> 4), b + uint64_t((col * L::CH64 + inner) >> 4),
                     idesc, kk > 0 ? 1u : 0u);
  }
}

// D[tmem] (+)= A x B, A from TMEM (128 lanes x 64 fp16 = 32 columns), B = a [64, D] tile read MN-major.
template <int D>
__device__ __forceinline__ void mma_tmem_x_tile64(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_mn, uint32_t idesc,
                                                  uint32_t accumulate) {
  using L = BwdLayout<D>;
  asm volatile("" : "+l"(b_mn));
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma_f16_ts_elect(d_tmem, a_tmem + kk * 8, b_mn + uint64_t((kk * 16 * L::SWB) >> 4), idesc,
                     kk > 0 ? 1u : accumulate);
}

__device__ __forceinline__ int cta_order(int nct, int zh, bool longest_first, int* bh) {
  if (longest_first) {
    *bh = blockIdx.x % zh;
    return blockIdx.x / zh;
  }
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
  if (EMU) return f2_unpack(exp2_poly_x2(x));
  const float2 v = f2_unpack(x);
  return make_float2(ex2_approx(v.x), ex2_approx(v.y));
}
// Of every 8 column pairs, this many take exp2 on the FMA pipe.
constexpr int kBwdEmuPairs = 2;

// =============================================================================================== dQ
template <int D>
struct DqCfg {
  using L = BwdLayout<D>;
  static constexpr int BN = 64;
  static constexpr int NS = 4;
  static constexpr int OFF_Q = 0;                              // TPC query tiles
  static constexpr int OFF_DO = L::TPC * L::T128;              // TPC dO tiles
  static constexpr int OFF_K = 2 * L::TPC * L::T128;           // NS key blocks
  static constexpr int OFF_V = OFF_K + NS * L::T64;            // NS value blocks
  static constexpr int OFF_BAR = OFF_V + NS * L::T64;
  // q_full, kv_full[NS], kv_empty[2][NS], s_full[2], s_free[2], ds_full[2], dq_done[2], fin[2]
  static constexpr int NBARS = 1 + 3 * NS + 10;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  static constexpr uint32_t T_S = 0, T_DP = 64, T_DS = 128, T_DQ = 160;  // per-tile offsets
  static constexpr uint32_t TILE_COLS = (160 + D + 31) / 32 * 32;
  static_assert(L::TPC * TILE_COLS <= 512, "TMEM budget");
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BN, false);
  static constexpr uint32_t IDESC_DQ = idesc_f16_f32(128, D, true);
};

// dS = P * (dP - D_r) for 64 columns of one row; P = exp2(S * scale - M_r). MASK zeroes columns >= lim.
template <bool MASK>
__device__ __forceinline__ void ds_row64(const uint32_t* s, const uint32_t* dp, uint32_t* ds, uint64_t scale2,
                                         uint64_t negm2, uint64_t negd2, int lim) {
#pragma unroll
  for (int c = 0; c < 64; c += 2) {
    const uint64_t x = ffma2(f2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), scale2, negm2);
    float2 e = (((c / 2) & 7) < kBwdEmuPairs) ? exp2_pair<true>(x) : exp2_pair<false>(x);
    if (MASK) {
      e.x = c < lim ? e.x : 0.f;
      e.y = c + 1 < lim ? e.y : 0.f;
    }
    const uint64_t d = fadd2(f2(__uint_as_float(dp[c]), __uint_as_float(dp[c + 1])), negd2);
    const float2 v = f2_unpack(fmul2(f2(e.x, e.y), d));
    ds[c / 2] = pack_half2(v.x, v.y);
  }
}

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(BwdLayout<D>::THREADS, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  const BwdArgs args) {
  using C = DqCfg<D>;
  using L = BwdLayout<D>;
  constexpr int TPC = L::TPC;
  constexpr int TMA_WARP = 4 * TPC, ALLOC_WARP = 4 * TPC + 3;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q = bars;
  uint64_t* bar_kv_full = bars + 1;                 // [NS]
  uint64_t* bar_kv_empty = bars + 1 + C::NS;        // [2][NS]
  uint64_t* bar_s_full = bars + 1 + 3 * C::NS;      // [2]
  uint64_t* bar_s_free = bar_s_full + 2;            // [2]
  uint64_t* bar_ds_full = bar_s_full + 4;           // [2]
  uint64_t* bar_dq_done = bar_s_full + 6;           // [2]
  uint64_t* bar_fin = bar_s_full + 8;               // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int zh = args.Z * args.H;
  const int nct = (N + 128 * TPC - 1) / (128 * TPC);
  int bh;
  int cta = cta_order(nct, zh, CAUSAL, &bh);
  if (CAUSAL) cta = nct - 1 - cta;  // longest-first: the highest query tiles see the most keys
  const int zi = bh / args.H, hi = bh % args.H;
  const int NBk = (N + C::BN - 1) / C::BN;
  const int row0_0 = 128 * TPC * cta, row0_1 = row0_0 + 128;
  const int n0 = row0_0 >= N ? 0 : (CAUSAL ? min((row0_0 + 128) / C::BN, NBk) : NBk);
  const int n1 = (TPC < 2 || row0_1 >= N) ? 0 : (CAUSAL ? min((row0_1 + 128) / C::BN, NBk) : NBk);
  const int nmax = max(n0, n1);

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 1);
      mbar_init(&bar_kv_empty[C::NS + s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_s_full[i], 1);
      mbar_init(&bar_s_free[i], 128);
      mbar_init(&bar_ds_full[i], 128);
      mbar_init(&bar_dq_done[i], 1);
      mbar_init(&bar_fin[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == ALLOC_WARP) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == TMA_WARP && lane == 0) {
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

  if (warp >= TMA_WARP) {
    if constexpr (TPC == 2) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == TMA_WARP && lane == 0) {
      // -------------------------------------------------------------- TMA producer
      const uint32_t qbytes = ((n0 > 0) + (n1 > 0)) * 2 * L::T128;
      mbar_arrive_expect_tx(bar_q, qbytes);
      for (int t = 0; t < TPC; ++t) {
        if ((t ? n1 : n0) == 0) continue;
        const int r0 = t ? row0_1 : row0_0;
        for (int ch = 0; ch < L::NCH; ++ch) {
          tma_load_4d(sQ + t * L::T128 + ch * L::CH128, &tm_q, ch * L::CW, r0, hi, zi, bar_q);
          tma_load_4d(sDO + t * L::T128 + ch * L::CH128, &tm_do, ch * L::CW, r0, hi, zi, bar_q);
        }
      }
      int j = 0;
      bool ok = true;
      for (; ok && j < nmax; ++j) {
        const int st = j % C::NS;
        if (j >= C::NS) {  // every tile that used this stage's previous block must be done with it
          const int old = j - C::NS;
          for (int t = 0; t < TPC && ok; ++t)
            if (old < (t ? n1 : n0) && !mbar_wait(&bar_kv_empty[t * C::NS + st], ((j / C::NS) - 1) & 1, ab)) ok = false;
          if (!ok) break;
        }
        mbar_arrive_expect_tx(&bar_kv_full[st], 2 * L::T64);
        for (int ch = 0; ch < L::NCH; ++ch) {
          tma_load_4d(sK + st * L::T64 + ch * L::CH64, &tm_k, ch * L::CW, j * C::BN, hi, zi, &bar_kv_full[st]);
          tma_load_4d(sV + st * L::T64 + ch * L::CH64, &tm_v, ch * L::CW, j * C::BN, hi, zi, &bar_kv_full[st]);
        }
      }
      const unsigned long long lim = 100ull * 1000ull * 1000ull;
      mbar_drain(bar_q, 0, lim);
      for (int jj = max(0, j - C::NS); jj < j; ++jj) mbar_drain(&bar_kv_full[jj % C::NS], (jj / C::NS) & 1, lim);
    } else if (warp > TMA_WARP && warp <= TMA_WARP + TPC) {
      // -------------------------------------------------------------- MMA issuer of tile t
      const int t = warp - TMA_WARP - 1;
      const int n = t ? n1 : n0;
      const uint32_t tb = tmem + t * C::TILE_COLS;
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      const uint64_t dQ = smem_desc(sQ + t * L::T128, 16, 8 * L::SWB, L::LAYOUT);
      const uint64_t dDO = smem_desc(sDO + t * L::T128, 16, 8 * L::SWB, L::LAYOUT);
      const uint64_t dK = smem_desc(sK, 16, 8 * L::SWB, L::LAYOUT);
      const uint64_t dV = smem_desc(sV, 16, 8 * L::SWB, L::LAYOUT);
      const uint64_t dKmn = smem_desc(sK, L::CH64, 8 * L::SWB, L::LAYOUT);
      auto issue_s_dp = [&](int b) {
        const uint64_t so = uint64_t(((b % C::NS) * L::T64) >> 4);
        mma_rows_x_rows64<D, L::CH128>(tb + C::T_S, dQ, dK + so, idesc_s);
        mma_rows_x_rows64<D, L::CH128>(tb + C::T_DP, dDO, dV + so, C::IDESC_S);
        mma_commit_elect(&bar_s_full[t]);
      };
      bool ok = n > 0 && warp_wait(bar_q, 0, ab) && warp_wait(&bar_kv_full[0], 0, ab);
      if (ok) {
        tc_fence_after();
        issue_s_dp(0);
      }
      for (int j = 0; ok && j < n; ++j) {
        if (j + 1 < n) {
          const int b = j + 1;
          if (!warp_wait(&bar_s_free[t], j & 1, ab) || !warp_wait(&bar_kv_full[b % C::NS], (b / C::NS) & 1, ab)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s_dp(b);
        }
        if (!warp_wait(&bar_ds_full[t], j & 1, ab)) { ok = false; break; }
        tc_fence_after();
        mma_tmem_x_tile64<D>(tb + C::T_DQ, tb + C::T_DS, dKmn + uint64_t(((j % C::NS) * L::T64) >> 4), C::IDESC_DQ,
                             j > 0 ? 1u : 0u);
        mma_commit_elect(&bar_dq_done[t]);
        mma_commit_elect(&bar_kv_empty[t * C::NS + j % C::NS]);
      }
      mma_commit_elect(&bar_fin[t]);
      mbar_drain(&bar_fin[t], 0, 100ull * 1000ull * 1000ull);
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    if constexpr (TPC == 2) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kComputeRegs));
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
    const uint64_t scale2 = f2(scale, scale), negm2 = f2(-m_r, -m_r), negd2 = f2(-d_r, -d_r);
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!warp_wait(&bar_s_full[t], j & 1, ab)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[64], dp[64];
      tmem_load_cols<64>(tb + C::T_S, s);
      tmem_load_cols<64>(tb + C::T_DP, dp);
      tmem_wait_ld();
      reg_fence<64>(s);
      reg_fence<64>(dp);
      tc_fence_before();
      mbar_arrive(&bar_s_free[t]);  // the tensor core may now write S/dP of the next block
      const int col0 = j * C::BN;
      const bool masked = (col0 + C::BN > N) || (CAUSAL && col0 + C::BN - 1 > row0);
      const int lim = (CAUSAL ? min(N, row + 1) : N) - col0;  // valid columns: c < lim
      uint32_t ds[32];
      if (masked)
        ds_row64<true>(s, dp, ds, scale2, negm2, negd2, lim);
      else
        ds_row64<false>(s, dp, ds, scale2, negm2, negd2, lim);
      if (j > 0) {  // the dQ MMA of the previous block has read dS
        if (!warp_wait(&bar_dq_done[t], (j - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
      }
      tmem_store_cols<32>(tb + C::T_DS, ds);
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
        tmem_load_cols<W>(tb + C::T_DQ + c0, o);
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
  if (warp == ALLOC_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================================ dK/dV
template <int D>
struct DkvCfg {
  using L = BwdLayout<D>;
  static constexpr int BQ = 64;                           // query rows per block
  static constexpr int NS = 4;
  static constexpr int OFF_K = 0;                         // TPC key tiles
  static constexpr int OFF_V = L::TPC * L::T128;          // TPC value tiles
  static constexpr int OFF_Q = 2 * L::TPC * L::T128;      // NS query blocks
  static constexpr int OFF_DO = OFF_Q + NS * L::T64;      // NS dO blocks
  static constexpr int OFF_MD = OFF_DO + NS * L::T64;     // per tile: 2 buffers x (64 M + 64 delta) fp32
  static constexpr int OFF_BAR = OFF_MD + L::TPC * 2 * 128 * 4;
  // kv_full, q_full[NS], q_empty[2][NS], s_full[2], p_full[2], acc_done[2], fin[2]
  static constexpr int NBARS = 1 + 3 * NS + 8;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16;
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  static constexpr uint32_t TILE_COLS = 128 + 2 * D;      // S^T, dP^T, dV, dK
  static_assert(L::TPC * TILE_COLS <= 512, "TMEM budget");
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BQ, false);
  static constexpr uint32_t IDESC_ACC = idesc_f16_f32(128, D, true);
};

// P^T and dS^T for 64 query columns of one key row. MASK keeps only columns c_lo <= c < c_hi.
template <bool MASK>
__device__ __forceinline__ void pds_row64(const uint32_t* s, const uint32_t* dp, const float* mq, const float* dq,
                                          uint32_t* pt, uint32_t* dst, uint64_t scale2, int c_lo, int c_hi) {
#pragma unroll
  for (int c = 0; c < 64; c += 4) {
    const float4 mv = *reinterpret_cast<const float4*>(mq + c);
    const float4 dv = *reinterpret_cast<const float4*>(dq + c);
#pragma unroll
    for (int h = 0; h < 4; h += 2) {
      const int cc = c + h;
      const uint64_t negm = f2(-(h ? mv.z : mv.x), -(h ? mv.w : mv.y));
      const uint64_t negd = f2(-(h ? dv.z : dv.x), -(h ? dv.w : dv.y));
      const uint64_t x = ffma2(f2(__uint_as_float(s[cc]), __uint_as_float(s[cc + 1])), scale2, negm);
      float2 e = (((cc / 2) & 7) < kBwdEmuPairs) ? exp2_pair<true>(x) : exp2_pair<false>(x);
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

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(BwdLayout<D>::THREADS, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const BwdArgs args) {
  using C = DkvCfg<D>;
  using L = BwdLayout<D>;
  constexpr int TPC = L::TPC;
  constexpr int TMA_WARP = 4 * TPC, ALLOC_WARP = 4 * TPC + 3;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_kv = bars;
  uint64_t* bar_q_full = bars + 1;                  // [NS]
  uint64_t* bar_q_empty = bars + 1 + C::NS;         // [2][NS]
  uint64_t* bar_s_full = bars + 1 + 3 * C::NS;      // [2]
  uint64_t* bar_p_full = bar_s_full + 2;            // [2]
  uint64_t* bar_acc = bar_s_full + 4;               // [2]
  uint64_t* bar_fin = bar_s_full + 6;               // [2]
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
  // Key tile t: keys [k0_t, k0_t + 128), query blocks [lo_t, NBq).
  const int k0_0 = 128 * TPC * cta, k0_1 = k0_0 + 128;
  const bool valid_0 = k0_0 < N, valid_1 = TPC == 2 && k0_1 < N;
  const int lo_0 = CAUSAL ? k0_0 / C::BQ : 0, lo_1 = CAUSAL ? k0_1 / C::BQ : 0;
  const int i_begin = lo_0;
  const int nq = NBq - i_begin;  // query blocks this CTA walks (tile 0 is always valid)

  if (threadIdx.x == 0) {
    mbar_init(bar_kv, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&bar_q_full[s], 1);
      mbar_init(&bar_q_empty[s], 1);
      mbar_init(&bar_q_empty[C::NS + s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bar_s_full[t], 1);
      mbar_init(&bar_p_full[t], 128);
      mbar_init(&bar_acc[t], 1);
      mbar_init(&bar_fin[t], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == ALLOC_WARP) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == TMA_WARP && lane == 0) {
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

  if (warp >= TMA_WARP) {
    if constexpr (TPC == 2) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == TMA_WARP && lane == 0) {
      // -------------------------------------------------------------- TMA producer
      const uint32_t kvbytes = (valid_0 ? 2 * L::T128 : 0) + (valid_1 ? 2 * L::T128 : 0);
      mbar_arrive_expect_tx(bar_kv, kvbytes);
      for (int t = 0; t < TPC; ++t) {
        if (!(t ? valid_1 : valid_0)) continue;
        const int k0 = t ? k0_1 : k0_0;
        for (int ch = 0; ch < L::NCH; ++ch) {
          tma_load_4d(sK + t * L::T128 + ch * L::CH128, &tm_k, ch * L::CW, k0, hi, zi, bar_kv);
          tma_load_4d(sV + t * L::T128 + ch * L::CH128, &tm_v, ch * L::CW, k0, hi, zi, bar_kv);
        }
      }
      int it = 0;
      bool ok = true;
      for (; ok && it < nq; ++it) {
        const int st = it % C::NS;
        const int i = i_begin + it;
        if (it >= C::NS) {  // every tile that used this stage's previous block must be done with it
          if (valid_0 && !mbar_wait(&bar_q_empty[st], ((it / C::NS) - 1) & 1, ab)) ok = false;
          if (ok && valid_1 && !mbar_wait(&bar_q_empty[C::NS + st], ((it / C::NS) - 1) & 1, ab)) ok = false;
          if (!ok) break;
        }
        mbar_arrive_expect_tx(&bar_q_full[st], 2 * L::T64);
        for (int ch = 0; ch < L::NCH; ++ch) {
          tma_load_4d(sQ + st * L::T64 + ch * L::CH64, &tm_q, ch * L::CW, i * C::BQ, hi, zi, &bar_q_full[st]);
          tma_load_4d(sDO + st * L::T64 + ch * L::CH64, &tm_do, ch * L::CW, i * C::BQ, hi, zi, &bar_q_full[st]);
        }
      }
      const unsigned long long lim = 100ull * 1000ull * 1000ull;
      mbar_drain(bar_kv, 0, lim);
      for (int jj = max(0, it - C::NS); jj < it; ++jj) mbar_drain(&bar_q_full[jj % C::NS], (jj / C::NS) & 1, lim);
    } else if (warp > TMA_WARP && warp <= TMA_WARP + TPC) {
      // -------------------------------------------------------------- MMA issuer of key tile t
      const int t = warp - TMA_WARP - 1;
      const bool valid = t ? valid_1 : valid_0;
      const int lo = t ? lo_1 : lo_0;
      const int n = valid ? NBq - lo : 0;
      const int it0 = lo - i_begin;  // first ring slot this tile reads
      const uint32_t tb = tmem + t * C::TILE_COLS;
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      const uint64_t dKt = smem_desc(sK + t * L::T128, 16, 8 * L::SWB, L::LAYOUT);
      const uint64_t dVt = smem_desc(sV + t * L::T128, 16, 8 * L::SWB, L::LAYOUT);
      const uint64_t dQk = smem_desc(sQ, 16, 8 * L::SWB, L::LAYOUT);
      const uint64_t dDOk = smem_desc(sDO, 16, 8 * L::SWB, L::LAYOUT);
      const uint64_t dQmn = smem_desc(sQ, L::CH64, 8 * L::SWB, L::LAYOUT);
      const uint64_t dDOmn = smem_desc(sDO, L::CH64, 8 * L::SWB, L::LAYOUT);
      // Ring slots before it0 are never read by this tile: release each once, in order (it0 < NS),
      // so this tile's q_empty phases line up with the producer's slot count.
      if (valid && lane == 0) {
        for (int it = 0; it < it0 && it < nq; ++it) mbar_arrive(&bar_q_empty[t * C::NS + it % C::NS]);
      }
      __syncwarp();
      auto issue_s = [&](int it) {
        const uint64_t so = uint64_t(((it % C::NS) * L::T64) >> 4);
        mma_rows_x_rows64<D, L::CH128>(tb, dKt, dQk + so, idesc_s);
        mma_rows_x_rows64<D, L::CH128>(tb + 64, dVt, dDOk + so, C::IDESC_S);
        mma_commit_elect(&bar_s_full[t]);
      };
      bool ok = n > 0 && warp_wait(bar_kv, 0, ab) && warp_wait(&bar_q_full[it0 % C::NS], (it0 / C::NS) & 1, ab);
      if (ok) {
        tc_fence_after();
        issue_s(it0);
      }
      for (int cnt = 0; ok && cnt < n; ++cnt) {
        const int it = it0 + cnt;
        const uint64_t so = uint64_t(((it % C::NS) * L::T64) >> 4);
        if (!warp_wait(&bar_p_full[t], cnt & 1, ab)) { ok = false; break; }
        tc_fence_after();
        mma_tmem_x_tile64<D>(tb + 128, tb, dDOmn + so, C::IDESC_ACC, cnt > 0 ? 1u : 0u);      // dV += P^T dO
        mma_tmem_x_tile64<D>(tb + 128 + D, tb + 64, dQmn + so, C::IDESC_ACC, cnt > 0 ? 1u : 0u);  // dK += dS^T Q
        mma_commit_elect(&bar_q_empty[t * C::NS + it % C::NS]);
        if (cnt + 1 < n) {
          const int it1 = it + 1;
          if (!warp_wait(&bar_q_full[it1 % C::NS], (it1 / C::NS) & 1, ab)) { ok = false; break; }
          tc_fence_after();
          issue_s(it1);
        }
      }
      mma_commit_elect(&bar_acc[t]);
      mma_commit_elect(&bar_fin[t]);
      mbar_drain(&bar_fin[t], 0, 100ull * 1000ull * 1000ull);
    }
  } else {
    // ------------------------------------------------------------------ compute warpgroups
    if constexpr (TPC == 2) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kComputeRegs));
    const int t = warp / 4;
    const int r = threadIdx.x % 128;
    const int k0 = t ? k0_1 : k0_0;
    const int lo = t ? lo_1 : lo_0;
    const int key = k0 + r;
    const int n = (t ? valid_1 : valid_0) ? NBq - lo : 0;
    const uint32_t tb = tmem + (uint32_t((warp % 4) * 32) << 16) + t * C::TILE_COLS;
    const uint64_t scale2 = f2(args.qk_scale, args.qk_scale);
    float* mdt = md + t * 256;  // [2 buffers][64 M | 64 delta]
    const float* mrow = args.m + int64_t(bh) * N;
    const float* drow = args.delta + int64_t(bh) * N;
    // Prefetch M (threads 0-63) or delta (64-127) of the first query block into a register.
    float pre = 0.f;
    if (n > 0) {
      const int q = lo * C::BQ + (r & 63);
      pre = q < N ? (r < 64 ? mrow[q] : drow[q]) : 0.f;
    }
    bool ok = true;
    for (int cnt = 0; cnt < n; ++cnt) {
      const int i = lo + cnt;
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
      const int q0 = i * C::BQ;
      const bool masked = (q0 + C::BQ > N) || (CAUSAL && q0 < k0 + 127) || (k0 + 128 > N);
      // valid query columns c: c_lo <= c < c_hi
      const int c_lo = CAUSAL ? max(0, key - q0) : 0;
      const int c_hi = key < N ? N - q0 : 0;
      uint32_t pt[32], dst[32];
      if (masked)
        pds_row64<true>(s, dp, mq, mq + 64, pt, dst, scale2, c_lo, c_hi);
      else
        pds_row64<false>(s, dp, mq, mq + 64, pt, dst, scale2, c_lo, c_hi);
      tmem_store_cols<32>(tb, pt);
      tmem_store_cols<32>(tb + 64, dst);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_p_full[t]);
    }
    if (ok && n > 0 && warp_wait(&bar_acc[t], 0, ab)) {
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
  if (warp == ALLOC_WARP) {
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
  using L = BwdLayout<D>;
  const long long grid = (long long)((a.N + 128 * L::TPC - 1) / (128 * L::TPC)) * a.Z * a.H;
  return launch_common(bwd_dq_kernel<D, CAUSAL>, DqCfg<D>::SMEM_BYTES, L::THREADS, grid, tq, tk, tv, tdo, a, s);
}

template <int D, bool CAUSAL>
cudaError_t dkdv_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                      const BwdArgs& a, cudaStream_t s) {
  using L = BwdLayout<D>;
  const long long grid = (long long)((a.N + 128 * L::TPC - 1) / (128 * L::TPC)) * a.Z * a.H;
  return launch_common(bwd_dkdv_kernel<D, CAUSAL>, DkvCfg<D>::SMEM_BYTES, L::THREADS, grid, tq, tk, tv, tdo, a, s);
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
