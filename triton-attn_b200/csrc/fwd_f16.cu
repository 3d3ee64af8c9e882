// FlashAttention-2 forward for fp16 on sm_100a: TMA-fed shared-memory tiles, tcgen05 MMAs with TMEM
// accumulators, warp-specialised roles.
//
// Algorithm (the reference's _fwd_kernel, src/tattn/kernels.py:57-148): for each 128-row query tile,
// loop over key blocks, S = Q K^T, online softmax in base 2 (scores scaled by sm_scale*log2(e), exp2),
// O = sum(P V) / l, and M = m + log2(l) saved per row. Causal tiles stop at the diagonal block.
//
// B200 mapping (one CTA per SM, 384 threads = 3 warpgroups):
//   warpgroup 0 (warps 0-3)   softmax for query tile 0 (thread t owns TMEM lane t = query row t)
//   warpgroup 1 (warps 4-7)   softmax for query tile 1
//   warpgroup 2: warp 8       TMA producer (Q tiles once, then K/V blocks through an NS-stage ring)
//                warps 9, 10  MMA issuers for tile 0 and tile 1 (one elected lane issues)
//                warp 11      TMEM allocator
// setmaxnreg moves registers from warpgroup 2 (56 per thread) to the softmax warpgroups (216), so a
// softmax thread keeps its whole score row in registers and reads S from TMEM once.
// TMEM (512 columns): S0, S1 [BN each] | P0, P1 [BN/2 each, fp16 pairs] | O0, O1 [D each]. P has its own
// buffer, so the tensor core computes S(j+1) of a tile while that tile's softmax still exponentiates
// S(j): as soon as a softmax warpgroup has S(j) in registers it releases the S buffer (s_free) and
// its tile's issuer starts the next QK^T. P then feeds the PV MMA as the A operand straight from
// TMEM. The two warpgroups ping-pong on the exponent pass (the MUFU-bound part) through a token pair
// of mbarriers; a warpgroup hands the turn over before its last quarter of columns.
// The running max is rescaled lazily: O (in TMEM) and l are only corrected when a row's max grows by
// more than kRescaleThreshold (log2 units); P values stay below 2^kRescaleThreshold, exact in fp16.
#include "common.cuh"
#include "kernels.h"
#include "tiles.h"

namespace tattn {
namespace {

constexpr float kRescaleThreshold = 8.0f;
// Of every 8 column pairs of a row, this many take exp2 on the FMA pipe (exp2_poly_x2) and the rest
// on MUFU (16 results/clk/SM), whose rate alone caps the D = 64 forward near half the tensor rate.
constexpr int kEmuPairs = 2;
// Register split (setmaxnreg): launch = 384 threads x 168 registers = 64512; softmax warpgroups take
// 216 and warpgroup 2 keeps 56: 8*32*216 + 4*32*56 = 62464 <= 64512.
constexpr int kSoftmaxRegs = 216;
constexpr int kProducerRegs = 56;

// Geometry of one tile variant (tiles.h, kFwdTiles): head dim D, BN_ keys per block, NS_ ring stages.
template <int D, int BN_, int NS_>
struct FwdCfg {
  static constexpr int BM = 128;                        // rows per query tile (2 tiles per CTA)
  static constexpr int BN = BN_;                        // keys per block
  static constexpr int NS = NS_;                        // K/V ring depth
  static constexpr int CW = D < 64 ? D : 64;            // columns per swizzle chunk
  static constexpr int NCH = D / CW;                    // chunks per row (2 for D = 128)
  static constexpr int SWB = CW * 2;                    // swizzle span in bytes (32/64/128)
  static constexpr uint32_t LAYOUT = SWB == 128 ? 2u : (SWB == 64 ? 4u : 6u);
  static constexpr int QCHUNK = BM * SWB;               // one 128-row chunk
  static constexpr int QTILE = QCHUNK * NCH;            // one [128, D] fp16 query tile
  static constexpr int KCHUNK = BN * SWB;               // one BN-row chunk
  static constexpr int KTILE = KCHUNK * NCH;            // one [BN, D] fp16 key / value block
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = 2 * QTILE;
  static constexpr int OFF_V = OFF_K + NS * KTILE;
  static constexpr int OFF_BAR = OFF_V + NS * KTILE;
  // q_full, k_full[NS], v_full[NS], kv_empty[2][NS], s_full[2], o_done[2], exp_done[2], fin[2],
  // s_free[2], p_full[2]
  static constexpr int NBARS = 1 + 4 * NS + 12;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;  // tmem base (u32), abort flag (int), head index (int)
  static constexpr int SMEM_USED = OFF_MISC + 16;
  // Request at least ~116 KB so exactly one CTA (which owns all 512 TMEM columns) fits per SM.
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  // TMEM: S_i [BN], P_i [BN / 2, fp16 pairs], O_i [D] per tile. Where S, P and O of both tiles do not
  // fit 512 columns (D = 128 with 128-key blocks), P_i is written over the first half of S_i (ALIAS_P):
  // the MMAs of a CTA run in issue order, so S_i(j + 1), issued after PV_i(j), overwrites P_i(j) only
  // once PV_i(j) has read it.
  static constexpr bool ALIAS_P = 3 * BN + 2 * D > 512;
  static constexpr uint32_t TM_S = 0;                             // + i * BN
  static constexpr uint32_t TM_P = ALIAS_P ? TM_S : 2 * BN;       // + i * BN (ALIAS_P) or i * BN / 2
  static constexpr uint32_t TM_O = ALIAS_P ? 2 * BN : 3 * BN;     // + i * D
  static constexpr uint32_t P_STRIDE = ALIAS_P ? BN : BN / 2;     // columns between P_0 and P_1
  static_assert((ALIAS_P ? 2 * BN : 3 * BN) + 2 * D <= 512, "TMEM budget");
  static_assert(OFF_MISC + 16 + 1024 <= 232448, "shared memory budget");
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BN, false);
  static constexpr uint32_t IDESC_PV = idesc_f16_f32(128, D, true);
};

// S_i = Q_i K^T for the K block in ring stage ST: D/16 MMAs (K = 16 each). All descriptor offsets are
// compile-time constants added to loop-invariant base descriptors.
template <typename C, int D, int ST>
__device__ __forceinline__ void issue_qk_st(int i, uint32_t d_tmem, uint64_t dQ, uint64_t dK, uint32_t idesc) {
  // Opaque copies: keep the compiler from hoisting every stage's descriptors into registers.
  asm volatile("" : "+l"(dQ), "+l"(dK));
  const uint64_t a0 = i ? dQ + uint64_t(C::QTILE >> 4) : dQ;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int col = kk * 16 / C::CW, inner = ((kk * 16) % C::CW) * 2;
    mma_f16_ss_elect(d_tmem, a0 + uint64_t((col * C::QCHUNK + inner) >> 4),
                     dK + uint64_t((ST * C::KTILE + col * C::KCHUNK + inner) >> 4), idesc, kk > 0 ? 1u : 0u);
  }
}
// Ring stage `st` (runtime) to the stage-specialised issue (compile-time offsets).
template <typename C, int D, int ST = 0>
__device__ __forceinline__ void issue_qk_stage(int st, int i, uint32_t d_tmem, uint64_t dQ, uint64_t dK,
                                               uint32_t idesc) {
  if constexpr (ST + 1 < C::NS) {
    if (st != ST) {
      issue_qk_stage<C, D, ST + 1>(st, i, d_tmem, dQ, dK, idesc);
      return;
    }
  }
  issue_qk_st<C, D, ST>(i, d_tmem, dQ, dK, idesc);
}

// O_i += P_i V for the V block in ring stage ST: BN/16 MMAs with P (fp16) read from TMEM.
template <typename C, int D, int ST>
__device__ __forceinline__ void issue_pv_st(uint32_t d_tmem, uint32_t p_tmem, uint64_t dV, uint32_t accumulate) {
  asm volatile("" : "+l"(dV));
#pragma unroll
  for (int kk = 0; kk < C::BN / 16; ++kk)
    mma_f16_ts_elect(d_tmem, p_tmem + kk * 8, dV + uint64_t((ST * C::KTILE + kk * 16 * C::SWB) >> 4), C::IDESC_PV,
                     kk > 0 ? 1u : accumulate);
}
template <typename C, int D, int ST = 0>
__device__ __forceinline__ void issue_pv_stage(int st, uint32_t d_tmem, uint32_t p_tmem, uint64_t dV,
                                               uint32_t accumulate) {
  if constexpr (ST + 1 < C::NS) {
    if (st != ST) {
      issue_pv_stage<C, D, ST + 1>(st, d_tmem, p_tmem, dV, accumulate);
      return;
    }
  }
  issue_pv_st<C, D, ST>(d_tmem, p_tmem, dV, accumulate);
}

// Max of one row of raw scores; MASK ignores columns >= lim.
template <int BN, bool MASK>
__device__ __forceinline__ float row_max(const uint32_t* s, int lim) {
  float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int c = 0; c < BN; c += 2) {
    float a = __uint_as_float(s[c]), b = __uint_as_float(s[c + 1]);
    if (MASK) {
      a = c < lim ? a : -INFINITY;
      b = c + 1 < lim ? b : -INFINITY;
    }
    m[(c / 2) & 3] = fmax3(m[(c / 2) & 3], a, b);
  }
  return fmax3(fmaxf(m[0], m[1]), m[2], m[3]);
}

// One row of P = exp2(S * scale - m) for columns [C0, C1) as fp16 pairs (p[c/2] = columns c, c+1) and
// its fp32 sum. kEmuPairs of every 8 column pairs use the FMA-pipe exp2, the rest MUFU. MASK zeroes
// columns >= lim.
template <int C0, int C1, bool MASK>
__device__ __forceinline__ float exp_cols(const uint32_t* s, uint32_t* p, uint64_t scale2, uint64_t negm2, int lim) {
  uint64_t acc0 = 0, acc1 = 0;
#pragma unroll
  for (int c = C0; c < C1; c += 2) {
    const uint64_t x = ffma2(f2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), scale2, negm2);
    float2 e;
    if (((c / 2) & 7) < kEmuPairs) {
      e = f2_unpack(exp2_poly_x2(x));
    } else {
      const float2 xv = f2_unpack(x);
      e = make_float2(ex2_approx(xv.x), ex2_approx(xv.y));
    }
    if (MASK) {
      e.x = c < lim ? e.x : 0.f;
      e.y = c + 1 < lim ? e.y : 0.f;
    }
    if ((c / 2) & 1)
      acc1 = fadd2(acc1, f2(e.x, e.y));
    else
      acc0 = fadd2(acc0, f2(e.x, e.y));
    p[c / 2] = pack_half2(e.x, e.y);
  }
  const float2 t = f2_unpack(fadd2(acc0, acc1));
  return t.x + t.y;
}

template <int D, bool CAUSAL, int BN_, int NS_>
__global__ void __launch_bounds__(384, 1)
    fwd_f16_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const FwdArgs args) {
  using C = FwdCfg<D, BN_, NS_>;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q = bars;
  uint64_t* bar_k_full = bars + 1;                   // [NS]
  uint64_t* bar_v_full = bars + 1 + C::NS;           // [NS]
  uint64_t* bar_kv_empty = bars + 1 + 2 * C::NS;     // [2][NS]: tile i is done with the block in stage s
  uint64_t* bar_s_full = bars + 1 + 4 * C::NS;       // [2]
  uint64_t* bar_o_done = bar_s_full + 2;             // [2]
  uint64_t* bar_exp_done = bar_s_full + 4;           // [2]: warpgroup i finished the exponent pass
  uint64_t* bar_fin = bar_s_full + 6;                // [2]
  uint64_t* bar_s_free = bar_s_full + 8;             // [2]: the tile's softmax holds S(j) in registers
  uint64_t* bar_p_full = bar_s_full + 10;            // [2]: the tile's softmax has stored P(j)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status, args.wait_limit_ns};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int nct = (N + 2 * C::BM - 1) / (2 * C::BM);  // CTAs per (z, h)
  int bh, cta;
  if (CAUSAL) {  // longest first within groups of heads whose K/V fit in L2 (the highest row blocks see the most keys)
    cta = nct - 1 - causal_cta_rank(nct, args.Z * args.H, N, D, &bh);
  } else {  // row blocks of one head adjacent: K/V of a head stay hot in L2
    bh = blockIdx.x / nct;
    cta = blockIdx.x % nct;
  }
  const int zi = bh / args.H, hi = bh % args.H;
  const int NB = (N + BN - 1) / BN;
  // Query tile i of this CTA: rows [row0_i, row0_i + 128), key blocks [0, n_i).
  const int row0_0 = 2 * cta * C::BM, row0_1 = row0_0 + C::BM;
  const int n_0 = row0_0 >= N ? 0 : (CAUSAL ? min((row0_0 + C::BM + BN - 1) / BN, NB) : NB);
  const int n_1 = row0_1 >= N ? 0 : (CAUSAL ? min((row0_1 + C::BM + BN - 1) / BN, NB) : NB);
  const int nmax = max(n_0, n_1);

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&bar_k_full[s], 1);
      mbar_init(&bar_v_full[s], 1);
      mbar_init(&bar_kv_empty[s], 1);
      mbar_init(&bar_kv_empty[C::NS + s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_s_full[i], 1);
      mbar_init(&bar_o_done[i], 1);
      mbar_init(&bar_exp_done[i], 128);
      mbar_init(&bar_fin[i], 1);
      mbar_init(&bar_s_free[i], 128);
      mbar_init(&bar_p_full[i], 128);
    }
    *abort_flag = 0;
    *reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8) = bh;  // for the softmax epilogue
    fence_mbar_init();
  }
  if (warp == 11) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const uint32_t sQ = base_u32 + C::OFF_Q, sK = base_u32 + C::OFF_K, sV = base_u32 + C::OFF_V;

  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == 8 && lane == 0) {
      // -------------------------------------------------------------- TMA producer
      const uint32_t qbytes = (n_0 > 0 ? C::QTILE : 0) + (n_1 > 0 ? C::QTILE : 0);
      mbar_arrive_expect_tx(bar_q, qbytes);
      for (int i = 0; i < 2; ++i) {
        if ((i ? n_1 : n_0) == 0) continue;
        for (int ch = 0; ch < C::NCH; ++ch)
          tma_load_4d(sQ + i * C::QTILE + ch * C::QCHUNK, &tm_q, ch * C::CW, i ? row0_1 : row0_0, hi, zi, bar_q);
      }
      int j = 0;
      bool ok = true;
      for (; ok && j < nmax; ++j) {
        const int st = j % C::NS;
        if (j >= C::NS) {  // both tiles that used the stage's previous block must be done with it
          const int old = j - C::NS;
          for (int i = 0; i < 2 && ok; ++i)
            if (old < (i ? n_1 : n_0) && !mbar_wait(&bar_kv_empty[i * C::NS + st], ((j / C::NS) - 1) & 1, ab))
              ok = false;
          if (!ok) break;
        }
        mbar_arrive_expect_tx(&bar_k_full[st], C::KTILE);
        for (int ch = 0; ch < C::NCH; ++ch)
          tma_load_4d(sK + st * C::KTILE + ch * C::KCHUNK, &tm_k, ch * C::CW, j * BN, hi, zi, &bar_k_full[st]);
        mbar_arrive_expect_tx(&bar_v_full[st], C::KTILE);
        for (int ch = 0; ch < C::NCH; ++ch)
          tma_load_4d(sV + st * C::KTILE + ch * C::KCHUNK, &tm_v, ch * C::CW, j * BN, hi, zi, &bar_v_full[st]);
      }
      // Every copy this CTA issued must land before the CTA exits (instant on the normal path).
      const unsigned long long lim = 100ull * 1000ull * 1000ull;
      mbar_drain(bar_q, 0, lim);
      for (int jj = max(0, j - C::NS); jj < j; ++jj) {
        mbar_drain(&bar_k_full[jj % C::NS], (jj / C::NS) & 1, lim);
        mbar_drain(&bar_v_full[jj % C::NS], (jj / C::NS) & 1, lim);
      }
    } else if (warp == 9 || warp == 10) {
      // -------------------------------------------------------------- MMA issuer of tile i
      // Order within a tile = the order its softmax releases inputs: S(j+1) once the softmax holds
      // S(j) in registers (s_free), then PV(j) once it has stored P(j) (p_full). The whole warp runs
      // the loop; elect.sync inside each MMA picks the issuing lane, and every descriptor is a
      // loop-invariant base plus a compile-time constant, so the MMAs go out at tensor-core rate.
      const int i = warp - 9;
      const int n = i ? n_1 : n_0;
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      const uint64_t dQ = smem_desc(sQ, 16, 8 * C::SWB, C::LAYOUT);
      const uint64_t dK = smem_desc(sK, 16, 8 * C::SWB, C::LAYOUT);
      const uint64_t dV = smem_desc(sV, C::KCHUNK, 8 * C::SWB, C::LAYOUT);
      const uint32_t tS = tmem + C::TM_S + i * BN, tP = tmem + C::TM_P + i * C::P_STRIDE, tO = tmem + C::TM_O + i * D;
      bool ok = n > 0 && warp_wait(bar_q, 0, ab) && warp_wait(&bar_k_full[0], 0, ab);
      if (ok) {
        tc_fence_after();
        issue_qk_stage<C, D>(0, i, tS, dQ, dK, idesc_s);
        mma_commit_elect(&bar_s_full[i]);
      }
      for (int j = 0; ok && j < n; ++j) {
        if (C::ALIAS_P) {
          // PV(j) reads P(j) where S(j) was, then S(j + 1) overwrites both (in issue order).
          if (!warp_wait(&bar_p_full[i], j & 1, ab) || !warp_wait(&bar_v_full[j % C::NS], (j / C::NS) & 1, ab)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv_stage<C, D>(j % C::NS, tO, tP, dV, j > 0 ? 1u : 0u);
          mma_commit_elect(&bar_o_done[i]);
          mma_commit_elect(&bar_kv_empty[i * C::NS + j % C::NS]);
          if (j + 1 < n) {
            const int b = j + 1;
            if (!warp_wait(&bar_k_full[b % C::NS], (b / C::NS) & 1, ab)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_qk_stage<C, D>(b % C::NS, i, tS, dQ, dK, idesc_s);
            mma_commit_elect(&bar_s_full[i]);
          }
          continue;
        }
        if (j + 1 < n) {
          const int b = j + 1;
          if (!warp_wait(&bar_s_free[i], j & 1, ab) || !warp_wait(&bar_k_full[b % C::NS], (b / C::NS) & 1, ab)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_qk_stage<C, D>(b % C::NS, i, tS, dQ, dK, idesc_s);
          mma_commit_elect(&bar_s_full[i]);
        }
        if (!warp_wait(&bar_p_full[i], j & 1, ab) || !warp_wait(&bar_v_full[j % C::NS], (j / C::NS) & 1, ab)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv_stage<C, D>(j % C::NS, tO, tP, dV, j > 0 ? 1u : 0u);
        mma_commit_elect(&bar_o_done[i]);
        mma_commit_elect(&bar_kv_empty[i * C::NS + j % C::NS]);
      }
      // Every MMA of this tile must retire before TMEM is released.
      mma_commit_elect(&bar_fin[i]);
      mbar_drain(&bar_fin[i], 0, 100ull * 1000ull * 1000ull);
    }
  } else {
    // ------------------------------------------------------------------ softmax warpgroups
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    const int i = warp / 4;
    const int t = threadIdx.x % 128;
    const int row = (i ? row0_1 : row0_0) + t;
    const int n = i ? n_1 : n_0;
    const uint32_t lane_off = uint32_t((warp % 4) * 32) << 16;
    const uint32_t tS = tmem + lane_off + C::TM_S + i * BN;
    const uint32_t tP = tmem + lane_off + C::TM_P + i * C::P_STRIDE;
    const uint32_t tO = tmem + lane_off + C::TM_O + i * D;
    const float scale = args.qk_scale;
    const uint64_t scale2 = f2(scale, scale);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!warp_wait(&bar_s_full[i], j & 1, ab)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[BN];
      tmem_load_cols<BN>(tS, s);
      tmem_wait_ld();
      reg_fence<BN>(s);
      tc_fence_before();
      if (!C::ALIAS_P) mbar_arrive(&bar_s_free[i]);  // the tensor core may now write S(j+1) of this tile

      // Columns past N (ragged tail) only occur in the last block; columns above the diagonal
      // (causal) in every block that reaches past the tile's first row (the last BM / BN blocks).
      const int col0 = j * BN;
      const bool last = (col0 + BN > N) || (CAUSAL && col0 + BN - 1 > row - t);
      int lim = N - col0;
      if (CAUSAL) lim = min(lim, row - col0 + 1);
      const float m_cand = (last ? row_max<BN, true>(s, lim) : row_max<BN, false>(s, lim)) * scale;
      float alpha = 1.f;
      bool need = false;
      if (j == 0) {
        m_run = m_cand;
      } else if (m_cand > m_run + kRescaleThreshold) {
        alpha = ex2_approx(m_run - m_cand);
        m_run = m_cand;
        l_run *= alpha;
        need = true;
      }

      // Ping-pong: the two warpgroups take turns on the exponent pass (the MUFU-bound part), so one
      // exponentiates while the other loads S, reduces the max and stores P. Order: tile 0 block j,
      // tile 1 block j, tile 0 block j+1, ...; a turn is only awaited if the other tile has that block.
      const int other_n = i ? n_0 : n_1;
      if (i == 1 ? (j < other_n) : (j >= 1 && j - 1 < other_n)) {
        if (!warp_wait(&bar_exp_done[1 - i], (i == 1 ? j : j - 1) & 1, ab)) { ok = false; break; }
      }
      // P = exp2(S * scale - m); the masked variant only runs for blocks that need it, so the column
      // tests never cost the unmasked blocks anything.
      // With 128-key blocks the turn is handed over after seven eighths of the columns, so the other
      // tile's pass starts while this one finishes and the exponent unit does not idle across the
      // hand-off (measured at BN = 128: 7/8 best, 3/4 within 1%, 1/2 8% slower; slower at BN = 64).
      constexpr int kSplit = BN == 128 ? BN * 7 / 8 : BN;
      uint32_t p[BN / 2];
      const uint64_t negm2 = f2(-m_run, -m_run);
      l_run += last ? exp_cols<0, kSplit, true>(s, p, scale2, negm2, lim) : exp_cols<0, kSplit, false>(s, p, scale2, negm2, lim);
      mbar_arrive(&bar_exp_done[i]);
      if constexpr (kSplit < BN)
        l_run += last ? exp_cols<kSplit, BN, true>(s, p, scale2, negm2, lim)
                      : exp_cols<kSplit, BN, false>(s, p, scale2, negm2, lim);

      // PV(j-1) must have landed before P and O of this tile are touched again (ALIAS_P: it has, since
      // S(j) was issued after it and has completed).
      if (!C::ALIAS_P && j > 0) {
        if (!warp_wait(&bar_o_done[i], (j - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          constexpr int W = D < 32 ? D : 32;
          uint32_t o[W];
          tmem_load_cols<W>(tO + c0, o);
          tmem_wait_ld();
          reg_fence<W>(o);
#pragma unroll
          for (int c = 0; c < W; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_store_cols<W>(tO + c0, o);
        }
      }
      tmem_store_cols<BN / 2>(tP, p);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar_p_full[i]);
    }

    if (ok && n > 0 && warp_wait(&bar_o_done[i], (n - 1) & 1, ab)) {
      tc_fence_after();
      const float inv_l = 1.f / l_run;
      // The head index from shared memory rather than a register held through the block loop (one
      // spilled register fewer).
      const int bh_e = *reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8);
      const int zi_e = bh_e / args.H, hi_e = bh_e % args.H;
      __half* orow = reinterpret_cast<__half*>(args.o) + zi_e * args.so.z + hi_e * args.so.h + int64_t(row) * args.so.n;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        constexpr int W = D < 32 ? D : 32;
        uint32_t o[W];
        tmem_load_cols<W>(tO + c0, o);
        tmem_wait_ld();
        reg_fence<W>(o);
        uint32_t h[W / 2];
#pragma unroll
        for (int c = 0; c < W; c += 2)
          h[c / 2] = pack_half2(__uint_as_float(o[c]) * inv_l, __uint_as_float(o[c + 1]) * inv_l);
        if (row < N) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
          for (int v = 0; v < W / 8; ++v) dst[v] = make_uint4(h[4 * v], h[4 * v + 1], h[4 * v + 2], h[4 * v + 3]);
        }
      }
      if (row < N) args.m[int64_t(bh_e) * N + row] = m_run + log2f(l_run);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 11) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool CAUSAL, int BN, int NS>
cudaError_t launch_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const FwdArgs& a,
                        cudaStream_t s) {
  using C = FwdCfg<D, BN, NS>;
  auto kern = fwd_f16_kernel<D, CAUSAL, BN, NS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const int nct = (a.N + 2 * C::BM - 1) / (2 * C::BM);
  const long long grid = (long long)nct * a.Z * a.H;
  if (grid <= 0) return cudaSuccess;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  kern<<<dim3((unsigned)grid), dim3(384), C::SMEM_BYTES, s>>>(tq, tk, tv, a);
  return cudaGetLastError();
}

// Variant v (tiles.h, kFwdTiles) for head dim D; variants whose blocks do not fit D's TMEM budget are
// not instantiated.
template <int D, bool CAUSAL>
cudaError_t launch_variant(int v, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                           const FwdArgs& a, cudaStream_t s) {
  static_assert(kNumFwdTiles == 3, "variant dispatch");
  switch (v) {
    case 0:
      if constexpr (D <= 64) return launch_impl<D, CAUSAL, kFwdTiles[0].block_n, kFwdTiles[0].stages>(tq, tk, tv, a, s);
      break;
    case 1:
      return launch_impl<D, CAUSAL, kFwdTiles[1].block_n, kFwdTiles[1].stages>(tq, tk, tv, a, s);
    case 2:
      return launch_impl<D, CAUSAL, kFwdTiles[2].block_n, kFwdTiles[2].stages>(tq, tk, tv, a, s);
    default:
      break;
  }
  return cudaErrorNotSupported;
}

}  // namespace

int fwd_f16_kv_rows(int D, int variant) {
  return tile_supported(0, variant, D) ? kFwdTiles[variant].block_n : 0;
}

cudaError_t launch_fwd_f16(int D, bool causal, int variant, const CUtensorMap& tq, const CUtensorMap& tk,
                           const CUtensorMap& tv, const FwdArgs& a, cudaStream_t s) {
  if (!tile_supported(0, variant, D)) return cudaErrorNotSupported;
#define TATTN_FWD_CASE(DD)                                                                     \
  case DD:                                                                                     \
    return causal ? launch_variant<DD, true>(variant, tq, tk, tv, a, s)                        \
                  : launch_variant<DD, false>(variant, tq, tk, tv, a, s);
  switch (D) {
    TATTN_FWD_CASE(16)
    TATTN_FWD_CASE(32)
    TATTN_FWD_CASE(64)
    TATTN_FWD_CASE(128)
    default:
      return cudaErrorInvalidValue;
  }
#undef TATTN_FWD_CASE
}

}  // namespace tattn
