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
//                warp 9       TMEM allocator + MMA issuer (one thread, event loop)
//                warps 10-11  idle (they complete the warpgroup for the register split)
// setmaxnreg moves registers from warpgroup 2 (48 per thread) to the softmax warpgroups (224), so a
// softmax thread keeps its whole score row in registers and reads S from TMEM once.
// TMEM (512 columns): S0, S1 [BN each] | P0, P1 [BN/2 each, fp16 pairs] | O0, O1 [D each]. P has its own
// buffer, so the tensor core computes S(j+1) of a tile while that tile's softmax still exponentiates
// S(j): as soon as a softmax warpgroup has S(j) in registers it releases the S buffer (s_free), and
// the MMA issuer starts the next QK^T. P then feeds the PV MMA as the A operand straight from TMEM.
// The running max is rescaled lazily: O (in TMEM) and l are only corrected when a row's max grows by
// more than kRescaleThreshold (log2 units); P values stay below 2^kRescaleThreshold, exact in fp16.
#include "common.cuh"
#include "kernels.h"

namespace tattn {
namespace {

constexpr float kRescaleThreshold = 8.0f;
// Of every 8 column pairs of a row, this many take exp2 on the FMA pipe (exp2_poly_x2) and the rest
// on MUFU (16 results/clk/SM), whose rate alone caps the D = 64 forward near half the tensor rate.
constexpr int kEmuPairs = 0;
// Register split (setmaxnreg): launch = 384 threads x 168 registers = 64512; softmax warpgroups take
// 224 and warpgroup 2 keeps 48: 8*32*224 + 4*32*48 = 63488 <= 64512.
constexpr int kSoftmaxRegs = 224;
constexpr int kProducerRegs = 48;

template <int D>
struct FwdCfg {
  static constexpr int BM = 128;                        // rows per query tile (2 tiles per CTA)
  static constexpr int BN = D == 128 ? 64 : 128;        // keys per block
  static constexpr int NS = 4;                          // K/V ring depth
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
  // q_full, k_full[NS], v_full[NS], kv_empty[NS], s_full[2], s_free[2], p_full[2], o_done[2], fin
  static constexpr int NBARS = 1 + 3 * NS + 9;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;  // tmem base (u32), abort flag (int)
  static constexpr int SMEM_USED = OFF_MISC + 16;
  // Request at least ~116 KB so exactly one CTA (which owns all 512 TMEM columns) fits per SM.
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  static constexpr uint32_t TM_S = 0;                   // + i * BN
  static constexpr uint32_t TM_P = 2 * BN;              // + i * BN / 2
  static constexpr uint32_t TM_O = 3 * BN;              // + i * D
  static_assert(3 * BN + 2 * D <= 512, "TMEM budget");
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BN, false);
  static constexpr uint32_t IDESC_PV = idesc_f16_f32(128, D, true);
};

template <int D>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_base, uint32_t k_base, uint32_t idesc) {
  using C = FwdCfg<D>;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t col = kk * 16 / C::CW, inner = ((kk * 16) % C::CW) * 2;
    const uint64_t a = smem_desc(q_base + col * C::QCHUNK + inner, 16, 8 * C::SWB, C::LAYOUT);
    const uint64_t b = smem_desc(k_base + col * C::KCHUNK + inner, 16, 8 * C::SWB, C::LAYOUT);
    mma_f16_ss(d_tmem, a, b, idesc, kk > 0 ? 1u : 0u);
  }
}

template <int D>
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_base, bool accumulate) {
  using C = FwdCfg<D>;
#pragma unroll
  for (int kk = 0; kk < C::BN / 16; ++kk) {
    const uint64_t b = smem_desc(v_base + kk * 16 * C::SWB, C::KCHUNK, 8 * C::SWB, C::LAYOUT);
    mma_f16_ts(d_tmem, p_tmem + kk * 8, b, C::IDESC_PV, (accumulate || kk > 0) ? 1u : 0u);
  }
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(384, 1)
    fwd_f16_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const FwdArgs args) {
  using C = FwdCfg<D>;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_u32 - raw_u32);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q = bars;
  uint64_t* bar_k_full = bars + 1;
  uint64_t* bar_v_full = bars + 1 + C::NS;
  uint64_t* bar_kv_empty = bars + 1 + 2 * C::NS;
  uint64_t* bar_s_full = bars + 1 + 3 * C::NS;
  uint64_t* bar_s_free = bar_s_full + 2;
  uint64_t* bar_p_full = bar_s_full + 4;
  uint64_t* bar_o_done = bar_s_full + 6;
  uint64_t* bar_fin = bar_s_full + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const CtaAbort ab{abort_flag, args.status};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int N = args.N;
  const int nct = (N + 2 * C::BM - 1) / (2 * C::BM);  // CTAs per (z, h)
  int bh, cta;
  if (CAUSAL) {  // longest-first: all heads' heaviest row blocks are scheduled first
    bh = blockIdx.x % (args.Z * args.H);
    cta = nct - 1 - blockIdx.x / (args.Z * args.H);
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
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_s_full[i], 1);
      mbar_init(&bar_s_free[i], 128);
      mbar_init(&bar_p_full[i], 128);
      mbar_init(&bar_o_done[i], 1);
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
      for (; j < nmax; ++j) {
        const int st = j % C::NS;
        if (j >= C::NS && !mbar_wait(&bar_kv_empty[st], ((j / C::NS) - 1) & 1, ab)) break;
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
    } else if (warp == 9 && lane == 0) {
      // -------------------------------------------------------------- MMA issuer (event loop)
      // Per tile: S(b) needs the tile's S buffer released (s_free of b-1) and K(b); PV(b) needs P(b)
      // (p_full of b) and V(b). Whatever is ready is issued; a K/V stage is released once every tile
      // that uses block b has issued PV(b).
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      bool ok = mbar_wait(bar_q, 0, ab);
      int next_s0 = 0, next_s1 = 0, next_pv0 = 0, next_pv1 = 0, released = 0;
      unsigned long long idle_since = 0;
      while (ok && (next_pv0 < n_0 || next_pv1 < n_1)) {
        bool progress = false;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int n = i ? n_1 : n_0;
          int& ns = i ? next_s1 : next_s0;
          int& np = i ? next_pv1 : next_pv0;
          if (ns < n && (ns == 0 || mbar_test(&bar_s_free[i], (ns - 1) & 1)) &&
              mbar_test(&bar_k_full[ns % C::NS], (ns / C::NS) & 1)) {
            tc_fence_after();
            issue_qk<D>(tmem + C::TM_S + i * BN, sQ + i * C::QTILE, sK + (ns % C::NS) * C::KTILE, idesc_s);
            mma_commit(&bar_s_full[i]);
            ++ns;
            progress = true;
          }
          if (np < ns && mbar_test(&bar_p_full[i], np & 1) && mbar_test(&bar_v_full[np % C::NS], (np / C::NS) & 1)) {
            tc_fence_after();
            issue_pv<D>(tmem + C::TM_O + i * D, tmem + C::TM_P + i * (BN / 2), sV + (np % C::NS) * C::KTILE, np > 0);
            mma_commit(&bar_o_done[i]);
            ++np;
            progress = true;
          }
        }
        while (released < nmax && (released >= n_0 || next_pv0 > released) && (released >= n_1 || next_pv1 > released)) {
          mma_commit(&bar_kv_empty[released % C::NS]);
          ++released;
        }
        if (progress) {
          idle_since = 0;
        } else {
          const unsigned long long now = globaltimer_ns();
          if (idle_since == 0) {
            idle_since = now;
          } else if (now - idle_since > kWaitLimitNs || *abort_flag) {
            if (!*abort_flag) {
              *abort_flag = 1;
              atomicOr(ab.status, kStatusWaitTimeout);
            }
            ok = false;
          }
        }
      }
      // All MMAs must retire before TMEM is released.
      mma_commit(bar_fin);
      mbar_drain(bar_fin, 0, 100ull * 1000ull * 1000ull);
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
    const uint32_t tP = tmem + lane_off + C::TM_P + i * (BN / 2);
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
      mbar_arrive(&bar_s_free[i]);  // the tensor core may now write S(j+1) of this tile

      // Columns past N (ragged tail) only occur in the last block; columns above the diagonal
      // (causal) in every block that reaches past the tile's first row (the last BM / BN blocks).
      const int col0 = j * BN;
      const bool last = (col0 + BN > N) || (CAUSAL && col0 + BN - 1 > row - t);
      int lim = N - col0;
      if (CAUSAL) lim = min(lim, row - col0 + 1);
      if (last) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c >= lim) s[c] = __float_as_uint(-INFINITY);
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; c += 4) {
        mx0 = fmax3(mx0, __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
        mx1 = fmax3(mx1, __uint_as_float(s[c + 2]), __uint_as_float(s[c + 3]));
      }
      const float m_cand = fmaxf(mx0, mx1) * scale;
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

      // P = exp2(S * scale - m): kEmuPairs of every 8 column pairs on the FMA pipe, the rest on MUFU.
      const uint64_t negm2 = f2(-m_run, -m_run);
      float ls0 = 0.f, ls1 = 0.f, ls2 = 0.f, ls3 = 0.f;
      uint32_t p[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const uint64_t x = ffma2(f2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), scale2, negm2);
        float2 e;
        if (((c / 2) & 7) < kEmuPairs) {
          e = f2_unpack(exp2_poly_x2(x));
        } else {
          const float2 xv = f2_unpack(x);
          e = make_float2(ex2_approx(xv.x), ex2_approx(xv.y));
        }
        if (last) {
          e.x = c < lim ? e.x : 0.f;
          e.y = c + 1 < lim ? e.y : 0.f;
        }
        if ((c / 2) & 1) {
          ls2 += e.x;
          ls3 += e.y;
        } else {
          ls0 += e.x;
          ls1 += e.y;
        }
        p[c / 2] = pack_half2(e.x, e.y);
      }
      l_run += (ls0 + ls1) + (ls2 + ls3);

      // PV(j-1) must have landed before P and O of this tile are touched again.
      if (j > 0) {
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
      __half* orow = reinterpret_cast<__half*>(args.o) + zi * args.so.z + hi * args.so.h + int64_t(row) * args.so.n;
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
      if (row < N) args.m[int64_t(bh) * N + row] = m_run + log2f(l_run);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool CAUSAL>
cudaError_t launch_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const FwdArgs& a,
                        cudaStream_t s) {
  using C = FwdCfg<D>;
  auto kern = fwd_f16_kernel<D, CAUSAL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const int nct = (a.N + 2 * C::BM - 1) / (2 * C::BM);
  const long long grid = (long long)nct * a.Z * a.H;
  if (grid <= 0) return cudaSuccess;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  kern<<<dim3((unsigned)grid), dim3(384), C::SMEM_BYTES, s>>>(tq, tk, tv, a);
  return cudaGetLastError();
}

}  // namespace

int fwd_f16_kv_rows(int D) {
  switch (D) {
    case 16: return FwdCfg<16>::BN;
    case 32: return FwdCfg<32>::BN;
    case 64: return FwdCfg<64>::BN;
    case 128: return FwdCfg<128>::BN;
    default: return 0;
  }
}

cudaError_t launch_fwd_f16(int D, bool causal, int tile_cfg, const CUtensorMap& tq, const CUtensorMap& tk,
                           const CUtensorMap& tv, const FwdArgs& a, cudaStream_t s) {
  (void)tile_cfg;  // one tile shape per head dim for now
#define TATTN_FWD_CASE(DD)                                                         \
  case DD:                                                                         \
    return causal ? launch_impl<DD, true>(tq, tk, tv, a, s) : launch_impl<DD, false>(tq, tk, tv, a, s);
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
