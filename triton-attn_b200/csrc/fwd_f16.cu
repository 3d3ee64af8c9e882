// FlashAttention-2 forward for fp16 on sm_100a: TMA-fed shared-memory tiles, tcgen05 MMAs with TMEM
// accumulators, warp-specialised roles.
//
// Algorithm (the reference's _fwd_kernel, src/tattn/kernels.py:57-148): for each 128-row query tile,
// loop over 128-key blocks, S = Q K^T, online softmax in base 2 (scores scaled by sm_scale*log2(e),
// exp2), O = sum(P V) / l, and M = m + log2(l) saved per row. Causal tiles stop at the diagonal block.
//
// B200 mapping (one CTA per SM, 320 threads):
//   warps 0-3  softmax warpgroup for query tile 0 (thread t owns TMEM lane t = query row t)
//   warps 4-7  softmax warpgroup for query tile 1
//   warp 8     TMA producer: Q tiles once, then K/V blocks through an NS-stage ring
//   warp 9     TMEM allocator + MMA issuer (one thread)
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D). P (fp16) overwrites the
// first 64 columns of its S buffer and is the A operand of the PV MMA straight from TMEM.
// The two softmax warpgroups ping-pong: while one exponentiates its S tile, the tensor core runs the
// other tile's PV and next QK^T.
// The running max is rescaled lazily: O (in TMEM) and l are only corrected when a row's max grows by
// more than kRescaleThreshold (log2 units); P values stay below 2^kRescaleThreshold, exact in fp16.
#include "common.cuh"
#include "kernels.h"

namespace tattn {
namespace {

constexpr float kRescaleThreshold = 8.0f;

template <int D>
struct FwdCfg {
  static constexpr int BM = 128;                        // rows per query tile (2 tiles per CTA)
  static constexpr int BN = 128;                        // keys per block
  static constexpr int NS = D <= 64 ? 3 : 2;            // K/V ring depth
  static constexpr int CW = D < 64 ? D : 64;            // columns per swizzle chunk
  static constexpr int NCH = D / CW;                    // chunks per row (2 for D = 128)
  static constexpr int SWB = CW * 2;                    // swizzle span in bytes (32/64/128)
  static constexpr uint32_t LAYOUT = SWB == 128 ? 2u : (SWB == 64 ? 4u : 6u);
  static constexpr int CHUNK_BYTES = 128 * SWB;         // one 128-row chunk
  static constexpr int TILE_BYTES = CHUNK_BYTES * NCH;  // one [128, D] fp16 tile
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = 2 * TILE_BYTES;
  static constexpr int OFF_V = OFF_K + NS * TILE_BYTES;
  static constexpr int OFF_BAR = OFF_V + NS * TILE_BYTES;
  // barriers: q_full, k_full[NS], v_full[NS], kv_empty[NS], s_full[2], p_full[2], o_done[2], fin
  static constexpr int NBARS = 1 + 3 * NS + 7;
  static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;  // tmem base (u32), abort flag (int)
  static constexpr int SMEM_USED = OFF_MISC + 16;
  // Request at least ~116 KB so exactly one CTA (which owns all 512 TMEM columns) fits per SM.
  static constexpr int SMEM_BYTES = (SMEM_USED > 118784 ? SMEM_USED : 118784) + 1024;
  static constexpr uint32_t TM_S0 = 0, TM_S1 = 128, TM_O0 = 256, TM_O1 = 256 + D;
  static constexpr uint32_t IDESC_S = idesc_f16_f32(128, BN, false);
  static constexpr uint32_t IDESC_PV = idesc_f16_f32(128, D, true);
};

template <int D>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_base, uint32_t k_base, uint32_t idesc) {
  using C = FwdCfg<D>;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = (kk * 16 / C::CW) * C::CHUNK_BYTES + ((kk * 16) % C::CW) * 2;
    const uint64_t a = smem_desc(q_base + off, 16, 8 * C::SWB, C::LAYOUT);
    const uint64_t b = smem_desc(k_base + off, 16, 8 * C::SWB, C::LAYOUT);
    mma_f16_ss(d_tmem, a, b, idesc, kk > 0 ? 1u : 0u);
  }
}

template <int D>
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_base, bool accumulate) {
  using C = FwdCfg<D>;
#pragma unroll
  for (int kk = 0; kk < C::BN / 16; ++kk) {
    const uint64_t b = smem_desc(v_base + kk * 16 * C::SWB, C::CHUNK_BYTES, 8 * C::SWB, C::LAYOUT);
    mma_f16_ts(d_tmem, p_tmem + kk * 8, b, C::IDESC_PV, (accumulate || kk > 0) ? 1u : 0u);
  }
}

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(320, 1)
    fwd_f16_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const FwdArgs args) {
  using C = FwdCfg<D>;
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
  uint64_t* bar_p_full = bar_s_full + 2;
  uint64_t* bar_o_done = bar_s_full + 4;
  uint64_t* bar_fin = bar_s_full + 6;
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
  const int NB = (N + C::BN - 1) / C::BN;
  int row0[2], nblk[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    row0[i] = (2 * cta + i) * C::BM;
    nblk[i] = row0[i] >= N ? 0 : (CAUSAL ? min(2 * cta + i + 1, NB) : NB);
  }
  const int nmax = max(nblk[0], nblk[1]);

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&bar_k_full[s], 1);
      mbar_init(&bar_v_full[s], 1);
      mbar_init(&bar_kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_s_full[i], 1);
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

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t qbytes = 0;
      for (int i = 0; i < 2; ++i) qbytes += nblk[i] > 0 ? C::TILE_BYTES : 0;
      mbar_arrive_expect_tx(bar_q, qbytes);
      for (int i = 0; i < 2; ++i) {
        if (nblk[i] == 0) continue;
        for (int ch = 0; ch < C::NCH; ++ch)
          tma_load_4d(sQ + i * C::TILE_BYTES + ch * C::CHUNK_BYTES, &tm_q, ch * C::CW, row0[i], hi, zi, bar_q);
      }
      int j = 0;
      for (; j < nmax; ++j) {
        const int st = j % C::NS;
        if (j >= C::NS && !mbar_wait(&bar_kv_empty[st], ((j / C::NS) - 1) & 1, ab)) break;
        mbar_arrive_expect_tx(&bar_k_full[st], C::TILE_BYTES);
        for (int ch = 0; ch < C::NCH; ++ch)
          tma_load_4d(sK + st * C::TILE_BYTES + ch * C::CHUNK_BYTES, &tm_k, ch * C::CW, j * C::BN, hi, zi,
                      &bar_k_full[st]);
        mbar_arrive_expect_tx(&bar_v_full[st], C::TILE_BYTES);
        for (int ch = 0; ch < C::NCH; ++ch)
          tma_load_4d(sV + st * C::TILE_BYTES + ch * C::CHUNK_BYTES, &tm_v, ch * C::CW, j * C::BN, hi, zi,
                      &bar_v_full[st]);
      }
      // Every copy this CTA issued must land before the CTA exits (instant on the normal path).
      const unsigned long long lim = 100ull * 1000ull * 1000ull;
      mbar_drain(bar_q, 0, lim);
      for (int jj = max(0, j - C::NS); jj < j; ++jj) {
        mbar_drain(&bar_k_full[jj % C::NS], (jj / C::NS) & 1, lim);
        mbar_drain(&bar_v_full[jj % C::NS], (jj / C::NS) & 1, lim);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = C::IDESC_S | (args.negate_s ? (1u << 13) : 0u);
      const uint32_t tS[2] = {tmem + C::TM_S0, tmem + C::TM_S1};
      const uint32_t tO[2] = {tmem + C::TM_O0, tmem + C::TM_O1};
      bool ok = mbar_wait(bar_q, 0, ab);
      if (ok && nmax > 0) ok = mbar_wait(&bar_k_full[0], 0, ab);
      if (ok) {
        tc_fence_after();
        for (int i = 0; i < 2; ++i) {
          if (nblk[i] == 0) continue;
          issue_qk<D>(tS[i], sQ + i * C::TILE_BYTES, sK, idesc_s);
          mma_commit(&bar_s_full[i]);
        }
      }
      for (int j = 0; ok && j < nmax; ++j) {
        const int st = j % C::NS;
        if (!mbar_wait(&bar_v_full[st], (j / C::NS) & 1, ab)) { ok = false; break; }
        for (int i = 0; i < 2 && ok; ++i) {
          if (j >= nblk[i]) continue;
          if (!mbar_wait(&bar_p_full[i], j & 1, ab)) { ok = false; break; }
          tc_fence_after();
          issue_pv<D>(tO[i], tS[i], sV + st * C::TILE_BYTES, j > 0);
          mma_commit(&bar_o_done[i]);
          if (j + 1 < nblk[i]) {
            const int st1 = (j + 1) % C::NS;
            if (!mbar_wait(&bar_k_full[st1], ((j + 1) / C::NS) & 1, ab)) { ok = false; break; }
            tc_fence_after();
            issue_qk<D>(tS[i], sQ + i * C::TILE_BYTES, sK + st1 * C::TILE_BYTES, idesc_s);
            mma_commit(&bar_s_full[i]);
          }
        }
        if (!ok) break;
        mma_commit(&bar_kv_empty[st]);
      }
      // All MMAs must retire before TMEM is released.
      mma_commit(bar_fin);
      mbar_drain(bar_fin, 0, 100ull * 1000ull * 1000ull);
    }
  } else {
    // ------------------------------------------------------------------ softmax warpgroups
    const int i = warp / 4;
    const int t = threadIdx.x % 128;
    const int row = row0[i] + t;
    const int n = nblk[i];
    const uint32_t lane_off = uint32_t((warp % 4) * 32) << 16;
    const uint32_t tS = tmem + lane_off + (i ? C::TM_S1 : C::TM_S0);
    const uint32_t tO = tmem + lane_off + (i ? C::TM_O1 : C::TM_O0);
    const float scale = args.qk_scale;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!warp_wait(&bar_s_full[i], j & 1, ab)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[128];
      tmem_load_cols<128>(tS, s);
      tmem_wait_ld();
      reg_fence<128>(s);

      // Columns past N (ragged tail) and above the diagonal (causal) only occur in the last block.
      const bool last = (j == n - 1);
      const int col0 = j * C::BN;
      int lim = N - col0;
      if (CAUSAL) lim = min(lim, row - col0 + 1);
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (last) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          mx[c & 3] = fmaxf(mx[c & 3], c < lim ? __uint_as_float(s[c]) : -INFINITY);
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) mx[c & 3] = fmaxf(mx[c & 3], __uint_as_float(s[c]));
      }
      const float m_cand = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale;

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
      if (__any_sync(0xffffffffu, need)) {
        // Rescale this warp's 32 rows of O once the previous PV MMA has landed.
        if (!warp_wait(&bar_o_done[i], (j - 1) & 1, ab)) { ok = false; break; }
        tc_fence_after();
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

      const float neg_m = -m_run;
      uint32_t p[64];
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
      if (last) {
#pragma unroll
        for (int c = 0; c < 128; c += 2) {
          const float p0 = c < lim ? ex2_approx(fmaf(__uint_as_float(s[c]), scale, neg_m)) : 0.f;
          const float p1 = c + 1 < lim ? ex2_approx(fmaf(__uint_as_float(s[c + 1]), scale, neg_m)) : 0.f;
          ls[(c >> 1) & 3] += p0 + p1;
          p[c >> 1] = pack_half2(p0, p1);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; c += 2) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(s[c]), scale, neg_m));
          const float p1 = ex2_approx(fmaf(__uint_as_float(s[c + 1]), scale, neg_m));
          ls[(c >> 1) & 3] += p0 + p1;
          p[c >> 1] = pack_half2(p0, p1);
        }
      }
      l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      tmem_store_cols<64>(tS, p);
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
  kern<<<dim3((unsigned)grid), dim3(320), C::SMEM_BYTES, s>>>(tq, tk, tv, a);
  return cudaGetLastError();
}

}  // namespace

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
