// Shared device helpers for the sm_100a attention kernels: mbarriers with bounded waits, TMA tile
// loads, tcgen05 (TMEM allocation, MMA issue/commit, TMEM loads/stores) and UMMA descriptors.
//
// Every wait in these kernels is bounded: a wait that has not completed after the launch's wait limit
// (FwdArgs/BwdArgs::wait_limit_ns, set process-wide with tattn_set_wait_limit_ns; 1 s by default) sets
// a bit in the caller-supplied status word and returns false, and the kernel then unwinds (drains its
// own copies in flight, frees TMEM, exits) instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace tattn {

// Status bits written by kernels into the device status word (see include/tattn.h).
enum : int {
  kStatusWaitTimeout = 1 << 0,  // an mbarrier wait exceeded the launch's wait limit
  kStatusAborted = 1 << 1,      // a CTA unwound because a sibling role timed out
};

constexpr unsigned long long kDefaultWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Per-CTA unwinding state shared by all roles of a warp-specialised kernel.
struct CtaAbort {
  volatile int* flag;           // shared memory: nonzero once any role of this CTA gave up
  int* status;                  // global status word
  unsigned long long limit_ns;  // how long one wait may take before the CTA gives up
};

// Wait until the phase with the given parity of `bar` has completed. Returns false (after setting
// the status bits and the CTA abort flag) if the wait exceeds ab.limit_ns or another role of the
// CTA has already given up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const CtaAbort& ab) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(a, parity)) return true;
    if ((it & 63u) == 0) {
      if (*ab.flag) return false;
      if (globaltimer_ns() - t0 > ab.limit_ns) {
        *ab.flag = 1;
        atomicOr(ab.status, kStatusWaitTimeout);
        return false;
      }
    }
  }
}

// Drain wait used while unwinding: bounded, never raises new status bits.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, unsigned long long limit_ns) {
  const uint32_t a = smem_u32(bar);
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(a, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return;
  }
}

// Warp-uniform bounded wait: every lane waits (each gets acquire ordering), then the lanes agree, so
// the warp stays converged for the .sync.aligned tcgen05 instructions that follow.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const CtaAbort& ab) {
  const bool ok = mbar_wait(bar, parity, ab);
  return __all_sync(0xffffffffu, ok);
}

// ----------------------------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ----------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t smem_dst, const CUtensorMap* tm, int c0, int c1, int c2,
                                            int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// TMA tile store from shared memory (bulk-group completion). The source must be visible to the async
// proxy first (fence_proxy_async_smem after the generic stores). Coordinates are never negative here.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* tm, uint32_t smem_src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(smem_src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
// Element-wise add of a shared-memory box into global memory (the tensor map's element type, here fp32),
// performed at L2; completes through the same bulk groups as the stores.
__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* tm, uint32_t smem_src, int c0, int c1, int c2,
                                                  int c3) {
  asm volatile("cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(smem_src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed store of this thread has finished reading its shared-memory source.
__device__ __forceinline__ void tma_store_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until every committed store of this thread has completed.
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Byte offset of the 16-byte unit at `byte` inside a TMA/UMMA swizzled region whose rows are SWB bytes
// (SWB = 128, 64, 32): the unit index is XORed with address bits [7, 7 + log2(SWB/16)).
template <int SWB>
__device__ __forceinline__ uint32_t swizzle_offset(uint32_t byte) {
  return byte ^ (((byte >> 7) & uint32_t(SWB / 16 - 1)) << 4);
}

// ----------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, fences, MMA, commit
// ----------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A * B, A from shared memory (_ss) or TMEM (_ts), B from shared memory; commit: arrive
// (once) on `bar` when every tcgen05 operation the electing lane issued so far has completed.
// Warp-converged issue: every lane of the issuing warp executes these with the same (warp-uniform)
// operands and elect.sync picks one lane (the lowest, i.e. the same lane every time while the warp is
// converged, so the commits track that lane's MMAs). Keeping the warp converged and the descriptors
// loop-invariant lets back-to-back MMAs issue at the tensor core's rate; per-MMA descriptor arithmetic
// on a single divergent lane costs ~90-180 cycles per MMA instead.
__device__ __forceinline__ void mma_f16_ss_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 rx;\n\t"
      "elect.sync rx|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_f16_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 rx;\n\t"
      "elect.sync rx|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 rx;\n\t"
      "elect.sync rx|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// Instruction descriptor for kind::f16 with fp16 A/B and fp32 accumulation.
//   bits 4-5 D format (1 = f32), 7-9 A format (0 = f16), 10-12 B format (0 = f16),
//   15 A major (0 = K), 16 B major (1 = MN), 17-22 N>>3, 24-28 M>>4.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N, bool b_mn_major) {
  return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
// The same with the A operand MN-major (transposed: M contiguous in shared memory) as well.
__host__ __device__ constexpr uint32_t idesc_f16_f32_amn(int M, int N, bool b_mn_major) {
  return idesc_f16_f32(M, N, b_mn_major) | (1u << 15);
}

// Shared-memory matrix descriptor (sm100 version field = 1).
//   layout: 2 = 128B swizzle, 4 = 64B swizzle, 6 = 32B swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (uint64_t(layout) << 61);
}

// ----------------------------------------------------------------------------------------------
// TMEM <-> registers (32x32b shape: thread i of the warp owns TMEM lane (warp_lane_base + i))
// ----------------------------------------------------------------------------------------------
#define TATTN_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), \
                    "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define TATTN_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), \
                    "r"(r[i + 6]), "r"(r[i + 7])

__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : TATTN_R8(0)
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : TATTN_R8(0), TATTN_R8(8)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : TATTN_R8(0), TATTN_R8(8), TATTN_R8(16), TATTN_R8(24)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               TATTN_W8(0)
               : "memory");
}
__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      TATTN_W8(0), TATTN_W8(8)
      : "memory");
}
__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      TATTN_W8(0), TATTN_W8(8), TATTN_W8(16), TATTN_W8(24)
      : "memory");
}
#undef TATTN_R8
#undef TATTN_W8

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Register fence: values loaded by tcgen05.ld are only valid after tcgen05.wait::ld. Routing them
// through an empty asm after the wait stops the compiler from using them earlier.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// Load `N` (multiple of 8, <= 128) consecutive fp32 columns of this thread's TMEM lane.
template <int N>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, uint32_t* r) {
  static_assert(N % 8 == 0 && N <= 128, "column count");
#pragma unroll
  for (int c = 0; c + 32 <= N; c += 32) tmem_ld_x32(taddr + c, r + c);
  if constexpr (N % 32 >= 16) tmem_ld_x16(taddr + (N / 32) * 32, r + (N / 32) * 32);
  if constexpr (N % 16 == 8) tmem_ld_x8(taddr + (N / 16) * 16, r + (N / 16) * 16);
}

template <int N>
__device__ __forceinline__ void tmem_store_cols(uint32_t taddr, const uint32_t* r) {
  static_assert(N % 8 == 0 && N <= 128, "column count");
#pragma unroll
  for (int c = 0; c + 32 <= N; c += 32) tmem_st_x32(taddr + c, r + c);
  if constexpr (N % 32 >= 16) tmem_st_x16(taddr + (N / 32) * 32, r + (N / 32) * 32);
  if constexpr (N % 16 == 8) tmem_st_x8(taddr + (N / 16) * 16, r + (N / 16) * 16);
}

// ----------------------------------------------------------------------------------------------
// CTA order of one-tile-per-CTA causal grids
// ----------------------------------------------------------------------------------------------
// Causal tiles differ in cost, so the grid runs them longest first and the hardware's CTA dispatch
// balances the rest. Longest first across all heads, though, spreads the CTAs running at any time over
// as many heads as there are SMs, and every CTA streams its head's whole K/V (or Q/dO): with 1,024 heads
// that working set is far beyond L2 and each CTA reads it from DRAM. So heads are grouped so that one
// group's K and V (2 * N * D fp16 each) take at most ~48 MiB, and the order is longest first within a
// group, one group after another. Returns the CTA's position in its head's longest-first order (0 = the
// longest tile) and sets *bh.
__device__ __forceinline__ int causal_cta_rank(int nct, int zh, int N, int D, int* bh) {
  const long long per_head = 4ll * N * D;
  const int hg = int(per_head <= 0 ? zh : max(1ll, min((long long)zh, (48ll << 20) / per_head)));
  const int per_group = hg * nct;
  const int grp = int(blockIdx.x) / per_group;
  const int h0 = grp * hg;
  const int gh = min(hg, zh - h0);             // heads in this group (the last one may be short)
  const int r = int(blockIdx.x) - grp * per_group;  // < gh * nct
  *bh = h0 + r % gh;
  return r / gh;
}

// ----------------------------------------------------------------------------------------------
// Math
// ----------------------------------------------------------------------------------------------
// Hardware base-2 exponential (MUFU). exp2(-inf) = +0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---- packed fp32 pairs (sm_100 f32x2 instructions: one issue slot for two lanes' worth of math)
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair on the FMA/ALU pipes, leaving MUFU free for the other exponentials of a row.
// Method: Cody-Waite style reduction x = j + f with j = round-to-nearest(x) obtained by adding the
// shifter 1.5*2^23 (j lands in the low mantissa bits of t = x + shifter), f = x - j in [-0.5, 0.5];
// 2^f by a degree-3 polynomial minimising the maximum relative error on [-0.5, 0.5] (Remez exchange;
// coefficients derived by csrc/fit_exp2_poly.py, max relative error 7.5e-5), then 2^j applied by adding
// j << 23 to the result's exponent field. x is clamped to >= -126 so the exponent never underflows;
// results below 2^-24 vanish in the fp16 P anyway. Valid for x <= 127 (callers pass x <= 8).
__device__ __forceinline__ uint64_t exp2_poly_x2(uint64_t x2) {
  float2 x = f2_unpack(x2);
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const uint64_t xc = f2(x.x, x.y);
  const uint64_t shifter = f2(12582912.f, 12582912.f);
  const uint64_t t = fadd2(xc, shifter);
  const uint64_t f = fsub2(xc, fsub2(t, shifter));
  uint64_t p = ffma2(f2(0.0551716685295105f, 0.0551716685295105f), f, f2(0.2426111251115799f, 0.2426111251115799f));
  p = ffma2(p, f, f2(0.6932609677314758f, 0.6932609677314758f));
  p = ffma2(p, f, f2(0.9999280571937561f, 0.9999280571937561f));
  const float2 pv = f2_unpack(p), tv = f2_unpack(t);
  return f2(__int_as_float(__float_as_int(pv.x) + (__float_as_int(tv.x) << 23)),
            __int_as_float(__float_as_int(pv.y) + (__float_as_int(tv.y) << 23)));
}

// The same with a degree-4 polynomial (max relative error 2.7e-6, one more packed FMA): accurate enough
// that a gradient summed over thousands of query rows stays within the fp16 bound (the backward).
__device__ __forceinline__ uint64_t exp2_poly4_x2(uint64_t x2) {
  float2 x = f2_unpack(x2);
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const uint64_t xc = f2(x.x, x.y);
  const uint64_t shifter = f2(12582912.f, 12582912.f);
  const uint64_t t = fadd2(xc, shifter);
  const uint64_t f = fsub2(xc, fsub2(t, shifter));
  uint64_t p = ffma2(f2(0.009570102207362652f, 0.009570102207362652f), f, f2(0.05591785907745361f, 0.05591785907745361f));
  p = ffma2(p, f, f2(0.240247443318367f, 0.240247443318367f));
  p = ffma2(p, f, f2(0.6931217908859253f, 0.6931217908859253f));
  p = ffma2(p, f, f2(0.9999992847442627f, 0.9999992847442627f));
  const float2 pv = f2_unpack(p), tv = f2_unpack(t);
  return f2(__int_as_float(__float_as_int(pv.x) + (__float_as_int(tv.x) << 23)),
            __int_as_float(__float_as_int(pv.y) + (__float_as_int(tv.y) << 23)));
}

}  // namespace tattn
