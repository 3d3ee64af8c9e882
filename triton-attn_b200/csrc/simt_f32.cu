// fp32 attention on CUDA cores (FFMA), plus the backward preprocess for both dtypes.
//
// tcgen05 has no fp32 MMA (only kind::tf32, ~1e-3 relative error), and the path's fp32 contract is a
// 1e-4 max-abs error, so fp32 inputs run these exact-fp32 kernels. They follow the same block
// algorithm as the reference (src/tattn/kernels.py:57-148 forward, 151-239 dK/dV, 242-321 dQ,
// 324-337 preprocess): base-2 online softmax with the exact running max, M = m + log2(l), P rebuilt
// from M in the backward, atomic-free dK/dV (one CTA per key block) and dQ (one CTA per query block).
// fp32 is a correctness path, not a throughput target.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace tattn {
namespace {

constexpr int SIMT_THREADS = 128;

// Rows per block (= keys per block) and threads per row; 16 rows at D = 128 keeps static shared
// memory under 48 KB. Thread tid owns row tid / G and every G-th column starting at tid % G.
template <int D>
struct Simt {
  static constexpr int SB = D == 128 ? 16 : 32;
  static constexpr int G = SIMT_THREADS / SB;
};

template <int G>
__device__ __forceinline__ float group_max(float x) {
#pragma unroll
  for (int o = 1; o < G; o *= 2) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
template <int G>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = 1; o < G; o *= 2) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ float ld_f32(const float* p) { return __ldg(p); }

template <int D>
__global__ void __launch_bounds__(SIMT_THREADS)
    fwd_f32_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                   Strides4 sq, Strides4 sk, Strides4 sv, FwdArgs a, float qk_scale, bool causal) {
  constexpr int SB = Simt<D>::SB, G = Simt<D>::G;
  __shared__ float Qs[SB][D + 1];
  __shared__ float Ks[SB][D + 1];
  __shared__ float Vs[SB][D + 1];
  __shared__ float Ps[SB][SB + 1];
  const int N = a.N;
  const int bh = blockIdx.y, zi = bh / a.H, hi = bh % a.H;
  const int rb = blockIdx.x * SB;
  const int tid = threadIdx.x, r = tid / G, g = tid % G;
  const float* qb = q + zi * sq.z + hi * sq.h;
  const float* kb = k + zi * sk.z + hi * sk.h;
  const float* vb = v + zi * sv.z + hi * sv.h;
  for (int e = tid; e < SB * D; e += SIMT_THREADS) {
    const int rr = e / D, d = e % D;
    Qs[rr][d] = (rb + rr < N) ? ld_f32(qb + int64_t(rb + rr) * sq.n + d * sq.d) : 0.f;
  }
  const int row = rb + r;
  float m_i = -INFINITY, l_i = 0.f;
  float acc[D / G];
#pragma unroll
  for (int dd = 0; dd < D / G; ++dd) acc[dd] = 0.f;
  const int hi_col = causal ? min(rb + SB, N) : N;
  for (int cb = 0; cb < hi_col; cb += SB) {
    __syncthreads();
    for (int e = tid; e < SB * D; e += SIMT_THREADS) {
      const int cc = e / D, d = e % D;
      const bool ok = cb + cc < N;
      Ks[cc][d] = ok ? ld_f32(kb + int64_t(cb + cc) * sk.n + d * sk.d) : 0.f;
      Vs[cc][d] = ok ? ld_f32(vb + int64_t(cb + cc) * sv.n + d * sv.d) : 0.f;
    }
    __syncthreads();
    float x[SB / G];
    float mx = -INFINITY;
#pragma unroll
    for (int t = 0; t < SB / G; ++t) {
      const int c = g + G * t, col = cb + c;
      float s = 0.f;
#pragma unroll 16
      for (int d = 0; d < D; ++d) s = fmaf(Qs[r][d], Ks[c][d], s);
      s *= qk_scale;
      if (col >= N || (causal && col > row)) s = -INFINITY;
      x[t] = s;
      mx = fmaxf(mx, s);
    }
    mx = group_max<G>(mx);
    const float m_new = fmaxf(m_i, mx);
    const float m_use = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = exp2f(m_i - m_use);
    float ps = 0.f;
#pragma unroll
    for (int t = 0; t < SB / G; ++t) {
      const float p = exp2f(x[t] - m_use);
      Ps[r][g + G * t] = p;
      ps += p;
    }
    ps = group_sum<G>(ps);
    l_i = l_i * alpha + ps;
    m_i = m_new;
    __syncwarp();
#pragma unroll
    for (int dd = 0; dd < D / G; ++dd) {
      const int d = g + G * dd;
      float o = acc[dd] * alpha;
#pragma unroll 8
      for (int c = 0; c < SB; ++c) o = fmaf(Ps[r][c], Vs[c][d], o);
      acc[dd] = o;
    }
  }
  if (row < N) {
    float* o = reinterpret_cast<float*>(a.o) + zi * a.so.z + hi * a.so.h + int64_t(row) * a.so.n;
    const float inv = 1.f / l_i;
#pragma unroll
    for (int dd = 0; dd < D / G; ++dd) o[(g + G * dd) * a.so.d] = acc[dd] * inv;
    if (g == 0) a.m[int64_t(bh) * N + row] = m_i + log2f(l_i);
  }
}

// dQ for one block of SB query rows (reference: _bwd_dq_kernel, kernels.py:242-321).
template <int D>
__global__ void __launch_bounds__(SIMT_THREADS) bwd_dq_f32_kernel(BwdArgs a, bool causal) {
  constexpr int SB = Simt<D>::SB, G = Simt<D>::G;
  __shared__ float Qs[SB][D + 1];
  __shared__ float DOs[SB][D + 1];
  __shared__ float Ks[SB][D + 1];
  __shared__ float Vs[SB][D + 1];
  __shared__ float DSs[SB][SB + 1];
  const int N = a.N;
  const int bh = blockIdx.y, zi = bh / a.H, hi = bh % a.H;
  const int rb = blockIdx.x * SB;
  const int tid = threadIdx.x, r = tid / G, g = tid % G;
  const float* q = reinterpret_cast<const float*>(a.q) + zi * a.sq.z + hi * a.sq.h;
  const float* k = reinterpret_cast<const float*>(a.k) + zi * a.sk.z + hi * a.sk.h;
  const float* v = reinterpret_cast<const float*>(a.v) + zi * a.sv.z + hi * a.sv.h;
  const float* dout = reinterpret_cast<const float*>(a.dout) + zi * a.sdo.z + hi * a.sdo.h;
  for (int e = tid; e < SB * D; e += SIMT_THREADS) {
    const int rr = e / D, d = e % D;
    const bool ok = rb + rr < N;
    Qs[rr][d] = ok ? ld_f32(q + int64_t(rb + rr) * a.sq.n + d * a.sq.d) : 0.f;
    DOs[rr][d] = ok ? ld_f32(dout + int64_t(rb + rr) * a.sdo.n + d * a.sdo.d) : 0.f;
  }
  const int row = rb + r;
  const float qks = a.sm_scale * 1.4426950408889634f;
  const float m_r = row < N ? a.m[int64_t(bh) * N + row] : 0.f;
  const float d_r = row < N ? a.delta[int64_t(bh) * N + row] : 0.f;
  float acc[D / G];
#pragma unroll
  for (int dd = 0; dd < D / G; ++dd) acc[dd] = 0.f;
  const int hi_col = causal ? min(rb + SB, N) : N;
  for (int cb = 0; cb < hi_col; cb += SB) {
    __syncthreads();
    for (int e = tid; e < SB * D; e += SIMT_THREADS) {
      const int cc = e / D, d = e % D;
      const bool ok = cb + cc < N;
      Ks[cc][d] = ok ? ld_f32(k + int64_t(cb + cc) * a.sk.n + d * a.sk.d) : 0.f;
      Vs[cc][d] = ok ? ld_f32(v + int64_t(cb + cc) * a.sv.n + d * a.sv.d) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < SB / G; ++t) {
      const int c = g + G * t, col = cb + c;
      float s = 0.f, dp = 0.f;
#pragma unroll 16
      for (int d = 0; d < D; ++d) {
        s = fmaf(Qs[r][d], Ks[c][d], s);
        dp = fmaf(DOs[r][d], Vs[c][d], dp);
      }
      const bool keep = row < N && col < N && !(causal && col > row);
      const float p = keep ? exp2f(s * qks - m_r) : 0.f;
      DSs[r][c] = p * (dp - d_r);
    }
    __syncwarp();
#pragma unroll
    for (int dd = 0; dd < D / G; ++dd) {
      const int d = g + G * dd;
      float o = acc[dd];
#pragma unroll 8
      for (int c = 0; c < SB; ++c) o = fmaf(DSs[r][c], Ks[c][d], o);
      acc[dd] = o;
    }
  }
  if (row < N) {
    float* dq = reinterpret_cast<float*>(a.dq) + (int64_t(bh) * N + row) * D;
#pragma unroll
    for (int dd = 0; dd < D / G; ++dd) dq[g + G * dd] = acc[dd] * a.sm_scale;
  }
}

// dK, dV for one block of SB keys (reference: _bwd_dkdv_kernel, kernels.py:151-239).
template <int D>
__global__ void __launch_bounds__(SIMT_THREADS) bwd_dkdv_f32_kernel(BwdArgs a, bool causal) {
  constexpr int SB = Simt<D>::SB, G = Simt<D>::G;
  __shared__ float Ks[SB][D + 1];
  __shared__ float Vs[SB][D + 1];
  __shared__ float Qs[SB][D + 1];
  __shared__ float DOs[SB][D + 1];
  __shared__ float Pt[SB][SB + 1];
  __shared__ float DSt[SB][SB + 1];
  __shared__ float Ms[SB], Ds[SB];
  const int N = a.N;
  const int bh = blockIdx.y, zi = bh / a.H, hi = bh % a.H;
  const int cb = blockIdx.x * SB;
  const int tid = threadIdx.x, c = tid / G, g = tid % G;
  const float* q = reinterpret_cast<const float*>(a.q) + zi * a.sq.z + hi * a.sq.h;
  const float* k = reinterpret_cast<const float*>(a.k) + zi * a.sk.z + hi * a.sk.h;
  const float* v = reinterpret_cast<const float*>(a.v) + zi * a.sv.z + hi * a.sv.h;
  const float* dout = reinterpret_cast<const float*>(a.dout) + zi * a.sdo.z + hi * a.sdo.h;
  for (int e = tid; e < SB * D; e += SIMT_THREADS) {
    const int cc = e / D, d = e % D;
    const bool ok = cb + cc < N;
    Ks[cc][d] = ok ? ld_f32(k + int64_t(cb + cc) * a.sk.n + d * a.sk.d) : 0.f;
    Vs[cc][d] = ok ? ld_f32(v + int64_t(cb + cc) * a.sv.n + d * a.sv.d) : 0.f;
  }
  const int col = cb + c;
  const float qks = a.sm_scale * 1.4426950408889634f;
  float dk[D / G], dv[D / G];
#pragma unroll
  for (int dd = 0; dd < D / G; ++dd) dk[dd] = dv[dd] = 0.f;
  const int lo = causal ? cb : 0;  // query rows before this key block never see it
  for (int rb = lo; rb < N; rb += SB) {
    __syncthreads();
    for (int e = tid; e < SB * D; e += SIMT_THREADS) {
      const int rr = e / D, d = e % D;
      const bool ok = rb + rr < N;
      Qs[rr][d] = ok ? ld_f32(q + int64_t(rb + rr) * a.sq.n + d * a.sq.d) : 0.f;
      DOs[rr][d] = ok ? ld_f32(dout + int64_t(rb + rr) * a.sdo.n + d * a.sdo.d) : 0.f;
    }
    if (tid < SB) {
      const bool ok = rb + tid < N;
      Ms[tid] = ok ? a.m[int64_t(bh) * N + rb + tid] : 0.f;
      Ds[tid] = ok ? a.delta[int64_t(bh) * N + rb + tid] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < SB / G; ++t) {
      const int rr = g + G * t, row = rb + rr;
      float s = 0.f, dp = 0.f;
#pragma unroll 16
      for (int d = 0; d < D; ++d) {
        s = fmaf(Qs[rr][d], Ks[c][d], s);
        dp = fmaf(DOs[rr][d], Vs[c][d], dp);
      }
      const bool keep = row < N && col < N && !(causal && col > row);
      const float p = keep ? exp2f(s * qks - Ms[rr]) : 0.f;
      Pt[c][rr] = p;
      DSt[c][rr] = p * (dp - Ds[rr]);
    }
    __syncwarp();
#pragma unroll
    for (int dd = 0; dd < D / G; ++dd) {
      const int d = g + G * dd;
      float x = dv[dd], y = dk[dd];
#pragma unroll 8
      for (int rr = 0; rr < SB; ++rr) {
        x = fmaf(Pt[c][rr], DOs[rr][d], x);
        y = fmaf(DSt[c][rr], Qs[rr][d], y);
      }
      dv[dd] = x;
      dk[dd] = y;
    }
  }
  if (col < N) {
    float* dkp = reinterpret_cast<float*>(a.dk) + (int64_t(bh) * N + col) * D;
    float* dvp = reinterpret_cast<float*>(a.dv) + (int64_t(bh) * N + col) * D;
#pragma unroll
    for (int dd = 0; dd < D / G; ++dd) {
      dkp[g + G * dd] = dk[dd] * a.sm_scale;
      dvp[g + G * dd] = dv[dd];
    }
  }
}

// delta[bh, i] = sum_d O[i, d] * dO[i, d] in fp32 (reference: _bwd_preprocess, kernels.py:324-337).
// L lanes cooperate on one row with 16-byte loads; rows need a unit D stride and 16-byte alignment.
// With a.dq_acc set (fused backward) the row's fp32 dQ workspace is zeroed as well.
template <typename T, int D>
__global__ void __launch_bounds__(256) preprocess_kernel(BwdArgs a) {
  constexpr int VEC = 16 / sizeof(T);  // elements per 16-byte load
  constexpr int L = D / VEC;           // lanes per row (2..32)
  constexpr int RPW = 32 / L;          // rows per warp per step
  const int N = a.N;
  const int64_t rows_total = int64_t(a.Z) * a.H * N;
  const int lane = threadIdx.x % 32, sub = lane % L;
  const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int64_t row_g = warp_global * RPW + lane / L;
  float acc = 0.f;
  const bool valid = row_g < rows_total;
  if (valid) {
    const int64_t bh = row_g / N;
    const int row = int(row_g % N);
    const int zi = int(bh / a.H), hi = int(bh % a.H);
    const T* o = reinterpret_cast<const T*>(a.o) + zi * a.so.z + hi * a.so.h + int64_t(row) * a.so.n;
    const T* g = reinterpret_cast<const T*>(a.dout) + zi * a.sdo.z + hi * a.sdo.h + int64_t(row) * a.sdo.n;
    const uint4 ov = __ldg(reinterpret_cast<const uint4*>(o) + sub);
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(g) + sub);
    if constexpr (sizeof(T) == 2) {
      const __half2* oh = reinterpret_cast<const __half2*>(&ov);
      const __half2* gh = reinterpret_cast<const __half2*>(&gv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 of = __half22float2(oh[e]), gf = __half22float2(gh[e]);
        acc = fmaf(of.x, gf.x, acc);
        acc = fmaf(of.y, gf.y, acc);
      }
    } else {
      const float* of = reinterpret_cast<const float*>(&ov);
      const float* gf = reinterpret_cast<const float*>(&gv);
#pragma unroll
      for (int e = 0; e < 4; ++e) acc = fmaf(of[e], gf[e], acc);
    }
  }
#pragma unroll
  for (int off = L / 2; off > 0; off /= 2) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (valid && sub == 0) a.delta[row_g] = acc;
  if (valid && a.dq_acc != nullptr) {  // the fused backward's fp32 dQ row: D floats, D / L per lane
    uint4* dst = reinterpret_cast<uint4*>(a.dq_acc + row_g * D + sub * (D / L));
#pragma unroll
    for (int e = 0; e < D / L / 4; ++e) dst[e] = make_uint4(0u, 0u, 0u, 0u);
  }
  if (a.grid_sync != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *a.grid_sync = 0u;  // its grid barrier
}

template <int D>
cudaError_t fwd_f32_impl(bool causal, const void* q, const void* k, const void* v, Strides4 sq, Strides4 sk,
                         Strides4 sv, const FwdArgs& a, float qk_scale, cudaStream_t s) {
  constexpr int SB = Simt<D>::SB;
  dim3 grid((a.N + SB - 1) / SB, a.Z * a.H);
  fwd_f32_kernel<D><<<grid, SIMT_THREADS, 0, s>>>(static_cast<const float*>(q), static_cast<const float*>(k),
                                                  static_cast<const float*>(v), sq, sk, sv, a, qk_scale, causal);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fwd_f32(int D, bool causal, const void* q, const void* k, const void* v, Strides4 sq,
                           Strides4 sk, Strides4 sv, const FwdArgs& a, float sm_scale, cudaStream_t s) {
  const float qk = sm_scale * 1.4426950408889634f;
  if (a.N == 0 || a.Z * a.H == 0) return cudaSuccess;
  switch (D) {
    case 16: return fwd_f32_impl<16>(causal, q, k, v, sq, sk, sv, a, qk, s);
    case 32: return fwd_f32_impl<32>(causal, q, k, v, sq, sk, sv, a, qk, s);
    case 64: return fwd_f32_impl<64>(causal, q, k, v, sq, sk, sv, a, qk, s);
    case 128: return fwd_f32_impl<128>(causal, q, k, v, sq, sk, sv, a, qk, s);
    default: return cudaErrorInvalidValue;
  }
}

template <int D>
cudaError_t bwd_f32_impl(bool dq_pass, bool causal, const BwdArgs& a, cudaStream_t s) {
  constexpr int SB = Simt<D>::SB;
  dim3 grid((a.N + SB - 1) / SB, a.Z * a.H);
  if (dq_pass)
    bwd_dq_f32_kernel<D><<<grid, SIMT_THREADS, 0, s>>>(a, causal);
  else
    bwd_dkdv_f32_kernel<D><<<grid, SIMT_THREADS, 0, s>>>(a, causal);
  return cudaGetLastError();
}

static cudaError_t bwd_f32_dispatch(int D, bool dq_pass, bool causal, const BwdArgs& a, cudaStream_t s) {
  if (a.N == 0 || a.Z * a.H == 0) return cudaSuccess;
  switch (D) {
    case 16: return bwd_f32_impl<16>(dq_pass, causal, a, s);
    case 32: return bwd_f32_impl<32>(dq_pass, causal, a, s);
    case 64: return bwd_f32_impl<64>(dq_pass, causal, a, s);
    case 128: return bwd_f32_impl<128>(dq_pass, causal, a, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_bwd_dq_f32(int D, bool causal, const BwdArgs& a, cudaStream_t s) {
  return bwd_f32_dispatch(D, true, causal, a, s);
}

cudaError_t launch_bwd_dkdv_f32(int D, bool causal, const BwdArgs& a, cudaStream_t s) {
  return bwd_f32_dispatch(D, false, causal, a, s);
}

cudaError_t launch_bwd_preprocess(int D, bool is_f16, const BwdArgs& a, cudaStream_t s) {
  const int64_t rows = int64_t(a.Z) * a.H * a.N;
  if (rows == 0) return cudaSuccess;
  const int vec = is_f16 ? 8 : 4;
  const int rpw = 32 / (D / vec);
  const int64_t warps = (rows + rpw - 1) / rpw;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
#define TATTN_PRE(T, DD) preprocess_kernel<T, DD><<<unsigned(blocks), 256, 0, s>>>(a)
  if (is_f16) {
    switch (D) {
      case 16: TATTN_PRE(__half, 16); break;
      case 32: TATTN_PRE(__half, 32); break;
      case 64: TATTN_PRE(__half, 64); break;
      case 128: TATTN_PRE(__half, 128); break;
      default: return cudaErrorInvalidValue;
    }
  } else {
    switch (D) {
      case 16: TATTN_PRE(float, 16); break;
      case 32: TATTN_PRE(float, 32); break;
      case 64: TATTN_PRE(float, 64); break;
      case 128: TATTN_PRE(float, 128); break;
      default: return cudaErrorInvalidValue;
    }
  }
#undef TATTN_PRE
  return cudaGetLastError();
}

}  // namespace tattn
