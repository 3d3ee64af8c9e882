// Diagnostic kernels for the library's own math building blocks (no reference counterpart).
// tattn_selftest_exp2 evaluates the FMA-pipe exp2 of the forward (exp2_poly_x2, degree 3) next to the
// hardware exponential (ex2.approx) and CUDA's exp2f on caller-given inputs, and
// tattn_selftest_exp2_poly4 the backward's (exp2_poly4_x2, degree 4), so tests can check the
// polynomials against CUDA's outputs and their error bounds.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tattn.h"
#include "common.cuh"

namespace {

__global__ void exp2_selftest_kernel(const float* __restrict__ x, float* __restrict__ y_poly,
                                     float* __restrict__ y_hw, float* __restrict__ y_lib, int n) {
  const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float x0 = x[i], x1 = (i + 1 < n) ? x[i + 1] : 0.f;
  const float2 p = tattn::f2_unpack(tattn::exp2_poly_x2(tattn::f2(x0, x1)));
  y_poly[i] = p.x;
  y_hw[i] = tattn::ex2_approx(x0);
  y_lib[i] = exp2f(x0);
  if (i + 1 < n) {
    y_poly[i + 1] = p.y;
    y_hw[i + 1] = tattn::ex2_approx(x1);
    y_lib[i + 1] = exp2f(x1);
  }
}

__global__ void exp2_poly4_selftest_kernel(const float* __restrict__ x, float* __restrict__ y, int n) {
  const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float x0 = x[i], x1 = (i + 1 < n) ? x[i + 1] : 0.f;
  const float2 p = tattn::f2_unpack(tattn::exp2_poly4_x2(tattn::f2(x0, x1)));
  y[i] = p.x;
  if (i + 1 < n) y[i + 1] = p.y;
}

}  // namespace

extern "C" int tattn_selftest_exp2_poly4(const float* x, float* y, int n, void* stream) {
  if (n < 0 || (n > 0 && (!x || !y))) return TATTN_ERR_INVALID_ARGUMENT;
  if (n == 0) return TATTN_OK;
  const int pairs = (n + 1) / 2;
  exp2_poly4_selftest_kernel<<<(pairs + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
  return cudaGetLastError() == cudaSuccess ? TATTN_OK : TATTN_ERR_CUDA;
}

extern "C" int tattn_selftest_exp2(const float* x, float* y_poly, float* y_hw, float* y_lib, int n, void* stream) {
  if (n < 0 || (n > 0 && (!x || !y_poly || !y_hw || !y_lib))) return TATTN_ERR_INVALID_ARGUMENT;
  if (n == 0) return TATTN_OK;
  const int pairs = (n + 1) / 2;
  exp2_selftest_kernel<<<(pairs + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y_poly, y_hw,
                                                                                             y_lib, n);
  return cudaGetLastError() == cudaSuccess ? TATTN_OK : TATTN_ERR_CUDA;
}
