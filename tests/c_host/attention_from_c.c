/* A host program in plain C -- no C++, no Python, no PyTorch -- that uses the library the way a cgo, JNI
 * or C caller would: it includes tattn.h, allocates device buffers with the CUDA runtime, runs the forward
 * (tattn_fwd) and the backward (tattn_bwd_fused) through the C ABI, and compares O, M, dq, dk and dv with
 * attention and its gradients computed here in double precision on the CPU.
 *
 * Exit status: 0 when every value of every case is within tolerance (|got - ref| <= 2e-3 + 2e-3 |ref| for
 * O and the gradients, <= 1e-3 for M, base-2 log-sum-exp), 1 on a mismatch, 2 on a set-up or library
 * error. Built and run by tests/test_c_host.py. */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "tattn.h"

/* fp16 bits of x, for x = k / 128 with |k| <= 128 (exact in fp16: normal, at most 8 significant bits). */
static uint16_t half_exact(float x) {
  if (x == 0.f) return 0;
  uint32_t b;
  memcpy(&b, &x, 4);
  const uint32_t sign = (b >> 16) & 0x8000u;
  const int e = (int)((b >> 23) & 0xffu) - 127 + 15;
  return (uint16_t)(sign | ((uint32_t)e << 10) | ((b >> 13) & 0x3ffu));
}

static double half_value(uint16_t h) {
  const int sign = (h >> 15) & 1, e = (h >> 10) & 31, mant = h & 1023;
  double v;
  if (e == 0) v = ldexp((double)mant, -24);
  else if (e == 31) v = mant ? NAN : INFINITY;
  else v = ldexp(1.0 + mant / 1024.0, e - 15);
  return sign ? -v : v;
}

static uint32_t lcg_state = 12345u;
static float next_input(void) {  /* k / 128 for k uniform in [-128, 128] */
  lcg_state = lcg_state * 1664525u + 1013904223u;
  return (float)((int)((lcg_state >> 8) % 257u) - 128) / 128.f;
}

#define CHECK_CUDA(x)                                                            \
  do {                                                                           \
    cudaError_t e_ = (x);                                                        \
    if (e_ != cudaSuccess) {                                                     \
      fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));                   \
      return 2;                                                                  \
    }                                                                            \
  } while (0)
#define CHECK_TATTN(x)                                                           \
  do {                                                                           \
    int r_ = (x);                                                                \
    if (r_ != TATTN_OK) {                                                        \
      fprintf(stderr, "%s: %s\n", #x, tattn_status_string(r_));                  \
      return 2;                                                                  \
    }                                                                            \
  } while (0)

/* Attention of one (batch, head) in double: inputs [N, D] row-major; outputs O, M (base 2) and the
 * gradients for the output gradient dO. */
static void reference(int N, int D, int causal, double scale, const double* q, const double* k, const double* v,
                      const double* dout, double* o, double* m2, double* dq, double* dk, double* dv) {
  double* p = (double*)malloc(sizeof(double) * (size_t)N * N);
  double* ds = (double*)malloc(sizeof(double) * (size_t)N * N);
  for (int i = 0; i < N; ++i) {
    double mx = -INFINITY, l = 0.0;
    for (int j = 0; j < N; ++j) {
      double s = -INFINITY;
      if (!causal || j <= i) {
        s = 0.0;
        for (int d = 0; d < D; ++d) s += q[i * D + d] * k[j * D + d];
        s *= scale;
      }
      p[(size_t)i * N + j] = s;
      if (s > mx) mx = s;
    }
    for (int j = 0; j < N; ++j) {
      const double e = isinf(p[(size_t)i * N + j]) ? 0.0 : exp(p[(size_t)i * N + j] - mx);
      p[(size_t)i * N + j] = e;
      l += e;
    }
    for (int j = 0; j < N; ++j) p[(size_t)i * N + j] /= l;
    m2[i] = (mx + log(l)) / log(2.0);
    for (int d = 0; d < D; ++d) {
      double acc = 0.0;
      for (int j = 0; j < N; ++j) acc += p[(size_t)i * N + j] * v[j * D + d];
      o[i * D + d] = acc;
    }
  }
  for (int i = 0; i < N; ++i) {
    double delta = 0.0;
    for (int d = 0; d < D; ++d) delta += dout[i * D + d] * o[i * D + d];
    for (int j = 0; j < N; ++j) {
      double dp = 0.0;
      for (int d = 0; d < D; ++d) dp += dout[i * D + d] * v[j * D + d];
      ds[(size_t)i * N + j] = p[(size_t)i * N + j] * (dp - delta);
    }
  }
  for (int i = 0; i < N; ++i)
    for (int d = 0; d < D; ++d) {
      double aq = 0.0, ak = 0.0, av = 0.0;
      for (int j = 0; j < N; ++j) {
        aq += ds[(size_t)i * N + j] * k[j * D + d];
        ak += ds[(size_t)j * N + i] * q[j * D + d];
        av += p[(size_t)j * N + i] * dout[j * D + d];
      }
      dq[i * D + d] = aq * scale;
      dk[i * D + d] = ak * scale;
      dv[i * D + d] = av;
    }
  free(p);
  free(ds);
}

/* Largest |got - ref| / (atol + rtol |ref|) over n values (<= 1 passes). */
static double worst(const uint16_t* got, const double* ref, size_t n, double* max_abs) {
  double w = 0.0;
  *max_abs = 0.0;
  for (size_t i = 0; i < n; ++i) {
    const double err = fabs(half_value(got[i]) - ref[i]);
    const double r = err / (2e-3 + 2e-3 * fabs(ref[i]));
    if (!(r <= w)) w = r;  /* also catches NaN */
    if (err > *max_abs) *max_abs = err;
  }
  return w;
}

static int run_case(int Z, int H, int N, int D, int causal) {
  const size_t per = (size_t)N * D, n = (size_t)Z * H * per, rows = (size_t)Z * H * N;
  const double scale = 1.0 / sqrt((double)D);
  uint16_t* h_in[4];
  double* d_in[4];
  for (int t = 0; t < 4; ++t) {
    h_in[t] = (uint16_t*)malloc(n * 2);
    d_in[t] = (double*)malloc(n * sizeof(double));
    for (size_t i = 0; i < n; ++i) {
      const float x = next_input();
      h_in[t][i] = half_exact(x);
      d_in[t][i] = x;
    }
  }
  void *q, *k, *v, *o, *dout, *dq, *dk, *dv, *ws;
  float *m, *delta;
  CHECK_CUDA(cudaMalloc(&q, n * 2));
  CHECK_CUDA(cudaMalloc(&k, n * 2));
  CHECK_CUDA(cudaMalloc(&v, n * 2));
  CHECK_CUDA(cudaMalloc(&dout, n * 2));
  CHECK_CUDA(cudaMalloc(&o, n * 2));
  CHECK_CUDA(cudaMalloc(&dq, n * 2));
  CHECK_CUDA(cudaMalloc(&dk, n * 2));
  CHECK_CUDA(cudaMalloc(&dv, n * 2));
  CHECK_CUDA(cudaMalloc((void**)&m, rows * 4));
  CHECK_CUDA(cudaMalloc((void**)&delta, rows * 4));
  const int64_t ws_bytes = tattn_bwd_fused_workspace_bytes(Z, H, N, D);
  if (ws_bytes < 0) {
    fprintf(stderr, "tattn_bwd_fused_workspace_bytes refused the shape\n");
    return 2;
  }
  CHECK_CUDA(cudaMalloc(&ws, (size_t)ws_bytes));
  CHECK_CUDA(cudaMemcpy(q, h_in[0], n * 2, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(k, h_in[1], n * 2, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(v, h_in[2], n * 2, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dout, h_in[3], n * 2, cudaMemcpyHostToDevice));

  /* Dense [Z, H, N, D]: element strides (z, h, n, d), once per tensor. */
  int64_t strides[20];
  for (int t = 0; t < 5; ++t) {
    strides[4 * t + 0] = (int64_t)H * N * D;
    strides[4 * t + 1] = (int64_t)N * D;
    strides[4 * t + 2] = D;
    strides[4 * t + 3] = 1;
  }
  CHECK_TATTN(tattn_fwd(q, k, v, o, m, strides, Z, H, N, D, TATTN_F16, causal, (float)scale, 0, NULL));
  CHECK_TATTN(tattn_bwd_fused(q, k, v, o, dout, dq, dk, dv, m, delta, ws, strides, Z, H, N, D, TATTN_F16, causal,
                              (float)scale, NULL));
  CHECK_CUDA(cudaDeviceSynchronize());
  int status = -1;
  CHECK_TATTN(tattn_device_status(NULL, &status, 1));
  if (status != 0) {
    fprintf(stderr, "device status word %d\n", status);
    return 2;
  }

  uint16_t* h_out[4];
  void* d_out[4] = {o, dq, dk, dv};
  for (int t = 0; t < 4; ++t) {
    h_out[t] = (uint16_t*)malloc(n * 2);
    CHECK_CUDA(cudaMemcpy(h_out[t], d_out[t], n * 2, cudaMemcpyDeviceToHost));
  }
  float* h_m = (float*)malloc(rows * 4);
  CHECK_CUDA(cudaMemcpy(h_m, m, rows * 4, cudaMemcpyDeviceToHost));

  double* ref[4];
  double* ref_m = (double*)malloc(rows * sizeof(double));
  for (int t = 0; t < 4; ++t) ref[t] = (double*)malloc(n * sizeof(double));
  for (int bh = 0; bh < Z * H; ++bh) {
    const size_t off = (size_t)bh * per;
    reference(N, D, causal, scale, d_in[0] + off, d_in[1] + off, d_in[2] + off, d_in[3] + off, ref[0] + off,
              ref_m + (size_t)bh * N, ref[1] + off, ref[2] + off, ref[3] + off);
  }
  const char* names[4] = {"o", "dq", "dk", "dv"};
  int ok = 1;
  printf("case Z=%d H=%d N=%d D=%d causal=%d:", Z, H, N, D, causal);
  for (int t = 0; t < 4; ++t) {
    double max_abs;
    const double w = worst(h_out[t], ref[t], n, &max_abs);
    printf(" %s %.3g", names[t], max_abs);
    if (!(w <= 1.0)) ok = 0;
  }
  double m_err = 0.0;
  for (size_t i = 0; i < rows; ++i) {
    const double e = fabs((double)h_m[i] - ref_m[i]);
    if (!(e <= m_err)) m_err = e;
  }
  printf(" m %.3g %s\n", m_err, ok && m_err <= 1e-3 ? "ok" : "MISMATCH");
  if (m_err > 1e-3) ok = 0;

  void* bufs[11] = {q, k, v, dout, o, dq, dk, dv, m, delta, ws};
  for (int t = 0; t < 11; ++t) cudaFree(bufs[t]);
  for (int t = 0; t < 4; ++t) {
    free(h_in[t]);
    free(d_in[t]);
    free(h_out[t]);
    free(ref[t]);
  }
  free(h_m);
  free(ref_m);
  return ok ? 0 : 1;
}

int main(void) {
  printf("tattn ABI version %d (header %d)\n", tattn_abi_version(), TATTN_ABI_VERSION);
  if (tattn_abi_version() != TATTN_ABI_VERSION) return 2;
  /* one ragged block, causal; several blocks, not causal; head dim 128 (transposed dQ part), causal */
  const int cases[3][5] = {{1, 2, 77, 64, 1}, {2, 1, 300, 64, 0}, {1, 2, 300, 128, 1}};
  int worst_rc = 0;
  for (int c = 0; c < 3; ++c) {
    const int rc = run_case(cases[c][0], cases[c][1], cases[c][2], cases[c][3], cases[c][4]);
    if (rc > worst_rc) worst_rc = rc;
  }
  return worst_rc;
}
