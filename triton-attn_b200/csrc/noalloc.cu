// tattn_bwd_noalloc: the whole backward (preprocess, dK/dV, dQ) in one call that allocates nothing.
//
// The regular backward needs one fp32 value per query row (delta = rowsum(dO * O)) between its
// preprocess kernel and the dK/dV and dQ kernels, and its callers supply that buffer. Some callers
// cannot: a runtime that serves every device byte from a fixed, pre-planned arena has no slot for an
// extra workspace, and a host binding (cgo, JNI, a C plugin) may only be able to pass the buffers its
// user handed it. For them this entry point keeps delta in a file-scope device array that every GPU
// loading this library holds from module load until process exit.
//
// Limits and sharing:
//   * at most TATTN_BWD_NOALLOC_MAX_ROWS = Z*H*N query rows (16 MiB of fp32); larger problems are
//     rejected with TATTN_ERR_TOO_LARGE before anything is launched;
//   * every call on a device uses the same array. Each call rewrites all Z*H*N entries it reads (the
//     preprocess fills them before dK/dV and dQ run), so nothing needs clearing between calls, but two
//     calls whose kernels overlap on the GPU (different streams, no ordering between them) race on it;
//   * the first call on a device resolves the array's device address (cudaGetSymbolAddress, with that
//     device current); make that first call before any stream capture.
// No cudaMalloc, cudaFree or allocating library routine is called here or in the entry points it uses.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/tattn.h"

namespace {

constexpr long long kMaxRows = TATTN_BWD_NOALLOC_MAX_ROWS;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_delta_scratch[kMaxRows];

std::mutex g_scratch_mu;
bool g_scratch_init[kMaxDevices] = {};
int g_scratch_rc[kMaxDevices] = {};
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_delta_scratch on the current device (resolved once per device). The host-side
// name `g_delta_scratch` is only a stand-in for the symbol and must never be passed to a kernel. The
// device is checked first: on a GPU that is not sm_100 the library's kernels cannot load, so the symbol
// cannot be resolved either, and the answer is TATTN_ERR_NO_DEVICE (the runtime's error from the
// failed lookup, if any, is cleared so it does not surface in an unrelated later launch check).
int scratch_for_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return TATTN_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return TATTN_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_init[dev]) {
    g_scratch_init[dev] = true;
    int major = 0;
    void* p = nullptr;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
      (void)cudaGetLastError();
      g_scratch_rc[dev] = TATTN_ERR_CUDA;
    } else if (major != 10) {
      g_scratch_rc[dev] = TATTN_ERR_NO_DEVICE;
    } else if (cudaGetSymbolAddress(&p, g_delta_scratch) != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      g_scratch_rc[dev] = TATTN_ERR_CUDA;
    } else {
      g_scratch_rc[dev] = TATTN_OK;
      g_scratch_ptr[dev] = static_cast<float*>(p);
    }
  }
  *out = g_scratch_ptr[dev];
  return g_scratch_rc[dev];
}

}  // namespace

extern "C" int tattn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                                 void* dq, void* dk, void* dv, const float* m, const int64_t* strides, int Z,
                                 int H, int N, int D, int dtype, int causal, float sm_scale, void* stream) {
  if (!strides || Z < 0 || H < 0 || N < 0 || (D != 16 && D != 32 && D != 64 && D != 128))
    return TATTN_ERR_INVALID_ARGUMENT;
  if (Z == 0 || H == 0 || N == 0) return TATTN_OK;
  // Z*H*N rows, bounded without forming a product that could overflow.
  if ((long long)N > kMaxRows / Z / H) return TATTN_ERR_TOO_LARGE;
  float* delta = nullptr;
  int rc = scratch_for_current_device(&delta);
  if (rc != TATTN_OK) return rc;
  // strides: q, k, v, o, dout, each (z, h, n, d)
  const int64_t* sq = strides;
  const int64_t* sk = strides + 4;
  const int64_t* sv = strides + 8;
  const int64_t* so = strides + 12;
  const int64_t* sdo = strides + 16;
  const int64_t pre_strides[8] = {so[0], so[1], so[2], so[3], sdo[0], sdo[1], sdo[2], sdo[3]};
  const int64_t qkvdo[16] = {sq[0], sq[1], sq[2], sq[3], sk[0], sk[1], sk[2], sk[3],
                             sv[0], sv[1], sv[2], sv[3], sdo[0], sdo[1], sdo[2], sdo[3]};
  rc = tattn_bwd_preprocess(o, dout, delta, pre_strides, Z, H, N, D, dtype, stream);
  if (rc != TATTN_OK) return rc;
  rc = tattn_bwd_dkdv(q, k, v, dout, dk, dv, m, delta, qkvdo, Z, H, N, D, dtype, causal, sm_scale, 0, stream);
  if (rc != TATTN_OK) return rc;
  return tattn_bwd_dq(q, k, v, dout, dq, m, delta, qkvdo, Z, H, N, D, dtype, causal, sm_scale, 0, stream);
}
