// C-ABI boundary (include/tattn.h): argument validation, TMA tensor-map encoding, dispatch to the
// kernel launchers, and the per-device status word that kernels write when a bounded wait runs out.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../../include/tattn.h"
#include "common.cuh"
#include "kernels.h"
#include "tiles.h"

namespace tattn {
namespace {

constexpr int kMaxDevices = 64;
constexpr float kLog2e = 1.4426950408889634f;

// Kernel-side failure bits (tattn_device_status). One word per device, in the module's own global
// memory; kernels get its address as a plain pointer.
__device__ int g_status_word;

struct DeviceState {
  bool init = false;
  int err = TATTN_OK;
  int* status = nullptr;
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
// Bound of every mbarrier wait in the kernels launched from now on (tattn_set_wait_limit_ns).
std::atomic<unsigned long long> g_wait_limit_ns{kDefaultWaitLimitNs};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

// The caller's current device. Also makes its primary context current on this thread: a thread that
// has not used CUDA yet (e.g. the autograd engine's worker) has none, and the driver's tensor-map
// encoder, called before any launch, then fails.
int current_device(int* dev) {
  if (cudaGetDevice(dev) != cudaSuccess) return TATTN_ERR_CUDA;
  if (*dev < 0 || *dev >= kMaxDevices) return TATTN_ERR_NO_DEVICE;
  if (cudaSetDevice(*dev) != cudaSuccess) return TATTN_ERR_CUDA;
  return TATTN_OK;
}

// Once per device (with that device current): check it is sm_100 and resolve the status word address.
int device_setup(DeviceState** out) {
  int dev;
  int rc = current_device(&dev);
  if (rc != TATTN_OK) return rc;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& st = g_dev[dev];
  if (!st.init) {
    st.init = true;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
      st.err = TATTN_ERR_CUDA;
    } else if (prop.major != 10) {
      st.err = TATTN_ERR_NO_DEVICE;
    } else if (cudaGetSymbolAddress(reinterpret_cast<void**>(&st.status), g_status_word) != cudaSuccess) {
      st.err = TATTN_ERR_CUDA;
    } else if (g_encode == nullptr) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr) {
        st.err = TATTN_ERR_NO_DEVICE;
      } else {
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      }
    }
  }
  *out = &st;
  return st.err;
}

bool valid_dims(int Z, int H, int N, int D) {
  return Z >= 0 && H >= 0 && N >= 0 && (D == 16 || D == 32 || D == 64 || D == 128);
}

Strides4 load_strides(const int64_t* s) { return Strides4{s[0], s[1], s[2], s[3]}; }

// Strides of extent-1 dimensions never move an address; replace them by the dense value so the TMA
// stride rules only see strides that matter.
Strides4 normalize(Strides4 s, int Z, int H, int N, int D) {
  if (N <= 1) s.n = D;
  if (H <= 1) s.h = int64_t(N) * s.n;
  if (Z <= 1) s.z = int64_t(H) * s.h;
  return s;
}

bool layout_ok(const void* p, Strides4 s, int Z, int H, int N, int D) {
  s = normalize(s, Z, H, N, D);
  if (s.d != 1) return false;
  if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return false;
  const int64_t lim = int64_t(1) << 38;
  for (int64_t x : {s.n, s.h, s.z}) {
    if (x <= 0 || x % 8 != 0 || x >= lim) return false;
  }
  return true;
}

// [Z, H, N, D] fp16 tensor as a 4-D TMA map {D, N, H, Z}; box = {box_cols columns (default min(D, 64)),
// box_rows rows} with the swizzle that matches one box row (16 bytes: none; 32/64/128 bytes).
int encode_f16(CUtensorMap* tm, const void* p, Strides4 s, int Z, int H, int N, int D, int box_rows, int box_cols = 0) {
  s = normalize(s, Z, H, N, D);
  const int cw = box_cols > 0 ? box_cols : (D < 64 ? D : 64);
  cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(N), cuuint64_t(H), cuuint64_t(Z)};
  cuuint64_t strides[3] = {cuuint64_t(s.n) * 2, cuuint64_t(s.h) * 2, cuuint64_t(s.z) * 2};
  cuuint32_t box[4] = {cuuint32_t(cw), cuuint32_t(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle sw = cw == 64   ? CU_TENSOR_MAP_SWIZZLE_128B
                                : cw == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : cw == 16 ? CU_TENSOR_MAP_SWIZZLE_32B
                                           : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(p), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TATTN_OK : TATTN_ERR_LAYOUT;
}

// Dense [Z, H, N, D] fp32 tensor as a 4-D TMA map {D, N, H, Z} with boxes of box_cols x box_rows and
// the swizzle of one box row (box_cols * 4 bytes: 32, 64 or 128).
int encode_f32_dense(CUtensorMap* tm, void* p, int Z, int H, int N, int D, int box_rows, int box_cols) {
  cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(N), cuuint64_t(H), cuuint64_t(Z)};
  cuuint64_t strides[3] = {cuuint64_t(D) * 4, cuuint64_t(N) * D * 4, cuuint64_t(H) * N * D * 4};
  cuuint32_t box[4] = {cuuint32_t(box_cols), cuuint32_t(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const int row_bytes = box_cols * 4;
  const CUtensorMapSwizzle sw = row_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : row_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                  : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TATTN_OK : TATTN_ERR_LAYOUT;
}

int cuda_rc(cudaError_t e) {
  if (e == cudaSuccess) return TATTN_OK;
  if (e == cudaErrorNotSupported) return TATTN_ERR_UNSUPPORTED;
  return TATTN_ERR_CUDA;
}

}  // namespace
}  // namespace tattn

using namespace tattn;

extern "C" int tattn_fwd(const void* q, const void* k, const void* v, void* o, float* m, const int64_t* strides,
                         int Z, int H, int N, int D, int dtype, int causal, float sm_scale, int tile_cfg,
                         void* stream) {
  if (!strides || !valid_dims(Z, H, N, D) || (dtype != TATTN_F16 && dtype != TATTN_F32) || tile_cfg < 0 ||
      tile_cfg > kNumFwdTiles)
    return TATTN_ERR_INVALID_ARGUMENT;
  const int variant = tile_cfg == 0 ? tile_default(0, D, causal != 0) : tile_cfg - 1;
  if (dtype == TATTN_F16 && !tile_supported(0, variant, D)) return TATTN_ERR_UNSUPPORTED;
  if (int64_t(Z) * H * N == 0) return TATTN_OK;
  if (!q || !k || !v || !o || !m) return TATTN_ERR_INVALID_ARGUMENT;
  DeviceState* st;
  int rc = device_setup(&st);
  if (rc != TATTN_OK) return rc;
  const Strides4 sq = load_strides(strides), sk = load_strides(strides + 4), sv = load_strides(strides + 8),
                 so = load_strides(strides + 12);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  FwdArgs a{};
  a.o = o;
  a.m = m;
  a.so = so;
  a.Z = Z;
  a.H = H;
  a.N = N;
  a.status = st->status;
  a.wait_limit_ns = g_wait_limit_ns.load();
  if (dtype == TATTN_F32) {
    a.qk_scale = sm_scale * kLog2e;
    return cuda_rc(launch_fwd_f32(D, causal != 0, q, k, v, sq, sk, sv, a, sm_scale, s));
  }
  if (!layout_ok(q, sq, Z, H, N, D) || !layout_ok(k, sk, Z, H, N, D) || !layout_ok(v, sv, Z, H, N, D) ||
      !layout_ok(o, so, Z, H, N, D))
    return TATTN_ERR_LAYOUT;
  a.so = normalize(so, Z, H, N, D);
  a.qk_scale = (sm_scale < 0.f ? -sm_scale : sm_scale) * kLog2e;
  a.negate_s = sm_scale < 0.f ? 1 : 0;
  CUtensorMap tq, tk, tv;
  const int kv_rows = fwd_f16_kv_rows(D, variant);  // must match the kernel's K/V shared-memory slots
  if ((rc = encode_f16(&tq, q, sq, Z, H, N, D, 128)) != TATTN_OK) return rc;
  if ((rc = encode_f16(&tk, k, sk, Z, H, N, D, kv_rows)) != TATTN_OK) return rc;
  if ((rc = encode_f16(&tv, v, sv, Z, H, N, D, kv_rows)) != TATTN_OK) return rc;
  return cuda_rc(launch_fwd_f16(D, causal != 0, variant, tq, tk, tv, a, s));
}

extern "C" int tattn_bwd_preprocess(const void* o, const void* dout, float* delta, const int64_t* strides, int Z,
                                    int H, int N, int D, int dtype, void* stream) {
  if (!strides || !valid_dims(Z, H, N, D) || (dtype != TATTN_F16 && dtype != TATTN_F32))
    return TATTN_ERR_INVALID_ARGUMENT;
  if (int64_t(Z) * H * N == 0) return TATTN_OK;
  if (!o || !dout || !delta) return TATTN_ERR_INVALID_ARGUMENT;
  DeviceState* st;
  int rc = device_setup(&st);
  if (rc != TATTN_OK) return rc;
  BwdArgs a{};
  a.o = o;
  a.dout = dout;
  a.so = load_strides(strides);
  a.sdo = load_strides(strides + 4);
  // Rows are read with 16-byte vector loads: same rules as the TMA path (fp32 rows are 16-byte
  // aligned whenever fp16-style strides hold with half the element count, checked here directly).
  const int esz = dtype == TATTN_F16 ? 2 : 4;
  for (const auto& pr : {std::make_pair(o, a.so), std::make_pair(dout, a.sdo)}) {
    Strides4 s = normalize(pr.second, Z, H, N, D);
    if (s.d != 1 || (reinterpret_cast<uintptr_t>(pr.first) & 15u) != 0) return TATTN_ERR_LAYOUT;
    for (int64_t x : {s.n, s.h, s.z})
      if ((x * esz) % 16 != 0) return TATTN_ERR_LAYOUT;
  }
  a.so = normalize(a.so, Z, H, N, D);
  a.sdo = normalize(a.sdo, Z, H, N, D);
  a.delta = delta;
  a.Z = Z;
  a.H = H;
  a.N = N;
  a.status = st->status;
  return cuda_rc(launch_bwd_preprocess(D, dtype == TATTN_F16, a, static_cast<cudaStream_t>(stream)));
}

namespace {

int bwd_common(bool dq_pass, const void* q, const void* k, const void* v, const void* dout, void* dq, void* dk,
               void* dv, const float* m, const float* delta, const int64_t* strides, int Z, int H, int N, int D,
               int dtype, int causal, float sm_scale, int tile_cfg, void* stream) {
  if (!strides || !valid_dims(Z, H, N, D) || (dtype != TATTN_F16 && dtype != TATTN_F32) || tile_cfg < 0 ||
      tile_cfg > kNumBwdTiles)
    return TATTN_ERR_INVALID_ARGUMENT;
  const int variant = tile_cfg == 0 ? tile_default(1, D, causal != 0) : tile_cfg - 1;
  if (dtype == TATTN_F16 && !tile_supported(1, variant, D)) return TATTN_ERR_UNSUPPORTED;
  if (int64_t(Z) * H * N == 0) return TATTN_OK;
  if (!q || !k || !v || !dout || !m || !delta) return TATTN_ERR_INVALID_ARGUMENT;
  if (dq_pass ? !dq : (!dk || !dv)) return TATTN_ERR_INVALID_ARGUMENT;
  DeviceState* st;
  int rc = device_setup(&st);
  if (rc != TATTN_OK) return rc;
  BwdArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.dout = dout;
  a.sq = load_strides(strides);
  a.sk = load_strides(strides + 4);
  a.sv = load_strides(strides + 8);
  a.sdo = load_strides(strides + 12);
  a.m = m;
  a.delta = const_cast<float*>(delta);
  a.dq = dq;
  a.dk = dk;
  a.dv = dv;
  a.Z = Z;
  a.H = H;
  a.N = N;
  a.sm_scale = sm_scale;
  a.qk_scale = (sm_scale < 0.f ? -sm_scale : sm_scale) * kLog2e;
  a.negate_s = sm_scale < 0.f ? 1 : 0;
  a.status = st->status;
  a.wait_limit_ns = g_wait_limit_ns.load();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TATTN_F32)
    return cuda_rc(dq_pass ? launch_bwd_dq_f32(D, causal != 0, a, s) : launch_bwd_dkdv_f32(D, causal != 0, a, s));
  if (!layout_ok(q, a.sq, Z, H, N, D) || !layout_ok(k, a.sk, Z, H, N, D) || !layout_ok(v, a.sv, Z, H, N, D) ||
      !layout_ok(dout, a.sdo, Z, H, N, D))
    return TATTN_ERR_LAYOUT;
  if ((reinterpret_cast<uintptr_t>(dq_pass ? dq : dk) & 15u) != 0 || (!dq_pass && (reinterpret_cast<uintptr_t>(dv) & 15u)))
    return TATTN_ERR_LAYOUT;
  CUtensorMap tq, tk, tv, tdo;
  // dQ: query tiles of 128 rows, key blocks of the variant's block_n rows; dK/dV: key tiles of 128 rows,
  // query blocks of block_n rows.
  int q_rows = 0, kv_rows = 0;
  bwd_f16_box_rows(D, dq_pass, variant, &q_rows, &kv_rows);  // must match the kernels' shared-memory slots
  if ((rc = encode_f16(&tq, q, a.sq, Z, H, N, D, q_rows)) != TATTN_OK) return rc;
  if ((rc = encode_f16(&tk, k, a.sk, Z, H, N, D, kv_rows)) != TATTN_OK) return rc;
  if ((rc = encode_f16(&tv, v, a.sv, Z, H, N, D, kv_rows)) != TATTN_OK) return rc;
  if ((rc = encode_f16(&tdo, dout, a.sdo, Z, H, N, D, q_rows)) != TATTN_OK) return rc;
  // dQ / dK / dV are dense [Z, H, N, D]; the kernels write them through TMA store maps (dQ: each
  // compute warpgroup stores half of the columns).
  const Strides4 dense{int64_t(H) * N * D, int64_t(N) * D, D, 1};
  if (dq_pass) {
    CUtensorMap tdq;
    if ((rc = encode_f16(&tdq, dq, dense, Z, H, N, D, kBwdStoreRows, D <= 64 ? D / 2 : 0)) != TATTN_OK) return rc;
    return cuda_rc(launch_bwd_dq_f16(D, causal != 0, variant, tq, tk, tv, tdo, tdq, a, s));
  }
  CUtensorMap tdk, tdv;
  if ((rc = encode_f16(&tdk, dk, dense, Z, H, N, D, kBwdStoreRows, D <= 64 ? D / 2 : 0)) != TATTN_OK) return rc;
  if ((rc = encode_f16(&tdv, dv, dense, Z, H, N, D, kBwdStoreRows, D <= 64 ? D / 2 : 0)) != TATTN_OK) return rc;
  return cuda_rc(launch_bwd_dkdv_f16(D, causal != 0, variant, tq, tk, tv, tdo, tdk, tdv, a, s));
}

}  // namespace

extern "C" int tattn_bwd_dkdv(const void* q, const void* k, const void* v, const void* dout, void* dk, void* dv,
                              const float* m, const float* delta, const int64_t* strides, int Z, int H, int N,
                              int D, int dtype, int causal, float sm_scale, int tile_cfg, void* stream) {
  return bwd_common(false, q, k, v, dout, nullptr, dk, dv, m, delta, strides, Z, H, N, D, dtype, causal, sm_scale,
                    tile_cfg, stream);
}

extern "C" int tattn_bwd_dq(const void* q, const void* k, const void* v, const void* dout, void* dq,
                            const float* m, const float* delta, const int64_t* strides, int Z, int H, int N, int D,
                            int dtype, int causal, float sm_scale, int tile_cfg, void* stream) {
  return bwd_common(true, q, k, v, dout, dq, nullptr, nullptr, m, delta, strides, Z, H, N, D, dtype, causal,
                    sm_scale, tile_cfg, stream);
}

extern "C" int tattn_bwd_fused(const void* q, const void* k, const void* v, const void* o, const void* dout,
                               void* dq, void* dk, void* dv, const float* m, float* delta, void* workspace,
                               const int64_t* strides, int Z, int H, int N, int D, int dtype, int causal,
                               float sm_scale, void* stream) {
  if (!strides || !valid_dims(Z, H, N, D) || (dtype != TATTN_F16 && dtype != TATTN_F32))
    return TATTN_ERR_INVALID_ARGUMENT;
  if (dtype != TATTN_F16) return TATTN_ERR_UNSUPPORTED;
  if (int64_t(Z) * H * N == 0) return TATTN_OK;
  if (!q || !k || !v || !o || !dout || !dq || !dk || !dv || !m || !delta || !workspace)
    return TATTN_ERR_INVALID_ARGUMENT;
  float* dq_acc = static_cast<float*>(workspace);
  DeviceState* st;
  int rc = device_setup(&st);
  if (rc != TATTN_OK) return rc;
  BwdArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.o = o;
  a.dout = dout;
  a.sq = load_strides(strides);
  a.sk = load_strides(strides + 4);
  a.sv = load_strides(strides + 8);
  a.so = load_strides(strides + 12);
  a.sdo = load_strides(strides + 16);
  a.m = m;
  a.delta = delta;
  a.dq = dq;
  a.dk = dk;
  a.dv = dv;
  a.dq_acc = dq_acc;
  a.grid_sync = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + int64_t(Z) * H * N * D * 4);
  a.Z = Z;
  a.H = H;
  a.N = N;
  a.sm_scale = sm_scale;
  a.qk_scale = (sm_scale < 0.f ? -sm_scale : sm_scale) * kLog2e;
  a.negate_s = sm_scale < 0.f ? 1 : 0;
  a.status = st->status;
  a.wait_limit_ns = g_wait_limit_ns.load();
  if (!layout_ok(q, a.sq, Z, H, N, D) || !layout_ok(k, a.sk, Z, H, N, D) || !layout_ok(v, a.sv, Z, H, N, D) ||
      !layout_ok(o, a.so, Z, H, N, D) || !layout_ok(dout, a.sdo, Z, H, N, D))
    return TATTN_ERR_LAYOUT;
  for (const void* p : {static_cast<const void*>(dq), static_cast<const void*>(dk), static_cast<const void*>(dv),
                        static_cast<const void*>(dq_acc)})
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return TATTN_ERR_LAYOUT;
  CUtensorMap tq, tk, tv, tdo, tdk, tdv, tdqacc;
  // 128-row key tiles; query blocks of 128 rows (64 at D = 128). The dQ workspace is added to in boxes
  // of D/2 columns (32 at D = 128, where each warp holds 32 head dims of 32 queries).
  const int q_rows = bwd_fused_query_rows(D), acc_cols = D == 128 ? 32 : D / 2;
  if ((rc = encode_f16(&tq, q, a.sq, Z, H, N, D, q_rows)) != TATTN_OK) return rc;
  if ((rc = encode_f16(&tk, k, a.sk, Z, H, N, D, 128)) != TATTN_OK) return rc;
  if ((rc = encode_f16(&tv, v, a.sv, Z, H, N, D, 128)) != TATTN_OK) return rc;
  if ((rc = encode_f16(&tdo, dout, a.sdo, Z, H, N, D, q_rows)) != TATTN_OK) return rc;
  const Strides4 dense{int64_t(H) * N * D, int64_t(N) * D, D, 1};
  if ((rc = encode_f16(&tdk, dk, dense, Z, H, N, D, kBwdStoreRows, D / 2)) != TATTN_OK) return rc;
  if ((rc = encode_f16(&tdv, dv, dense, Z, H, N, D, kBwdStoreRows, D / 2)) != TATTN_OK) return rc;
  if ((rc = encode_f32_dense(&tdqacc, dq_acc, Z, H, N, D, kBwdStoreRows, acc_cols)) != TATTN_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = cuda_rc(launch_bwd_preprocess(D, true, a, s))) != TATTN_OK) return rc;  // delta, zeroed workspace
  return cuda_rc(launch_bwd_fused_f16(D, causal != 0, tq, tk, tv, tdo, tdk, tdv, tdqacc, a, s));
}

extern "C" int64_t tattn_bwd_fused_workspace_bytes(int Z, int H, int N, int D) {
  if (!valid_dims(Z, H, N, D) || double(Z) * H * N * (4.0 * D + 4.0) > 4e18) return -1;
  return bwd_fused_workspace_bytes(Z, H, N, D);
}

namespace tattn {
namespace {

// One CTA of two warps that runs the attention kernels' unwinding protocol without their data
// movement. Warp 0 waits on a barrier phase that nothing completes; warp 1 waits on a barrier that warp
// 0 would arrive on once its own wait succeeded. Warp 0's bounded wait runs out after the launch's wait
// limit: it records kStatusWaitTimeout in the status word and raises the CTA's abort flag; warp 1 sees
// the flag inside its own bounded wait and gives up as well; the TMEM columns allocated at the start
// (as every tensor-core kernel here does) are released, and the kernel returns.
__global__ void __launch_bounds__(64) wait_selftest_kernel(int* status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x / 32;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 32);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const CtaAbort ab{&abort_flag, status, limit_ns};
  if (warp == 0) {
    if (warp_wait(&bars[0], 0, ab)) mbar_arrive(&bars[1]);  // bars[0] never receives an arrival
  } else {
    warp_wait(&bars[1], 0, ab);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_slot, 32);
  }
}

}  // namespace
}  // namespace tattn

extern "C" int tattn_set_wait_limit_ns(uint64_t limit_ns) {
  g_wait_limit_ns.store(limit_ns == 0 ? kDefaultWaitLimitNs : static_cast<unsigned long long>(limit_ns));
  return TATTN_OK;
}

extern "C" uint64_t tattn_get_wait_limit_ns(void) { return g_wait_limit_ns.load(); }

extern "C" int tattn_selftest_wait(void* stream) {
  DeviceState* st;
  int rc = device_setup(&st);
  if (rc != TATTN_OK) return rc;
  wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(st->status, g_wait_limit_ns.load());
  return cudaGetLastError() == cudaSuccess ? TATTN_OK : TATTN_ERR_CUDA;
}

extern "C" int tattn_layout_ok(const void* ptr, const int64_t* strides, int Z, int H, int N, int D) {
  if (!strides || !valid_dims(Z, H, N, D)) return 0;
  return layout_ok(ptr, load_strides(strides), Z, H, N, D) ? 1 : 0;
}

extern "C" int tattn_tile_configs(int kind) { return kind == 0 ? kNumFwdTiles : kind == 1 ? kNumBwdTiles : 0; }

extern "C" int tattn_tile_config_info(int kind, int tile_cfg, int* block_m, int* block_n, int* stages) {
  if (!block_m || !block_n || !stages || tile_cfg < 1 || tile_cfg > tattn_tile_configs(kind))
    return TATTN_ERR_INVALID_ARGUMENT;
  const TileVariant& t = kind == 0 ? kFwdTiles[tile_cfg - 1] : kBwdTiles[tile_cfg - 1];
  *block_m = t.block_m;
  *block_n = t.block_n;
  *stages = t.stages;
  return TATTN_OK;
}

extern "C" int tattn_tile_default(int kind, int D, int causal, int dtype) {
  if ((kind != 0 && kind != 1) || (D != 16 && D != 32 && D != 64 && D != 128)) return -1;
  if (dtype == TATTN_F32) return 0;
  if (dtype != TATTN_F16) return -1;
  return tile_default(kind, D, causal != 0) + 1;
}

extern "C" int tattn_tile_supported(int kind, int tile_cfg, int D) {
  if (tile_cfg == 0) return (D == 16 || D == 32 || D == 64 || D == 128) ? 1 : 0;
  return tile_supported(kind, tile_cfg - 1, D) ? 1 : 0;
}

extern "C" int tattn_device_status(void* stream, int* out, int clear) {
  if (!out) return TATTN_ERR_INVALID_ARGUMENT;
  DeviceState* st;
  int rc = device_setup(&st);
  if (rc != TATTN_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return TATTN_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, st->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return TATTN_ERR_CUDA;
  if (clear && v != 0) {
    const int zero = 0;
    if (cudaMemcpy(st->status, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return TATTN_ERR_CUDA;
  }
  *out = v;
  return TATTN_OK;
}

extern "C" const char* tattn_status_string(int status) {
  switch (status) {
    case TATTN_OK: return "ok";
    case TATTN_ERR_INVALID_ARGUMENT: return "invalid argument (dims, dtype, head dim or null pointer)";
    case TATTN_ERR_LAYOUT: return "layout not addressable by TMA (needs unit D stride, 16-byte alignment)";
    case TATTN_ERR_CUDA: return "CUDA runtime or launch failure";
    case TATTN_ERR_NO_DEVICE: return "current device is not an sm_100 GPU (or the TMA encoder is unavailable)";
    case TATTN_ERR_DEVICE_STATUS: return "a kernel recorded a failure in the device status word";
    case TATTN_ERR_UNSUPPORTED: return "not implemented by this build";
    case TATTN_ERR_TOO_LARGE: return "problem larger than the fixed no-allocation buffer (Z*H*N > TATTN_BWD_NOALLOC_MAX_ROWS)";
    default: return "unknown status";
  }
}

extern "C" int tattn_abi_version(void) { return TATTN_ABI_VERSION; }
