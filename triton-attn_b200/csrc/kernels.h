// Host-side launcher interface between the C-ABI layer (capi.cu) and the kernel translation units.
// Nothing here is exported from the shared library; include/tattn.h is the public boundary.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tattn {

// Element strides of one [Z, H, N, D] tensor (the D stride is always 1 for the fp16 kernels).
struct Strides4 {
  int64_t z, h, n, d;
};

struct FwdArgs {
  void* o;           // [Z, H, N, D], strides `so`
  float* m;          // [Z, H, N] dense fp32: rowmax + log2(rowsum), base-2 units
  Strides4 so;
  int Z, H, N;
  float qk_scale;    // |sm_scale| * log2(e); the sign goes into the S MMA (negate A) for fp16
  int negate_s;      // 1 when sm_scale < 0 (fp16 path)
  int* status;       // device status word
  unsigned long long wait_limit_ns;  // bound of every mbarrier wait (tattn_set_wait_limit_ns)
};

struct BwdArgs {
  // inputs
  const void* q; const void* k; const void* v; const void* o; const void* dout;
  Strides4 sq, sk, sv, so, sdo;
  const float* m;    // [Z, H, N]
  float* delta;      // [Z, H, N]: rowsum(dO * O)
  // outputs (dense [Z, H, N, D])
  void* dq; void* dk; void* dv;
  float* dq_acc;     // fused backward: dense fp32 [Z, H, N, D] dQ workspace (zeroed by the preprocess), or null
  unsigned* grid_sync;  // fused backward: its grid-barrier counter (zeroed by the preprocess), or null
  int Z, H, N;
  float sm_scale;    // signed
  float qk_scale;    // |sm_scale| * log2(e)
  int negate_s;
  int* status;
  unsigned long long wait_limit_ns;  // bound of every mbarrier wait (tattn_set_wait_limit_ns)
};

// `variant` below is a 0-based tile variant of tiles.h (kFwdTiles / kBwdTiles); launchers return
// cudaErrorNotSupported for a variant that does not fit head dim D.
// Rows per K/V block of the fp16 forward variant for head dim D: the TMA box height of its K and V
// tensor maps (the Q map always uses 128-row boxes); 0 if the variant does not fit D.
int fwd_f16_kv_rows(int D, int variant);
// TMA box heights of the fp16 split-backward kernels' Q/dO and K/V tensor maps for head dim D, dQ pass
// or dK/dV pass, and tile variant.
void bwd_f16_box_rows(int D, bool dq_pass, int variant, int* q_rows, int* kv_rows);

// fp16 tcgen05 kernels (tensor maps describe [Z, H, N, D] tensors as 4-D {D, N, H, Z}).
cudaError_t launch_fwd_f16(int D, bool causal, int variant, const CUtensorMap& tq, const CUtensorMap& tk,
                           const CUtensorMap& tv, const FwdArgs& a, cudaStream_t s);
// tdq: store map of the dense dQ output, kBwdStoreRows-row boxes of D/2 columns (D <= 64).
cudaError_t launch_bwd_dq_f16(int D, bool causal, int variant, const CUtensorMap& tq, const CUtensorMap& tk,
                              const CUtensorMap& tv, const CUtensorMap& tdo, const CUtensorMap& tdq, const BwdArgs& a,
                              cudaStream_t s);
// tdk / tdv: store maps of the dense dK / dV outputs, kBwdStoreRows-row boxes of D/2 columns (D <= 64).
cudaError_t launch_bwd_dkdv_f16(int D, bool causal, int variant, const CUtensorMap& tq, const CUtensorMap& tk,
                                const CUtensorMap& tv, const CUtensorMap& tdo, const CUtensorMap& tdk,
                                const CUtensorMap& tdv, const BwdArgs& a, cudaStream_t s);
// Fused backward kernel (any supported D, causal or not; one cooperative launch): dK, dV and the dQ
// sums into the fp32 workspace a.dq_acc [Z, H, N, D], then a grid barrier and a.dq = sm_scale * dq_acc
// as fp16. a.dq_acc, a.delta and the barrier counter a.grid_sync come from launch_bwd_preprocess.
// tq/tdo with boxes of bwd_fused_query_rows(D) rows, tk/tv 128-row boxes, tdk/tdv store maps of
// kBwdStoreRows-row boxes of D/2 columns, tdqacc a reduce map over a.dq_acc (kBwdStoreRows-row boxes
// of D/2 columns; 32 columns at D = 128).
cudaError_t launch_bwd_fused_f16(int D, bool causal, const CUtensorMap& tq, const CUtensorMap& tk,
                                 const CUtensorMap& tv, const CUtensorMap& tdo, const CUtensorMap& tdk,
                                 const CUtensorMap& tdv, const CUtensorMap& tdqacc, const BwdArgs& a, cudaStream_t s);
// Box height of the backward's output store maps (one warp's 32 TMEM lanes).
constexpr int kBwdStoreRows = 32;
// Query rows per block of the fused backward (its Q / dO box height): 128, or 64 at D = 128.
__host__ __device__ constexpr int bwd_fused_query_rows(int D) { return D == 128 ? 64 : 128; }
// Workspace of tattn_bwd_fused: the fp32 dQ rows [Z, H, N, D], then 16 bytes for the grid-barrier counter.
inline int64_t bwd_fused_workspace_bytes(int Z, int H, int N, int D) { return int64_t(Z) * H * N * D * 4 + 16; }

// SIMT kernels (fp32 inputs; any strides).
cudaError_t launch_fwd_f32(int D, bool causal, const void* q, const void* k, const void* v, Strides4 sq,
                           Strides4 sk, Strides4 sv, const FwdArgs& a, float sm_scale, cudaStream_t s);
cudaError_t launch_bwd_dq_f32(int D, bool causal, const BwdArgs& a, cudaStream_t s);
cudaError_t launch_bwd_dkdv_f32(int D, bool causal, const BwdArgs& a, cudaStream_t s);

// delta = rowsum(dO * O) in fp32 (fp16 or fp32 inputs); also zeroes the rows of a.dq_acc and the
// counter a.grid_sync when they are set (the fused backward's workspace).
cudaError_t launch_bwd_preprocess(int D, bool is_f16, const BwdArgs& a, cudaStream_t s);

}  // namespace tattn
