/*
 * tattn_b200 -- C ABI of the B200-native FlashAttention-2 forward/backward.
 *
 * This is the drop-in boundary for the reference's kernel layer (amaanmithani/triton-attn,
 * src/tattn/kernels.py): each entry point replaces one Triton kernel launch made by the reference's
 * host glue (src/tattn/api.py). Plain pointers and sizes only; any host language binds it through
 * its FFI (the Python package `tattn` uses ctypes).
 *
 * Conventions shared by every entry point
 *   - Tensors are logically [Z, H, N, D] (batch, heads, sequence, head dim) and are given by a device
 *     pointer plus four element strides in (z, h, n, d) order, exactly like the reference kernels'
 *     (stride_*z, stride_*h, stride_*m|n, stride_*d) arguments (kernels.py:63-88, 157-179, 248-269).
 *   - dtype: TATTN_F16 (IEEE half; runs on the tcgen05 tensor cores) or TATTN_F32 (runs exact fp32
 *     CUDA-core kernels). D must be 16, 32, 64 or 128 (api.py:53).
 *   - M and delta are dense fp32 [Z, H, N] (index (z*H + h)*N + n), as kernels.py:143 / 193-194.
 *     M = rowmax + log2(rowsum) of the base-2 scaled scores S*sm_scale*log2(e).
 *   - Gradients dq, dk, dv are written dense and contiguous [Z, H, N, D] (api.py:111-113).
 *   - The causal mask keeps row >= col (top-left aligned, equal query and key length).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Calls are asynchronous; they only
 *     enqueue work. The caller allocates every buffer; the library allocates no device memory.
 *   - fp16 tensors read through TMA need: unit D stride, 16-byte aligned base, and (z, h, n) strides
 *     that are multiples of 8 elements (strides of extent-1 dimensions are ignored). Otherwise the
 *     call returns TATTN_ERR_LAYOUT and the caller makes the tensor contiguous (and aligned).
 *   - Return value: TATTN_OK or one of the TATTN_ERR_* codes below; nothing is launched on error.
 *   - Kernel-side failures (a bounded wait that ran out) are recorded in a per-device status word,
 *     read with tattn_device_status().
 */
#ifndef TATTN_B200_H_
#define TATTN_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TATTN_ABI_VERSION 3

#if defined(__GNUC__)
#define TATTN_API __attribute__((visibility("default")))
#else
#define TATTN_API
#endif

enum tattn_dtype { TATTN_F16 = 0, TATTN_F32 = 1 };

enum tattn_status {
  TATTN_OK = 0,
  TATTN_ERR_INVALID_ARGUMENT = 1, /* bad dims, dtype, head dim, null pointer */
  TATTN_ERR_LAYOUT = 2,           /* strides/alignment not addressable by TMA: make contiguous */
  TATTN_ERR_CUDA = 3,             /* a CUDA runtime/driver call or a launch failed */
  TATTN_ERR_NO_DEVICE = 4,        /* current device is not sm_100 or the TMA encoder is missing */
  TATTN_ERR_DEVICE_STATUS = 5,    /* a kernel recorded a failure in the device status word */
  TATTN_ERR_UNSUPPORTED = 6,      /* valid request this build does not implement */
  TATTN_ERR_TOO_LARGE = 7         /* problem exceeds a fixed-size library buffer (tattn_bwd_noalloc) */
};

/* Device status word bits (tattn_device_status). */
#define TATTN_DEV_WAIT_TIMEOUT 1 /* an mbarrier wait exceeded the wait limit (tattn_set_wait_limit_ns); the CTA unwound */
#define TATTN_DEV_ABORTED 2

/* Forward: O = softmax(Q K^T * sm_scale) V and M, for one attention call.
 * Replaces the launch of _fwd_kernel (src/tattn/kernels.py:57-148) made by _forward
 * (src/tattn/api.py:78-99). strides: 16 int64 = q, k, v, o each (z, h, n, d).
 * tile_cfg: 0 = the default tile for (D, causal, dtype); 1..n = an explicit variant (tattn_tile_configs). */
TATTN_API int tattn_fwd(const void* q, const void* k, const void* v, void* o, float* m, const int64_t* strides, int Z,
              int H, int N, int D, int dtype, int causal, float sm_scale, int tile_cfg, void* stream);

/* Backward preprocess: delta = rowsum(dO * O) in fp32.
 * Replaces _bwd_preprocess (src/tattn/kernels.py:324-337), launched at api.py:122.
 * strides: 8 int64 = o, dout each (z, h, n, d); both need a unit D stride and 16-byte aligned rows. */
TATTN_API int tattn_bwd_preprocess(const void* o, const void* dout, float* delta, const int64_t* strides, int Z, int H,
                         int N, int D, int dtype, void* stream);

/* Backward dK/dV, one CTA per key block, no atomics: dV = P^T dO, dK = dS^T Q * sm_scale.
 * Replaces _bwd_dkdv_kernel (src/tattn/kernels.py:151-239), launched at api.py:124-142.
 * strides: 16 int64 = q, k, v, dout each (z, h, n, d). dk, dv: dense [Z, H, N, D]. */
TATTN_API int tattn_bwd_dkdv(const void* q, const void* k, const void* v, const void* dout, void* dk, void* dv,
                   const float* m, const float* delta, const int64_t* strides, int Z, int H, int N, int D,
                   int dtype, int causal, float sm_scale, int tile_cfg, void* stream);

/* Backward dQ, one CTA per query block: dQ = dS K * sm_scale.
 * Replaces _bwd_dq_kernel (src/tattn/kernels.py:242-321), launched at api.py:143-145.
 * strides: 16 int64 = q, k, v, dout each (z, h, n, d). dq: dense [Z, H, N, D]. */
TATTN_API int tattn_bwd_dq(const void* q, const void* k, const void* v, const void* dout, void* dq, const float* m,
                 const float* delta, const int64_t* strides, int Z, int H, int N, int D, int dtype, int causal,
                 float sm_scale, int tile_cfg, void* stream);

/* The whole backward in two kernels: delta = rowsum(dO * O) (tattn_bwd_preprocess's job) into the
 * caller's fp32 [Z, H, N] buffer, then dQ, dK and dV in one pass in which each (key block, query
 * block) pair's scores, P and dS are computed once; the reference's two kernels (src/tattn/kernels.py:
 * 151-239 and 242-321, launched at api.py:122-145) each recompute S and dO V^T. dQ is accumulated by
 * fp32 additions at L2 into `workspace` (caller-provided, tattn_bwd_fused_workspace_bytes bytes,
 * 16-byte aligned; zeroed by the first kernel): dense fp32 [Z, H, N, D] sums, then a grid-barrier
 * counter. The second kernel is one cooperative launch (one CTA per SM at most, all resident): once
 * every CTA's additions have completed it scales the sums into dq itself. The order of the additions
 * varies from run to run, so dq is not bitwise reproducible (dk and dv are).
 * strides: 20 int64 = q, k, v, o, dout each (z, h, n, d); dq, dk, dv dense [Z, H, N, D].
 * fp16 only (every supported D, causal or not; at D = 128 the query blocks are 64 rows and each block's
 * dQ part is computed transposed, dQ^T = K^T dS^T, to fit tensor memory): fp32 requests return
 * TATTN_ERR_UNSUPPORTED (use the three calls). */
TATTN_API int tattn_bwd_fused(const void* q, const void* k, const void* v, const void* o, const void* dout,
                    void* dq, void* dk, void* dv, const float* m, float* delta, void* workspace,
                    const int64_t* strides, int Z, int H, int N, int D, int dtype, int causal, float sm_scale,
                    void* stream);

/* Bytes of the workspace tattn_bwd_fused needs for a [Z, H, N, D] call (a multiple of 16), or -1 for
 * invalid dimensions. */
TATTN_API int64_t tattn_bwd_fused_workspace_bytes(int Z, int H, int N, int D);

/* Largest Z*H*N accepted by tattn_bwd_noalloc (its fixed fp32 row buffer: 16 MiB per GPU). */
#define TATTN_BWD_NOALLOC_MAX_ROWS 4194304

/* The whole backward (delta preprocess, dK/dV, dQ) in one call that allocates no device memory.
 * No counterpart in the reference: it exists for callers that cannot provide the fp32 row buffer
 * (delta) the three-call backward needs -- e.g. runtimes that hand out every device byte from a fixed,
 * pre-planned arena, or host bindings that can only pass the buffers their user gave them. delta lives
 * instead in a file-scope device array of TATTN_BWD_NOALLOC_MAX_ROWS floats that every GPU loading this
 * library holds until exit; larger problems return TATTN_ERR_TOO_LARGE. All calls on a device share
 * that array: each call rewrites every entry it reads, but calls that overlap on the GPU (unordered
 * streams) race on it. The first call on a device resolves the array's address; make it before any
 * stream capture. strides: 20 int64 = q, k, v, o, dout each (z, h, n, d); dq, dk, dv: dense
 * [Z, H, N, D]; other conventions as tattn_bwd_dkdv / tattn_bwd_dq (tile_cfg 0). */
TATTN_API int tattn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                                void* dq, void* dk, void* dv, const float* m, const int64_t* strides, int Z,
                                int H, int N, int D, int dtype, int causal, float sm_scale, void* stream);

/* Can the fp16 tensor-core path read this tensor in place? Returns 1 (yes) or 0 (make it contiguous).
 * strides: 4 int64 (z, h, n, d). Mirrors the check every fp16 entry point applies. */
TATTN_API int tattn_layout_ok(const void* ptr, const int64_t* strides, int Z, int H, int N, int D);

/* Tile variants. They stand in for the reference's autotune spaces (src/tattn/kernels.py:21-41, keyed
 * per (N bucket, D, causal) at api.py:59-62) and for its explicit-config bypass (_launch, api.py:69-75):
 * a static list per kernel family (kind 0 = forward, tattn_fwd; kind 1 = the split backward,
 * tattn_bwd_dkdv and tattn_bwd_dq) and a fixed default per (D, causal, dtype) measured on a B200.
 * tile_cfg 0 runs that default; tile_cfg i in 1..tattn_tile_configs(kind) runs variant i whatever the
 * shape, and an fp16 call whose variant does not fit its head dim returns TATTN_ERR_UNSUPPORTED. fp32
 * calls run CUDA-core kernels with no tile choice: tile_cfg is validated and otherwise ignored. */
/* Number of explicit variants of family `kind` (0 for an unknown kind). */
TATTN_API int tattn_tile_configs(int kind);
/* Shape of variant tile_cfg (1-based): query rows per CTA (block_m), rows of each inner block the CTA
 * loops over (block_n: keys in the forward and dQ pass, queries in the dK/dV pass), ring stages. */
TATTN_API int tattn_tile_config_info(int kind, int tile_cfg, int* block_m, int* block_n, int* stages);
/* The variant (1-based) that tile_cfg 0 runs for (D, causal, dtype); 0 when the dtype has no tile choice
 * (fp32); -1 for an invalid kind, head dim or dtype. */
TATTN_API int tattn_tile_default(int kind, int D, int causal, int dtype);
/* 1 if variant tile_cfg of family `kind` can run fp16 head dim D (tile_cfg 0 always can), else 0. */
TATTN_API int tattn_tile_supported(int kind, int tile_cfg, int D);

/* Diagnostic (no reference counterpart): evaluate, for n inputs x, the FMA-pipe exp2 the kernels use
 * for part of each softmax row (y_poly), the hardware ex2.approx (y_hw) and CUDA's exp2f (y_lib), so
 * a test can hold the polynomial to its error bound against CUDA's own outputs. Device pointers. */
TATTN_API int tattn_selftest_exp2(const float* x, float* y_poly, float* y_hw, float* y_lib, int n, void* stream);

/* The backward's FMA-pipe exp2 (degree-4 polynomial) on n caller-given inputs: y[i] ~ 2^x[i], for
 * tests of its error bound (2.7e-6 relative for results above 2^-24). */
TATTN_API int tattn_selftest_exp2_poly4(const float* x, float* y, int n, void* stream);

/* Bound of every wait inside the tensor-core kernels (no reference counterpart; the Triton kernels have
 * no such waits). A wait that has not completed after limit_ns nanoseconds makes its CTA give up: it
 * sets TATTN_DEV_WAIT_TIMEOUT in the device status word, drains its own copies in flight, frees its
 * TMEM and exits, so a fault elsewhere can never leave a kernel spinning. Applies to launches made after
 * the call, process-wide; 0 restores the default of 1 s. A limit shorter than a kernel's normal waits
 * makes it fail (status set, outputs incomplete); keep the default outside tests. */
TATTN_API int tattn_set_wait_limit_ns(uint64_t limit_ns);
TATTN_API uint64_t tattn_get_wait_limit_ns(void);

/* Diagnostic (no reference counterpart): one small kernel that runs the tensor-core kernels' unwinding
 * path on purpose. Its first bounded wait is on a barrier that nothing completes, so after the current
 * wait limit it records TATTN_DEV_WAIT_TIMEOUT, its other warp gives up through the CTA's abort flag, it
 * frees its TMEM and returns. The GPU and the context stay usable; read (and clear) the bit with
 * tattn_device_status. */
TATTN_API int tattn_selftest_wait(void* stream);

/* Synchronise `stream`, then report the current device's status word (TATTN_DEV_* bits) in *out and
 * clear it when `clear` is nonzero. Returns TATTN_OK, or TATTN_ERR_CUDA if the sync failed. */
TATTN_API int tattn_device_status(void* stream, int* out, int clear);

/* Static description of a status code. */
TATTN_API const char* tattn_status_string(int status);

/* TATTN_ABI_VERSION of the loaded library. */
TATTN_API int tattn_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TATTN_B200_H_ */
