/* liteweight_b200 C ABI: the drop-in boundary of liteweight's weight-only
 * dequant-matmul hot path and of the decode step that drives it, built for
 * NVIDIA B200 (sm_100a).
 *
 * Conventions
 *   - Plain device pointers and sizes; tensors are row-major and contiguous.
 *   - fp16 = IEEE binary16 (2 bytes); int8/uint8 are raw bytes.
 *   - Every entry point enqueues work on `stream` (a cudaStream_t; NULL = the
 *     legacy default stream), never synchronises the host and never allocates
 *     device memory, so it can be captured in a CUDA graph.
 *   - Every entry point returns an lw_status (0 = success). Nothing calls
 *     exit(), traps on the device or prints.
 *
 * Reference interfaces replaced (paths inside the liteweight project):
 *   kernels/matmul_int8.py:103-145  matmul_int8(act, qweight, scales, group_size)
 *   kernels/matmul_int4.py:122-165  matmul_int4(act, qweight, scales, group_size)
 *   kernels/matmul_fp16.py:67-85    matmul_fp16(a, b)
 *   liteweight/quantize.py:30-43    dequantize_int8
 *   liteweight/quantize.py:102-128  dequantize_int4
 */
#ifndef LITEWEIGHT_B200_H
#define LITEWEIGHT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* lw_stream_t;

typedef enum {
  LW_OK = 0,
  LW_ERR_NULL_POINTER = 1,   /* a required pointer is NULL */
  LW_ERR_BAD_SHAPE = 2,      /* M, N or K <= 0, or K / N inconsistent with the format */
  LW_ERR_BAD_GROUP = 3,      /* group_size <= 0 or K % group_size != 0 */
  LW_ERR_ALIGNMENT = 4,      /* a pointer is not aligned to its element size */
  LW_ERR_UNSUPPORTED = 5,    /* valid input this build does not handle */
  LW_ERR_LAUNCH = 6,         /* the CUDA launch failed (cudaGetLastError) */
  LW_ERR_WORKSPACE = 7,      /* workspace missing or too small */
  LW_ERR_TIMEOUT = 8         /* a bounded device-side wait gave up */
} lw_status;

/* Human-readable name of a status code (static string). */
const char* lw_status_string(int status);

/* ABI version of this library (major * 100 + minor). */
int lw_abi_version(void);

/* Number of CUDA kernels this library has enqueued since it was loaded
 * (telemetry; no counterpart in the reference). */
unsigned long long lw_launch_count(void);

/* ---- dequant matmul: out[M,N] = act[M,K] @ dequant(W)[N,K]^T (+ bias) ----
 * fp32 accumulation of fp16 activations times fp16 dequantized weights, one
 * fp16 rounding at the end, then `+ bias` in fp16 when bias != NULL. This is
 * the arithmetic of liteweight/quantize.py:60 (the oracle the reference's
 * Triton kernels are tested against) followed by quantlinear.py:63-64.
 *
 * lw_gemm_w8a16 replaces kernels/matmul_int8.py:103-145:
 *   act fp16 [M,K], qweight int8 [N,K], scales fp16 [N,K/group_size],
 *   bias fp16 [N] or NULL, out fp16 [M,N].
 * lw_gemm_w4a16 replaces kernels/matmul_int4.py:122-165:
 *   qweight uint8 [N,K/2] (even k in the low nibble), K even.
 *
 * workspace (optional; may be NULL with workspace_bytes = 0): device scratch
 * of at least lw_gemm_workspace_size() bytes, 256-byte aligned, ZEROED before
 * its first use; every completed call leaves it zeroed again. With it, a
 * weight tile may be split between warps (better balance for small N); the
 * partial sums are combined in a fixed order, so results are deterministic
 * for a given shape and device. Calls that run concurrently (different
 * streams) must not share a workspace.
 */
int lw_gemm_w8a16(const void* act, const void* qweight, const void* scales, const void* bias,
                  void* out, int M, int N, int K, int group_size, void* workspace,
                  size_t workspace_bytes, lw_stream_t stream);
int lw_gemm_w4a16(const void* act, const void* qweight, const void* scales, const void* bias,
                  void* out, int M, int N, int K, int group_size, void* workspace,
                  size_t workspace_bytes, lw_stream_t stream);

/* Workspace bytes the matmul entry points can use for these sizes (bits = 4,
 * 8 or 16); 0 when no tile is split. Needs a current CUDA device. No
 * counterpart in the reference (its Triton kernels need no scratch). */
size_t lw_gemm_workspace_size(int bits, int M, int N, int K);

/* fp16 matmul with the weight in nn.Linear layout: out[M,N] = a[M,K] @ w[N,K]^T.
 * Replaces kernels/matmul_fp16.py:67-85 when `b` is the transpose of a
 * contiguous [N,K] tensor (how bench/benchmark.py:133 calls it: `W.T`), and
 * is the engine's un-quantized lm_head. */
int lw_gemm_f16(const void* a, const void* w, void* out, int M, int N, int K, void* workspace,
                size_t workspace_bytes, lw_stream_t stream);

/* fp16 matmul with a row-major b[K,N]: replaces kernels/matmul_fp16.py:67-85
 * for a contiguous b. */
int lw_gemm_f16_kn(const void* a, const void* b, void* out, int M, int N, int K, lw_stream_t stream);

/* ---- dequantization (bit-exact with liteweight/quantize.py:30-43, :102-128) ----
 * out fp16 [N,K] = fp16((float)code * (float)scale). */
int lw_dequant_w8(const void* qweight, const void* scales, void* out, int N, int K, int group_size,
                  lw_stream_t stream);
int lw_dequant_w4(const void* qweight, const void* scales, void* out, int N, int K, int group_size,
                  lw_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LITEWEIGHT_B200_H */
