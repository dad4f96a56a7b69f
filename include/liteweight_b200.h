/* liteweight_b200 C ABI: the drop-in boundary of liteweight's weight-only
 * dequant-matmul hot path and of the decode step that drives it, built for
 * NVIDIA B200 (sm_100a).
 *
 * Conventions
 *   - Plain device pointers and sizes; tensors are row-major and contiguous.
 *   - fp16 = IEEE binary16 (2 bytes); int8/uint8 are raw bytes.
 *   - Every compute entry point enqueues work on `stream` (a cudaStream_t;
 *     NULL = the legacy default stream), never synchronises the host and
 *     never allocates device memory, so it can be captured in a CUDA graph.
 *     The lw_peer_* setup calls are the exception and say so.
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
  LW_ERR_UNSUPPORTED = 5,    /* valid input the library does not handle */
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

/* Reads and clears the library's device-side error flags on the current
 * device: LW_ERR_TIMEOUT if a bounded wait inside one of its kernels gave up
 * since the last call (that launch's results are invalid), else LW_OK.
 * Synchronises the device. No counterpart in the reference. */
int lw_take_device_error(void);

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
 * of at least lw_gemm_workspace_size() bytes, 256-byte aligned, whose first
 * 64 KiB (per-tile counters) are ZEROED before its first use; every completed
 * call leaves them zeroed again, the rest is scratch. With it, a
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

/* lw_gemm_w4a16 without a caller workspace, for callers that cannot allocate
 * device memory (a runtime whose device memory is all planned at start-up, a
 * plugin host that forbids cudaMalloc after initialisation, code that only
 * receives its inputs and outputs). No counterpart in the reference. Its
 * scratch is a fixed 4 MiB array inside the library, held on every GPU that
 * loads it until exit; problems needing more (lw_gemm_workspace_size) return
 * LW_ERR_WORKSPACE. The first call on a device looks the array up, so make
 * it before any stream capture; the address is cached for the process, so do
 * not call it after cudaDeviceReset. All calls share the array: calls that
 * overlap on the GPU race. */
int lw_gemm_w4a16_noalloc(const void* act, const void* qweight, const void* scales, const void* bias,
                          void* out, int M, int N, int K, int group_size, lw_stream_t stream);

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

/* ---- quantization on the GPU (bit-exact with liteweight/quantize.py:7-27, :65-99) ----
 * weight [N,K] fp16 (weight_fp32 = 0) or fp32 (1); per group of group_size
 * consecutive k: scale = max(absmax / 127 (INT8) or / 7 (INT4), 1e-8) in fp32,
 * code = round-half-even(w / scale) clipped to [-127,127] / [-8,7], scales
 * stored fp16 [N,K/group_size]; INT4 codes packed uint8 [N,K/2], even k in the
 * low nibble. Replaces quantize_int8 / quantize_int4 for device tensors
 * (liteweight/quantize.py:7, :65); weights must be finite. */
int lw_quantize_int8(const void* weight, int weight_fp32, void* qweight, void* scales, int N, int K,
                     int group_size, lw_stream_t stream);
int lw_quantize_int4(const void* weight, int weight_fp32, void* qweight, void* scales, int N, int K,
                     int group_size, lw_stream_t stream);

/* ---- dequantization (bit-exact with liteweight/quantize.py:30-43, :102-128) ----
 * out fp16 [N,K] = fp16((float)code * (float)scale). */
int lw_dequant_w8(const void* qweight, const void* scales, void* out, int N, int K, int group_size,
                  lw_stream_t stream);
int lw_dequant_w4(const void* qweight, const void* scales, void* out, int N, int K, int group_size,
                  lw_stream_t stream);

/* ---- decode step (one new token per sequence) -----------------------------
 * The kernels of one decode step of the HF LlamaForCausalLM that liteweight's
 * generate() drives (liteweight/generate.py:106-124; transformers
 * modeling_llama.py:290-335, which the reference calls through
 * QuantLinear.forward, liteweight/quantlinear.py:54-66). No single
 * counterpart in the reference: there each op is a separate torch/HF call.
 * Every kernel reads the current position from device memory, so a captured
 * CUDA graph of one step replays every step. */

/* How the fused GEMV stages its activation. */
enum {
  LW_PRO_PLAIN = 0,      /* act as given */
  LW_PRO_NORM = 1,       /* RMSNorm(act) * gamma (modeling_llama.py:63-68) */
  LW_PRO_RESID_NORM = 2, /* x_out = act + fp16(psum) (CTA 0 writes it), then RMSNorm */
  LW_PRO_PEER_RESID_NORM = 3  /* as LW_PRO_RESID_NORM with psum = the sum over r = 0..world-1,
                                 in rank order (fp32), of the partials of exchange xin (src =
                                 8-byte words [world][M][K]), each read once its flag is current */
};

/* What the fused GEMV does with each output. */
enum {
  LW_EPI_PLAIN = 0,    /* out = fp16(y) (+bias) (+residual); residual may alias out */
  LW_EPI_ROPE_KV = 1,  /* q|k|v rows (rope-pair order): RoPE q,k; q -> q_out, k,v -> cache at *pos
                          (with prefill_seq: row m is position *pos + m of sequence *prefill_seq) */
  LW_EPI_SWIGLU = 2,   /* gate|up rows interleaved by 8: out[i] = silu(gate_i) * up_i */
  LW_EPI_F32 = 3,      /* out_f32 = y unrounded (tensor-parallel partial sum) */
  LW_EPI_ARGMAX = 4,   /* out = fp16 logits; argmax_keys[m] = max(key) (first max wins) */
  LW_EPI_PEER_F32 = 5, /* y unrounded as flagged words [M][ldo] into xout->dst[d] on every rank d */
  LW_EPI_PEER_ARGMAX = 6  /* as LW_EPI_ARGMAX; the last CTA then sends this rank's keys as flagged
                             words [M] to xout->dst[d] on every rank d */
};

/* ---- tensor-parallel exchange through peer memory --------------------------
 * Replaces the NCCL all-reduce of the o_proj / down_proj partial sums and the
 * all-reduce MAX of the argmax keys of a vocabulary-sharded lm_head (no
 * counterpart in the reference, which runs on one device). An exchange is one
 * all-reduce point of a step. Every rank owns a receive buffer per exchange in
 * device memory from lw_peer_alloc, which the other ranks map with
 * lw_peer_export / lw_peer_import (CUDA IPC over NVLink).
 *
 * Each value travels as one 8-byte word that also carries a flag, so it is
 * either wholly old or wholly new (8-byte stores and loads are single-copy
 * atomic): a partial sum as (flag << 32) | fp32 bits, a key as (flag16 << 48)
 * | 48-bit key. The producer stores its words straight into every rank's
 * buffer; the consumer re-reads each word until its flag is this exchange's
 * flag for this step. No fences, counters or resets are needed.
 *   flag   = s * tags_per_step + tag + 1 (32-bit; 1 if that wraps to 0)
 *   flag16 = flag % 65535 + 1
 * where s = *step, the number of decode steps every rank has completed (the
 * sampler advances it), and tag numbers the exchange within the step.
 * Waits are bounded: after timeout_ns the kernel sets *error =
 * LW_ERR_TIMEOUT and carries on with whatever data is there.
 * Plain peer loads and stores only (no multicast objects). */
#define LW_MAX_RANKS 8

typedef struct {
  int world;            /* ranks taking part, 1..LW_MAX_RANKS */
  int rank;             /* this rank */
  void* dst[LW_MAX_RANKS];  /* rank d's receive buffer (mapped here); this rank's words go at
                               word offset rank * M * ldo (partials) or rank * M (keys) */
  const int* step;      /* device: decode steps completed; the same on every rank */
  int tag, tags_per_step;
  int* arrivals;        /* LW_EPI_PEER_ARGMAX: local int, zero before first use and left zero */
} lw_exchange_out;

typedef struct {
  int world;
  int tag, tags_per_step;
  const void* src;      /* local receive buffer: rank r's words at r * M * K (partials) or r * M (keys) */
  const int* step;
  int* error;           /* device: set to LW_ERR_TIMEOUT when a wait gives up (may be NULL) */
  long long timeout_ns; /* wait limit */
  int* slice_flags;     /* NULL: every CTA of the consuming GEMV sums every rank's partials for the
                           whole K. Else (>= 1024 local ints, zero before first use): CTA b sums
                           slice b of K, writes it to x_out and sets slice_flags[b] to the exchange's
                           flag; every CTA then reads the whole new residual from x_out. Same bits. */
} lw_exchange_in;

typedef struct {
  int bits;          /* 4, 8 (liteweight formats) or 16 (fp16 weight) */
  int prologue;      /* LW_PRO_* */
  int epilogue;      /* LW_EPI_* */
  int pdl;           /* 1: programmatic dependent launch (overlaps the previous kernel) */
  int fold_scales;   /* 0: dequantize exactly (fp16(code * scale), as liteweight does);
                        1: sum codes * act per 4-lane chunk and scale the chunk sum in fp32
                        (skips that fp16 rounding; within the row-scaled tolerance, not bit-identical) */
  int M, N, K, group_size;  /* M <= 32 rows */
  int lda, ldo;
  const void* act;      /* fp16 [M][lda] (the residual stream for the norm prologues) */
  const void* weight;   /* [N][K*bits/8] */
  const void* scales;   /* fp16 [N][K/group_size] (bits 4, 8) */
  const void* bias;     /* fp16 [N] or NULL (LW_EPI_PLAIN) */
  const void* residual; /* fp16 [M][ldo] or NULL (LW_EPI_PLAIN) */
  void* out;            /* fp16 [M][ldo] */
  const void* gamma;    /* fp16 [K] RMSNorm weight */
  const float* psum;    /* fp32 [M][K] (LW_PRO_RESID_NORM) */
  void* x_out;          /* fp16 [M][lda] (LW_PRO_RESID_NORM); must not alias act */
  float eps;
  int head_dim, n_q_heads, n_kv_heads, max_seq;
  int argmax_offset;    /* vocabulary index of weight row 0 (vocab-sharded lm_head) */
  const void* rope_cos; /* fp16 [max_seq][head_dim] */
  const void* rope_sin;
  const int* pos;       /* device position of this step */
  void* q_out;          /* fp16 [M][n_q_heads*head_dim] */
  void* k_cache;        /* fp16 [M][n_kv_heads][max_seq][head_dim] */
  void* v_cache;
  float* out_f32;       /* fp32 [M][ldo] (LW_EPI_F32) */
  unsigned long long* argmax_keys; /* [M], zero before the launch (LW_EPI_ARGMAX) */
  void* workspace;      /* as for lw_gemm_w8a16 */
  size_t workspace_bytes;
  const lw_exchange_in* xin;    /* LW_PRO_PEER_RESID_NORM; read at the call */
  const lw_exchange_out* xout;  /* LW_EPI_PEER_*; read at the call */
  const int* prefill_seq;       /* NULL: decode (row m = sequence m). Else a prompt chunk: the M
                                   rows are positions *pos .. *pos + M - 1 of sequence *prefill_seq */
  int sched_set;                /* reserved (ignored): the ring GEMV's schedule is static */
  int kernel;                   /* 0: the shared-memory ring GEMV when the shape suits it (M <= 8),
                                   else the register-pipeline GEMV; 1: the register-pipeline GEMV */
} lw_fused_gemv_args;

int lw_fused_gemv(const lw_fused_gemv_args* args, lw_stream_t stream);
size_t lw_fused_gemv_workspace_size(const lw_fused_gemv_args* args);

/* GQA attention of one query per sequence over cache positions 0..*pos
 * (modeling_llama.py:197-222 with repeat_kv): scores scaled by
 * head_dim^-0.5, fp32 softmax, fp16 output [batch][n_q_heads*head_dim].
 * head_dim 64 or 128; n_q_heads / n_kv_heads in {1, 2, 4, 8}. Each
 * (sequence, kv head) is one 8-CTA thread-block cluster whose CTAs split the
 * positions and merge through distributed shared memory: no workspace. */
typedef struct {
  const void* q;
  const void* k_cache;   /* fp16 [batch][n_kv_heads][max_seq][head_dim] */
  const void* v_cache;
  void* out;
  const int* pos;
  int batch, n_q_heads, n_kv_heads, head_dim, max_seq, pdl;
  const int* prefill_seq;  /* NULL: query row b is sequence b over positions 0..*pos. Else a prompt
                              chunk of `batch` rows: row b is position *pos + b of sequence
                              *prefill_seq, over positions 0..*pos + b (causal) */
} lw_attention_args;

int lw_attention_decode(const lw_attention_args* args, lw_stream_t stream);

/* sizeof(lw_fused_gemv_args) for which = 0, sizeof(lw_attention_args) for
 * which = 1, sizeof(lw_exchange_out) for 2, sizeof(lw_exchange_in) for 3,
 * sizeof(lw_prefill_gemm_args) for 4, else 0: lets a binding check its
 * struct layouts at load time. */
size_t lw_struct_size(int which);

/* x[b] = embed[tokens[*pos][b]] (tokens int32 [max_seq+1][batch]). */
int lw_embed_tokens(const int* tokens, const void* embed, void* x, const int* pos, int batch, int hidden,
                    int pdl, lw_stream_t stream);

/* Next token per sequence: tokens[*pos+1][b] if it is >= 0 (a prompt token),
 * else the argmax decoded from keys[b], which is then stored there; writes
 * its embedding to x, clears keys and advances *pos by one (done: an int
 * kept zero between calls). generate.py:49-52 (greedy pick).
 * step (may be NULL): advanced by one with *pos; never reset, it numbers the
 * steps for the exchanges. xin (may be NULL): the pick is the maximum of the
 * world ranks' keys of a tensor-parallel exchange (src = flagged words
 * [world][batch]), each read once its flag is current; keys (this rank's
 * lm_head keys) is still cleared. */
int lw_sample_tokens(int* tokens, unsigned long long* keys, const void* embed, void* x, int* pos, int* done,
                     int* step, const lw_exchange_in* xin, int batch, int hidden, int pdl, lw_stream_t stream);

/* ---- chunked prefill: the prompt runs through the decode kernels M
 * positions at a time (one sequence per chunk, rows = positions), so every
 * weight is read once per chunk instead of once per prompt token. A chunk is
 * lw_prefill_embed, the layers' kernels with prefill_seq set, then
 * lw_prefill_advance (not the last chunk) or, for the last chunk, the
 * lm_head GEMV and lw_prefill_sample. No counterpart in the reference, whose
 * generate() runs the prompt through one HF forward call. */

/* x[m] = embed[tokens[(*pos + m) * batch + *seq]] for m < rows. */
int lw_prefill_embed(const int* tokens, const void* embed, void* x, const int* pos, const int* seq, int rows,
                     int batch, int hidden, int pdl, lw_stream_t stream);

/* *pos += rows and, when step != NULL, *step += 1 (after every earlier kernel of the stream). */
int lw_prefill_advance(int* pos, int* step, int rows, int pdl, lw_stream_t stream);

/* The token at position *pos + rows of sequence *seq: tokens[..] if >= 0,
 * else the argmax decoded from keys[rows - 1] (or, with xin, the maximum of
 * the world ranks' flagged keys of row rows - 1), then stored. Its embedding
 * goes to x_out[*seq] (the decode step's residual stream); keys[0..rows) are
 * cleared; *pos += rows; *step += 1 when step != NULL. */
int lw_prefill_sample(int* tokens, unsigned long long* keys, const void* embed, void* x_out, int* pos, int* step,
                      const int* seq, const lw_exchange_in* xin, int rows, int batch, int hidden, int pdl,
                      lw_stream_t stream);

/* ---- prompt-chunk GEMM on the 5th-generation tensor cores ----------------
 * out[m][n] for the M rows of a prompt chunk (M <= 256) and N weight rows
 * (a multiple of 128): D = act[M][K] . dequant(W)[N][K]^T, fp32 sums in
 * tensor memory (tcgen05.mma kind::f16, 128-row weight tiles, K in blocks of
 * 64 through a shared-memory ring fed by TMA), then one epilogue:
 *   LW_TC_EPI_RESID:  out = fp16(fp16(y) + residual)   (residual may alias out)
 *   LW_TC_EPI_SWIGLU: gate|up rows interleaved by 8, out[m][i] = silu(gate) * up
 *   LW_TC_EPI_ROPE_KV: q|k|v rows in rope-pair order; RoPE q, k at position
 *                      *pos + m; q -> q_out, k, v -> the cache of sequence *seq
 *                      (seq NULL: decode rows, row m is sequence m at *pos)
 *   LW_TC_EPI_F32:    out is fp32 [M][ldo], out = y (a tensor-parallel rank's
 *                      partial sum of a row-split linear, to be all-reduced)
 *   LW_TC_EPI_ARGMAX: out = fp16 logits; argmax_keys[m] = atomic max of
 *                      (order key of the fp16 logit) << 32 | ~(n + argmax_offset)
 *                      over the N rows (the keys lw_fused_gemv's argmax writes;
 *                      zero before, as the sampler leaves them). The only
 *                      epilogue that also takes fp16 weights (bits 16, scales NULL:
 *                      the lm_head of a large decode batch)
 * Weights dequantize exactly (fp16(code * scale)) as the GEMV does; the sums
 * differ from it only in order. K a multiple of 64, INT4 or INT8, group size a
 * power of two >= 32 dividing K. No counterpart in the reference (its prompt
 * runs through one HF forward over QuantLinear's dequantize + matmul). */
enum { LW_TC_EPI_RESID = 0, LW_TC_EPI_SWIGLU = 1, LW_TC_EPI_ROPE_KV = 2, LW_TC_EPI_F32 = 3, LW_TC_EPI_ARGMAX = 4 };

typedef struct {
  int bits, epilogue, pdl;
  int M, N, K, group_size;
  int lda, ldo;
  const void* act;       /* fp16 [M][lda] */
  const void* weight;    /* [N][K * bits / 8] */
  const void* scales;    /* fp16 [N][K / group_size] */
  void* out;             /* fp16 [M][ldo] (fp32 for LW_TC_EPI_F32) */
  const void* residual;  /* fp16 [M][ldo] (LW_TC_EPI_RESID; may be NULL) */
  int head_dim, n_q_heads, n_kv_heads, max_seq;
  const void* rope_cos;  /* fp16 [max_seq][head_dim] */
  const void* rope_sin;
  const int* pos;
  const int* seq;        /* NULL: decode rows (row m = sequence m at *pos) */
  void* q_out;           /* fp16 [M][n_q_heads * head_dim] */
  void* k_cache;         /* fp16 [batch][n_kv_heads][max_seq][head_dim] */
  void* v_cache;
  unsigned long long* argmax_keys;   /* LW_TC_EPI_ARGMAX: [M] */
  int argmax_offset;                 /* LW_TC_EPI_ARGMAX: global index of weight row 0 */
} lw_prefill_gemm_args;

int lw_prefill_gemm(const lw_prefill_gemm_args* args, lw_stream_t stream);

/* h[m] = RMSNorm(x[m]) * gamma for m < M (modeling_llama.py:63-68 rounding points). */
int lw_rmsnorm_rows(const void* x, const void* gamma, void* h, int M, int K, float eps, int pdl,
                    lw_stream_t stream);

/* x[m] = fp16(x[m] + fp16(psum[m])) in place (psum fp32 [M][K], the all-reduced
 * partial sums of a row-split linear), then h[m] = RMSNorm(x[m]) * gamma: the
 * residual add and norm between the linears of a tensor-parallel prompt chunk,
 * at the rounding points of the GEMV prologue LW_PRO_RESID_NORM
 * (modeling_llama.py:63-68 and the residual add of :290-335). */
int lw_resid_rmsnorm_rows(void* x, const float* psum, const void* gamma, void* h, int M, int K, float eps, int pdl,
                          lw_stream_t stream);

/* ---- peer memory for the exchanges (setup calls: these allocate, map and
 * synchronise; they are not stream-ordered and must not be graph-captured) */

/* cudaMalloc'd, zeroed device memory that other processes can map. */
int lw_peer_alloc(size_t bytes, void** ptr);
int lw_peer_free(void* ptr);
/* Bytes of the opaque handle lw_peer_export writes (a cudaIpcMemHandle_t). */
size_t lw_peer_handle_size(void);
int lw_peer_export(void* ptr, void* handle);
/* Map another process's lw_peer_alloc block on this process's current device. */
int lw_peer_import(const void* handle, void** ptr);
int lw_peer_close(void* ptr);

#ifdef __cplusplus
}
#endif

#endif /* LITEWEIGHT_B200_H */
