// Prompt-chunk GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// out[m][n] for the M rows of a prompt chunk: D[n][m] = sum_k W[n][k] * X[m][k]
// with W the liteweight-packed weight, dequantized exactly (fp16(code * scale),
// liteweight/quantize.py:30-43, :102-128), and X the fp16 activation.
//
// One CTA (or one cluster of `splits` CTAs, each a slice of K) per 128-row
// weight tile. K is cut into blocks of 64; each block is one stage of an
// S-stage ring (S <= 8, as many as fit) holding in shared memory
//   B operand          Mpad activation rows x 64 fp16 (TMA, 128-byte swizzle:
//                      16-byte chunk c of row r at chunk c ^ (r & 7), rows 128
//                      bytes apart, 8-row groups 1024 bytes apart; K-major)
//   raw weight codes   128 rows x 32 / 64 bytes (TMA, no swizzle)
// and in tensor memory the A operand, 128 weight rows (lanes) x 64 fp16 (32
// columns), written by the dequantizing threads with tcgen05.st: the MMA
// reads A from tensor memory ("TS" form), so shared memory carries only the
// copies in, the codes out and B into the tensor core (a 128 x 128 x 64
// stage moves ~40 KB through it instead of ~72 KB with A staged there, which
// bounded the stage rate at the shared-memory bandwidth). The CTA's eighteen
// warps are specialised:
//   warp 16  one lane issues the two TMA tile copies of each stage (weights
//            first, before griddepcontrol.wait: they do not depend on the
//            previous kernel) once the tensor core has released the stage;
//   warps 0-15 unpack the stage's raw codes, scale them (fp16 hmul, the
//            reference's rounding) and store the A operand to tensor memory:
//            four groups of four warps (one weight row per thread, the warp's
//            own 32 lanes) take the stages in turn;
//   warp 17  owns the tensor memory; one lane issues four tcgen05.mma
//            (K = 16 each) per stage into the fp32 accumulator (128 lanes =
//            tile rows, columns [0, Mpad) = activation rows) and commits the
//            stage back to the producer.
// After the last stage, warps 0-15 read the accumulator with tcgen05.ld. With
// one CTA per tile they apply the epilogue directly; with a cluster, every CTA
// writes its partial tile to its own shared memory, and CTA c sums column
// slice c of all partials over distributed shared memory in rank order (the
// same sums on every run) and applies the epilogue to it. Epilogues: residual
// add / SwiGLU / RoPE + KV-cache append, at the GEMV kernels' rounding points.
//
// Every mbarrier wait is bounded (global timer): on expiry the kernel records
// LW_ERR_TIMEOUT, the other roles stop at their next wait, the producer waits
// (bounded) for the copies it issued, and the tensor memory is released; the
// results of that launch are then invalid.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "gemv_host.cuh"
#include "tma_host.cuh"

namespace lw {

constexpr int kTcDeqWarps = 16;      // warps 0-15: dequantize, then the epilogue
constexpr int kTcDeqThreads = kTcDeqWarps * 32;
constexpr int kTcDeqGroups = kTcDeqWarps / 4;     // a group of 128 threads converts a whole block
constexpr int kTcProducerWarp = kTcDeqWarps;       // TMA producer
constexpr int kTcMmaWarp = kTcDeqWarps + 1;        // MMA issuer, tensor-memory owner
constexpr int kTcThreads = kTcDeqThreads + 64;
constexpr int kTcMaxStages = 8;
constexpr int kTcTileN = 128;        // weight rows per CTA (UMMA M)
constexpr int kTcKBlock = 64;        // K per stage (one 128-byte swizzle row of fp16)
constexpr int kTcMaxM = 256;         // activation rows (UMMA N)
constexpr int kTcMaxSplits = 4;
constexpr size_t kTcSmemMax = 225 * 1024;
constexpr long long kTcWaitNs = 500000000;

struct TcGemmParams {
  CUtensorMap tm_w;   // weights: [N rows][K * BITS / 8 bytes] u8, box {block bytes, 128}
  CUtensorMap tm_x;   // activations: [M rows][K] fp16 (row stride lda), box {64, Mpad}, 128-byte swizzle
  const __half* scales;
  __half* out;
  const __half* residual;
  const __half* bias;   // LW_TC_EPI_RESID: fp16 [N] added to the fp16 result (QuantLinear's bias), or null
  int ldo;
  int M, Mpad, N, K, G, gshift, kblocks;
  int splits, kb_per, stages;
  uint32_t stage_bytes, b_bytes, w_bytes;
  uint32_t idesc;
  int tmem_cols;
  int acc_cols;       // accumulator columns [0, acc_cols); A operand of ring slot s at acc_cols + 32 s
  // rope / kv
  const __half* rope_cos;
  const __half* rope_sin;
  const int* pos;
  const int* seq;      // prompt chunk: row m = position *pos + m of sequence *seq; null: row m = sequence m
  int head_dim, n_q_heads, n_kv_heads, max_seq;
  __half* q_out;
  __half* k_cache;
  __half* v_cache;
  // argmax (LW_TC_EPI_ARGMAX)
  unsigned long long* keys;   // [M]: max over the rows n of (order key of fp16 y) << 32 | ~(n + argmax_offset)
  int argmax_offset;
};

// ---- tcgen05 / mbarrier helpers (PTX ISA 8.7, sm_100a)

LW_DEV void tmem_alloc(uint32_t dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(cols)
               : "memory");
}
LW_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
LW_DEV void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
LW_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
LW_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LW_DEV void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D (tensor memory) += A (tensor memory, 128 lanes x 16 fp16 in 8 columns) x B (shared memory).
LW_DEV void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 registers per thread -> 32 consecutive columns of this warp's 32 lanes.
LW_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
LW_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
LW_DEV void tc_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar) : "memory");
}
LW_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// 32 lanes x 32 consecutive fp32 columns of tensor memory -> 32 registers per thread.
LW_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
LW_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled operand
// whose 8-row groups are 1024 bytes apart (start address and offsets in
// 16-byte units; descriptor version 1; layout type 2 = 128-byte swizzle).
LW_DEV uint64_t sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;                    // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;          // stride byte offset: next 8-row group
  d |= (uint64_t)1u << 46;                    // version
  d |= (uint64_t)2u << 61;                    // 128-byte swizzle
  return d;
}


// 8 codes of one 32-bit word -> 8 fp16 in natural k order, each fp16(code * scale).
template <int BITS>
LW_DEV uint4 dequant8(uint32_t lo, uint32_t hi, uint32_t s2) {
  uint4 o;
  if constexpr (BITS == 4) {
    uint32_t A[4];
    unpack_int4_word(lo, A);   // pairs (0,4) (1,5) (2,6) (3,7)
#pragma unroll
    for (int i = 0; i < 4; ++i) A[i] = hmul2_rn(A[i], s2);
    o.x = __byte_perm(A[0], A[1], 0x5410);   // (0,1)
    o.y = __byte_perm(A[2], A[3], 0x5410);   // (2,3)
    o.z = __byte_perm(A[0], A[1], 0x7632);   // (4,5)
    o.w = __byte_perm(A[2], A[3], 0x7632);   // (6,7)
  } else {
    uint32_t a[2], b[2];
    dequant_int8_word(lo, a);   // (0,1) (2,3)
    dequant_int8_word(hi, b);   // (4,5) (6,7)
    o.x = hmul2_rn(a[0], s2);
    o.y = hmul2_rn(a[1], s2);
    o.z = hmul2_rn(b[0], s2);
    o.w = hmul2_rn(b[1], s2);
  }
  return o;
}

LW_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// One lane of the (fully active) warp returns true.
LW_DEV bool elect_one_sync() {
  uint32_t elected;
  asm volatile(
      "{\n"
      " .reg .pred P;\n"
      " elect.sync _|P, 0xffffffff;\n"
      " selp.u32 %0, 1, 0, P;\n"
      "}\n"
      : "=r"(elected));
  return elected != 0;
}
LW_DEV void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Epilogue of one accumulator value: tile row n (lane `lane` of its warp),
// activation row m. Every lane of the warp calls it for the same m.
template <int EPI>
LW_DEV void tc_epilogue(const TcGemmParams& p, int n, int m, float y, int lane) {
  if constexpr (EPI == LW_TC_EPI_F32) {
    if (m < p.M && n < p.N) reinterpret_cast<float*>(p.out)[(size_t)m * p.ldo + n] = y;
  } else if constexpr (EPI == LW_TC_EPI_RESID) {
    if (m >= p.M || n >= p.N) return;
    y = r16(y);
    if (p.bias) y = r16(y + __half2float(p.bias[n]));
    if (p.residual) y = r16(__half2float(p.residual[(size_t)m * p.ldo + n]) + y);
    p.out[(size_t)m * p.ldo + n] = __float2half_rn(y);
  } else if constexpr (EPI == LW_TC_EPI_ARGMAX) {
    // logits and the first index of their maximum (the GEMV argmax's keys):
    // the warp's 32 rows reduce to one key per row m, then one atomic
    unsigned long long key = 0ull;
    if (m < p.M && n < p.N) {
      const __half h = __float2half_rn(y);
      p.out[(size_t)m * p.ldo + n] = h;
      key = ((unsigned long long)f16_order_key(h) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)(n + p.argmax_offset));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
      key = other > key ? other : key;
    }
    if (lane == 0 && key) atomicMax(p.keys + m, key);
  } else {
    // rows g and g + 8 of every 16-row tile are partners (gate/up, or the
    // rotate_half pair): the lower lane of each pair finishes both
    const float partner = __shfl_down_sync(0xffffffffu, y, 8);
    const bool lower = (lane & 15) < 8;
    if (!lower || m >= p.M || n >= p.N) return;
    const int t16 = n >> 4, g = n & 7;
    if constexpr (EPI == LW_TC_EPI_SWIGLU) {
      const float gt = r16(y), up = r16(partner);
      const float a = r16(silu_f32(gt));
      p.out[(size_t)m * p.ldo + t16 * 8 + g] = __float2half_rn(a * up);
    } else {
      const int hd = p.head_dim, nq = p.n_q_heads, nkv = p.n_kv_heads;
      const int head = (t16 * 16) / hd, jt = t16 % (hd / 16);
      const int d_lo = 8 * jt + g, d_hi = d_lo + hd / 2;
      // a prompt chunk: row m is position *pos + m of sequence *seq; decode
      // rows (seq null): row m is sequence m at position *pos
      const int pos = p.seq ? *p.pos + m : *p.pos, row = p.seq ? *p.seq : m;
      const float y_lo = r16(y), y_hi = r16(partner);
      float o_lo = y_lo, o_hi = y_hi;
      if (head < nq + nkv) {
        const float c_lo = __half2float(p.rope_cos[(size_t)pos * hd + d_lo]);
        const float c_hi = __half2float(p.rope_cos[(size_t)pos * hd + d_hi]);
        const float s_lo = __half2float(p.rope_sin[(size_t)pos * hd + d_lo]);
        const float s_hi = __half2float(p.rope_sin[(size_t)pos * hd + d_hi]);
        o_lo = r16(r16(y_lo * c_lo) + r16(-y_hi * s_lo));
        o_hi = r16(r16(y_hi * c_hi) + r16(y_lo * s_hi));
      }
      __half* dst;
      if (head < nq) dst = p.q_out + (size_t)m * nq * hd + (size_t)head * hd;
      else if (head < nq + nkv) dst = p.k_cache + (((size_t)row * nkv + (head - nq)) * p.max_seq + pos) * hd;
      else dst = p.v_cache + (((size_t)row * nkv + (head - nq - nkv)) * p.max_seq + pos) * hd;
      dst[d_lo] = __float2half_rn(o_lo);
      dst[d_hi] = __float2half_rn(o_hi);
    }
  }
}

template <int BITS, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const __grid_constant__ TcGemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) unsigned long long bar_raw[kTcMaxStages], bar_a[kTcMaxStages], bar_empty[kTcMaxStages];
  __shared__ __align__(8) unsigned long long bar_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = (int)(blockIdx.x % (unsigned)p.splits), tile = (int)(blockIdx.x / (unsigned)p.splits);
  const int n0 = tile * kTcTileN;
  const int kb0 = split * p.kb_per, nkb = max(0, min(p.kblocks, kb0 + p.kb_per) - kb0);
  const int S = p.stages;
  // stages on 1024-byte boundaries (the swizzle pattern follows address bits 4-9):
  // B operand at +0, raw weight codes after it
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - smem_u32(smem_raw));

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&bar_raw[s]), 1);
      mbar_init(smem_u32(&bar_a[s]), kTcDeqThreads / kTcDeqGroups);
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    mbar_init(smem_u32(&bar_done), 1);
    abort_s = 0;
    fence_mbar_init();
  }
  if (warp == kTcMmaWarp) {
    tmem_alloc(smem_u32(&tmem_base_s), (uint32_t)p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  // Bounded wait shared by the roles: the first to give up makes the others
  // stop at their next wait.
  auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_s) return false;
    if (mbar_wait_bounded(bar, parity, kTcWaitNs)) return true;
    abort_s = 1;
    return false;
  };

  // The producer and MMA roles run as whole warps: their loop state and the
  // operand descriptors stay warp-uniform (uniform registers), and one elected
  // lane issues each TMA copy / tcgen05 instruction.
  // Every lane of the warp polls (measured faster than one polling lane
  // followed by a shuffle); lane 0's answer is the warp's.
  auto warp_wait = [&](uint32_t bar, uint32_t parity) -> bool {
    return __shfl_sync(0xffffffffu, wait(bar, parity) ? 1u : 0u, 0) != 0;
  };

  if (warp == kTcProducerWarp) {
    // ---- TMA producer
    const bool leader = elect_one_sync();
    if (leader) {
      tma_prefetch_map(&p.tm_w);
      tma_prefetch_map(&p.tm_x);
    }
    const int first = min(S, nkb);
    const int wx = kTcKBlock * BITS / 8;   // weight bytes per row per block
    for (int i = 0; i < first; ++i) {
      const uint32_t st = base + i * p.stage_bytes, bar = smem_u32(&bar_raw[i]);
      if (leader) {
        mbar_arrive_expect_tx(bar, p.w_bytes + p.b_bytes);
        tma_load_2d(st + p.b_bytes, &p.tm_w, (kb0 + i) * wx, n0, bar);
      }
    }
    pdl_wait();   // activations come from the previous kernel
    pdl_launch_dependents();
    for (int i = 0; i < first; ++i)
      if (leader)
        tma_load_2d(base + i * p.stage_bytes, &p.tm_x, (kb0 + i) * kTcKBlock, 0, smem_u32(&bar_raw[i]));
    __syncwarp();
    int issued = first;
    uint32_t phase = 0;   // parity of the empty-barrier phase awaited in the current pass over the ring
    for (int i = first, s = 0; i < nkb; ++i) {
      if (!warp_wait(smem_u32(&bar_empty[s]), phase)) break;
      const uint32_t st = base + s * p.stage_bytes, bar = smem_u32(&bar_raw[s]);
      if (leader) {
        mbar_arrive_expect_tx(bar, p.w_bytes + p.b_bytes);
        tma_load_2d(st + p.b_bytes, &p.tm_w, (kb0 + i) * wx, n0, bar);
        tma_load_2d(st, &p.tm_x, (kb0 + i) * kTcKBlock, 0, bar);
      }
      __syncwarp();
      issued = i + 1;
      if (++s == S) {
        s = 0;
        phase ^= 1u;
      }
    }
    // no copy may land after the CTA has exited: wait (bounded) for the last
    // one issued into every stage (immediate unless a wait gave up)
    if (leader) {
      for (int s = 0; s < min(S, issued); ++s) {
        const int last = (issued - 1 - s) / S;   // use index of stage s's last copy
        mbar_wait_bounded(smem_u32(&bar_raw[s]), last & 1, kTcWaitNs);
      }
    }
  } else if (warp == kTcMmaWarp) {
    // ---- MMA issuer: B descriptor of stage 0, advanced by the stage offset and
    // by 32 bytes (2 in 16-byte units) per K = 16 step; A in tensor memory,
    // 8 columns per K = 16 step
    const uint64_t db0 = sw128_desc(base);
    uint32_t phase = 0;
    for (int i = 0, s = 0; i < nkb; ++i) {
      if (!warp_wait(smem_u32(&bar_a[s]), phase)) break;
      tc_fence_after();
      const uint64_t off = (uint64_t)(((uint32_t)s * p.stage_bytes) >> 4);
      if (elect_one_sync()) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc_mma_f16_ts(tmem, tmem + (uint32_t)(p.acc_cols + 32 * s + 8 * j), db0 + off + 2 * j, p.idesc,
                        (i | j) != 0);
        tc_commit(smem_u32(&bar_empty[s]));
      }
      __syncwarp();
      if (++s == S) {
        s = 0;
        phase ^= 1u;
      }
    }
    if (elect_one_sync()) tc_commit(smem_u32(&bar_done));   // arrives once every MMA issued above has completed
    __syncwarp();
  } else {
    // ---- dequantize: group dg (4 warps) converts blocks dg, dg + 4, ... of
    // this CTA; thread ar of the group owns weight row ar (64 codes)
    const int dg = tid >> 7, ar = tid & 127;
    const int ngroups = p.K / p.G;
    const unsigned short* ssrc =
        BITS < 16 ? reinterpret_cast<const unsigned short*>(p.scales) + (size_t)min(n0 + ar, p.N - 1) * ngroups
                  : nullptr;
    auto scales_of = [&](int kb, unsigned short& s0, unsigned short& s1) {
      if constexpr (BITS < 16) {
        s0 = __ldg(ssrc + min((kb * kTcKBlock) >> p.gshift, ngroups - 1));
        s1 = __ldg(ssrc + min((kb * kTcKBlock + 32) >> p.gshift, ngroups - 1));
      }
    };
    const uint32_t raw_off = p.b_bytes + (uint32_t)ar * (uint32_t)(kTcKBlock * BITS / 8);
    // this warp's 32 lanes of tensor memory (a warp reaches lanes 32 (warp % 4) ..)
    const uint32_t a_taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)p.acc_cols;
    int i = dg, s = dg;   // block index within this CTA's K slice, its ring slot (S >= kTcDeqGroups)
    uint32_t phase = 0;
    unsigned short n0s = 0, n1s = 0;
    if (i < nkb) scales_of(kb0 + i, n0s, n1s);
    for (; i < nkb; i += kTcDeqGroups) {
      const uint32_t s2a = (uint32_t)n0s | ((uint32_t)n0s << 16), s2b = (uint32_t)n1s | ((uint32_t)n1s << 16);
      if (i + kTcDeqGroups < nkb) scales_of(kb0 + i + kTcDeqGroups, n0s, n1s);
      if (!warp_wait(smem_u32(&bar_raw[s]), phase)) break;
      tc_fence_after();   // the MMAs that read this slot's A columns before have completed
      uint8_t* st = base_ptr + (size_t)s * p.stage_bytes;
      uint4 o[8];
      if constexpr (BITS == 16) {
        // fp16 weights as they are: row ar's eight 16-byte chunks, stored
        // 128-byte swizzled (chunk j of row r at j ^ (r % 8)) so that the 32
        // rows of a warp spread over the banks
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = lds128(st + raw_off + (uint32_t)((j ^ (ar & 7)) << 4));
      } else if constexpr (BITS == 4) {
        const uint4 q0 = lds128(st + raw_off), q1 = lds128(st + raw_off + 16);
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = dequant8<4>(qw[j], 0u, j < 4 ? s2a : s2b);
      } else {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const uint4 q = lds128(st + raw_off + 16 * h);
          o[2 * h] = dequant8<8>(q.x, q.y, h < 2 ? s2a : s2b);
          o[2 * h + 1] = dequant8<8>(q.z, q.w, h < 2 ? s2a : s2b);
        }
      }
      // row ar of the A operand: 64 fp16 (natural k order) in 32 columns of lane ar
      uint32_t r[32];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        r[4 * j] = o[j].x;
        r[4 * j + 1] = o[j].y;
        r[4 * j + 2] = o[j].z;
        r[4 * j + 3] = o[j].w;
      }
      tmem_st32(a_taddr + (uint32_t)(32 * s), r);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&bar_a[s]));
      s += kTcDeqGroups;
      if (s >= S) {
        s -= S;
        phase ^= 1u;
      }
    }
  }
  __syncwarp();   // the producer and MMA warps reconverge with their single working lane

  // ---- epilogue (warps 0-15): warp w reads lanes 32*(w%4).. (tile rows) and
  // every fourth 32-column chunk (starting at 32*(w/4)); a chunk starts below
  // Mpad and the allocation is a power of two >= 32 and >= Mpad, so every read
  // is inside it
  constexpr int kChunkWarps = kTcDeqWarps / 4;
  const int lg = warp & 3, ch = warp >> 2;
  const int r = lg * 32 + lane;   // tile row
  const int n = n0 + r;
  // partial-tile row stride (floats): whole 32-column chunks are stored, +1
  // so that the 32 lanes (rows) of a warp hit distinct banks
  const int RS = ((p.Mpad + 31) & ~31) + 1;
  float* red = reinterpret_cast<float*>(base_ptr);
  if (warp < kTcDeqWarps) {
    pdl_wait();   // the residual input comes from a previous kernel
    uint32_t done = 1;
    if (lane == 0) {
      done = mbar_wait_bounded(smem_u32(&bar_done), 0, kTcWaitNs) ? 1u : 0u;
      if (!done) abort_s = 1;   // this CTA's partial tile will be missing: the cluster must know
    }
    const bool ok = __shfl_sync(0xffffffffu, done, 0) && !abort_s;
    tc_fence_after();
    if (ok) {
      for (int c0 = ch * 32; c0 < p.Mpad; c0 += 32 * kChunkWarps) {
        uint32_t v[32];
        __syncwarp();   // tcgen05.ld is warp-collective (.sync.aligned)
        tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)c0, v);
        tmem_wait_ld();
        if (p.splits == 1) {
#pragma unroll
          for (int j = 0; j < 32; ++j) tc_epilogue<EPI>(p, n, c0 + j, __uint_as_float(v[j]), lane);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) red[r * RS + c0 + j] = __uint_as_float(v[j]);
        }
      }
    }
  }
  if (p.splits > 1) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();   // every partial tile (and every CTA's abort flag) is in its CTA's shared memory
    // A CTA that gave up on a wait left its partial tile unwritten: if any
    // did, no CTA combines (the error flag is set; the outputs keep their
    // previous contents instead of sums built from stale shared memory).
    bool any_abort = false;
    for (int q = 0; q < p.splits; ++q)
      any_abort |= *static_cast<volatile int*>(cluster.map_shared_rank(const_cast<int*>(&abort_s), q)) != 0;
    if (warp < kTcDeqWarps && !any_abort) {
      const int cw = p.Mpad / p.splits, m0 = split * cw;
      for (int j = ch; j < cw; j += kChunkWarps) {
        float y = 0.f;
        for (int q = 0; q < p.splits; ++q) y += cluster.map_shared_rank(red, q)[r * RS + m0 + j];
        tc_epilogue<EPI>(p, n, m0 + j, y, lane);
      }
    }
    cluster.sync();   // no CTA leaves while its partial tile is still being read
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTcMmaWarp) tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
}

// h[m] = fp16(gamma * fp16(x * rstd)), rstd = 1 / sqrt(mean(x^2) + eps) in fp32.
// With psum, x[m] first becomes fp16(x + fp16(psum)) (written back; the
// second pass reads the new values, which this block wrote before its barrier).
__global__ void rmsnorm_rows_kernel(__half* x, const float* __restrict__ psum, const __half* __restrict__ gamma,
                                    __half* __restrict__ h, int K, float eps) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float part[32];
  const int m = blockIdx.x;
  __half* xr = x + (size_t)m * K;
  float sq = 0.f;
  for (int i = threadIdx.x * 8; i < K; i += blockDim.x * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(xr + i);
    if (psum) {
      const float4 a = *reinterpret_cast<const float4*>(psum + (size_t)m * K + i);
      const float4 b = *reinterpret_cast<const float4*>(psum + (size_t)m * K + i + 4);
      const float ps[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      __half* hv = reinterpret_cast<__half*>(&v);
#pragma unroll
      for (int e = 0; e < 8; ++e) hv[e] = __float2half_rn(__half2float(hv[e]) + r16(ps[e]));
      *reinterpret_cast<uint4*>(xr + i) = v;
    }
    const __half* hv = reinterpret_cast<const __half*>(&v);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float f = __half2float(hv[e]);
      sq = fmaf(f, f, sq);
    }
  }
  sq = warp_sum(sq);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) part[0] = t;
  }
  __syncthreads();
  const float rstd = 1.0f / sqrtf(part[0] / (float)K + eps);
  for (int i = threadIdx.x * 8; i < K; i += blockDim.x * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(xr + i);
    const uint4 gm = ldg_nc(gamma + i);
    __half* hv = reinterpret_cast<__half*>(&v);
    const __half* hg = reinterpret_cast<const __half*>(&gm);
#pragma unroll
    for (int e = 0; e < 8; ++e) hv[e] = __float2half_rn(__half2float(hg[e]) * r16(__half2float(hv[e]) * rstd));
    *reinterpret_cast<uint4*>(h + (size_t)m * K + i) = v;
  }
}

}  // namespace lw

namespace {

inline bool al(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// UMMA instruction descriptor: fp16 A and B, fp32 D, both K-major, M = 128, N = mpad.
uint32_t tc_idesc(int mpad) {
  uint32_t d = 0;
  d |= 1u << 4;                              // D format fp32
  d |= 0u << 7;                              // A fp16
  d |= 0u << 10;                             // B fp16
  d |= (uint32_t)(mpad >> 3) << 17;          // N
  d |= (uint32_t)(lw::kTcTileN >> 4) << 24;  // M
  return d;
}

using lw::encode_2d;

int sm_count() {
  static int counts[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!counts[dev] && cudaDeviceGetAttribute(&counts[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    counts[dev] = 148;
  return counts[dev];
}

template <int BITS, int EPI>
cudaError_t tc_launch(const lw::TcGemmParams& p, size_t smem, cudaStream_t s, bool pdl) {
  auto kern = lw::gemm_tc_kernel<BITS, EPI>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  lw_count_launch();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N / lw::kTcTileN) * p.splits);
  cfg.blockDim = dim3(lw::kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (p.splits > 1) {   // the CTAs of one tile (its K slices) form a cluster
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)p.splits;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace

int lw_gemm_tc_take_error() { return lw_tu_take_error(); }

extern "C" {

namespace {
int prefill_gemm(const lw_prefill_gemm_args* a, const void* bias, lw_stream_t stream);
}

int lw_prefill_gemm(const lw_prefill_gemm_args* a, lw_stream_t stream) { return prefill_gemm(a, nullptr, stream); }

}  // extern "C"

// out[M, N] = act[M, K] @ dequant(W)^T (+ bias), the drop-in matmul past the
// GEMV crossover: lw_prefill_gemm's plain epilogue in row blocks of up to
// kTcMaxM rows. The caller has checked the shape (N % 128, K % 64, a group
// size of >= 32 that is a power of two or K, 16-byte aligned act and weight).
int lw_tc_matmul(int bits, const void* act, const void* w, const void* scales, const void* bias, void* out, int M,
                 int N, int K, int G, cudaStream_t s) {
  for (int m0 = 0; m0 < M; m0 += lw::kTcMaxM) {
    lw_prefill_gemm_args a = {};
    a.bits = bits;
    a.epilogue = LW_TC_EPI_RESID;
    a.M = std::min(lw::kTcMaxM, M - m0);
    a.N = N;
    a.K = K;
    a.group_size = G;
    a.lda = K;
    a.ldo = N;
    a.act = static_cast<const __half*>(act) + (size_t)m0 * K;
    a.weight = w;
    a.scales = scales;
    a.out = static_cast<__half*>(out) + (size_t)m0 * N;
    const int st = prefill_gemm(&a, bias, reinterpret_cast<lw_stream_t>(s));
    if (st) return st;
  }
  return LW_OK;
}

extern "C" {
namespace {
int prefill_gemm(const lw_prefill_gemm_args* a, const void* bias, lw_stream_t stream) {
  if (!a || !a->act || !a->weight || !a->out) return LW_ERR_NULL_POINTER;
  if (a->bits != 4 && a->bits != 8 && a->bits != 16) return LW_ERR_UNSUPPORTED;
  if (a->bits != 16 && !a->scales) return LW_ERR_NULL_POINTER;
  if (a->bits == 16 && a->epilogue != LW_TC_EPI_ARGMAX) return LW_ERR_UNSUPPORTED;   // fp16 weights: the lm_head
  if (a->M <= 0 || a->M > lw::kTcMaxM || a->N <= 0 || a->N % lw::kTcTileN || a->K <= 0 || a->K % lw::kTcKBlock)
    return LW_ERR_BAD_SHAPE;
  const int group = a->bits == 16 ? a->K : a->group_size;
  if (group < 32 || a->K % group || lw::group_shift(a->K, group) < 0) return LW_ERR_BAD_GROUP;
  if (a->lda < a->K || a->lda % 8 || a->ldo % 8) return LW_ERR_BAD_SHAPE;
  if (!al(a->act, 16) || !al(a->weight, 16) || !al(a->out, 2)) return LW_ERR_ALIGNMENT;
  switch (a->epilogue) {
    case LW_TC_EPI_RESID:
      if (a->ldo < a->N) return LW_ERR_BAD_SHAPE;
      break;
    case LW_TC_EPI_SWIGLU:
      if (a->ldo < a->N / 2) return LW_ERR_BAD_SHAPE;
      break;
    case LW_TC_EPI_F32:
      if (a->ldo < a->N || !al(a->out, 16)) return LW_ERR_BAD_SHAPE;
      break;
    case LW_TC_EPI_ROPE_KV:
      if (!a->q_out || !a->k_cache || !a->v_cache || !a->rope_cos || !a->rope_sin || !a->pos)
        return LW_ERR_NULL_POINTER;
      if (a->head_dim % 16 || a->N != (a->n_q_heads + 2 * a->n_kv_heads) * a->head_dim) return LW_ERR_BAD_SHAPE;
      break;
    case LW_TC_EPI_ARGMAX:
      if (!a->argmax_keys) return LW_ERR_NULL_POINTER;
      if (a->ldo < a->N || !al(a->argmax_keys, 8)) return LW_ERR_BAD_SHAPE;
      break;
    default:
      return LW_ERR_UNSUPPORTED;
  }
  lw::TcGemmParams p = {};
  p.scales = static_cast<const __half*>(a->scales);
  p.out = static_cast<__half*>(a->out);
  p.residual = static_cast<const __half*>(a->residual);
  p.bias = static_cast<const __half*>(bias);
  p.ldo = a->ldo;
  p.M = a->M;
  p.Mpad = (a->M + 15) / 16 * 16;
  p.N = a->N;
  p.K = a->K;
  p.G = group;
  p.gshift = lw::group_shift(a->K, group);
  p.kblocks = a->K / lw::kTcKBlock;
  p.idesc = tc_idesc(p.Mpad);
  int acc = 32;
  while (acc < p.Mpad) acc <<= 1;
  p.acc_cols = acc;
  p.rope_cos = static_cast<const __half*>(a->rope_cos);
  p.rope_sin = static_cast<const __half*>(a->rope_sin);
  p.pos = a->pos;
  p.seq = a->seq;
  p.head_dim = a->head_dim;
  p.n_q_heads = a->n_q_heads;
  p.n_kv_heads = a->n_kv_heads;
  p.max_seq = a->max_seq;
  p.q_out = static_cast<__half*>(a->q_out);
  p.k_cache = static_cast<__half*>(a->k_cache);
  p.v_cache = static_cast<__half*>(a->v_cache);
  p.keys = static_cast<unsigned long long*>(a->argmax_keys);
  p.argmax_offset = a->argmax_offset;

  // K slices per tile. The cluster combine of the partial tiles grows with the
  // rows: up to 64 rows, slices (up to 4) while the tiles alone leave at least
  // half the SMs idle and every slice keeps >= 8 blocks of 64; past 64 rows, two
  // slices for long rows (>= 128 blocks) only. Measured (INT4, 8B shapes, us):
  // at 32 / 64 rows q|k|v 17.6 / 21.1 in 2 slices vs 29.7 / 31.0 whole; at 256
  // rows q|k|v (48 tiles, 64 blocks) 30.0 whole vs 43.5 in 2 slices, o (32
  // tiles) 29.6 vs 42.1 / 57.1 in 2 / 4, down (224 blocks) 76.2 vs 66.7 in 2.
  const int tiles = p.N / lw::kTcTileN;
  int splits = 1;
  if (p.Mpad <= 64) {
    while (splits < lw::kTcMaxSplits && tiles * splits * 2 <= sm_count() && p.kblocks >= splits * 2 * 8) splits *= 2;
  } else if (p.kblocks >= 128 && tiles * 2 <= sm_count()) {
    splits = 2;
  }
  if (const char* e = getenv("LW_B200_TC_SPLITS")) {   // a fixed split (1, 2 or 4), for measurements
    const int v = atoi(e);
    if ((v == 1 || v == 2 || v == 4) && p.kblocks >= v * 8) splits = v;
  }
  p.splits = splits;
  p.kb_per = (p.kblocks + splits - 1) / splits;

  const uint32_t wx = (uint32_t)(lw::kTcKBlock * a->bits / 8);   // weight bytes per row per block
  p.w_bytes = wx * lw::kTcTileN;
  p.b_bytes = (uint32_t)p.Mpad * 128;
  p.stage_bytes = p.b_bytes + p.w_bytes;
  p.stages = (int)std::min<size_t>({(size_t)lw::kTcMaxStages, (lw::kTcSmemMax - 1024) / p.stage_bytes,
                                    (size_t)(512 - acc) / 32});
  int cols = 32;
  while (cols < acc + 32 * p.stages) cols <<= 1;
  p.tmem_cols = cols;
  const size_t red_bytes = (size_t)lw::kTcTileN * (((p.Mpad + 31) & ~31) + 1) * 4;
  if (p.stages < lw::kTcDeqGroups || (splits > 1 && red_bytes > (size_t)p.stages * p.stage_bytes)) return LW_ERR_BAD_SHAPE;
  const size_t smem = 1024 + (size_t)p.stages * p.stage_bytes;

  const size_t rowbytes = (size_t)a->K * a->bits / 8;
  // fp16 rows (128 bytes per block) land 128-byte swizzled: the reading
  // threads (one row each) then spread over the banks
  if (!encode_2d(&p.tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, a->weight, rowbytes, (uint64_t)a->N, rowbytes, wx,
                 lw::kTcTileN, a->bits == 16 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_2d(&p.tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a->act, (uint64_t)a->K, (uint64_t)a->M,
                 (uint64_t)a->lda * 2, lw::kTcKBlock, (uint32_t)p.Mpad, CU_TENSOR_MAP_SWIZZLE_128B))
    return LW_ERR_LAUNCH;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool pdl = a->pdl != 0;
  cudaGetLastError();
  cudaError_t e = cudaErrorInvalidValue;
#define LW_TC(B_, E_) \
  if (a->bits == B_ && a->epilogue == E_) e = tc_launch<B_, E_>(p, smem, s, pdl);
  LW_TC(4, LW_TC_EPI_RESID)
  LW_TC(4, LW_TC_EPI_SWIGLU)
  LW_TC(4, LW_TC_EPI_ROPE_KV)
  LW_TC(8, LW_TC_EPI_RESID)
  LW_TC(8, LW_TC_EPI_SWIGLU)
  LW_TC(8, LW_TC_EPI_ROPE_KV)
  LW_TC(4, LW_TC_EPI_F32)
  LW_TC(8, LW_TC_EPI_F32)
  LW_TC(16, LW_TC_EPI_ARGMAX)
  LW_TC(4, LW_TC_EPI_ARGMAX)
  LW_TC(8, LW_TC_EPI_ARGMAX)
#undef LW_TC
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}
}  // namespace

namespace {
int rmsnorm_rows_launch(void* x, const float* psum, const void* gamma, void* h, int M, int K, float eps, int pdl,
                        lw_stream_t stream) {
  if (!x || !gamma || !h) return LW_ERR_NULL_POINTER;
  if (M <= 0 || K <= 0 || K % 8) return LW_ERR_BAD_SHAPE;
  if (!al(x, 16) || !al(gamma, 16) || !al(h, 16) || (psum && !al(psum, 16))) return LW_ERR_ALIGNMENT;
  cudaGetLastError();
  cudaError_t e = lw_launch(lw::rmsnorm_rows_kernel, dim3(M), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                            pdl != 0, static_cast<__half*>(x), psum, static_cast<const __half*>(gamma),
                            static_cast<__half*>(h), K, eps);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}
}  // namespace

int lw_rmsnorm_rows(const void* x, const void* gamma, void* h, int M, int K, float eps, int pdl,
                    lw_stream_t stream) {
  // x is only read when psum is NULL
  return rmsnorm_rows_launch(const_cast<void*>(x), nullptr, gamma, h, M, K, eps, pdl, stream);
}

int lw_resid_rmsnorm_rows(void* x, const float* psum, const void* gamma, void* h, int M, int K, float eps, int pdl,
                          lw_stream_t stream) {
  if (!psum) return LW_ERR_NULL_POINTER;
  return rmsnorm_rows_launch(x, psum, gamma, h, M, K, eps, pdl, stream);
}

}  // extern "C"
