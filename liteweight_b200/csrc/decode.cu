// Decode-step kernels for a Llama-family model on B200 (sm_100a).
//
// One decode step (one new token per sequence) of the HF LlamaForCausalLM that
// liteweight's generate() drives (liteweight/generate.py:106-124 ->
// transformers modeling_llama.py:290-335) runs as 5 kernels per layer:
//
//   1. fused GEMV: RMSNorm prologue + q|k|v projection + RoPE + KV append
//   2. split-KV GQA attention over the cache (last CTA per head group combines)
//   3. fused GEMV: o_proj + residual add
//   4. fused GEMV: RMSNorm prologue + gate|up projection + SwiGLU
//   5. fused GEMV: down_proj + residual add
//
// then the final RMSNorm + lm_head + argmax GEMV and a sampling kernel that
// picks the next token (or takes the forced prompt token), writes its
// embedding as the next step's residual stream and advances the position.
// Every kernel reads the position from device memory, so one captured CUDA
// graph replays any step. With tensor parallelism the o/down projections
// produce fp32 partial sums instead, either written locally for an NCCL
// all-reduce by the caller or pushed to every rank through peer memory
// (decode_tp.cu), and the next norm prologue adds their sum to the residual.
#include "fused_host.cuh"

#include <cooperative_groups.h>
#include <type_traits>

namespace lw {

// ------------------------------------------------------------- attention

struct AttnParams {
  const __half* q;     // [B][nq * hd]
  const __half* k;     // [B][nkv][S][hd] (this layer)
  const __half* v;
  __half* out;         // [B][nq * hd]
  const int* pos;      // attend over positions 0..*pos
  const int* seq;      // prompt chunk: row b is position *pos + b of sequence *seq (causal)
  int B, nq, nkv, S;
  float scale_log2;    // head_dim^-0.5 * log2(e)
};

// Cluster attention: one thread-block cluster of CL CTAs per (sequence, kv
// head) - CL = kAttnCluster (8) while the grid stays within about two waves of
// the SMs, fewer for large batches; CTA r of the cluster and warp w of the CTA
// own positions [base + (r * W + w) * P, ... + P) of every round of
// CL * W * P positions (P = 8). Per round a warp computes, on the
// tensor cores, S = Q K^T for the GQA group's query heads (MMA rows; rows
// past GQ are zero) against its 8 positions (one m16n8k16 per 16 head dims),
// an online softmax per head (rows: max / sum over the 4 lanes of a row), and
// O += P V with m16n8k8 (P straight from the score fragments). Head dims are
// permuted the same way in q and K so that each lane's fragments are whole
// 16-byte loads: lane (g, t) holds K row g, 16-byte chunks 4q + t; V dims are
// assigned to output columns so that lane (g, t) holds rows 2t, 2t+1, dims
// [g HD/8, (g+1) HD/8) and pairs them with one byte permute per fragment.
// Warps merge through shared memory, then the cluster's CTAs merge through
// distributed shared memory after a cluster barrier - no global round trips,
// no counters. The first two rounds of positions before *pos are loaded before
// griddepcontrol.wait (they do not depend on the previous kernel).
constexpr int kAttnWarps = 8;
constexpr int kAttnCluster = 8;   // largest cluster (CTAs per sequence and kv head)
constexpr int kAttnPos = 8;   // positions per warp per round

LW_DEV void mma1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// CL: CTAs per cluster (8 for one or a few sequences: the latency of one
// sequence's positions split 8 ways; 1 for large batches, whose (sequence, kv
// head) pairs already fill the GPU several times over).
template <int HD, int GQ, int CL>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(const AttnParams p) {
  static_assert(GQ <= 8 && (HD == 64 || HD == 128), "GQA group of at most 8 heads, head_dim 64 or 128");
  namespace cg = cooperative_groups;
  constexpr int W = kAttnWarps;
  constexpr int KQ = HD / 32;    // 16-byte K chunks per lane per position (2 k-steps each)
  constexpr int DPL = HD / 8;    // V dims per lane group g
  constexpr int NV = DPL / 8;    // 16-byte V chunks per lane per position
  // per-warp partial outputs: head h, dim d at h * SAS + d + d / 32, so the
  // fragment stores (lanes = heads x 32-dim strides) fall in distinct banks
  constexpr int SAS = HD + HD / 32 + 4;
  __shared__ float sm_m[W][GQ], sm_l[W][GQ];
  __shared__ float sm_acc[W][GQ * SAS];
  __shared__ float cta_m[GQ], cta_l[GQ];
  __shared__ float cta_acc[GQ][HD];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  auto acc_at = [](int h, int d) { return h * SAS + d + (d >> 5); };
  const int per_round = CL * W * kAttnPos;
  const int first = (rank * W + warp) * kAttnPos;
  // Positions before *pos were written by earlier steps, not by the kernel
  // this one waits for: the first two rounds of them are loaded before
  // griddepcontrol.wait, so their DRAM latency overlaps the previous kernel.
  // (*pos itself is final before this grid launches: the kernel that advances
  // it completed before the previous kernel passed its own wait.)
  const int cs_pre = p.seq ? -1 : b;
  const int len_pre = p.seq ? 0 : *p.pos;              // prefetchable positions [0, len_pre)

  uint4 kr[2][KQ], vr[2][2][NV];   // per round: K row g; V rows 2t, 2t+1
  const __half* kb = nullptr;
  const __half* vb = nullptr;
  int len = 0;
  auto load_k = [&](int base, uint4 (&kk)[KQ]) {
    const int s = min(base + first + g, len - 1);   // clamped: positions past len are masked below
#pragma unroll
    for (int q = 0; q < KQ; ++q) kk[q] = *reinterpret_cast<const uint4*>(kb + (size_t)s * HD + (4 * q + t) * 8);
  };
  auto load_v = [&](int base, uint4 (&vv)[2][NV]) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int s = min(base + first + 2 * t + e, len - 1);
#pragma unroll
      for (int c = 0; c < NV; ++c)
        vv[e][c] = *reinterpret_cast<const uint4*>(vb + (size_t)s * HD + g * DPL + c * 8);
    }
  };
  auto load_round = [&](int base, int r) {
    load_k(base, kr[r]);
    load_v(base, vr[r]);
  };
  if (len_pre > 0) {
    kb = p.k + ((size_t)cs_pre * p.nkv + kvh) * p.S * HD;
    vb = p.v + ((size_t)cs_pre * p.nkv + kvh) * p.S * HD;
    len = len_pre;
    load_round(0, 0);
    load_round(per_round, 1);
  }
  pdl_wait();
  pdl_launch_dependents();   // the next kernel's CTAs may start on the SMs this grid leaves idle
  const int cs = p.seq ? *p.seq : b;                   // KV-cache sequence of this query row
  len = *p.pos + 1 + (p.seq ? b : 0);
  kb = p.k + ((size_t)cs * p.nkv + kvh) * p.S * HD;
  vb = p.v + ((size_t)cs * p.nkv + kvh) * p.S * HD;
  if (len_pre == 0 || len != len_pre + 1) {
    load_round(0, 0);   // nothing (or not the expected positions) prefetched
    load_round(per_round, 1);
  } else {
    // only position len - 1 (this step's, written by the previous kernel) is new
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      if (rr * per_round + first + g == len - 1) load_k(rr * per_round, kr[rr]);
      if (rr * per_round + first + 2 * t == len - 1 || rr * per_round + first + 2 * t + 1 == len - 1)
        load_v(rr * per_round, vr[rr]);
    }
  }
  // the queries come from the previous kernel: read after the wait. A
  // fragments: row g = query head kvh * GQ + g (zero past GQ), the same dim
  // permutation as K; rows g + 8 are zero.
  uint32_t qa[KQ][4];
  {
    const __half* qp = p.q + (size_t)b * p.nq * HD + (size_t)(kvh * GQ + min(g, GQ - 1)) * HD;
#pragma unroll
    for (int q = 0; q < KQ; ++q) {
      uint4 v = *reinterpret_cast<const uint4*>(qp + (4 * q + t) * 8);
      if (g >= GQ) v = make_uint4(0, 0, 0, 0);
      qa[q][0] = v.x;   // k-step 2q:   dims +0,1 / +2,3
      qa[q][1] = v.y;
      qa[q][2] = v.z;   // k-step 2q+1: dims +4,5 / +6,7
      qa[q][3] = v.w;
    }
  }
  float m_r = -INFINITY, l_r = 0.f;   // softmax state of head g (replicated over the row's 4 lanes)
  float o[DPL][4];
#pragma unroll
  for (int j = 0; j < DPL; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

  auto process = [&](int base, const uint4 (&kk)[KQ], const uint4 (&vv)[2][NV]) {
    const int n = min(kAttnPos, len - (base + first));
    if (n <= 0) return;
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < KQ; ++q) {
      mma16816(sc, qa[q][0], 0u, qa[q][1], 0u, kk[q].x, kk[q].y);
      mma16816(sc, qa[q][2], 0u, qa[q][3], 0u, kk[q].z, kk[q].w);
    }
    // scores of head g at positions 2t, 2t + 1 of the round (log2 domain)
    float s0 = 2 * t < n ? sc[0] * p.scale_log2 : -INFINITY;
    float s1 = 2 * t + 1 < n ? sc[1] * p.scale_log2 : -INFINITY;
    float mx = fmaxf(s0, s1);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m_r, mx);   // finite: position base + first < len
    const float corr = exp2f(m_r - mn);
    const float p0 = exp2f(s0 - mn), p1 = exp2f(s1 - mn);
    float sum = p0 + p1;
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    l_r = l_r * corr + sum;
    m_r = mn;
    const uint32_t pa = h2_as_u32(__floats2half2_rn(p0, p1));
    const uint32_t* v0 = reinterpret_cast<const uint32_t*>(&vv[0][0]);
    const uint32_t* v1 = reinterpret_cast<const uint32_t*>(&vv[1][0]);
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      o[j][0] *= corr;
      o[j][1] *= corr;
      // B[k = position 2t, 2t+1][n = g] for output columns j: dim g * DPL + j of the two rows
      const uint32_t bv = __byte_perm(v0[j >> 1], v1[j >> 1], (j & 1) ? 0x7632 : 0x5410);
      mma1688(o[j], pa, 0u, bv);
    }
  };
  // rounds 0 and 1 are in registers; later rounds load two ahead of use
  const int rounds = (len + per_round - 1) / per_round;
  for (int r = 0; r < rounds; r += 2) {
    process(r * per_round, kr[0], vr[0]);
    if (r + 2 < rounds) load_round((r + 2) * per_round, 0);
    if (r + 1 >= rounds) break;
    process((r + 1) * per_round, kr[1], vr[1]);
    if (r + 3 < rounds) load_round((r + 3) * per_round, 1);
  }
  // per-warp state to shared memory: o[j][0] / o[j][1] = head g, dims
  // (2t) DPL + j / (2t + 1) DPL + j
  if (g < GQ) {
    if (t == 0) {
      sm_m[warp][g] = m_r;
      sm_l[warp][g] = l_r;
    }
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      sm_acc[warp][acc_at(g, (2 * t) * DPL + j)] = o[j][0];
      sm_acc[warp][acc_at(g, (2 * t + 1) * DPL + j)] = o[j][1];
    }
  }
  __syncthreads();
  // warps -> CTA
  for (int i = threadIdx.x; i < GQ * HD; i += W * 32) {
    const int h = i / HD, d = i - h * HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, sm_m[w][h]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const float c = exp2f(sm_m[w][h] - M);
        L = fmaf(sm_l[w][h], c, L);
        A = fmaf(sm_acc[w][acc_at(h, d)], c, A);
      }
    }
    cta_acc[h][d] = A;
    if (d == 0) {
      cta_m[h] = M;
      cta_l[h] = L;
    }
  }
  // CTAs of the cluster -> output: CTA r finishes elements r, r + CL, ...
  cluster.sync();
  for (int i = rank * (W * 32) + threadIdx.x; i < GQ * HD; i += CL * W * 32) {
    const int h = i / HD, d = i - h * HD;
    // all remote reads issued together (independent distributed-shared-memory loads)
    float mc[CL], lc[CL], ac[CL];
#pragma unroll
    for (int c = 0; c < CL; ++c) {
      mc[c] = *cluster.map_shared_rank(&cta_m[h], c);
      lc[c] = *cluster.map_shared_rank(&cta_l[h], c);
      ac[c] = *cluster.map_shared_rank(&cta_acc[h][d], c);
    }
    float M = -INFINITY;
#pragma unroll
    for (int c = 0; c < CL; ++c) M = fmaxf(M, mc[c]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int c = 0; c < CL; ++c) {
      const float w = mc[c] == -INFINITY ? 0.f : exp2f(mc[c] - M);   // a CTA with no positions adds nothing
      L = fmaf(lc[c], w, L);
      A = fmaf(ac[c], w, A);
    }
    p.out[(size_t)b * p.nq * HD + (size_t)(kvh * GQ + h) * HD + d] = __float2half_rn(A / L);
  }
  cluster.sync();   // keep this CTA's shared memory alive until every remote read is done
}

// ------------------------------------------------------------- prompt-chunk attention
//
// Rows of a prompt chunk are consecutive positions p0 .. p0 + R - 1 of one
// sequence (causal: row r attends keys 0 .. p0 + r). One CTA per (16 query
// positions, kv head) with one warp per query head of the GQA group, so each
// K/V block is staged in shared memory once for the whole group. Per block of
// 64 keys a warp computes S = Q K^T (16 x 64) with mma.sync m16n8k16 (K
// fragments by ldmatrix), masks by position, updates an fp32 online softmax
// (row max / sum, exp2 of log2e-scaled scores), and accumulates O += P V with
// P taken straight from the score fragments (rounded to fp16, the precision
// of the reference's softmax output) and V fragments by ldmatrix.trans.
constexpr int kPfKeys = 64;
constexpr int kPfRows = 16;

LW_DEV void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
LW_DEV void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
LW_DEV uint32_t pack_h2(float lo, float hi) { return h2_as_u32(__floats2half2_rn(lo, hi)); }

template <int HD, int GQ>
__global__ void __launch_bounds__(GQ * 32) attn_prefill_kernel(const AttnParams p) {
  constexpr int RS = HD + 8;   // padded row (halves): rows 16 bytes apart modulo 128
  constexpr int NT = GQ * 32;
  __shared__ __align__(16) __half ks[kPfKeys * RS];
  __shared__ __align__(16) __half vs[kPfKeys * RS];
  const int qb = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  pdl_wait();
  pdl_launch_dependents();
  const int p0 = *p.pos, cs = *p.seq, R = p.B;
  const int r0 = qb * kPfRows;
  const int head = kvh * GQ + warp;
  const int kv_len = p0 + min(R, r0 + kPfRows);   // keys any row of this block may see
  const int qpos_lo = p0 + r0 + g, qpos_hi = qpos_lo + 8;

  // Q fragments (A operand: 16 rows x HD), rows past R are zero
  uint32_t qa[HD / 16][4];
  {
    const int rl = r0 + g, rh = r0 + g + 8;
    const __half* ql = p.q + (size_t)rl * p.nq * HD + (size_t)head * HD + 2 * t;
    const __half* qh = p.q + (size_t)rh * p.nq * HD + (size_t)head * HD + 2 * t;
#pragma unroll
    for (int kt = 0; kt < HD / 16; ++kt) {
      qa[kt][0] = rl < R ? *reinterpret_cast<const uint32_t*>(ql + kt * 16) : 0u;
      qa[kt][1] = rh < R ? *reinterpret_cast<const uint32_t*>(qh + kt * 16) : 0u;
      qa[kt][2] = rl < R ? *reinterpret_cast<const uint32_t*>(ql + kt * 16 + 8) : 0u;
      qa[kt][3] = rh < R ? *reinterpret_cast<const uint32_t*>(qh + kt * 16 + 8) : 0u;
    }
  }
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  const __half* kg = p.k + ((size_t)cs * p.nkv + kvh) * p.S * HD;
  const __half* vg = p.v + ((size_t)cs * p.nkv + kvh) * p.S * HD;
  const uint32_t ks_a = smem_u32(ks), vs_a = smem_u32(vs);

  for (int k0 = 0; k0 < kv_len; k0 += kPfKeys) {
    __syncthreads();   // the previous block is no longer read
    for (int i = threadIdx.x; i < kPfKeys * HD / 8; i += NT) {
      const int r = i / (HD / 8), c = (i % (HD / 8)) * 8;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (k0 + r < kv_len) {
        kv = *reinterpret_cast<const uint4*>(kg + (size_t)(k0 + r) * HD + c);
        vv = *reinterpret_cast<const uint4*>(vg + (size_t)(k0 + r) * HD + c);
      }
      sts128(ks + r * RS + c, kv);
      sts128(vs + r * RS + c, vv);
    }
    __syncthreads();

    // S = Q K^T over this block's 64 keys (8 tiles of 8 keys)
    float sc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
#pragma unroll
    for (int kt = 0; kt < HD / 16; ++kt) {
#pragma unroll
      for (int n2 = 0; n2 < 4; ++n2) {
        const int mi = lane >> 3;
        const int key = n2 * 16 + (mi >> 1) * 8 + (lane & 7), dim = kt * 16 + (mi & 1) * 8;
        uint32_t b[4];
        ldsm_x4(ks_a + (uint32_t)(key * RS + dim) * 2u, b);
        mma16816(sc[2 * n2], qa[kt][0], qa[kt][1], qa[kt][2], qa[kt][3], b[0], b[1]);
        mma16816(sc[2 * n2 + 1], qa[kt][0], qa[kt][1], qa[kt][2], qa[kt][3], b[2], b[3]);
      }
    }
    // scale, causal mask, online softmax (rows g and g + 8 of the lane)
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + nt * 8 + 2 * t + (e & 1);
        const int qp = e < 2 ? qpos_lo : qpos_hi;
        float v = sc[nt][e] * p.scale_log2;
        if (key > qp || key >= kv_len) v = -INFINITY;
        sc[nt][e] = v;
        if (e < 2) mx_lo = fmaxf(mx_lo, v);
        else mx_hi = fmaxf(mx_hi, v);
      }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
    }
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    const float c_lo = mn_lo == -INFINITY ? 1.f : exp2f(m_lo - mn_lo);
    const float c_hi = mn_hi == -INFINITY ? 1.f : exp2f(m_hi - mn_hi);
    float s_lo = 0.f, s_hi = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      sc[nt][0] = mn_lo == -INFINITY ? 0.f : exp2f(sc[nt][0] - mn_lo);
      sc[nt][1] = mn_lo == -INFINITY ? 0.f : exp2f(sc[nt][1] - mn_lo);
      sc[nt][2] = mn_hi == -INFINITY ? 0.f : exp2f(sc[nt][2] - mn_hi);
      sc[nt][3] = mn_hi == -INFINITY ? 0.f : exp2f(sc[nt][3] - mn_hi);
      s_lo += sc[nt][0] + sc[nt][1];
      s_hi += sc[nt][2] + sc[nt][3];
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      s_lo += __shfl_xor_sync(0xffffffffu, s_lo, off);
      s_hi += __shfl_xor_sync(0xffffffffu, s_hi, off);
    }
    l_lo = l_lo * c_lo + s_lo;
    l_hi = l_hi * c_hi + s_hi;
    m_lo = mn_lo;
    m_hi = mn_hi;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= c_lo;
      o[i][1] *= c_lo;
      o[i][2] *= c_hi;
      o[i][3] *= c_hi;
    }
    // O += P V: the score fragments of key tiles 2kk, 2kk+1 are the A fragment of keys 16kk..16kk+15
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a0 = pack_h2(sc[2 * kk][0], sc[2 * kk][1]);
      const uint32_t a1 = pack_h2(sc[2 * kk][2], sc[2 * kk][3]);
      const uint32_t a2 = pack_h2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
      const uint32_t a3 = pack_h2(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
      for (int d2 = 0; d2 < HD / 16; ++d2) {
        const int mi = lane >> 3;
        const int key = kk * 16 + (mi & 1) * 8 + (lane & 7), dim = d2 * 16 + (mi >> 1) * 8;
        uint32_t b[4];
        ldsm_x4_t(vs_a + (uint32_t)(key * RS + dim) * 2u, b);
        mma16816(o[2 * d2], a0, a1, a2, a3, b[0], b[1]);
        mma16816(o[2 * d2 + 1], a0, a1, a2, a3, b[2], b[3]);
      }
    }
  }
  // out rows r0 + g and r0 + g + 8
  const int rl = r0 + g, rh = r0 + g + 8;
  const float il = l_lo > 0.f ? 1.f / l_lo : 0.f, ih = l_hi > 0.f ? 1.f / l_hi : 0.f;
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    const int d = i * 8 + 2 * t;
    if (rl < R)
      *reinterpret_cast<uint32_t*>(p.out + (size_t)rl * p.nq * HD + (size_t)head * HD + d) =
          pack_h2(o[i][0] * il, o[i][1] * il);
    if (rh < R)
      *reinterpret_cast<uint32_t*>(p.out + (size_t)rh * p.nq * HD + (size_t)head * HD + d) =
          pack_h2(o[i][2] * ih, o[i][3] * ih);
  }
}

// ------------------------------------------------------------- tokens

// x[b] = embed[tokens[*pos][b]]
__global__ void embed_kernel(const int* __restrict__ tokens, const __half* __restrict__ embed,
                             __half* __restrict__ x, const int* pos, int B, int H) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int tok = tokens[(size_t)(*pos) * B + b];
  const uint4* src = reinterpret_cast<const uint4*>(embed + (size_t)tok * H);
  uint4* dst = reinterpret_cast<uint4*>(x + (size_t)b * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// Next token per sequence: the forced token at position *pos + 1 when the
// table holds one (>= 0, a prompt token), else the argmax of the logits
// (first index of the maximum, torch.argmax semantics; generate.py:51-52).
// Writes it to the table, loads its embedding as the next residual stream,
// clears the argmax key and, in the last block to finish, advances *pos (and
// *step). With a tensor-parallel exchange the keys are max'd in by every
// rank's lm_head: wait until all of them have arrived.
struct SampleParams {
  int* tokens;
  unsigned long long* keys;
  const __half* embed;
  __half* x;
  int* pos;
  int* done;
  int* step;             // may be null
  int B, H;
  int in_world;          // 0: the local keys are the pick
  int in_tag, in_tags;
  const unsigned long long* in_src;  // flagged keys [in_world][B]
  int* in_error;
  long long in_timeout_ns;
};

__global__ void sample_kernel(const SampleParams p) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int s_tok;
  const int b = blockIdx.x;
  const int p_next = *p.pos + 1;
  if (threadIdx.x == 0) {
    int tok = p.tokens[(size_t)p_next * p.B + b];
    if (tok < 0) {
      unsigned long long key = 0;
      if (p.in_world) {
        // the maximum of every rank's key, each read once its flag is current
        const unsigned long long f16 = exchange_flag16(exchange_flag(*p.step, p.in_tag, p.in_tags));
        WaitBudget wb;
        for (int r = 0; r < p.in_world; ++r) {
          unsigned long long w;
          do {
            w = ld_volatile_u64(p.in_src + (size_t)r * p.B + b);
          } while ((w >> 48) != f16 && wb.keep_waiting(p.in_timeout_ns, p.in_error));
          w &= 0xFFFFFFFFFFFFull;
          key = w > key ? w : key;
        }
      } else {
        key = __ldcg(p.keys + b);
      }
      tok = (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
      p.tokens[(size_t)p_next * p.B + b] = tok;
    }
    p.keys[b] = 0ull;
    s_tok = tok;
  }
  __syncthreads();
  const uint4* src = reinterpret_cast<const uint4*>(p.embed + (size_t)s_tok * p.H);
  uint4* dst = reinterpret_cast<uint4*>(p.x + (size_t)b * p.H);
  for (int i = threadIdx.x; i < p.H / 8; i += blockDim.x) dst[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(p.done, 1);
    if (old == p.B - 1) {
      *p.pos = p_next;
      if (p.step) *p.step += 1;
      *p.done = 0;
    }
  }
}

// ------------------------------------------------------------- prefill chunks

__global__ void prefill_embed_kernel(const int* __restrict__ tokens, const __half* __restrict__ embed,
                                     __half* __restrict__ x, const int* pos, const int* seq, int B, int H) {
  pdl_wait();
  pdl_launch_dependents();
  const int m = blockIdx.x;
  const int tok = tokens[(size_t)(*pos + m) * B + *seq];
  const uint4* src = reinterpret_cast<const uint4*>(embed + (size_t)tok * H);
  uint4* dst = reinterpret_cast<uint4*>(x + (size_t)m * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

__global__ void prefill_advance_kernel(int* pos, int* step, int rows) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    *pos += rows;
    if (step) *step += 1;
  }
}

struct PrefillSampleParams {
  int* tokens;
  unsigned long long* keys;   // this rank's lm_head keys of the chunk rows
  const __half* embed;
  __half* x;                  // the decode step's residual stream [B][H]
  int* pos;
  int* step;                  // may be null
  const int* seq;
  int rows, B, H;
  int in_world, in_tag, in_tags;   // in_world > 0: keys from the exchange (flagged words [in_world][rows])
  const unsigned long long* in_src;
  int* in_error;
  long long in_timeout_ns;
};

// One block: the token after the chunk's last row (forced prompt token, or
// the argmax of that row), its embedding as the decode residual of sequence
// *seq, the chunk keys cleared, the position advanced past the chunk.
__global__ void prefill_sample_kernel(const PrefillSampleParams p) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int s_tok, s_seq, s_next;
  if (threadIdx.x == 0) {
    const int seq = *p.seq;
    const int p_next = *p.pos + p.rows;
    int tok = p.tokens[(size_t)p_next * p.B + seq];
    if (tok < 0) {
      unsigned long long key = 0;
      const int r = p.rows - 1;
      if (p.in_world) {
        const unsigned long long f16 = exchange_flag16(exchange_flag(*p.step, p.in_tag, p.in_tags));
        WaitBudget wb;
        for (int k = 0; k < p.in_world; ++k) {
          unsigned long long w;
          do {
            w = ld_volatile_u64(p.in_src + (size_t)k * p.rows + r);
          } while ((w >> 48) != f16 && wb.keep_waiting(p.in_timeout_ns, p.in_error));
          w &= 0xFFFFFFFFFFFFull;
          key = w > key ? w : key;
        }
      } else {
        key = __ldcg(p.keys + r);
      }
      tok = (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
      p.tokens[(size_t)p_next * p.B + seq] = tok;
    }
    s_tok = tok;
    s_seq = seq;
    s_next = p_next;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < p.rows; i += blockDim.x) p.keys[i] = 0ull;
  const uint4* src = reinterpret_cast<const uint4*>(p.embed + (size_t)s_tok * p.H);
  uint4* dst = reinterpret_cast<uint4*>(p.x + (size_t)s_seq * p.H);
  for (int i = threadIdx.x; i < p.H / 8; i += blockDim.x) dst[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    *p.pos = s_next;
    if (p.step) *p.step += 1;
  }
}

}  // namespace lw

// ======================================================================= host

namespace {

inline bool al(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }


// The (bits, prologue, epilogue) combinations the decode step uses.
#define LW_FUSED_TABLE(X)                                   \
  X(4, lw::PRO_NORM, lw::EPI_ROPE_KV)                       \
  X(8, lw::PRO_NORM, lw::EPI_ROPE_KV)                       \
  X(4, lw::PRO_RESID_NORM, lw::EPI_ROPE_KV)                 \
  X(8, lw::PRO_RESID_NORM, lw::EPI_ROPE_KV)                 \
  X(4, lw::PRO_NORM, lw::EPI_SWIGLU)                        \
  X(8, lw::PRO_NORM, lw::EPI_SWIGLU)                        \
  X(4, lw::PRO_RESID_NORM, lw::EPI_SWIGLU)                  \
  X(8, lw::PRO_RESID_NORM, lw::EPI_SWIGLU)                  \
  X(4, lw::PRO_PLAIN, lw::EPI_PLAIN)                        \
  X(8, lw::PRO_PLAIN, lw::EPI_PLAIN)                        \
  X(4, lw::PRO_PLAIN, lw::EPI_F32)                          \
  X(8, lw::PRO_PLAIN, lw::EPI_F32)                          \
  X(16, lw::PRO_NORM, lw::EPI_ARGMAX)                       \
  X(16, lw::PRO_RESID_NORM, lw::EPI_ARGMAX)                 \
  X(4, lw::PRO_NORM, lw::EPI_ARGMAX)                        \
  X(8, lw::PRO_NORM, lw::EPI_ARGMAX)                        \
  X(4, lw::PRO_RESID_NORM, lw::EPI_ARGMAX)                  \
  X(8, lw::PRO_RESID_NORM, lw::EPI_ARGMAX)

int validate(const lw_fused_gemv_args* a) {
  if (!a) return LW_ERR_NULL_POINTER;
  if (!a->act || !a->weight) return LW_ERR_NULL_POINTER;
  if (a->bits != 4 && a->bits != 8 && a->bits != 16) return LW_ERR_UNSUPPORTED;
  if (a->M <= 0 || a->M > 32 || a->N <= 0 || a->K <= 0) return LW_ERR_BAD_SHAPE;
  if (a->bits != 16 && (!a->scales || a->group_size <= 0 || a->K % a->group_size)) return LW_ERR_BAD_GROUP;
  const int E = a->bits == 4 ? 32 : (a->bits == 8 ? 16 : 8);
  if ((size_t)a->K * a->bits / 8 % 64 || a->K % 8 ||
      (a->bits != 16 && (a->group_size % E || lw::group_shift(a->K, a->group_size) < 0)))
    return LW_ERR_UNSUPPORTED;
  if (!al(a->act, 16) || !al(a->weight, 16) || a->lda % 8) return LW_ERR_ALIGNMENT;
  const int KC = 4 * E;
  if ((size_t)a->M * ((a->K + KC - 1) / KC) * KC * 2 + lw::gamma_bytes(a->prologue, a->K) > (size_t)lw::kStageBudget)
    return LW_ERR_UNSUPPORTED;
  if (a->prologue != LW_PRO_PLAIN) {
    if (!a->gamma || !al(a->gamma, 16)) return LW_ERR_NULL_POINTER;
    if (a->prologue == LW_PRO_RESID_NORM && (!a->psum || !a->x_out || !al(a->psum, 16) || !al(a->x_out, 16)))
      return LW_ERR_NULL_POINTER;
    if (a->prologue == LW_PRO_PEER_RESID_NORM) {
      const lw_exchange_in* x = a->xin;
      if (!x || !x->src || !x->step || !a->x_out) return LW_ERR_NULL_POINTER;
      if (x->world < 1 || x->world > LW_MAX_RANKS || x->timeout_ns <= 0 || x->tags_per_step <= 0 ||
          x->tag < 0 || x->tag >= x->tags_per_step)
        return LW_ERR_BAD_SHAPE;
      if (!al(x->src, 16) || !al(a->x_out, 16)) return LW_ERR_ALIGNMENT;
    }
  }
  if (a->epilogue == LW_EPI_PEER_F32 || a->epilogue == LW_EPI_PEER_ARGMAX) {
    const lw_exchange_out* x = a->xout;
    if (!x || !x->step) return LW_ERR_NULL_POINTER;
    if (x->world < 1 || x->world > LW_MAX_RANKS || x->rank < 0 || x->rank >= x->world ||
        x->tags_per_step <= 0 || x->tag < 0 || x->tag >= x->tags_per_step)
      return LW_ERR_BAD_SHAPE;
    for (int d = 0; d < x->world; ++d) {
      if (!x->dst[d]) return LW_ERR_NULL_POINTER;
      if (!al(x->dst[d], 8)) return LW_ERR_ALIGNMENT;
    }
    if (a->epilogue == LW_EPI_PEER_F32 && a->ldo < a->N) return LW_ERR_BAD_SHAPE;
    if (a->epilogue == LW_EPI_PEER_ARGMAX && (!a->out || !a->argmax_keys || !x->arrivals)) return LW_ERR_NULL_POINTER;
  }
  switch (a->epilogue) {
    case LW_EPI_PEER_F32:
    case LW_EPI_PEER_ARGMAX:
      break;
    case LW_EPI_PLAIN:
      if (!a->out) return LW_ERR_NULL_POINTER;
      break;
    case LW_EPI_F32:
      if (!a->out_f32) return LW_ERR_NULL_POINTER;
      break;
    case LW_EPI_ROPE_KV:
      if (!a->q_out || !a->k_cache || !a->v_cache || !a->rope_cos || !a->rope_sin || !a->pos)
        return LW_ERR_NULL_POINTER;
      if (a->head_dim % 16 || a->N != (a->n_q_heads + 2 * a->n_kv_heads) * a->head_dim) return LW_ERR_BAD_SHAPE;
      break;
    case LW_EPI_SWIGLU:
      if (!a->out) return LW_ERR_NULL_POINTER;
      if (a->N % 16) return LW_ERR_BAD_SHAPE;
      break;
    case LW_EPI_ARGMAX:
      if (!a->out || !a->argmax_keys) return LW_ERR_NULL_POINTER;
      break;
    default:
      return LW_ERR_UNSUPPORTED;
  }
  if (a->workspace_bytes && !a->workspace) return LW_ERR_WORKSPACE;
  if (a->workspace && !al(a->workspace, 256)) return LW_ERR_ALIGNMENT;
  return LW_OK;
}

// CTAs per (sequence, kv head): the largest of 8, 4, 2, 1 that keeps the grid
// within about two waves of one CTA per SM.
inline int attn_cluster_size(int B, int nkv) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0)
    sms = 148;
  int cl = lw::kAttnCluster;
  while (cl > 1 && (long long)B * nkv * cl > 2LL * sms) cl /= 2;
  return cl;
}

template <int HD, int GQ, int CL>
cudaError_t attn_launch_cl(const lw::AttnParams& p, cudaStream_t s, bool pdl) {
  lw_count_launch();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, p.nkv, p.B);
  cfg.blockDim = dim3(lw::kAttnWarps * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  int na = 1;
  if (pdl) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, lw::attn_decode_kernel<HD, GQ, CL>, p);
}

template <int HD, int GQ>
cudaError_t attn_launch(const lw::AttnParams& p, cudaStream_t s, bool pdl) {
  switch (attn_cluster_size(p.B, p.nkv)) {
    case 8: return attn_launch_cl<HD, GQ, 8>(p, s, pdl);
    case 4: return attn_launch_cl<HD, GQ, 4>(p, s, pdl);
    case 2: return attn_launch_cl<HD, GQ, 2>(p, s, pdl);
    default: return attn_launch_cl<HD, GQ, 1>(p, s, pdl);
  }
}

}  // namespace

int lw_decode_take_error() { return lw_tu_take_error(); }

extern "C" {

int lw_fused_gemv(const lw_fused_gemv_args* a, lw_stream_t stream) {
  int st = validate(a);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaGetLastError();
  cudaError_t e = cudaErrorInvalidValue;
  bool found = false;
#define X(B_, P_, E_)                                                         \
  if (!found && a->bits == B_ && a->prologue == P_ && a->epilogue == E_) {  \
    found = true;                                                           \
    e = lw::fused_launch<B_, P_, E_>(a, s);                                 \
  }
  LW_FUSED_TABLE(X)
#undef X
  if (!found) found = lw::tp_fused_launch(a, s, &e);
  if (!found) return LW_ERR_UNSUPPORTED;
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

size_t lw_fused_gemv_workspace_size(const lw_fused_gemv_args* a) {
  if (validate(a) != LW_OK) return 0;
  size_t r = 0;
  bool found = false;
#define X(B_, P_, E_)                                                         \
  if (!found && a->bits == B_ && a->prologue == P_ && a->epilogue == E_) {  \
    found = true;                                                           \
    r = lw::fused_ws<B_, P_, E_>(a);                                        \
  }
  LW_FUSED_TABLE(X)
#undef X
  if (!found) lw::tp_fused_ws(a, &r);
  return r;
}

int lw_attention_decode(const lw_attention_args* a, lw_stream_t stream) {
  if (!a || !a->q || !a->k_cache || !a->v_cache || !a->out || !a->pos) return LW_ERR_NULL_POINTER;
  if (a->batch <= 0 || a->n_kv_heads <= 0 || a->n_q_heads % a->n_kv_heads || a->max_seq <= 0)
    return LW_ERR_BAD_SHAPE;

  lw::AttnParams p = {};
  p.q = static_cast<const __half*>(a->q);
  p.k = static_cast<const __half*>(a->k_cache);
  p.v = static_cast<const __half*>(a->v_cache);
  p.out = static_cast<__half*>(a->out);
  p.pos = a->pos;
  p.seq = a->prefill_seq;
  p.B = a->batch;
  p.nq = a->n_q_heads;
  p.nkv = a->n_kv_heads;
  p.S = a->max_seq;
  p.scale_log2 = (1.0f / sqrtf((float)a->head_dim)) * 1.4426950408889634f;
  const int gq = a->n_q_heads / a->n_kv_heads;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool pdl = a->pdl != 0;
  cudaGetLastError();
  cudaError_t e;
  if (p.seq) {   // a prompt chunk: rows are positions of one sequence
    dim3 grid((p.B + lw::kPfRows - 1) / lw::kPfRows, p.nkv);
#define LW_PF(HD_, GQ_)                                                                                    \
  if (a->head_dim == HD_ && gq == GQ_) {                                                                   \
    e = lw_launch(lw::attn_prefill_kernel<HD_, GQ_>, grid, dim3(GQ_ * 32), 0, s, pdl, p);                  \
    if (e == cudaSuccess) e = cudaGetLastError();                                                          \
    return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;                                                       \
  }
    LW_PF(128, 1) LW_PF(128, 2) LW_PF(128, 4) LW_PF(128, 8) LW_PF(64, 1) LW_PF(64, 2) LW_PF(64, 4) LW_PF(64, 8)
#undef LW_PF
    return LW_ERR_UNSUPPORTED;
  }
  if (a->head_dim == 128 && gq == 4) e = attn_launch<128, 4>(p, s, pdl);
  else if (a->head_dim == 128 && gq == 8) e = attn_launch<128, 8>(p, s, pdl);
  else if (a->head_dim == 128 && gq == 2) e = attn_launch<128, 2>(p, s, pdl);
  else if (a->head_dim == 128 && gq == 1) e = attn_launch<128, 1>(p, s, pdl);
  else if (a->head_dim == 64 && gq == 4) e = attn_launch<64, 4>(p, s, pdl);
  else if (a->head_dim == 64 && gq == 2) e = attn_launch<64, 2>(p, s, pdl);
  else if (a->head_dim == 64 && gq == 8) e = attn_launch<64, 8>(p, s, pdl);
  else if (a->head_dim == 64 && gq == 1) e = attn_launch<64, 1>(p, s, pdl);
  else return LW_ERR_UNSUPPORTED;
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

size_t lw_struct_size(int which) {
  if (which == 0) return sizeof(lw_fused_gemv_args);
  if (which == 1) return sizeof(lw_attention_args);
  if (which == 2) return sizeof(lw_exchange_out);
  if (which == 3) return sizeof(lw_exchange_in);
  if (which == 4) return sizeof(lw_prefill_gemm_args);
  return 0;
}

int lw_embed_tokens(const int* tokens, const void* embed, void* x, const int* pos, int batch, int hidden, int pdl,
                    lw_stream_t stream) {
  if (!tokens || !embed || !x || !pos) return LW_ERR_NULL_POINTER;
  if (batch <= 0 || hidden <= 0 || hidden % 8) return LW_ERR_BAD_SHAPE;
  if (!al(embed, 16) || !al(x, 16)) return LW_ERR_ALIGNMENT;
  cudaGetLastError();
  cudaError_t e = lw_launch(lw::embed_kernel, dim3(batch), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                            pdl != 0, tokens, static_cast<const __half*>(embed), static_cast<__half*>(x), pos, batch,
                            hidden);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

int lw_sample_tokens(int* tokens, unsigned long long* keys, const void* embed, void* x, int* pos, int* done,
                     int* step, const lw_exchange_in* xin, int batch, int hidden, int pdl, lw_stream_t stream) {
  if (!tokens || !keys || !embed || !x || !pos || !done) return LW_ERR_NULL_POINTER;
  if (batch <= 0 || hidden <= 0 || hidden % 8) return LW_ERR_BAD_SHAPE;
  if (!al(embed, 16) || !al(x, 16)) return LW_ERR_ALIGNMENT;
  lw::SampleParams p = {};
  p.tokens = tokens;
  p.keys = keys;
  p.embed = static_cast<const __half*>(embed);
  p.x = static_cast<__half*>(x);
  p.pos = pos;
  p.done = done;
  p.step = step;
  p.B = batch;
  p.H = hidden;
  if (xin) {
    if (!xin->src || !step) return LW_ERR_NULL_POINTER;
    if (xin->world < 1 || xin->world > LW_MAX_RANKS || xin->timeout_ns <= 0 || xin->tags_per_step <= 0 ||
        xin->tag < 0 || xin->tag >= xin->tags_per_step)
      return LW_ERR_BAD_SHAPE;
    if (!al(xin->src, 8)) return LW_ERR_ALIGNMENT;
    p.in_world = xin->world;
    p.in_tag = xin->tag;
    p.in_tags = xin->tags_per_step;
    p.in_src = static_cast<const unsigned long long*>(xin->src);
    p.in_error = xin->error;
    p.in_timeout_ns = xin->timeout_ns;
  }
  cudaGetLastError();
  cudaError_t e = lw_launch(lw::sample_kernel, dim3(batch), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                            pdl != 0, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

int lw_prefill_embed(const int* tokens, const void* embed, void* x, const int* pos, const int* seq, int rows,
                     int batch, int hidden, int pdl, lw_stream_t stream) {
  if (!tokens || !embed || !x || !pos || !seq) return LW_ERR_NULL_POINTER;
  if (rows <= 0 || batch <= 0 || hidden <= 0 || hidden % 8) return LW_ERR_BAD_SHAPE;
  if (!al(embed, 16) || !al(x, 16)) return LW_ERR_ALIGNMENT;
  cudaGetLastError();
  cudaError_t e = lw_launch(lw::prefill_embed_kernel, dim3(rows), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                            pdl != 0, tokens, static_cast<const __half*>(embed), static_cast<__half*>(x), pos, seq,
                            batch, hidden);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

int lw_prefill_advance(int* pos, int* step, int rows, int pdl, lw_stream_t stream) {
  if (!pos) return LW_ERR_NULL_POINTER;
  if (rows <= 0) return LW_ERR_BAD_SHAPE;
  cudaGetLastError();
  cudaError_t e = lw_launch(lw::prefill_advance_kernel, dim3(1), dim3(32), 0, reinterpret_cast<cudaStream_t>(stream),
                            pdl != 0, pos, step, rows);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

int lw_prefill_sample(int* tokens, unsigned long long* keys, const void* embed, void* x_out, int* pos, int* step,
                      const int* seq, const lw_exchange_in* xin, int rows, int batch, int hidden, int pdl,
                      lw_stream_t stream) {
  if (!tokens || !keys || !embed || !x_out || !pos || !seq) return LW_ERR_NULL_POINTER;
  if (rows <= 0 || batch <= 0 || hidden <= 0 || hidden % 8) return LW_ERR_BAD_SHAPE;
  if (!al(embed, 16) || !al(x_out, 16)) return LW_ERR_ALIGNMENT;
  lw::PrefillSampleParams p = {};
  p.tokens = tokens;
  p.keys = keys;
  p.embed = static_cast<const __half*>(embed);
  p.x = static_cast<__half*>(x_out);
  p.pos = pos;
  p.step = step;
  p.seq = seq;
  p.rows = rows;
  p.B = batch;
  p.H = hidden;
  if (xin) {
    if (!xin->src || !step) return LW_ERR_NULL_POINTER;
    if (xin->world < 1 || xin->world > LW_MAX_RANKS || xin->timeout_ns <= 0 || xin->tags_per_step <= 0 ||
        xin->tag < 0 || xin->tag >= xin->tags_per_step)
      return LW_ERR_BAD_SHAPE;
    if (!al(xin->src, 8)) return LW_ERR_ALIGNMENT;
    p.in_world = xin->world;
    p.in_tag = xin->tag;
    p.in_tags = xin->tags_per_step;
    p.in_src = static_cast<const unsigned long long*>(xin->src);
    p.in_error = xin->error;
    p.in_timeout_ns = xin->timeout_ns;
  }
  cudaGetLastError();
  cudaError_t e = lw_launch(lw::prefill_sample_kernel, dim3(1), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                            pdl != 0, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

}  // extern "C"
