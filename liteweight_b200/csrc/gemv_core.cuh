// Persistent stream-K dequant GEMV core for B200 (sm_100a), shared by the
// plain matmul entry points and the fused decode-step kernels.
//
// out[m, n] = sum_k act[m, k] * W[n, k], W in liteweight's INT8 / packed INT4
// format (or fp16), each weight dequantized exactly as
// liteweight/quantize.py:30-43 / :102-128 do, fp32 accumulation, one fp16
// rounding (liteweight/quantize.py:60).
//
// Work decomposition. The weight matrix is cut into 16-row tiles; each tile's
// K extent is cut into chunks of 4 lanes x 16 bytes per row. The flattened
// (tile, chunk) sequence is divided into equal contiguous runs, one per warp
// of a persistent grid, so every warp streams the same number of bytes. A
// warp streams its run with a two-deep register double buffer (the loads of
// the next batch are in flight while the current one is dequantized and fed
// to the tensor core), so each SM keeps tens of KB of weight loads
// outstanding all the time. A tile that lies inside one warp's run is
// finished by that warp directly; a tile shared by several warps is combined
// deterministically: each contributor writes its fp32 fragment to its own
// slot of a scratch area and bumps the tile's counter; the last arriver sums
// the slots in slot order, applies the epilogue and resets the counter.
//
// Inner loop (per warp, per 16-byte piece and row pair): the codes are
// unpacked to exact fp16 integers with integer tricks, scaled with one fp16
// multiply (bit-identical to the reference's fp32 product rounded to fp16),
// and used directly from registers as the A operand of mma.sync.m16n8k16;
// the activation, staged once per CTA in shared memory in the element order
// the unpack produces, is the B operand; batch rows are the n8 columns.
//
// Prologues (activation staging): plain copy; RMSNorm of the residual stream
// (modeling_llama.py:63-68 rounding points); residual update + RMSNorm for
// tensor parallelism. Epilogues (per lane, rows g and g+8 of a tile are in
// the same lane): plain (+bias, +residual), RoPE + KV-cache append for the
// fused QKV projection, SwiGLU for the fused gate/up projection, raw fp32
// partial sums (tensor-parallel row split), logits + argmax.
#pragma once

#include "lw_common.cuh"

namespace lw {

template <int BITS>
struct WT;
template <>
struct WT<4> {
  static constexpr int E = 32;  // elements per 16-byte piece
};
template <>
struct WT<8> {
  static constexpr int E = 16;
};
template <>
struct WT<16> {
  static constexpr int E = 8;
};

enum { PRO_PLAIN = 0, PRO_NORM = 1, PRO_RESID_NORM = 2, PRO_PEER_RESID_NORM = 3 };
enum { EPI_PLAIN = 0, EPI_ROPE_KV = 1, EPI_SWIGLU = 2, EPI_F32 = 3, EPI_ARGMAX = 4, EPI_PEER_F32 = 5,
       EPI_PEER_ARGMAX = 6 };

template <int PRO>
constexpr bool kResidPro = PRO == PRO_RESID_NORM || PRO == PRO_PEER_RESID_NORM;
template <int EPI>
constexpr bool kPeerEpi = EPI == EPI_PEER_F32 || EPI == EPI_PEER_ARGMAX;

constexpr int kStreamThreads = 256;
#ifndef LW_STREAM_MIN_BLOCKS
#define LW_STREAM_MIN_BLOCKS 2
#endif
constexpr int kStreamMinBlocks = LW_STREAM_MIN_BLOCKS;   // CTAs per SM the register budget must allow
#ifndef LW_PREFETCH_BATCHES
#define LW_PREFETCH_BATCHES 4
#endif
constexpr int kPrefetch = LW_PREFETCH_BATCHES;   // batches of L2 prefetch ahead of the register loads
constexpr int kMaxM = 32;

struct StreamParams {
  // matmul
  const __half* act;       // [M][lda]; the residual stream x for the norm prologues
  const uint8_t* w;        // [N][K * BITS / 8]
  const __half* scales;    // [N][K / G]
  const __half* bias;      // [N] or null (EPI_PLAIN)
  const __half* residual;  // [M][ldo] or null (EPI_PLAIN): out = residual + y
  __half* out;             // [M][ldo]
  int lda, ldo;
  int M, N, K, G;
  int kchunks;  // chunks per tile row
  int tiles;    // ceil(N / 16)
  int per;      // chunks per warp
  int cp;       // staged activation row stride, halves
  int gshift;   // scale group of element k = k >> gshift (group size a power of two, or 31 when G == K)
  // prologue
  const __half* gamma;     // [K] RMSNorm weight
  float eps;
  const float* psum;       // PRO_RESID_NORM: fp32 [M][K] to add to the residual
  __half* x_out;           // PRO_RESID_NORM: updated residual, written by CTA 0
  // epilogue
  const __half* rope_cos;  // [max_seq][head_dim] fp16
  const __half* rope_sin;
  const int* pos;          // device: position written this step
  int head_dim, n_q_heads, n_kv_heads, max_seq;
  __half* q_out;           // [M][n_q_heads * head_dim]
  __half* k_cache;         // [M][n_kv_heads][max_seq][head_dim] (this layer)
  __half* v_cache;
  float* out_f32;          // EPI_F32: [M][ldo]
  unsigned long long* argmax_keys;  // EPI_ARGMAX: [M], zero before the launch
  int argmax_offset;       // EPI_ARGMAX: index of row 0 in the full vocabulary (vocab shards)
  // split-tile combination (scratch)
  float* slots;            // [tiles][max_slots][32 lanes][4 * MT]
  int* counters;           // [tiles], zero before the first launch, left zero
  int max_slots;
  int ring_slots;          // gemv_tma_kernel: shared-memory slots per warp
  const int* seq;          // prompt chunk (EPI_ROPE_KV): row m is position *pos + m of sequence *seq
  // tensor-parallel exchange, consumer (PRO_PEER_RESID_NORM): flagged words
  int in_world, in_tag, in_tags;
  const unsigned long long* in_src;    // local [in_world][M][K]
  const int* in_step;                  // decode steps completed
  int* in_error;
  long long in_timeout_ns;
  int* in_slice_flags;                 // non-null: the CTAs reduce slices of K (see stage_activation)
  // tensor-parallel exchange, producer (EPI_PEER_*)
  int out_world, out_rank, out_tag, out_tags;
  const int* out_step;
  unsigned long long* out_dst[kMaxRanks];  // rank d's receive buffer; this rank's words at out_rank * M * ldo (or * M)
  int* out_arrivals;                   // EPI_PEER_ARGMAX: local, zero, left zero
};

LW_DEV uint32_t bcast_h(const __half* p) {
  const unsigned short s = __ldg(reinterpret_cast<const unsigned short*>(p));
  return (uint32_t)s | ((uint32_t)s << 16);
}

// Activation fragments come from shared memory rows arow[mt] (lane row g + 8*mt,
// clamped to the last real row: batch columns >= M are computed and dropped,
// so they may read any valid data). Out-of-range weight pieces meet the zero
// padding of the staged activation, so no operand needs zeroing.
template <int MT>
LW_DEV uint4 act16(const __half* const (&arow)[MT], int mt, int off) {
  return *reinterpret_cast<const uint4*>(arow[mt] + off);
}

// Exact dequant: fp16(code) * fp16(scale) in fp16 (one rounding of the exact
// product, bit-identical to liteweight's dequantize), fp32 tensor-core sums.
template <int BITS, int MT>
LW_DEV void gemv_piece(float (&acc)[MT][4], const uint4& qa, const uint4& qb, uint32_t sa, uint32_t sb,
                       const __half* const (&arow)[MT], int off) {
  const uint32_t* a32 = reinterpret_cast<const uint32_t*>(&qa);
  const uint32_t* b32 = reinterpret_cast<const uint32_t*>(&qb);
  if constexpr (BITS == 4) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t A[4], B[4];
      unpack_int4_word(a32[w], A);
      unpack_int4_word(b32[w], B);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        A[i] = hmul2_rn(A[i], sa);
        B[i] = hmul2_rn(B[i], sb);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint4 av = act16(arow, mt, off + w * 32);
        mma16816(acc[mt], A[0], B[0], A[1], B[1], av.x, av.y);
        mma16816(acc[mt], A[2], B[2], A[3], B[3], av.z, av.w);
      }
    }
  } else if constexpr (BITS == 8) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint4 av[MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) av[mt] = act16(arow, mt, off + j * 32);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t A[2], B[2];
        dequant_int8_word(a32[2 * j + h], A);
        dequant_int8_word(b32[2 * j + h], B);
        A[0] = hmul2_rn(A[0], sa);
        A[1] = hmul2_rn(A[1], sa);
        B[0] = hmul2_rn(B[0], sb);
        B[1] = hmul2_rn(B[1], sb);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          mma16816(acc[mt], A[0], B[0], A[1], B[1], h ? av[mt].z : av[mt].x, h ? av[mt].w : av[mt].y);
      }
    }
  } else {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const uint4 av = act16(arow, mt, off);
      mma16816(acc[mt], qa.x, qb.x, qa.y, qb.y, av.x, av.y);
      mma16816(acc[mt], qa.z, qb.z, qa.w, qb.w, av.z, av.w);
    }
  }
}

// Unscaled piece: exact integer codes times activations, accumulated in fp32
// by the tensor core; the caller multiplies the chunk sum by the row scale.
template <int BITS, int MT>
LW_DEV void gemv_piece_codes(float (&acc)[MT][4], const uint4& qa, const uint4& qb,
                             const __half* const (&arow)[MT], int off) {
  const uint32_t* a32 = reinterpret_cast<const uint32_t*>(&qa);
  const uint32_t* b32 = reinterpret_cast<const uint32_t*>(&qb);
  if constexpr (BITS == 4) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t A[4], B[4];
      unpack_int4_word(a32[w], A);
      unpack_int4_word(b32[w], B);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint4 av = act16(arow, mt, off + w * 32);
        mma16816(acc[mt], A[0], B[0], A[1], B[1], av.x, av.y);
        mma16816(acc[mt], A[2], B[2], A[3], B[3], av.z, av.w);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint4 av[MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) av[mt] = act16(arow, mt, off + j * 32);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t A[2], B[2];
        dequant_int8_word(a32[2 * j + h], A);
        dequant_int8_word(b32[2 * j + h], B);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          mma16816(acc[mt], A[0], B[0], A[1], B[1], h ? av[mt].z : av[mt].x, h ? av[mt].w : av[mt].y);
      }
    }
  }
}

// Total order on fp16 values as unsigned keys (larger value -> larger key).
LW_DEV uint32_t f16_order_key(__half h) {
  const uint32_t u = __half_as_ushort(h);
  return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
}

LW_DEV float silu_f32(float x) { return x / (1.0f + expf(-x)); }

// Epilogue for one tile: v[mt][i] holds D(row, col) with rows n_lo = 16*tile +
// g (i = 0, 1) and n_hi = n_lo + 8 (i = 2, 3), cols m = 8*mt + 2t (+1 for odd i).
// g is the tile row of the lane's lower row: lane / 4 unless the kernel maps
// its lanes to the tile's rows in another order (gemv_ring.cuh).
template <int MT, int EPI>
LW_DEV void finish_tile(const StreamParams& p, int tile, const float (&v)[MT][4], int lane, uint32_t flag,
                        int g) {
  const int t = lane & 3;
  const int n_lo = tile * 16 + g, n_hi = n_lo + 8;
  if constexpr (EPI == EPI_PLAIN || EPI == EPI_F32 || EPI == EPI_PEER_F32) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = mt * 8 + 2 * t + (i & 1);
        const int n = (i < 2) ? n_lo : n_hi;
        if (m < p.M && n < p.N) {
          if constexpr (EPI == EPI_F32) {
            p.out_f32[(size_t)m * p.ldo + n] = v[mt][i];
          } else if constexpr (EPI == EPI_PEER_F32) {
            // straight into every rank's receive buffer (peer stores over NVLink)
            const unsigned long long word = ((unsigned long long)flag << 32) | __float_as_uint(v[mt][i]);
            const size_t at = ((size_t)p.out_rank * p.M + m) * p.ldo + n;
#pragma unroll
            for (int d = 0; d < kMaxRanks; ++d)
              if (d < p.out_world) st_relaxed_sys_u64(p.out_dst[d] + at, word);
          } else {
            float y = r16(v[mt][i]);
            if (p.bias) y = r16(y + __half2float(p.bias[n]));
            if (p.residual) y = r16(__half2float(p.residual[(size_t)m * p.ldo + n]) + y);
            p.out[(size_t)m * p.ldo + n] = __float2half_rn(y);
          }
        }
      }
  } else if constexpr (EPI == EPI_ROPE_KV) {
    // Rows of the fused q|k|v projection are stored so that tile rows g and
    // g+8 are head dims d and d + hd/2 (the rotate_half partners).
    const int hd = p.head_dim;
    const int head = (tile * 16) / hd;
    const int jt = tile % (hd / 16);
    const int d_lo = 8 * jt + g, d_hi = d_lo + hd / 2;
    const int pos0 = *p.pos;
    const int seq = p.seq ? *p.seq : -1;   // prompt chunk: rows are positions of one sequence
    const int nq = p.n_q_heads, nkv = p.n_kv_heads;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int m = mt * 8 + 2 * t + c;
        if (m >= p.M || n_lo >= p.N) continue;
        const int pos = seq >= 0 ? pos0 + m : pos0;
        const int row = seq >= 0 ? seq : m;   // KV-cache sequence
        const float y_lo = r16(v[mt][c]), y_hi = r16(v[mt][2 + c]);
        float o_lo = y_lo, o_hi = y_hi;
        if (head < nq + nkv) {
          // modeling_llama.py:161-162: q*cos + rotate_half(q)*sin, fp16 after each op
          const float c_lo = __half2float(p.rope_cos[(size_t)pos * hd + d_lo]);
          const float c_hi = __half2float(p.rope_cos[(size_t)pos * hd + d_hi]);
          const float s_lo = __half2float(p.rope_sin[(size_t)pos * hd + d_lo]);
          const float s_hi = __half2float(p.rope_sin[(size_t)pos * hd + d_hi]);
          o_lo = r16(r16(y_lo * c_lo) + r16(-y_hi * s_lo));
          o_hi = r16(r16(y_hi * c_hi) + r16(y_lo * s_hi));
        }
        __half* dst;
        if (head < nq) {
          dst = p.q_out + (size_t)m * nq * hd + (size_t)head * hd;
        } else if (head < nq + nkv) {
          dst = p.k_cache + (((size_t)row * nkv + (head - nq)) * p.max_seq + pos) * hd;
        } else {
          dst = p.v_cache + (((size_t)row * nkv + (head - nq - nkv)) * p.max_seq + pos) * hd;
        }
        dst[d_lo] = __float2half_rn(o_lo);
        dst[d_hi] = __float2half_rn(o_hi);
      }
  } else if constexpr (EPI == EPI_SWIGLU) {
    // Tile rows g = gate row 8*tile + g, g+8 = the matching up row.
    const int i_out = tile * 8 + g;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int m = mt * 8 + 2 * t + c;
        if (m >= p.M || n_lo >= p.N) continue;
        // modeling_llama.py:183: act_fn(gate) * up, fp16 after each op
        const float gt = r16(v[mt][c]), up = r16(v[mt][2 + c]);
        const float a = r16(silu_f32(gt));
        p.out[(size_t)m * p.ldo + i_out] = __float2half_rn(a * up);
      }
  } else if constexpr (EPI == EPI_ARGMAX || EPI == EPI_PEER_ARGMAX) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int m = mt * 8 + 2 * t + c;
        unsigned long long best = 0ull;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int n = h ? n_hi : n_lo;
          if (m < p.M && n < p.N) {
            const __half y = __float2half_rn(v[mt][2 * h + c]);
            p.out[(size_t)m * p.ldo + n] = y;
            const unsigned long long key =
                ((unsigned long long)f16_order_key(y) << 32) |
                (unsigned long long)(0xFFFFFFFFu - (uint32_t)(n + p.argmax_offset));
            best = key > best ? key : best;
          }
        }
        // lanes with the same t share the column: reduce over g
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
          best = other > best ? other : best;
        }
        if (g == 0 && m < p.M && best) atomicMax(p.argmax_keys + m, best);
      }
  }
}

// Stages the activation (M rows, K padded to whole chunks) into act_s in the
// element order the unpack produces (lane order), applying the prologue:
// RMSNorm (modeling_llama.py:65-68 rounding points), optionally after adding
// the all-reduced partial sum to the residual (CTA 0 writes the new residual).
// A thread issues the loads of up to kStageBatch of its 16-byte groups before
// storing any (each load is one L2 round trip after griddepcontrol.wait). The
// sum of squares is reduced per warp, then over the warps in warp order (the
// same fp32 sums on every run). ssq holds kMaxM * (NT / 32) floats. Called by
// all NT threads of the CTA; ends with a CTA barrier.
constexpr int kStageBatch = 8;

// Barrier over the NT threads that stage the activation: the whole CTA
// (BAR == 0), or named barrier BAR when other warps of the CTA do not take part.
template <int BAR, int NT>
LW_DEV void stage_sync() {
  if constexpr (BAR == 0) {
    __syncthreads();
  } else {
    asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
  }
}

template <int BITS, int PRO, int NT, int BAR = 0>
LW_DEV void stage_activation(const StreamParams& p, __half* act_s, const __half* gam_s, float* ssq, uint32_t in_flag,
                             WaitBudget& wb) {
  constexpr int E = WT<BITS>::E;
  constexpr int KC = 4 * E;
  constexpr int NW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = p.kchunks;
  const int groups8 = C * KC / 8;
  auto store = [&](int m, int k, uint4 v) {
    if constexpr (BITS == 4) v = perm_int4_pairs(v);
    const int c = k / KC, r = k - c * KC, tt = r / E, j = (r - tt * E) / 8;
    sts128(act_s + (size_t)m * p.cp + c * KC + (j * 4 + tt) * 8, v);
  };
  auto square_sum = [&](const uint4& v, float& sq) {
    const __half* hv = reinterpret_cast<const __half*>(&v);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float f = __half2float(hv[e]);
      sq = fmaf(f, f, sq);
    }
  };
  // Cooperative exchange (in_slice_flags): CTA b sums slice b of K (groups of
  // 8 elements) over the ranks - one (group, rank) word block per thread, then
  // the same rank-order sums as below - writes the new residual slice to x_out
  // and flags it; every CTA then reads the whole new residual back from x_out.
  // The same values, in the same order, as each CTA summing everything itself.
  bool coop = false;
  if constexpr (PRO == PRO_PEER_RESID_NORM) {
    const int G8 = (p.K + 7) / 8;
    const int per = (G8 + (int)gridDim.x - 1) / (int)gridDim.x;
    // (the scratch, M x per x world x 32 bytes, must fit the staged activation, M x cp x 2)
    coop = p.in_slice_flags != nullptr && gridDim.x <= kSliceFlagsMax && per * p.in_world * 16 <= p.cp;
    if (coop) {
      const int ga = (int)blockIdx.x * per, ng = max(0, min(G8, ga + per) - ga);
      const int W = p.in_world;
      const size_t rstride = (size_t)p.M * p.K;
      float* part = reinterpret_cast<float*>(act_s);   // scratch until the staging below: [M][ng][W][8]
      for (int t = tid; t < p.M * ng * W; t += NT) {
        const int m = t / (ng * W), rem = t - m * ng * W, gi = rem / W, r = rem - gi * W;
        float ps[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) ps[e] = 0.f;
        add_flagged8<1>(p.in_src + r * rstride + (size_t)m * p.K + (size_t)(ga + gi) * 8, rstride, 1, in_flag, ps,
                        wb, p.in_timeout_ns, p.in_error);
#pragma unroll
        for (int e = 0; e < 8; ++e) part[(size_t)t * 8 + e] = ps[e];
      }
      stage_sync<BAR, NT>();
      for (int t = tid; t < p.M * ng; t += NT) {
        const int m = t / ng, gi = t - m * ng, k = (ga + gi) * 8;
        float ps[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) ps[e] = 0.f;
        for (int r = 0; r < W; ++r)
#pragma unroll
          for (int e = 0; e < 8; ++e) ps[e] += part[((size_t)t * W + r) * 8 + e];
        uint4 v = ldg_nc(p.act + (size_t)m * p.lda + k);
        __half* hv = reinterpret_cast<__half*>(&v);
#pragma unroll
        for (int e = 0; e < 8; ++e) hv[e] = __float2half_rn(__half2float(hv[e]) + r16(ps[e]));
        *reinterpret_cast<uint4*>(p.x_out + (size_t)m * p.lda + k) = v;
      }
      stage_sync<BAR, NT>();
      if (tid == 0) {
        __threadfence();   // the slice is visible before its flag
        st_volatile_u32(reinterpret_cast<unsigned int*>(p.in_slice_flags) + blockIdx.x, in_flag);
      }
      for (int c = tid; c < (int)gridDim.x; c += NT) {
        while (ld_volatile_u32(reinterpret_cast<const unsigned int*>(p.in_slice_flags) + c) != in_flag)
          if (!wb.keep_waiting(p.in_timeout_ns, p.in_error)) break;
      }
      __threadfence();
      stage_sync<BAR, NT>();
    }
  }
  for (int m = 0; m < p.M; ++m) {
    float sq = 0.f;
    if (coop) {
      for (int i = tid; i < groups8; i += NT) {
        const int k = i * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (k < p.K) {
          v = __ldcg(reinterpret_cast<const uint4*>(p.x_out + (size_t)m * p.lda + k));
          square_sum(v, sq);
        }
        store(m, k, v);
      }
    } else if constexpr (PRO == PRO_PEER_RESID_NORM) {
      for (int i = tid; i < groups8; i += NT) {
        const int k = i * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (k < p.K) {
          v = ldg_nc(p.act + (size_t)m * p.lda + k);
          // the all-reduce itself: the world partials, summed in rank order,
          // each word read once it carries this step's flag; then
          // x_new = fp16(x + fp16(sum))
          float ps[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) ps[e] = 0.f;
          const size_t rstride = (size_t)p.M * p.K;
          for (int r = 0; r < p.in_world; r += 2)
            add_flagged8<2>(p.in_src + r * rstride + (size_t)m * p.K + k, rstride, min(2, p.in_world - r), in_flag,
                            ps, wb, p.in_timeout_ns, p.in_error);
          __half* hv = reinterpret_cast<__half*>(&v);
#pragma unroll
          for (int e = 0; e < 8; ++e) hv[e] = __float2half_rn(__half2float(hv[e]) + r16(ps[e]));
          if (blockIdx.x == 0) *reinterpret_cast<uint4*>(p.x_out + (size_t)m * p.lda + k) = v;
          square_sum(v, sq);
        }
        store(m, k, v);
      }
    } else {
      for (int i0 = tid; i0 < groups8; i0 += NT * kStageBatch) {
        uint4 v[kStageBatch];
        float4 pa[kStageBatch], pb[kStageBatch];
#pragma unroll
        for (int b = 0; b < kStageBatch; ++b) {
          const int k = (i0 + b * NT) * 8;
          v[b] = make_uint4(0, 0, 0, 0);
          if (k < p.K) {
            v[b] = ldg_nc(p.act + (size_t)m * p.lda + k);
            if constexpr (PRO == PRO_RESID_NORM) {
              pa[b] = __ldg(reinterpret_cast<const float4*>(p.psum + (size_t)m * p.K + k));
              pb[b] = __ldg(reinterpret_cast<const float4*>(p.psum + (size_t)m * p.K + k + 4));
            }
          }
        }
#pragma unroll
        for (int b = 0; b < kStageBatch; ++b) {
          const int i = i0 + b * NT, k = i * 8;
          if (i >= groups8) break;
          if (k < p.K) {
            if constexpr (PRO == PRO_RESID_NORM) {
              // x_new = fp16(x + fp16(psum)) (residual add of the all-reduced partial)
              const float ps[8] = {pa[b].x, pa[b].y, pa[b].z, pa[b].w, pb[b].x, pb[b].y, pb[b].z, pb[b].w};
              __half* hv = reinterpret_cast<__half*>(&v[b]);
#pragma unroll
              for (int e = 0; e < 8; ++e) hv[e] = __float2half_rn(__half2float(hv[e]) + r16(ps[e]));
              if (blockIdx.x == 0) *reinterpret_cast<uint4*>(p.x_out + (size_t)m * p.lda + k) = v[b];
            }
            if constexpr (PRO != PRO_PLAIN) square_sum(v[b], sq);
          }
          store(m, k, v[b]);
        }
      }
    }
    if constexpr (PRO != PRO_PLAIN) {
      sq = warp_sum(sq);
      if (lane == 0) ssq[m * NW + warp] = sq;
    }
  }
  if constexpr (PRO != PRO_PLAIN) {
    stage_sync<BAR, NT>();
    // modeling_llama.py:65-68: h = weight * fp16(x * rsqrt(mean(x^2) + eps))
    for (int m = 0; m < p.M; ++m) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) tot += ssq[m * NW + w];
      const float rstd = 1.0f / sqrtf(tot / (float)p.K + p.eps);
      for (int i = tid; i < groups8; i += NT) {
        const int k = i * 8;
        if (k >= p.K) continue;
        const int c = k / KC, r = k - c * KC, tt = r / E, j = (r - tt * E) / 8;
        __half* dst = act_s + (size_t)m * p.cp + c * KC + (j * 4 + tt) * 8;
        uint4 v = lds128(dst);
        uint4 gm = lds128(gam_s + k);
        if constexpr (BITS == 4) gm = perm_int4_pairs(gm);
        __half* hv = reinterpret_cast<__half*>(&v);
        const __half* hg = reinterpret_cast<const __half*>(&gm);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          hv[e] = __float2half_rn(__half2float(hg[e]) * r16(__half2float(hv[e]) * rstd));
        sts128(dst, v);
      }
    }
  }
  stage_sync<BAR, NT>();
}

// Copies the RMSNorm weight into shared memory (natural order). It does not
// depend on the previous kernel, so this runs before griddepcontrol.wait and
// its DRAM latency overlaps the previous kernel's tail. The copy is read after
// the first barrier of stage_activation.
template <int PRO, int NT>
LW_DEV void stage_gamma(const StreamParams& p, __half* gam_s) {
  if constexpr (PRO != PRO_PLAIN) {
    const int groups8 = (p.K + 7) / 8;
    for (int i = threadIdx.x; i < groups8; i += NT) sts128(gam_s + i * 8, ldg_nc(p.gamma + i * 8));
  }
}

// A warp's tile segment [seg_c0, end_c) is done: a whole tile runs the
// epilogue directly; a split tile writes its fp32 fragment to its slot, and
// the last contributor sums the slots in slot order and runs the epilogue.
template <int MT, int EPI>
LW_DEV void flush_tile(const StreamParams& p, int tile, int seg_c0, int end_c, int wid, const float (&acc)[MT][4],
                       int lane, uint32_t out_flag) {
  const int C = p.kchunks;
  const bool whole = (seg_c0 == 0) && (end_c == C);
  if (whole) {
    finish_tile<MT, EPI>(p, tile, acc, lane, out_flag, lane >> 2);
    return;
  }
  const int first = (tile * C) / p.per;
  const int last = ((tile + 1) * C - 1) / p.per;
  const int slot = wid - first, nslot = last - first + 1;
  float* base = p.slots + (size_t)tile * p.max_slots * 32 * 4 * MT;
  float4* mine = reinterpret_cast<float4*>(base + ((size_t)slot * 32 + lane) * 4 * MT);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) mine[mt] = make_float4(acc[mt][0], acc[mt][1], acc[mt][2], acc[mt][3]);
  __threadfence();
  __syncwarp();   // every lane's slot is stored and fenced before lane 0 counts the warp in
  int old = 0;
  if (lane == 0) old = atomicAdd(p.counters + tile, 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old == nslot - 1) {
    __threadfence();
    float sum[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) sum[mt][0] = sum[mt][1] = sum[mt][2] = sum[mt][3] = 0.f;
    for (int s = 0; s < nslot; ++s) {
      const float4* src = reinterpret_cast<const float4*>(base + ((size_t)s * 32 + lane) * 4 * MT);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const float4 f = __ldcg(src + mt);
        sum[mt][0] += f.x;
        sum[mt][1] += f.y;
        sum[mt][2] += f.z;
        sum[mt][3] += f.w;
      }
    }
    finish_tile<MT, EPI>(p, tile, sum, lane, out_flag, lane >> 2);
    if (lane == 0) p.counters[tile] = 0;
  }
}

// A cursor over a warp's run of flattened (tile, chunk) work.
struct RunCursor {
  int t, c, left;
  LW_DEV int take(int U, int C) {   // next batch: up to U chunks, never crossing a tile
    int n = min(U, min(C - c, left));
    if (n <= 0) return 0;
    left -= n;
    c += n;
    if (c == C) {
      c = 0;
      ++t;
    }
    return n;
  }
};

// FOLD: every 4-lane chunk lies in one scale group (G a multiple of the chunk),
// so the codes are summed unscaled per chunk and the sum is scaled once in fp32.
// Otherwise every piece is dequantized exactly (fp16 code * scale) first.
template <int BITS, int MT, int U, int PRO, int EPI, bool FOLD>
__global__ void __launch_bounds__(kStreamThreads, kStreamMinBlocks) gemv_stream_kernel(const StreamParams p) {
  constexpr int E = WT<BITS>::E;
  constexpr int KC = 4 * E;
  constexpr bool SCALED = BITS < 16;
  extern __shared__ __align__(16) uint8_t smem[];
  __half* act_s = reinterpret_cast<__half*>(smem);
  __half* gam_s = act_s + (size_t)p.M * p.cp;   // norm prologues: gamma [K], after the staged rows
  __shared__ float ssq[kMaxM * (kStreamThreads / 32)];

  const int tid = threadIdx.x, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wid = blockIdx.x * (kStreamThreads / 32) + (tid >> 5);
  const int C = p.kchunks;
  const int total = p.tiles * C;
  const int g0 = min(total, wid * p.per), g1 = min(total, g0 + p.per);
  const size_t rowbytes = (size_t)p.K * BITS / 8;
  const int ngroups = SCALED ? p.K / p.G : 1;

  // ---- the warp's run [g0, g1) of flattened (tile, chunk) work, cut into
  // tile segments. A segment sets its row, scale and activation pointers once
  // and steps through batches of U chunks; loads run two batches ahead of the
  // tensor cores (register double buffer) and L2 prefetches kPrefetch batches
  // ahead of the loads. Rows past N are clamped to N-1 (computed, never
  // stored). Rows are whole 64-byte chunks (the host routes other shapes to
  // the generic kernel), so no piece needs clamping; only a segment's last
  // batch may hold fewer than U chunks.
  const unsigned short* sbase = reinterpret_cast<const unsigned short*>(p.scales);
  const int toff = FOLD ? 0 : t * E;

  int s_tile = g0 / max(C, 1);
  int s_c0 = g0 - s_tile * C;
  int s_len = min(C - s_c0, g1 - g0);
  const uint8_t *w0 = nullptr, *w1 = nullptr;          // the lane's piece of chunk s_c0, rows g / g+8
  const unsigned short *sc0 = nullptr, *sc1 = nullptr;  // scale rows g / g+8
  auto seg_setup = [&]() {
    const int r0 = min(s_tile * 16 + g, p.N - 1), r1 = min(s_tile * 16 + g + 8, p.N - 1);
    const size_t piece = ((size_t)s_c0 * 4 + t) * 16;
    w0 = p.w + (size_t)r0 * rowbytes + piece;
    w1 = p.w + (size_t)r1 * rowbytes + piece;
    if constexpr (SCALED) {
      sc0 = sbase + (size_t)r0 * ngroups;
      sc1 = sbase + (size_t)r1 * ngroups;
    }
  };

  uint4 qa0[U], qb0[U], qa1[U], qb1[U];
  uint32_t sa0[U], sb0[U], sa1[U], sb1[U];
  // batch b of the current segment: chunks s_c0 + b*U + u (u < n)
  auto load = [&](int b, int n, uint4(&qa)[U], uint4(&qb)[U], uint32_t(&sa)[U], uint32_t(&sb)[U]) {
    const size_t off = (size_t)b * (U * 64);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (u < n) {
        qa[u] = ldg_stream(w0 + off + u * 64);
        qb[u] = ldg_stream(w1 + off + u * 64);
        if constexpr (SCALED) {
          const int grp = ((s_c0 + b * U + u) * KC + toff) >> p.gshift;
          const uint32_t h0 = __ldg(sc0 + grp), h1 = __ldg(sc1 + grp);
          if constexpr (FOLD) {
            sa[u] = __float_as_uint(__half2float(__ushort_as_half((unsigned short)h0)));
            sb[u] = __float_as_uint(__half2float(__ushort_as_half((unsigned short)h1)));
          } else {
            sa[u] = h0 | (h0 << 16);
            sb[u] = h1 | (h1 << 16);
          }
        }
      }
    }
  };

  // L2 prefetch cursor over the whole run: each lane takes one 64-byte line of
  // a batch (row lane % 16, chunk + lane / 16), crossing into the next tile.
  int pf_t = s_tile, pf_c = s_c0, pf_left = g1 - g0;
  auto pf_skip = [&]() {
    pf_left -= U;
    pf_c += U;
    if (pf_c >= C) {
      pf_c -= C;
      ++pf_t;
    }
  };
  auto prefetch_next = [&]() {
    if (pf_left <= 0) return;
    int ch = pf_c + (lane >> 4), tl = pf_t;
    if (ch >= C) {
      ch -= C;
      ++tl;
    }
    if ((lane >> 4) < pf_left) {
      const int row = min(tl * 16 + (lane & 15), p.N - 1);
      prefetch_l2_line(p.w + (size_t)row * rowbytes + (size_t)ch * 64);
    }
    pf_skip();
  };

  // Weights do not depend on the previous kernel: start streaming them first.
  int nb = (s_len + U - 1) / U;
  if (s_len > 0) {
    seg_setup();
    load(0, min(U, s_len), qa0, qb0, sa0, sb0);
    if (nb > 1) load(1, min(U, s_len - U), qa1, qb1, sa1, sb1);
  }
  pf_skip();   // the two batches loaded directly
  pf_skip();
#pragma unroll 1
  for (int i = 0; i < kPrefetch; ++i) prefetch_next();

  stage_gamma<PRO, kStreamThreads>(p, gam_s);
  pdl_wait();
  // Let the next kernel's CTAs launch as soon as this one's exit: they take
  // the SM slots freed by CTAs that finish early and stream their weights
  // (which do not depend on this kernel) while the last CTAs here finish.
  pdl_launch_dependents();

  // the previous kernels are complete: the step number is final
  uint32_t in_flag = 0, out_flag = 0;
  if constexpr (PRO == PRO_PEER_RESID_NORM) in_flag = exchange_flag(*p.in_step, p.in_tag, p.in_tags);
  if constexpr (kPeerEpi<EPI>) out_flag = exchange_flag(*p.out_step, p.out_tag, p.out_tags);
  WaitBudget wb;

  stage_activation<BITS, PRO, kStreamThreads>(p, act_s, gam_s, ssq, in_flag, wb);

  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
  const __half* arow[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) arow[mt] = act_s + (size_t)min(g + 8 * mt, p.M - 1) * p.cp + t * 8;

  // batch b of the segment, its first n chunks (a full batch has n == U)
  auto compute = [&](int b, int n, const uint4(&qa)[U], const uint4(&qb)[U], const uint32_t(&sa)[U],
                     const uint32_t(&sb)[U]) {
    const int off0 = (s_c0 + b * U) * KC;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (u < n) {
        const int off = off0 + u * KC;
        if constexpr (SCALED && FOLD) {
          float dc[MT][4];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) dc[mt][0] = dc[mt][1] = dc[mt][2] = dc[mt][3] = 0.f;
          gemv_piece_codes<BITS, MT>(dc, qa[u], qb[u], arow, off);
          const float s0f = __uint_as_float(sa[u]), s1f = __uint_as_float(sb[u]);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            acc[mt][0] = fmaf(dc[mt][0], s0f, acc[mt][0]);
            acc[mt][1] = fmaf(dc[mt][1], s0f, acc[mt][1]);
            acc[mt][2] = fmaf(dc[mt][2], s1f, acc[mt][2]);
            acc[mt][3] = fmaf(dc[mt][3], s1f, acc[mt][3]);
          }
        } else {
          gemv_piece<BITS, MT>(acc, qa[u], qb[u], sa[u], sb[u], arow, off);
        }
      }
    }
  };

  int done = 0;   // chunks of the run finished in earlier segments
  while (s_len > 0) {
    const int nfull = s_len / U;   // batches 0 .. nfull-1 hold U chunks; batch nfull the rest
    const int last = s_len - nfull * U;
    for (int b = 0;; b += 2) {
      if (b < nfull) compute(b, U, qa0, qb0, sa0, sb0);
      else compute(b, last, qa0, qb0, sa0, sb0);
      if (b + 2 < nb) {
        if (b + 2 < nfull) load(b + 2, U, qa0, qb0, sa0, sb0);
        else load(b + 2, last, qa0, qb0, sa0, sb0);
        prefetch_next();
      }
      if (b + 1 >= nb) break;
      if (b + 1 < nfull) compute(b + 1, U, qa1, qb1, sa1, sb1);
      else compute(b + 1, last, qa1, qb1, sa1, sb1);
      if (b + 3 < nb) {
        if (b + 3 < nfull) load(b + 3, U, qa1, qb1, sa1, sb1);
        else load(b + 3, last, qa1, qb1, sa1, sb1);
        prefetch_next();
      }
      if (b + 2 >= nb) break;
    }
    // the next segment (the next tile from its chunk 0) starts loading before
    // this one's partial sums are written out
    const int f_tile = s_tile, f_c0 = s_c0, f_end = s_c0 + s_len;
    done += s_len;
    ++s_tile;
    s_c0 = 0;
    s_len = min(C, (g1 - g0) - done);
    nb = (s_len + U - 1) / U;
    if (s_len > 0) {
      seg_setup();
      load(0, min(U, s_len), qa0, qb0, sa0, sb0);
      if (nb > 1) load(1, min(U, s_len - U), qa1, qb1, sa1, sb1);
      prefetch_next();
      prefetch_next();
    }
    flush_tile<MT, EPI>(p, f_tile, f_c0, f_end, wid, acc, lane, out_flag);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
  }
  if constexpr (EPI == EPI_PEER_ARGMAX) {
    // The last CTA to finish (every CTA's atomicMax is then in the local keys)
    // sends this rank's keys to every rank as flagged words.
    __shared__ int s_last;
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      s_last = atomicAdd(p.out_arrivals, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      const unsigned long long f16 = (unsigned long long)exchange_flag16(out_flag) << 48;
      for (int m = tid; m < p.M; m += kStreamThreads) {
        const unsigned long long word = (__ldcg(p.argmax_keys + m) & 0xFFFFFFFFFFFFull) | f16;
#pragma unroll
        for (int d = 0; d < kMaxRanks; ++d)
          if (d < p.out_world) st_relaxed_sys_u64(p.out_dst[d] + (size_t)p.out_rank * p.M + m, word);
      }
      if (tid == 0) *p.out_arrivals = 0;
    }
  }
}

}  // namespace lw
