// Prompt-chunk GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// out[m][n] for the M rows of a prompt chunk: D[n][m] = sum_k W[n][k] * X[m][k]
// with W the liteweight-packed weight, dequantized exactly (fp16(code * scale),
// liteweight/quantize.py:30-43, :102-128), and X the fp16 activation.
//
// One CTA per 128-row weight tile. The K dimension is cut into blocks of 64;
// each block is one stage of a 4-stage shared-memory pipeline holding the
// A operand (128 weight rows x 64, fp16) and the B operand (Mpad activation
// rows x 64, fp16), both K-major in the 128-byte-swizzled layout the tensor
// core reads (16-byte chunk c of row r stored at chunk c ^ (r & 7); rows 128
// bytes apart, 8-row groups 1024 bytes apart). All 256 threads fill a stage
// (weights: load, unpack, scale, reorder; activations: copy) and arrive on its
// "full" mbarrier; one elected thread waits for it and issues four
// tcgen05.mma (K = 16 each) accumulating into tensor memory (128 lanes = tile
// rows, Mpad fp32 columns = activation rows), then tcgen05.commit to the
// stage's "empty" mbarrier, which frees the stage for the producers. After the
// last block a final commit signals the epilogue: every warp reads its 32
// lanes x every other 32-column chunk with tcgen05.ld and applies the epilogue (residual
// add / SwiGLU / RoPE + KV-cache append, the GEMV kernels' rounding points).
//
// Every mbarrier wait is bounded (global timer): on expiry the kernel records
// LW_ERR_TIMEOUT, still drains, reads and releases its tensor memory, and
// returns; results of that launch are then invalid.
#include "gemv_host.cuh"

namespace lw {

constexpr int kTcThreads = 256;
constexpr int kTcStages = 4;
constexpr int kTcTileN = 128;     // weight rows per CTA (UMMA M)
constexpr int kTcKBlock = 64;     // K per stage (one 128-byte swizzle row of fp16)
constexpr int kTcMaxM = 256;      // activation rows (UMMA N)
constexpr long long kTcWaitNs = 500000000;

struct TcGemmParams {
  const uint8_t* w;
  const __half* scales;
  const __half* act;
  __half* out;
  const __half* residual;
  int lda, ldo;
  int M, Mpad, N, K, G, gshift, kblocks;
  uint32_t idesc;
  int tmem_cols;
  // rope / kv
  const __half* rope_cos;
  const __half* rope_sin;
  const int* pos;
  const int* seq;
  int head_dim, n_q_heads, n_kv_heads, max_seq;
  __half* q_out;
  __half* k_cache;
  __half* v_cache;
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

LW_DEV uint32_t swz(int row, int chunk) { return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4)); }

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

template <int BITS, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const TcGemmParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ __align__(8) unsigned long long bar_full[kTcStages], bar_empty[kTcStages], bar_done;
  __shared__ uint32_t tmem_base_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * kTcTileN;
  const uint32_t a_bytes = kTcTileN * 128;         // 16 KB
  const uint32_t b_bytes = (uint32_t)p.Mpad * 128;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  // stages on 1024-byte boundaries (the swizzle pattern follows address bits 4-9)
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - smem_u32(smem_raw));

  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(smem_u32(&bar_full[s]), kTcThreads);
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    mbar_init(smem_u32(&bar_done), 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_base_s), (uint32_t)p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  pdl_wait();
  pdl_launch_dependents();

  const size_t rowbytes = (size_t)p.K * BITS / 8;
  const int ngroups = p.K / p.G;
  // producer roles: weight row r = tid / 2, half h = tid & 1 (32 codes = 4 chunks)
  const int ar = tid >> 1, ah = tid & 1;
  const int wrow = min(n0 + ar, p.N - 1);
  const uint8_t* wsrc = p.w + (size_t)wrow * rowbytes;
  const unsigned short* ssrc = reinterpret_cast<const unsigned short*>(p.scales) + (size_t)wrow * ngroups;
  bool live = true;

  // Each thread's global loads of a k-block go to registers one block ahead of
  // their use (dequantize / store), so the load latency overlaps a block of work.
  constexpr int kBMax = kTcMaxM * 8 / kTcThreads;   // activation chunks per thread, at most
  struct Regs {
    uint4 w0, w1;
    unsigned short sc;
    uint4 b[kBMax];
  };
  auto load_block = [&](int kb, Regs& r) {
    const int k0 = kb * kTcKBlock + ah * 32;
    r.sc = __ldg(ssrc + min(k0 >> p.gshift, ngroups - 1));
    if constexpr (BITS == 4) {
      r.w0 = ldg_stream(wsrc + (size_t)k0 / 2);
    } else {
      r.w0 = ldg_stream(wsrc + (size_t)k0);
      r.w1 = ldg_stream(wsrc + (size_t)k0 + 16);
    }
#pragma unroll
    for (int j = 0; j < kBMax; ++j) {
      const int i = tid + j * kTcThreads;
      r.b[j] = make_uint4(0, 0, 0, 0);
      const int m = i >> 3, c = i & 7;   // rows past M stay zero
      if (i < p.Mpad * 8 && m < p.M) r.b[j] = ldg_nc(p.act + (size_t)m * p.lda + kb * kTcKBlock + c * 8);
    }
  };
  auto store_block = [&](int s, const Regs& r) {
    const uint32_t sa = base + s * stage_bytes, sb = sa + a_bytes;
    const uint32_t s2 = (uint32_t)r.sc | ((uint32_t)r.sc << 16);
    if constexpr (BITS == 4) {
      const uint32_t qw[4] = {r.w0.x, r.w0.y, r.w0.z, r.w0.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) sts128(base_ptr + (sa - base) + swz(ar, ah * 4 + j), dequant8<4>(qw[j], 0u, s2));
    } else {
      const uint32_t qw[8] = {r.w0.x, r.w0.y, r.w0.z, r.w0.w, r.w1.x, r.w1.y, r.w1.z, r.w1.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        sts128(base_ptr + (sa - base) + swz(ar, ah * 4 + j), dequant8<8>(qw[2 * j], qw[2 * j + 1], s2));
    }
#pragma unroll
    for (int j = 0; j < kBMax; ++j) {
      const int i = tid + j * kTcThreads;
      if (i < p.Mpad * 8) sts128(base_ptr + (sb - base) + swz(i >> 3, i & 7), r.b[j]);
    }
  };
  auto step = [&](int kb, const Regs& cur) {
    const int s = kb % kTcStages, use = kb / kTcStages;
    if (use > 0 && live) live = mbar_wait_bounded(smem_u32(&bar_empty[s]), (use - 1) & 1, kTcWaitNs);
    store_block(s, cur);
    fence_proxy_async_smem();   // the tensor core reads these through the async proxy
    mbar_arrive(smem_u32(&bar_full[s]));
    if (tid == 0) {
      if (live) live = mbar_wait_bounded(smem_u32(&bar_full[s]), use & 1, kTcWaitNs);
      tc_fence_after();
      if (live) {
        const uint32_t sa = base + s * stage_bytes, sb = sa + a_bytes;
#pragma unroll
        for (int j = 0; j < 4; ++j)   // K = 16 per instruction: 32 bytes further along each row
          tc_mma_f16(tmem, sw128_desc(sa + j * 32), sw128_desc(sb + j * 32), p.idesc, (kb | j) != 0);
      }
      tc_commit(smem_u32(&bar_empty[s]));
    }
  };

  Regs ra, rb;
  load_block(0, ra);
  for (int kb = 0; kb < p.kblocks; kb += 2) {
    if (kb + 1 < p.kblocks) load_block(kb + 1, rb);
    step(kb, ra);
    if (kb + 1 >= p.kblocks) break;
    if (kb + 2 < p.kblocks) load_block(kb + 2, ra);
    step(kb + 1, rb);
  }
  if (tid == 0) tc_commit(smem_u32(&bar_done));
  mbar_wait_bounded(smem_u32(&bar_done), 0, kTcWaitNs);
  tc_fence_after();

  // ---- epilogue: warp w reads lanes 32*(w%4).. (tile rows) and every other
  // 32-column chunk (starting at 32*(w/4)); a chunk starts below Mpad and the
  // allocation is a power of two >= 32 and >= Mpad, so every read is inside it
  const int lg = warp & 3, ch = warp >> 2;
  const int r = lg * 32 + lane;            // tile row
  const int n = n0 + r;
  for (int c0 = ch * 32; c0 < p.Mpad; c0 += 64) {
    uint32_t v[32];
    __syncwarp();                          // tcgen05.ld is warp-collective (.sync.aligned)
    tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)c0, v);
    tmem_wait_ld();
    if constexpr (EPI == LW_TC_EPI_RESID) {
      if (n < p.N) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int m = c0 + j;
          if (m >= p.M) break;
          float y = r16(__uint_as_float(v[j]));
          if (p.residual) y = r16(__half2float(p.residual[(size_t)m * p.ldo + n]) + y);
          p.out[(size_t)m * p.ldo + n] = __float2half_rn(y);
        }
      }
    } else {
      // rows g and g + 8 of every 16-row tile are partners (gate/up, or the
      // rotate_half pair): the lower lane of each pair finishes both
      const bool lower = (lane & 15) < 8;
      const int t16 = n >> 4, g = n & 7;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float y = __uint_as_float(v[j]);
        const float partner = __shfl_down_sync(0xffffffffu, y, 8);
        const int m = c0 + j;
        if (!lower || m >= p.M || n >= p.N) continue;
        if constexpr (EPI == LW_TC_EPI_SWIGLU) {
          const float gt = r16(y), up = r16(partner);
          const float a = r16(silu_f32(gt));
          p.out[(size_t)m * p.ldo + t16 * 8 + g] = __float2half_rn(a * up);
        } else {
          const int hd = p.head_dim, nq = p.n_q_heads, nkv = p.n_kv_heads;
          const int head = (t16 * 16) / hd, jt = t16 % (hd / 16);
          const int d_lo = 8 * jt + g, d_hi = d_lo + hd / 2;
          const int pos = *p.pos + m, row = *p.seq;
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
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
}

// h[m] = fp16(gamma * fp16(x * rstd)), rstd = 1 / sqrt(mean(x^2) + eps) in fp32.
__global__ void rmsnorm_rows_kernel(const __half* __restrict__ x, const __half* __restrict__ gamma,
                                    __half* __restrict__ h, int K, float eps) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float part[32];
  const int m = blockIdx.x;
  const __half* xr = x + (size_t)m * K;
  float sq = 0.f;
  for (int i = threadIdx.x * 8; i < K; i += blockDim.x * 8) {
    const uint4 v = ldg_nc(xr + i);
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
    uint4 v = ldg_nc(xr + i);
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

template <int BITS, int EPI>
cudaError_t tc_launch(const lw::TcGemmParams& p, size_t smem, cudaStream_t s, bool pdl) {
  auto kern = lw::gemm_tc_kernel<BITS, EPI>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return lw_launch(kern, dim3(p.N / lw::kTcTileN), dim3(lw::kTcThreads), smem, s, pdl, p);
}

}  // namespace

int lw_gemm_tc_take_error() { return lw_tu_take_error(); }

extern "C" {

int lw_prefill_gemm(const lw_prefill_gemm_args* a, lw_stream_t stream) {
  if (!a || !a->act || !a->weight || !a->scales || !a->out) return LW_ERR_NULL_POINTER;
  if (a->bits != 4 && a->bits != 8) return LW_ERR_UNSUPPORTED;
  if (a->M <= 0 || a->M > lw::kTcMaxM || a->N <= 0 || a->N % lw::kTcTileN || a->K <= 0 || a->K % lw::kTcKBlock)
    return LW_ERR_BAD_SHAPE;
  if (a->group_size < 32 || a->K % a->group_size || lw::group_shift(a->K, a->group_size) < 0) return LW_ERR_BAD_GROUP;
  if (a->lda < a->K || a->lda % 8 || a->ldo % 8) return LW_ERR_BAD_SHAPE;
  if (!al(a->act, 16) || !al(a->weight, 16) || !al(a->out, 2)) return LW_ERR_ALIGNMENT;
  switch (a->epilogue) {
    case LW_TC_EPI_RESID:
      if (a->ldo < a->N) return LW_ERR_BAD_SHAPE;
      break;
    case LW_TC_EPI_SWIGLU:
      if (a->ldo < a->N / 2) return LW_ERR_BAD_SHAPE;
      break;
    case LW_TC_EPI_ROPE_KV:
      if (!a->q_out || !a->k_cache || !a->v_cache || !a->rope_cos || !a->rope_sin || !a->pos || !a->seq)
        return LW_ERR_NULL_POINTER;
      if (a->head_dim % 16 || a->N != (a->n_q_heads + 2 * a->n_kv_heads) * a->head_dim) return LW_ERR_BAD_SHAPE;
      break;
    default:
      return LW_ERR_UNSUPPORTED;
  }
  lw::TcGemmParams p = {};
  p.w = static_cast<const uint8_t*>(a->weight);
  p.scales = static_cast<const __half*>(a->scales);
  p.act = static_cast<const __half*>(a->act);
  p.out = static_cast<__half*>(a->out);
  p.residual = static_cast<const __half*>(a->residual);
  p.lda = a->lda;
  p.ldo = a->ldo;
  p.M = a->M;
  p.Mpad = (a->M + 15) / 16 * 16;
  p.N = a->N;
  p.K = a->K;
  p.G = a->group_size;
  p.gshift = lw::group_shift(a->K, a->group_size);
  p.kblocks = a->K / lw::kTcKBlock;
  p.idesc = tc_idesc(p.Mpad);
  int cols = 32;
  while (cols < p.Mpad) cols <<= 1;
  p.tmem_cols = cols;
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
  const size_t smem = 1024 + (size_t)lw::kTcStages * (lw::kTcTileN * 128 + (size_t)p.Mpad * 128);
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
#undef LW_TC
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

int lw_rmsnorm_rows(const void* x, const void* gamma, void* h, int M, int K, float eps, int pdl,
                    lw_stream_t stream) {
  if (!x || !gamma || !h) return LW_ERR_NULL_POINTER;
  if (M <= 0 || K <= 0 || K % 8) return LW_ERR_BAD_SHAPE;
  if (!al(x, 16) || !al(gamma, 16) || !al(h, 16)) return LW_ERR_ALIGNMENT;
  cudaGetLastError();
  cudaError_t e = lw_launch(lw::rmsnorm_rows_kernel, dim3(M), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                            pdl != 0, static_cast<const __half*>(x), static_cast<const __half*>(gamma),
                            static_cast<__half*>(h), K, eps);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

}  // extern "C"
