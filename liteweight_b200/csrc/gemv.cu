// Weight-only dequant GEMV / skinny GEMM for B200 (sm_100a).
//
// Computes out[m, n] = sum_k act[m, k] * W[n, k] for the small-M (decode)
// regime, where the cost is streaming W from HBM once. Replaces the Triton
// kernels of liteweight (kernels/matmul_int8.py:26-100, matmul_int4.py:24-119,
// matmul_fp16.py:24-64); the arithmetic is that of liteweight/quantize.py:60:
// each weight is dequantized to fp16 exactly as dequantize_int{8,4} does, the
// products are accumulated in fp32, and the sum is rounded to fp16 once.
//
// Design (one CTA = RW row tiles x KW k-slices, one warp per (tile, slice)):
//   * a warp owns 16 weight rows; lane (g = lane/4, t = lane%4) streams rows
//     g and g+8 with 16-byte non-allocating loads, four lanes covering 64
//     contiguous bytes per row per chunk;
//   * the codes are turned into fp16 pairs in registers with integer tricks
//     (no conversion instructions) and scaled by an fp16 multiply, which is
//     bit-identical to the reference's fp32 product rounded to fp16;
//   * the dequantized pairs are the A operand of mma.sync.m16n8k16 directly in
//     registers, the activation (staged once per CTA in shared memory in the
//     element order the dequant produces) is the B operand, batch rows are
//     the n8 columns, fp32 accumulation in the tensor core;
//   * the KW k-slices of a tile are reduced through shared memory, then the
//     epilogue rounds to fp16, adds bias / residual and stores.
// Weights are read before griddepcontrol.wait so that, launched with
// programmatic dependent launch, the weight stream of this kernel overlaps the
// tail of the kernel that produces its activation.
#include "lw_common.cuh"

#include <algorithm>
#include <atomic>

static std::atomic<unsigned long long> g_launches{0};
void lw_count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

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

struct GemvParams {
  const __half* act;       // [M][lda]
  const uint8_t* w;        // [N][K * BITS / 8]
  const __half* scales;    // [N][K / G] (BITS < 16)
  const __half* bias;      // [N] or null
  const __half* residual;  // [M][ldo] or null: out = residual + y
  __half* out;             // [M][ldo]
  int lda, ldo;
  int M, N, K, G;
  int kchunks;  // ceil(K / (4 * E))
  int cp;       // staged activation row stride, halves
  int rw, kw;   // row tiles and k-slices per CTA
};

LW_DEV uint32_t bcast_h(const __half* p) {
  const unsigned short s = __ldg(reinterpret_cast<const unsigned short*>(p));
  return (uint32_t)s | ((uint32_t)s << 16);
}

template <int BITS, int MT>
LW_DEV void gemv_piece(float (&acc)[MT][4], const uint4& qa, const uint4& qb, uint32_t sa, uint32_t sb,
                       const __half* arow, int cp, int g, int M) {
  const uint32_t* a32 = reinterpret_cast<const uint32_t*>(&qa);
  const uint32_t* b32 = reinterpret_cast<const uint32_t*>(&qb);
  const uint4 z = make_uint4(0, 0, 0, 0);
  if constexpr (BITS == 4) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t A[4], B[4];
      dequant_int4_word(a32[w], A);
      dequant_int4_word(b32[w], B);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        A[i] = hmul2_u32(A[i], sa);
        B[i] = hmul2_u32(B[i], sb);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint4 av = (g + 8 * mt < M) ? lds128(arow + mt * 8 * cp + w * 32) : z;
        mma16816(acc[mt], A[0], B[0], A[1], B[1], av.x, av.y);
        mma16816(acc[mt], A[2], B[2], A[3], B[3], av.z, av.w);
      }
    }
  } else if constexpr (BITS == 8) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint4 av[MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) av[mt] = (g + 8 * mt < M) ? lds128(arow + mt * 8 * cp + j * 32) : z;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t A[2], B[2];
        dequant_int8_word(a32[2 * j + h], A);
        dequant_int8_word(b32[2 * j + h], B);
        A[0] = hmul2_u32(A[0], sa);
        A[1] = hmul2_u32(A[1], sa);
        B[0] = hmul2_u32(B[0], sb);
        B[1] = hmul2_u32(B[1], sb);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          mma16816(acc[mt], A[0], B[0], A[1], B[1], h ? av[mt].z : av[mt].x, h ? av[mt].w : av[mt].y);
      }
    }
  } else {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const uint4 av = (g + 8 * mt < M) ? lds128(arow + mt * 8 * cp) : z;
      mma16816(acc[mt], qa.x, qb.x, qa.y, qb.y, av.x, av.y);
      mma16816(acc[mt], qa.z, qb.z, qa.w, qb.w, av.z, av.w);
    }
  }
}

template <int BITS, int MT, int U>
__global__ void __launch_bounds__(512) gemv_kernel(const GemvParams p) {
  constexpr int E = WT<BITS>::E;
  constexpr int KC = 4 * E;
  extern __shared__ __align__(16) uint8_t smem[];
  __half* act_s = reinterpret_cast<__half*>(smem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rt = warp % p.rw, kwi = warp / p.rw;
  const int n_cta = blockIdx.x * p.rw * 16;
  const int r0 = n_cta + rt * 16 + g, r1 = r0 + 8;
  const bool v0 = r0 < p.N, v1 = r1 < p.N;
  const size_t rowbytes = (size_t)p.K * BITS / 8;
  const int npieces = (int)(rowbytes / 16);
  const uint8_t* w0 = p.w + (size_t)(v0 ? r0 : 0) * rowbytes;
  const uint8_t* w1 = p.w + (size_t)(v1 ? r1 : 0) * rowbytes;
  const int ngroups = (BITS < 16) ? p.K / p.G : 1;
  const __half* s0 = p.scales + (size_t)(v0 ? r0 : 0) * ngroups;
  const __half* s1 = p.scales + (size_t)(v1 ? r1 : 0) * ngroups;
  const int per = (p.kchunks + p.kw - 1) / p.kw;
  const int cb = kwi * per, ce = min(p.kchunks, cb + per);

  uint4 qa[U], qb[U];
  uint32_t sa[U], sb[U];
  auto load_batch = [&](int cbase) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = cbase + u;
      const int pc = c * 4 + t;
      const bool ok = (c < ce) && (pc < npieces);
      qa[u] = (ok && v0) ? ldg_stream(w0 + (size_t)pc * 16) : make_uint4(0, 0, 0, 0);
      qb[u] = (ok && v1) ? ldg_stream(w1 + (size_t)pc * 16) : make_uint4(0, 0, 0, 0);
      if constexpr (BITS < 16) {
        const int grp = (c * KC + t * E) / p.G;
        sa[u] = (ok && v0) ? bcast_h(s0 + grp) : 0u;
        sb[u] = (ok && v1) ? bcast_h(s1 + grp) : 0u;
      } else {
        sa[u] = sb[u] = 0u;
      }
    }
  };

  // Weights do not depend on the previous kernel: start streaming them first.
  load_batch(cb);
  pdl_wait();

  // Stage act[0:M][0:kchunks*KC] (zero padded past K) in the lane order.
  {
    const int groups8 = p.kchunks * KC / 8;
    for (int i = tid; i < p.M * groups8; i += blockDim.x) {
      const int m = i / groups8, k = (i - m * groups8) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (k < p.K) v = ldg_nc(p.act + (size_t)m * p.lda + k);
      if constexpr (BITS == 4) v = perm_int4_pairs(v);
      const int c = k / KC, r = k - c * KC, tt = r / E, j = (r - tt * E) / 8;
      sts128(act_s + (size_t)m * p.cp + c * KC + (j * 4 + tt) * 8, v);
    }
  }
  __syncthreads();

  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;

  const __half* abase = act_s + (size_t)g * p.cp + t * 8;
  for (int cc = cb; cc < ce; cc += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = cc + u;
      if (c < ce) gemv_piece<BITS, MT>(acc, qa[u], qb[u], sa[u], sb[u], abase + c * KC, p.cp, g, p.M);
    }
    if (cc + U < ce) load_batch(cc + U);
  }
  pdl_launch_dependents();

  // Reduce the KW k-slices of each row tile through shared memory.
  float* red = reinterpret_cast<float*>(smem + (size_t)p.M * p.cp * 2);
  const int CW = MT * 8;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    float* rb = red + ((size_t)(kwi * p.rw + rt) * CW + mt * 8 + 2 * t) * 16;
    rb[g] = acc[mt][0];
    rb[16 + g] = acc[mt][1];
    rb[g + 8] = acc[mt][2];
    rb[16 + g + 8] = acc[mt][3];
  }
  __syncthreads();

  const int rows = p.rw * 16;
  for (int i = tid; i < rows * p.M; i += blockDim.x) {
    const int m = i / rows, nl = i - m * rows;
    const int n = n_cta + nl;
    if (n >= p.N) continue;
    const int rti = nl >> 4, r = nl & 15;
    float s = 0.f;
    for (int k = 0; k < p.kw; ++k) s += red[((size_t)(k * p.rw + rti) * CW + m) * 16 + r];
    float y = r16(s);
    if (p.bias) y = r16(y + __half2float(p.bias[n]));
    if (p.residual) y = r16(__half2float(p.residual[(size_t)m * p.ldo + n]) + y);
    p.out[(size_t)m * p.ldo + n] = __float2half_rn(y);
  }
}

// ------------------------------------------------------------- generic path
// Any shape or alignment (e.g. the reference's 3x70x130 fp16 test): one warp
// per output row, scalar loads. KN selects a row-major b[K][N] fp16 weight.
template <int BITS, bool KN>
__global__ void gemv_generic_kernel(const GemvParams p) {
  const int n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (n >= p.N) return;
  const int ngroups = (BITS < 16) ? p.K / p.G : 1;
  for (int m = 0; m < p.M; ++m) {
    float s = 0.f;
    for (int k = lane; k < p.K; k += 32) {
      float wv;
      if constexpr (BITS == 16) {
        const __half* w16 = reinterpret_cast<const __half*>(p.w);
        wv = __half2float(KN ? w16[(size_t)k * p.N + n] : w16[(size_t)n * p.K + k]);
      } else {
        int code;
        if constexpr (BITS == 8) {
          code = (int)reinterpret_cast<const int8_t*>(p.w)[(size_t)n * p.K + k];
        } else {
          const uint8_t b = p.w[(size_t)n * (p.K / 2) + (k >> 1)];
          const int nib = (k & 1) ? (b >> 4) : (b & 15);
          code = nib >= 8 ? nib - 16 : nib;
        }
        const float sc = __half2float(p.scales[(size_t)n * ngroups + k / p.G]);
        wv = r16((float)code * sc);
      }
      s = fmaf(__half2float(p.act[(size_t)m * p.lda + k]), wv, s);
    }
    s = warp_sum(s);
    if (lane == 0) {
      float y = r16(s);
      if (p.bias) y = r16(y + __half2float(p.bias[n]));
      if (p.residual) y = r16(__half2float(p.residual[(size_t)m * p.ldo + n]) + y);
      p.out[(size_t)m * p.ldo + n] = __float2half_rn(y);
    }
  }
}

// ------------------------------------------------------------- fp16 b[K][N]
// Warp tile: 64 columns n x 16 k per step. Lane (g, t) loads b[k0 + 4t + i][n0
// + 8g .. +7] (i = 0..3, 16-byte rows) and pairs consecutive k with byte
// permutes into the A fragments of four m16n8k16 tiles whose rows are the
// columns n0 + 8g + 2j and +1 (j = 0..3).
template <int MT, int U>
__global__ void __launch_bounds__(512) gemm_f16_kn_kernel(const GemvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __half* act_s = reinterpret_cast<__half*>(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rt = warp % p.rw, kwi = warp / p.rw;
  const int n_cta = blockIdx.x * p.rw * 64;
  const int nc = n_cta + rt * 64 + 8 * g;  // first of this lane's 8 columns
  const bool vn = nc < p.N;                // N % 8 == 0 on this path
  const __half* b = reinterpret_cast<const __half*>(p.w);
  const int ksteps = (p.K + 15) / 16;
  const int per = (ksteps + p.kw - 1) / p.kw;
  const int sb = kwi * per, se = min(ksteps, sb + per);

  uint4 L[U][4];
  auto load_batch = [&](int s0) {
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = (s0 + u) * 16 + 4 * t + i;
        const bool ok = vn && (s0 + u < se) && (k < p.K);
        L[u][i] = ok ? ldg_stream(b + (size_t)k * p.N + nc) : make_uint4(0, 0, 0, 0);
      }
  };
  load_batch(sb);
  pdl_wait();
  {
    const int kpad = ksteps * 16;
    const int groups8 = kpad / 8;
    for (int i = tid; i < p.M * groups8; i += blockDim.x) {
      const int m = i / groups8, k = (i - m * groups8) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (k < p.K) v = ldg_nc(p.act + (size_t)m * p.lda + k);
      sts128(act_s + (size_t)m * p.cp + k, v);
    }
  }
  __syncthreads();

  float acc[MT][4][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[mt][j][0] = acc[mt][j][1] = acc[mt][j][2] = acc[mt][j][3] = 0.f;

  for (int s0 = sb; s0 < se; s0 += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (s0 + u < se) {
        const int kb = (s0 + u) * 16 + 4 * t;
        uint2 av[MT];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          if (g + 8 * mt < p.M) {
            av[mt] = *reinterpret_cast<const uint2*>(act_s + (size_t)(g + 8 * mt) * p.cp + kb);
          } else {
            av[mt] = make_uint2(0, 0);
          }
        }
        const uint32_t* l0 = reinterpret_cast<const uint32_t*>(&L[u][0]);
        const uint32_t* l1 = reinterpret_cast<const uint32_t*>(&L[u][1]);
        const uint32_t* l2 = reinterpret_cast<const uint32_t*>(&L[u][2]);
        const uint32_t* l3 = reinterpret_cast<const uint32_t*>(&L[u][3]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t a0 = __byte_perm(l0[j], l1[j], 0x5410);
          const uint32_t a1 = __byte_perm(l0[j], l1[j], 0x7632);
          const uint32_t a2 = __byte_perm(l2[j], l3[j], 0x5410);
          const uint32_t a3 = __byte_perm(l2[j], l3[j], 0x7632);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) mma16816(acc[mt][j], a0, a1, a2, a3, av[mt].x, av[mt].y);
        }
      }
    }
    if (s0 + U < se) load_batch(s0 + U);
  }
  pdl_launch_dependents();

  float* red = reinterpret_cast<float*>(smem + (size_t)p.M * p.cp * 2);
  const int CW = MT * 8;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float* rb = red + ((size_t)(kwi * p.rw + rt) * CW + mt * 8 + 2 * t) * 64;
      const int c = 8 * g + 2 * j;
      rb[c] = acc[mt][j][0];
      rb[64 + c] = acc[mt][j][1];
      rb[c + 1] = acc[mt][j][2];
      rb[64 + c + 1] = acc[mt][j][3];
    }
  __syncthreads();
  const int cols = p.rw * 64;
  for (int i = tid; i < cols * p.M; i += blockDim.x) {
    const int m = i / cols, nl = i - m * cols;
    const int n = n_cta + nl;
    if (n >= p.N) continue;
    const int rti = nl >> 6, r = nl & 63;
    float s = 0.f;
    for (int k = 0; k < p.kw; ++k) s += red[((size_t)(k * p.rw + rti) * CW + m) * 64 + r];
    p.out[(size_t)m * p.ldo + n] = __float2half_rn(s);
  }
}

// ------------------------------------------------------------- dequant
template <int BITS>
__global__ void dequant_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ scales,
                               __half* __restrict__ out, int N, int K, int G) {
  const size_t total = (size_t)N * K;
  const int ngroups = K / G;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(i / K), k = (int)(i - (size_t)n * K);
    int code;
    if constexpr (BITS == 8) {
      code = (int)reinterpret_cast<const int8_t*>(w)[i];
    } else {
      const uint8_t b = w[(size_t)n * (K / 2) + (k >> 1)];
      const int nib = (k & 1) ? (b >> 4) : (b & 15);
      code = nib >= 8 ? nib - 16 : nib;
    }
    out[i] = __float2half_rn((float)code * __half2float(scales[(size_t)n * ngroups + k / G]));
  }
}

}  // namespace lw

// ======================================================================= host

namespace {

using lw::GemvParams;

constexpr int kMaxStageBytes = 160 * 1024;
constexpr int kU = 4;

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <typename K>
cudaError_t set_smem(K kern, size_t bytes) {
  // Opt in to more than 48 KB of dynamic shared memory for this launch.
  if (bytes <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <int BITS, int MT>
cudaError_t launch_fast(GemvParams p, cudaStream_t s, bool pdl) {
  constexpr int E = lw::WT<BITS>::E, KC = 4 * E;
  p.kchunks = (p.K + KC - 1) / KC;
  const int kpad = p.kchunks * KC;
  p.cp = kpad + ((kpad % 64) == 0 ? 32 : 0);   // row stride = 64 mod 128 bytes
  const int tiles = (p.N + 15) / 16;
  int kw = std::min(16, std::max(1, (p.kchunks + kU - 1) / kU));
  int rw = 1;
  const int want = 2 * sm_count();
  while (rw * 2 * kw <= 16 && (tiles + rw * 2 - 1) / (rw * 2) >= want) rw *= 2;
  p.kw = kw;
  p.rw = rw;
  const size_t smem = (size_t)p.M * p.cp * 2 + (size_t)kw * rw * MT * 8 * 16 * 4;
  auto kern = lw::gemv_kernel<BITS, MT, kU>;
  cudaError_t e = set_smem(kern, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((tiles + rw - 1) / rw), block(32 * rw * kw);
  return lw_launch(kern, grid, block, smem, s, pdl, p);
}

template <int BITS>
cudaError_t launch_generic(GemvParams p, cudaStream_t s, bool kn) {
  dim3 block(256), grid((p.N * 32 + 255) / 256);
  if (kn) return lw_launch(lw::gemv_generic_kernel<16, true>, grid, block, 0, s, false, p);
  return lw_launch(lw::gemv_generic_kernel<BITS, false>, grid, block, 0, s, false, p);
}

// Stage-size limited M blocking: one launch per block of rows, each reading
// the weights again (they stay in L2 when they fit).
template <int BITS>
cudaError_t gemv_dispatch(GemvParams p, cudaStream_t s, bool pdl) {
  constexpr int E = lw::WT<BITS>::E, KC = 4 * E;
  const size_t rowbytes = (size_t)p.K * BITS / 8;
  const bool fast = (rowbytes % 16 == 0) && (p.K % 8 == 0) && aligned(p.w, 16) && aligned(p.act, 16) &&
                    (BITS == 16 || (p.G % E == 0));
  if (!fast) return launch_generic<BITS>(p, s, false);
  const int kpad = ((p.K + KC - 1) / KC) * KC + 32;
  const int rows_fit = std::max(1, kMaxStageBytes / (kpad * 2));
  const int mb_max = std::min(32, rows_fit);
  for (int m0 = 0; m0 < p.M; m0 += mb_max) {
    GemvParams q = p;
    q.M = std::min(mb_max, p.M - m0);
    q.act = p.act + (size_t)m0 * p.lda;
    q.out = p.out + (size_t)m0 * p.ldo;
    if (p.residual) q.residual = p.residual + (size_t)m0 * p.ldo;
    cudaError_t e;
    if (q.M <= 8)
      e = launch_fast<BITS, 1>(q, s, pdl);
    else if (q.M <= 16)
      e = launch_fast<BITS, 2>(q, s, pdl);
    else
      e = launch_fast<BITS, 4>(q, s, pdl);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int to_status(cudaError_t e) { return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH; }

int check_common(const void* act, const void* w, const void* out, int M, int N, int K) {
  if (!act || !w || !out) return LW_ERR_NULL_POINTER;
  if (M <= 0 || N <= 0 || K <= 0) return LW_ERR_BAD_SHAPE;
  if (!aligned(act, 2) || !aligned(out, 2)) return LW_ERR_ALIGNMENT;
  return LW_OK;
}

template <int BITS>
int gemm_quant(const void* act, const void* qweight, const void* scales, const void* bias, void* out, int M,
               int N, int K, int G, lw_stream_t stream) {
  int st = check_common(act, qweight, out, M, N, K);
  if (st) return st;
  if (!scales) return LW_ERR_NULL_POINTER;
  if (BITS == 4 && (K % 2)) return LW_ERR_BAD_SHAPE;
  if (G <= 0 || K % G) return LW_ERR_BAD_GROUP;
  if (!aligned(scales, 2) || (bias && !aligned(bias, 2))) return LW_ERR_ALIGNMENT;
  GemvParams p = {};
  p.act = static_cast<const __half*>(act);
  p.w = static_cast<const uint8_t*>(qweight);
  p.scales = static_cast<const __half*>(scales);
  p.bias = static_cast<const __half*>(bias);
  p.out = static_cast<__half*>(out);
  p.lda = K;
  p.ldo = N;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = G;
  cudaGetLastError();
  cudaError_t e = gemv_dispatch<BITS>(p, reinterpret_cast<cudaStream_t>(stream), false);
  if (e == cudaSuccess) e = cudaGetLastError();
  return to_status(e);
}

template <int MT>
cudaError_t launch_kn(GemvParams p, cudaStream_t s) {
  const int ksteps = (p.K + 15) / 16;
  p.cp = ksteps * 16 + 8;
  const int tiles = (p.N + 63) / 64;
  int kw = std::min(16, std::max(1, (ksteps + 2 * kU - 1) / (2 * kU)));
  int rw = 1;
  while (rw * 2 * kw <= 16 && (tiles + rw * 2 - 1) / (rw * 2) >= 2 * sm_count()) rw *= 2;
  p.kw = kw;
  p.rw = rw;
  const size_t smem = (size_t)p.M * p.cp * 2 + (size_t)kw * rw * MT * 8 * 64 * 4;
  auto kern = lw::gemm_f16_kn_kernel<MT, kU>;
  cudaError_t e = set_smem(kern, smem);
  if (e != cudaSuccess) return e;
  return lw_launch(kern, dim3((tiles + rw - 1) / rw), dim3(32 * rw * kw), smem, s, false, p);
}

}  // namespace

extern "C" {

const char* lw_status_string(int status) {
  switch (status) {
    case LW_OK: return "ok";
    case LW_ERR_NULL_POINTER: return "null pointer";
    case LW_ERR_BAD_SHAPE: return "bad shape";
    case LW_ERR_BAD_GROUP: return "bad group size";
    case LW_ERR_ALIGNMENT: return "misaligned pointer";
    case LW_ERR_UNSUPPORTED: return "unsupported";
    case LW_ERR_LAUNCH: return "CUDA launch failed";
    case LW_ERR_WORKSPACE: return "workspace missing or too small";
    case LW_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

int lw_abi_version(void) { return 100; }

unsigned long long lw_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int lw_gemm_w8a16(const void* act, const void* qweight, const void* scales, const void* bias, void* out, int M,
                  int N, int K, int group_size, lw_stream_t stream) {
  return gemm_quant<8>(act, qweight, scales, bias, out, M, N, K, group_size, stream);
}

int lw_gemm_w4a16(const void* act, const void* qweight, const void* scales, const void* bias, void* out, int M,
                  int N, int K, int group_size, lw_stream_t stream) {
  return gemm_quant<4>(act, qweight, scales, bias, out, M, N, K, group_size, stream);
}

int lw_gemm_f16(const void* a, const void* w, void* out, int M, int N, int K, lw_stream_t stream) {
  int st = check_common(a, w, out, M, N, K);
  if (st) return st;
  GemvParams p = {};
  p.act = static_cast<const __half*>(a);
  p.w = static_cast<const uint8_t*>(w);
  p.out = static_cast<__half*>(out);
  p.lda = K;
  p.ldo = N;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = K;
  cudaGetLastError();
  cudaError_t e = gemv_dispatch<16>(p, reinterpret_cast<cudaStream_t>(stream), false);
  if (e == cudaSuccess) e = cudaGetLastError();
  return to_status(e);
}

int lw_gemm_f16_kn(const void* a, const void* b, void* out, int M, int N, int K, lw_stream_t stream) {
  int st = check_common(a, b, out, M, N, K);
  if (st) return st;
  GemvParams p = {};
  p.act = static_cast<const __half*>(a);
  p.w = static_cast<const uint8_t*>(b);
  p.out = static_cast<__half*>(out);
  p.lda = K;
  p.ldo = N;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = K;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaGetLastError();
  cudaError_t e;
  const bool fast = (N % 8 == 0) && (K % 8 == 0) && aligned(a, 16) && aligned(b, 16);
  if (!fast) {
    e = launch_generic<16>(p, s, true);
  } else {
    const int kpad = ((K + 15) / 16) * 16 + 8;
    const int mb_max = std::min(32, std::max(1, kMaxStageBytes / (kpad * 2)));
    e = cudaSuccess;
    for (int m0 = 0; m0 < M && e == cudaSuccess; m0 += mb_max) {
      GemvParams q = p;
      q.M = std::min(mb_max, M - m0);
      q.act = p.act + (size_t)m0 * p.lda;
      q.out = p.out + (size_t)m0 * p.ldo;
      e = q.M <= 8 ? launch_kn<1>(q, s) : (q.M <= 16 ? launch_kn<2>(q, s) : launch_kn<4>(q, s));
    }
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  return to_status(e);
}

int lw_dequant_w8(const void* qweight, const void* scales, void* out, int N, int K, int G, lw_stream_t stream) {
  if (!qweight || !scales || !out) return LW_ERR_NULL_POINTER;
  if (N <= 0 || K <= 0) return LW_ERR_BAD_SHAPE;
  if (G <= 0 || K % G) return LW_ERR_BAD_GROUP;
  cudaGetLastError();
  lw_count_launch();
  lw::dequant_kernel<8><<<4 * sm_count(), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(qweight), static_cast<const __half*>(scales), static_cast<__half*>(out), N, K, G);
  return to_status(cudaGetLastError());
}

int lw_dequant_w4(const void* qweight, const void* scales, void* out, int N, int K, int G, lw_stream_t stream) {
  if (!qweight || !scales || !out) return LW_ERR_NULL_POINTER;
  if (N <= 0 || K <= 0 || K % 2) return LW_ERR_BAD_SHAPE;
  if (G <= 0 || K % G) return LW_ERR_BAD_GROUP;
  cudaGetLastError();
  lw_count_launch();
  lw::dequant_kernel<4><<<4 * sm_count(), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(qweight), static_cast<const __half*>(scales), static_cast<__half*>(out), N, K, G);
  return to_status(cudaGetLastError());
}

}  // extern "C"
