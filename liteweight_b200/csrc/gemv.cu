// Weight-only dequant matmul entry points for B200 (sm_100a): the C ABI of
// liteweight's kernels/matmul_int8.py, matmul_int4.py and matmul_fp16.py.
//
// The small-M path is the persistent stream-K GEMV of gemv_core.cuh. Shapes
// it cannot take (rows not 16-byte aligned, a group smaller than a 16-byte
// piece) go to a simple warp-per-row kernel; fp16 weights stored [K][N] use
// their own tensor-core kernel; dequant kernels expose the bit-exact unpack.
#include "gemv_host.cuh"

#include <algorithm>
#include <atomic>

static std::atomic<unsigned long long> g_launches{0};
void lw_count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

namespace lw {

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
  pdl_launch_dependents();
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

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int to_status(cudaError_t e) { return e == cudaSuccess ? LW_OK : LW_ERR_LAUNCH; }

cudaError_t launch_generic(GemvParams p, int bits, cudaStream_t s, bool kn) {
  dim3 block(256), grid((p.N * 32 + 255) / 256);
  if (kn) return lw_launch(lw::gemv_generic_kernel<16, true>, grid, block, 0, s, false, p);
  if (bits == 4) return lw_launch(lw::gemv_generic_kernel<4, false>, grid, block, 0, s, false, p);
  if (bits == 8) return lw_launch(lw::gemv_generic_kernel<8, false>, grid, block, 0, s, false, p);
  return lw_launch(lw::gemv_generic_kernel<16, false>, grid, block, 0, s, false, p);
}

template <int BITS>
bool stream_ok(const void* act, const void* w, int K, int G) {
  constexpr int E = lw::WT<BITS>::E;
  const size_t rowbytes = (size_t)K * BITS / 8;
  // the stream kernel reads whole 64-byte chunks of a row (true for every
  // group size liteweight uses: K is a multiple of the group)
  return (rowbytes % 64 == 0) && (K % 8 == 0) && aligned(w, 16) && aligned(act, 16) &&
         (BITS == 16 || (G % E == 0 && lw::group_shift(K, G) >= 0));
}

// The TMA-ring kernel's own conditions (gemv_ring.cuh): 16-byte activation
// rows and weight rows (it reads whole 16-byte pieces; a row's last 128-byte
// stage may run past K, the copy fills zeros there) and scale groups that
// hold whole 16-byte pieces.
template <int BITS>
bool ring_ok(const void* act, const void* w, int K, int G) {
  constexpr int E = lw::WT<BITS>::E;
  return (K % 8 == 0) && ((size_t)K * BITS / 8) % 16 == 0 && aligned(w, 16) && aligned(act, 16) &&
         (BITS == 16 || (G % E == 0 && lw::group_shift(K, G) >= 0));
}

}  // namespace

// The tcgen05 GEMM (gemm_tc.cu) as a plain matmul with bias.
int lw_tc_matmul(int bits, const void* act, const void* w, const void* scales, const void* bias, void* out, int M,
                 int N, int K, int G, cudaStream_t s);

namespace {

// Rows from which the drop-in matmuls run on the tensor cores (tcgen05 GEMM)
// instead of the GEMV: past them a GEMV launch stages at most 32 rows and
// re-reads the weights per row block, while the GEMM takes 256 rows per pass.
// LW_B200_TC_MIN_M overrides it (0 disables the GEMM route).
int tc_min_rows() {
  static const int m = [] {
    const char* v = getenv("LW_B200_TC_MIN_M");
    return v ? atoi(v) : 33;
  }();
  return m;
}

// Shapes the tcgen05 GEMM tiles: 128-row weight tiles, K in blocks of 64, a
// scale group of >= 32 that is a power of two or K, 16-byte aligned rows.
bool tc_ok(const void* act, const void* w, int M, int N, int K, int G) {
  const int min_m = tc_min_rows();
  return min_m > 0 && M >= min_m && N % 128 == 0 && K % 64 == 0 && G >= 32 && K % G == 0 &&
         lw::group_shift(K, G) >= 0 && aligned(act, 16) && aligned(w, 16);
}

// out[M,N] = act @ W^T (+bias): tcgen05 GEMM past the crossover, else the
// stream kernel in row blocks, or the generic kernel.
template <int BITS>
cudaError_t matmul_dispatch(const void* act, const void* w, const void* scales, const void* bias, void* out,
                            int M, int N, int K, int G, void* ws, size_t ws_bytes, cudaStream_t s) {
  if constexpr (BITS == 4 || BITS == 8) {
    if (tc_ok(act, w, M, N, K, G))
      return lw_tc_matmul(BITS, act, w, scales, bias, out, M, N, K, G, s) == LW_OK ? cudaSuccess
                                                                                   : cudaErrorInvalidValue;
  }
  if (!stream_ok<BITS>(act, w, K, G)) {
    // shapes the register-pipeline kernel cannot take may still suit the ring kernel
    lw::RingPlan rpl;
    if (M <= 8 && ring_ok<BITS>(act, w, K, G) && lw::plan_ring<BITS, lw::PRO_PLAIN>(M, N, K, G, w, scales, &rpl)) {
      lw::StreamParams p = {};
      p.M = M;
      p.act = static_cast<const __half*>(act);
      p.w = static_cast<const uint8_t*>(w);
      p.scales = static_cast<const __half*>(scales);
      p.bias = static_cast<const __half*>(bias);
      p.out = static_cast<__half*>(out);
      p.lda = K;
      p.ldo = N;
      p.N = N;
      p.K = K;
      p.G = G;
      // programmatic dependent launch with every global read after the wait:
      // the launch and barrier setup overlap whatever kernel came before
      return lw::launch_ring<BITS, lw::PRO_PLAIN, lw::EPI_PLAIN>(p, rpl, s, true, true);
    }
    GemvParams p = {};
    p.act = static_cast<const __half*>(act);
    p.w = static_cast<const uint8_t*>(w);
    p.scales = static_cast<const __half*>(scales);
    p.bias = static_cast<const __half*>(bias);
    p.out = static_cast<__half*>(out);
    p.lda = K;
    p.ldo = N;
    p.M = M;
    p.N = N;
    p.K = K;
    p.G = G;
    return launch_generic(p, BITS, s, false);
  }
  const int rows = lw::stage_rows<BITS>(K);
  for (int m0 = 0; m0 < M; m0 += rows) {
    lw::StreamParams p = {};
    p.M = std::min(rows, M - m0);
    p.act = static_cast<const __half*>(act) + (size_t)m0 * K;
    p.w = static_cast<const uint8_t*>(w);
    p.scales = static_cast<const __half*>(scales);
    p.bias = static_cast<const __half*>(bias);
    p.out = static_cast<__half*>(out) + (size_t)m0 * N;
    p.lda = K;
    p.ldo = N;
    p.N = N;
    p.K = K;
    p.G = G;
    // the ring kernel (M <= 8) launches with PDL, reading everything after the wait
    cudaError_t e = lw::launch_stream_block<BITS, lw::PRO_PLAIN, lw::EPI_PLAIN>(p, ws, ws_bytes, s, false, false,
                                                                                true, true);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int check_common(const void* act, const void* w, const void* out, int M, int N, int K) {
  if (!act || !w || !out) return LW_ERR_NULL_POINTER;
  if (M <= 0 || N <= 0 || K <= 0) return LW_ERR_BAD_SHAPE;
  if (!aligned(act, 2) || !aligned(out, 2)) return LW_ERR_ALIGNMENT;
  return LW_OK;
}

int check_workspace(const void* ws, size_t ws_bytes) {
  if (ws_bytes && !ws) return LW_ERR_WORKSPACE;
  if (ws && !aligned(ws, 256)) return LW_ERR_ALIGNMENT;
  return LW_OK;
}

template <int BITS>
int gemm_quant(const void* act, const void* qweight, const void* scales, const void* bias, void* out, int M,
               int N, int K, int G, void* ws, size_t ws_bytes, lw_stream_t stream) {
  int st = check_common(act, qweight, out, M, N, K);
  if (st) return st;
  if (!scales) return LW_ERR_NULL_POINTER;
  if (BITS == 4 && (K % 2)) return LW_ERR_BAD_SHAPE;
  if (G <= 0 || K % G) return LW_ERR_BAD_GROUP;
  if (!aligned(scales, 2) || (bias && !aligned(bias, 2))) return LW_ERR_ALIGNMENT;
  st = check_workspace(ws, ws_bytes);
  if (st) return st;
  cudaGetLastError();
  cudaError_t e = matmul_dispatch<BITS>(act, qweight, scales, bias, out, M, N, K, G, ws, ws_bytes,
                                        reinterpret_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaGetLastError();
  return to_status(e);
}

template <int MT>
cudaError_t launch_kn(GemvParams p, cudaStream_t s) {
  constexpr int U = 4;
  const int ksteps = (p.K + 15) / 16;
  p.cp = ksteps * 16 + 8;
  const int tiles = (p.N + 63) / 64;
  int kw = std::min(16, std::max(1, (ksteps + 2 * U - 1) / (2 * U)));
  int rw = 1;
  while (rw * 2 * kw <= 16 && (tiles + rw * 2 - 1) / (rw * 2) >= 2 * lw::device_sm_count()) rw *= 2;
  p.kw = kw;
  p.rw = rw;
  const size_t smem = (size_t)p.M * p.cp * 2 + (size_t)kw * rw * MT * 8 * 64 * 4;
  auto kern = lw::gemm_f16_kn_kernel<MT, U>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return lw_launch(kern, dim3((tiles + rw - 1) / rw), dim3(32 * rw * kw), smem, s, false, p);
}

}  // namespace

// Device error flags of the other translation units that launch kernels.
int lw_decode_take_error();
int lw_decode_tp_take_error();
int lw_gemm_tc_take_error();

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

int lw_abi_version(void) { return 113; }

int lw_take_device_error(void) {
  const int mine = lw_tu_take_error();
  const int dec = lw_decode_take_error();
  const int tp = lw_decode_tp_take_error();
  const int tc = lw_gemm_tc_take_error();
  return mine ? mine : (dec ? dec : (tp ? tp : tc));
}

unsigned long long lw_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

size_t lw_gemm_workspace_size(int bits, int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (bits == 4) return lw::stream_workspace<4, lw::PRO_PLAIN, lw::EPI_PLAIN>(M, N, K);
  if (bits == 8) return lw::stream_workspace<8, lw::PRO_PLAIN, lw::EPI_PLAIN>(M, N, K);
  if (bits == 16) return lw::stream_workspace<16, lw::PRO_PLAIN, lw::EPI_PLAIN>(M, N, K);
  return 0;
}

int lw_gemm_w8a16(const void* act, const void* qweight, const void* scales, const void* bias, void* out, int M,
                  int N, int K, int group_size, void* workspace, size_t workspace_bytes, lw_stream_t stream) {
  return gemm_quant<8>(act, qweight, scales, bias, out, M, N, K, group_size, workspace, workspace_bytes, stream);
}

int lw_gemm_w4a16(const void* act, const void* qweight, const void* scales, const void* bias, void* out, int M,
                  int N, int K, int group_size, void* workspace, size_t workspace_bytes, lw_stream_t stream) {
  return gemm_quant<4>(act, qweight, scales, bias, out, M, N, K, group_size, workspace, workspace_bytes, stream);
}

int lw_gemm_f16(const void* a, const void* w, void* out, int M, int N, int K, void* workspace,
                size_t workspace_bytes, lw_stream_t stream) {
  int st = check_common(a, w, out, M, N, K);
  if (st) return st;
  st = check_workspace(workspace, workspace_bytes);
  if (st) return st;
  cudaGetLastError();
  cudaError_t e = matmul_dispatch<16>(a, w, nullptr, nullptr, out, M, N, K, K, workspace, workspace_bytes,
                                      reinterpret_cast<cudaStream_t>(stream));
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
    e = launch_generic(p, 16, s, true);
  } else {
    const int kpad = ((K + 15) / 16) * 16 + 8;
    const int mb_max = std::min(32, std::max(1, (160 * 1024) / (kpad * 2)));
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
  lw::dequant_kernel<8><<<4 * lw::device_sm_count(), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(qweight), static_cast<const __half*>(scales), static_cast<__half*>(out), N, K, G);
  return to_status(cudaGetLastError());
}

int lw_dequant_w4(const void* qweight, const void* scales, void* out, int N, int K, int G, lw_stream_t stream) {
  if (!qweight || !scales || !out) return LW_ERR_NULL_POINTER;
  if (N <= 0 || K <= 0 || K % 2) return LW_ERR_BAD_SHAPE;
  if (G <= 0 || K % G) return LW_ERR_BAD_GROUP;
  cudaGetLastError();
  lw_count_launch();
  lw::dequant_kernel<4><<<4 * lw::device_sm_count(), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(qweight), static_cast<const __half*>(scales), static_cast<__half*>(out), N, K, G);
  return to_status(cudaGetLastError());
}

}  // extern "C"
