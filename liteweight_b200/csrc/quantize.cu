// liteweight's RTN quantizers on the GPU (sm_100a): bit-identical to
// liteweight/quantize.py:7-27 (INT8) and :65-99 (INT4).
//
// Per group of G consecutive K elements of a row: absmax in fp32, scale =
// absmax / 127 (INT8) or / 7 (INT4) as an IEEE fp32 division, clamped to
// >= 1e-8; code = round-half-even(w / scale) (IEEE fp32 division, rintf)
// clipped to [-127, 127] / [-8, 7]; the scale is stored rounded to fp16 (the
// codes use the unrounded fp32 scale). INT4 codes are packed two per byte,
// even k in the low nibble, 4-bit two's complement.
//
// One warp per (row, group) when a group holds whole bytes (INT8, or INT4 with
// an even G); INT4 with an odd G (a byte may straddle two groups) runs one
// thread per output byte that recomputes the absmax of its elements' groups.
// Used to build packed weights on the device (e.g. synthetic checkpoints of
// large architectures); no counterpart in the reference beyond the functions
// it restates, which run wherever their tensors are.
#include "lw_common.cuh"

namespace lw {

template <typename T>
LW_DEV float ldf(const T* p) {
  if constexpr (sizeof(T) == 2) {
    return __half2float(*reinterpret_cast<const __half*>(p));
  } else {
    return *reinterpret_cast<const float*>(p);
  }
}

// fp32 scale of a group (every lane of the warp gets it).
template <typename T>
LW_DEV float group_scale(const T* g, int G, int lane, float qmax) {
  float m = 0.f;
  for (int k = lane; k < G; k += 32) m = fmaxf(m, fabsf(ldf(g + k)));
  m = warp_max(m);
  return fmaxf(__fdiv_rn(m, qmax), 1e-8f);
}

LW_DEV int code_of(float w, float scale, int lo, int hi) {
  const float r = rintf(__fdiv_rn(w, scale));   // round half to even, as torch.round
  return (int)fminf(fmaxf(r, (float)lo), (float)hi);
}

template <typename T, int BITS>
__global__ void quantize_group_kernel(const T* __restrict__ w, uint8_t* __restrict__ q, __half* __restrict__ scales,
                                      int N, int K, int G) {
  const int lane = threadIdx.x & 31;
  const int ngroups = K / G;
  const long long total = (long long)N * ngroups;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long gi = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); gi < total; gi += warps) {
    const int n = (int)(gi / ngroups), grp = (int)(gi - (long long)n * ngroups);
    const T* src = w + (size_t)n * K + (size_t)grp * G;
    const float scale = group_scale(src, G, lane, BITS == 8 ? 127.f : 7.f);
    if (lane == 0) scales[gi] = __float2half_rn(scale);
    if constexpr (BITS == 8) {
      int8_t* dst = reinterpret_cast<int8_t*>(q) + (size_t)n * K + (size_t)grp * G;
      for (int k = lane; k < G; k += 32) dst[k] = (int8_t)code_of(ldf(src + k), scale, -127, 127);
    } else {
      uint8_t* dst = q + ((size_t)n * K + (size_t)grp * G) / 2;   // G even: the group starts on a byte
      for (int b = lane; b < G / 2; b += 32) {
        const int lo = code_of(ldf(src + 2 * b), scale, -8, 7), hi = code_of(ldf(src + 2 * b + 1), scale, -8, 7);
        dst[b] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
      }
    }
  }
}

// INT4 with an odd group size: one thread per byte; the scales come from a
// warp-per-group pass (scales_only), the codes recompute their group's absmax.
template <typename T>
__global__ void quantize_int4_bytes_kernel(const T* __restrict__ w, uint8_t* __restrict__ q, int N, int K, int G) {
  const long long total = (long long)N * (K / 2);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / (K / 2)), b = (int)(i - (long long)n * (K / 2));
    int codes[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int k = 2 * b + e;
      const T* g = w + (size_t)n * K + (size_t)(k / G) * G;
      float m = 0.f;
      for (int j = 0; j < G; ++j) m = fmaxf(m, fabsf(ldf(g + j)));
      const float scale = fmaxf(__fdiv_rn(m, 7.f), 1e-8f);
      codes[e] = code_of(ldf(w + (size_t)n * K + k), scale, -8, 7);
    }
    q[i] = (uint8_t)((codes[0] & 0xF) | ((codes[1] & 0xF) << 4));
  }
}

template <typename T>
__global__ void group_scales_kernel(const T* __restrict__ w, __half* __restrict__ scales, int N, int K, int G,
                                    float qmax) {
  const int lane = threadIdx.x & 31;
  const int ngroups = K / G;
  const long long total = (long long)N * ngroups;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long gi = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); gi < total; gi += warps) {
    const int n = (int)(gi / ngroups), grp = (int)(gi - (long long)n * ngroups);
    const float scale = group_scale(w + (size_t)n * K + (size_t)grp * G, G, lane, qmax);
    if (lane == 0) scales[gi] = __float2half_rn(scale);
  }
}

}  // namespace lw

namespace {

int sm_count_q() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 148;
  return n > 0 ? n : 148;
}

template <int BITS>
int quantize(const void* w, int w_fp32, void* qweight, void* scales, int N, int K, int G, lw_stream_t stream) {
  if (!w || !qweight || !scales) return LW_ERR_NULL_POINTER;
  if (N <= 0 || K <= 0 || (BITS == 4 && K % 2)) return LW_ERR_BAD_SHAPE;
  if (G <= 0 || K % G) return LW_ERR_BAD_GROUP;
  if (reinterpret_cast<uintptr_t>(w) % (w_fp32 ? 4 : 2) || reinterpret_cast<uintptr_t>(scales) % 2)
    return LW_ERR_ALIGNMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaGetLastError();
  const dim3 block(256), grid(8 * sm_count_q());
  uint8_t* q = static_cast<uint8_t*>(qweight);
  __half* sc = static_cast<__half*>(scales);
  if (BITS == 8 || G % 2 == 0) {
    lw_count_launch();
    if (w_fp32)
      lw::quantize_group_kernel<float, BITS><<<grid, block, 0, s>>>(static_cast<const float*>(w), q, sc, N, K, G);
    else
      lw::quantize_group_kernel<__half, BITS><<<grid, block, 0, s>>>(static_cast<const __half*>(w), q, sc, N, K, G);
  } else {
    lw_count_launch();
    lw_count_launch();
    if (w_fp32) {
      lw::group_scales_kernel<float><<<grid, block, 0, s>>>(static_cast<const float*>(w), sc, N, K, G, 7.f);
      lw::quantize_int4_bytes_kernel<float><<<grid, block, 0, s>>>(static_cast<const float*>(w), q, N, K, G);
    } else {
      lw::group_scales_kernel<__half><<<grid, block, 0, s>>>(static_cast<const __half*>(w), sc, N, K, G, 7.f);
      lw::quantize_int4_bytes_kernel<__half><<<grid, block, 0, s>>>(static_cast<const __half*>(w), q, N, K, G);
    }
  }
  return cudaGetLastError() == cudaSuccess ? LW_OK : LW_ERR_LAUNCH;
}

}  // namespace

extern "C" {

int lw_quantize_int8(const void* weight, int weight_fp32, void* qweight, void* scales, int N, int K, int group_size,
                     lw_stream_t stream) {
  return quantize<8>(weight, weight_fp32, qweight, scales, N, K, group_size, stream);
}

int lw_quantize_int4(const void* weight, int weight_fp32, void* qweight, void* scales, int N, int K, int group_size,
                     lw_stream_t stream) {
  return quantize<4>(weight, weight_fp32, qweight, scales, N, K, group_size, stream);
}

}  // extern "C"
