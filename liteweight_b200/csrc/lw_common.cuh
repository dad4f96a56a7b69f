// Shared device helpers for the liteweight B200 kernels (sm_100a).
//
// Weight formats (liteweight/quantize.py:7-27, :65-99, :102-128):
//   INT8  qweight int8  [N, K]      one code per byte, symmetric, codes -128..127
//   INT4  qweight uint8 [N, K/2]    byte p holds k = 2p (low nibble) and 2p + 1
//                                   (high nibble), 4-bit two's complement
//   scales fp16 [N, K/G]            dequant = fp16((float)q * (float)s), i.e. one
//                                   rounding of the exact product; an fp16 HMUL of
//                                   the exactly-converted code gives the same bits.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/liteweight_b200.h"

#define LW_DEV __device__ __forceinline__

namespace lw {

// ---------------------------------------------------------------- memory ops

// Streaming 16-byte load of weights: read once per call, keep out of L1.
LW_DEV uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

LW_DEV uint4 ldg_nc(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

LW_DEV uint4 lds128(const void* p) {
  uint4 v;
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}

LW_DEV void sts128(void* p, uint4 v) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w));
}

// Fire-and-forget bulk prefetch of [p, p + bytes) into L2 (16-byte multiples).
LW_DEV void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the previous kernel in the stream
// (no-op when the launch did not opt in) / let the next one start its prologue.
LW_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LW_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- tensor core

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col).
// Fragment ownership (lane = 4*g + t): a0 = A[g][2t..2t+1], a1 = A[g+8][2t..],
// a2 = A[g][2t+8..], a3 = A[g+8][2t+8..]; b0 = B[2t..2t+1][g], b1 = B[2t+8..][g];
// d0,d1 = D[g][2t..2t+1], d2,d3 = D[g+8][2t..2t+1].
LW_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                     uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------- half2 bits

LW_DEV uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
LW_DEV __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
LW_DEV uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  return h2_as_u32(__hmul2(u32_as_h2(a), u32_as_h2(b)));
}

// ---------------------------------------------------------------- dequant

// 8 INT4 codes in one 32-bit word (code i = nibble i = element k0 + i) to four
// half2 holding exact small integers, paired (0,4) (1,5) (2,6) (3,7).
// Trick: with u = nibble ^ 8 = code + 8 in 0..15, the fp16 with bits
// 0x6400 | u is 1024 + u, so subtracting 1032 gives the signed code; the
// nibbles at bits 4..7 land as 1024 + 16u and are rescaled by an exact fma.
LW_DEV void dequant_int4_word(uint32_t q, uint32_t (&o)[4]) {
  const uint32_t x = q ^ 0x88888888u;
  const uint32_t y = x >> 8;
  const uint32_t MAGIC = 0x64006400u;
  uint32_t h04 = (x & 0x000F000Fu) | MAGIC;
  uint32_t h15 = (x & 0x00F000F0u) | MAGIC;
  uint32_t h26 = (y & 0x000F000Fu) | MAGIC;
  uint32_t h37 = (y & 0x00F000F0u) | MAGIC;
  const __half2 k1032 = __half2half2(__ushort_as_half(0x6408));   // 1032.0
  const __half2 k1_16 = __half2half2(__ushort_as_half(0x2C00));   // 1/16
  const __half2 km72 = __half2half2(__ushort_as_half(0xD480));    // -72.0
  o[0] = h2_as_u32(__hsub2(u32_as_h2(h04), k1032));
  o[1] = h2_as_u32(__hfma2(u32_as_h2(h15), k1_16, km72));
  o[2] = h2_as_u32(__hsub2(u32_as_h2(h26), k1032));
  o[3] = h2_as_u32(__hfma2(u32_as_h2(h37), k1_16, km72));
}

// Same unpack without scaling, with the sign flip folded into each LOP3
// constant: (x & m) ^ c where c = 0x6400.. | 0x0008.. for the low nibbles.
LW_DEV void unpack_int4_word(uint32_t q, uint32_t (&o)[4]) {
  const uint32_t y = q >> 8;
  uint32_t h04, h15, h26, h37;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(h04) : "r"(q), "n"(0x000F000F), "n"(0x64086408));
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(h15) : "r"(q), "n"(0x00F000F0), "n"(0x64806480));
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(h26) : "r"(y), "n"(0x000F000F), "n"(0x64086408));
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(h37) : "r"(y), "n"(0x00F000F0), "n"(0x64806480));
  const __half2 k1032 = __half2half2(__ushort_as_half(0x6408));   // 1032.0
  const __half2 k1_16 = __half2half2(__ushort_as_half(0x2C00));   // 1/16
  const __half2 km72 = __half2half2(__ushort_as_half(0xD480));    // -72.0
  o[0] = h2_as_u32(__hsub2(u32_as_h2(h04), k1032));
  o[1] = h2_as_u32(__hfma2(u32_as_h2(h15), k1_16, km72));
  o[2] = h2_as_u32(__hsub2(u32_as_h2(h26), k1032));
  o[3] = h2_as_u32(__hfma2(u32_as_h2(h37), k1_16, km72));
}

// 4 INT8 codes (bytes 0..3 = elements k0..k0+3) to two half2 (0,1) (2,3).
// u = byte ^ 0x80 = code + 128; fp16 bits 0x64uu = 1024 + u; minus 1152.
LW_DEV void dequant_int8_word(uint32_t q, uint32_t (&o)[2]) {
  const uint32_t x = q ^ 0x80808080u;
  const __half2 k1152 = __half2half2(__ushort_as_half(0x6480));   // 1152.0
  o[0] = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(x, 0x64646464u, 0x4140)), k1152));
  o[1] = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(x, 0x64646464u, 0x4342)), k1152));
}

// Permute 8 halves (h0..h7) to (h0,h4)(h1,h5)(h2,h6)(h3,h7): the element
// pairing that dequant_int4_word produces.
LW_DEV uint4 perm_int4_pairs(uint4 v) {
  uint4 o;
  o.x = __byte_perm(v.x, v.z, 0x5410);
  o.y = __byte_perm(v.x, v.z, 0x7632);
  o.z = __byte_perm(v.y, v.w, 0x5410);
  o.w = __byte_perm(v.y, v.w, 0x7632);
  return o;
}

LW_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

LW_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// fp16 rounding of an fp32 value (round to nearest even), back to fp32.
LW_DEV float r16(float v) { return __half2float(__float2half_rn(v)); }

}  // namespace lw

// Number of kernels this library has enqueued (lw_launch_count()).
void lw_count_launch();

// Host-side launch helper: optional programmatic dependent launch.
template <typename Kernel, typename... Args>
static inline cudaError_t lw_launch(Kernel k, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                    bool pdl, Args... args) {
  lw_count_launch();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, k, args...);
}
