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

// Per-thread prefetch of the cache line holding p into L2 (one LSU instruction;
// the bulk prefetch is warp-uniform and serialises per-lane addresses).
LW_DEV void prefetch_l2_line(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// Programmatic dependent launch: wait for the previous kernel in the stream
// (no-op when the launch did not opt in) / let the next one start its prologue.
LW_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LW_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- peer exchange

constexpr int kMaxRanks = LW_MAX_RANKS;

// Flag of exchange `tag` at step `step` (never 0: receive buffers start zeroed).
LW_DEV uint32_t exchange_flag(int step, int tag, int tags_per_step) {
  const uint32_t f = (uint32_t)step * (uint32_t)tags_per_step + (uint32_t)tag + 1u;
  return f ? f : 1u;
}
LW_DEV uint32_t exchange_flag16(uint32_t flag) { return flag % 65535u + 1u; }

// 8-byte stores / loads that are single-copy atomic and coherent at system
// scope (the word may live on, or be written from, another GPU).
LW_DEV void st_relaxed_sys_u64(void* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
LW_DEV void ld_volatile_v2u64(const void* p, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0,%1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
LW_DEV unsigned long long ld_volatile_u64(const void* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// 4-byte flag words shared by the CTAs of one GPU.
LW_DEV unsigned int ld_volatile_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
LW_DEV void st_volatile_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Slice flags of a cooperatively reduced exchange: one per CTA of the consumer.
constexpr int kSliceFlagsMax = 1024;

LW_DEV unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// A thread's bounded wait for flagged words: `live` turns false, for good,
// once the thread has waited timeout_ns in total (from its first miss) or
// kMaxIters polls; *error is then set to LW_ERR_TIMEOUT. A thread that gave
// up reads what is there without waiting.
struct WaitBudget {
  unsigned long long t0 = 0;
  uint32_t iters = 0;
  bool live = true;
  LW_DEV bool keep_waiting(long long timeout_ns, int* error) {
    constexpr uint32_t kMaxIters = 1u << 24;
    if (!live) return false;
    if (t0 == 0) t0 = globaltimer_ns();
    ++iters;
    if ((iters & 63u) == 0u &&
        ((long long)(globaltimer_ns() - t0) > timeout_ns || iters >= kMaxIters)) {
      live = false;
      if (error) atomicExch(error, (int)LW_ERR_TIMEOUT);
      return false;
    }
    if (iters > 256u) __nanosleep(64);
    return true;
  }
};

// Adds, in rank order, the 8 consecutive flagged fp32 words of ranks
// r0 .. r0 + nr - 1 (nr <= RB; rank j's words at src + j * rank_stride) to
// acc, each read once its flag equals `flag` (bounded). The loads of all nr
// ranks are issued before the first flag is checked.
template <int RB>
LW_DEV void add_flagged8(const unsigned long long* src, size_t rank_stride, int nr, uint32_t flag,
                         float (&acc)[8], WaitBudget& wb, long long timeout_ns, int* error) {
  unsigned long long w[RB][8];
#pragma unroll
  for (int j = 0; j < RB; ++j)
    if (j < nr) {
#pragma unroll
      for (int i = 0; i < 4; ++i) ld_volatile_v2u64(src + j * rank_stride + 2 * i, w[j][2 * i], w[j][2 * i + 1]);
    }
#pragma unroll
  for (int j = 0; j < RB; ++j) {
    if (j >= nr) break;
    for (;;) {
      bool ok = true;
#pragma unroll
      for (int i = 0; i < 8; ++i) ok &= (uint32_t)(w[j][i] >> 32) == flag;
      if (ok || !wb.keep_waiting(timeout_ns, error)) break;
#pragma unroll
      for (int i = 0; i < 4; ++i) ld_volatile_v2u64(src + j * rank_stride + 2 * i, w[j][2 * i], w[j][2 * i + 1]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += __uint_as_float((uint32_t)w[j][i]);
  }
}

// ---------------------------------------------------------------- bulk copies

LW_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

LW_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// The initialised barriers become visible to the asynchronous (bulk copy) proxy.
LW_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// Order this thread's earlier generic-proxy shared-memory accesses before its
// later asynchronous-proxy ones (a bulk copy refilling a slot it has read).
LW_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
LW_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
LW_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that lets the thread sleep up to `ns` nanoseconds for the phase
// (it wakes when the phase completes), instead of returning at once.
LW_DEV bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Global -> shared bulk copy (16-byte aligned addresses, size a multiple of
// 16), its bytes counted on the mbarrier at `bar`.
LW_DEV void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Device error flag of this translation unit (each .cu file has its own copy:
// the library is built without relocatable device code). Bounded waits that
// give up record LW_ERR_TIMEOUT here; lw_take_device_error() reads them.
static __device__ int lw_tu_error;

LW_DEV void lw_record_error(int status) { atomicCAS(&lw_tu_error, 0, status); }

// Wait for phase `parity` of the mbarrier at `bar`, bounded by the global
// timer (timeout_ns) and an iteration cap; records LW_ERR_TIMEOUT on giving up.
LW_DEV bool mbar_wait_bounded(uint32_t bar, uint32_t parity, long long timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 1; it < (1u << 24); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u && (long long)(globaltimer_ns() - t0) > timeout_ns) break;
  }
  lw_record_error(LW_ERR_TIMEOUT);
  return false;
}

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

// ---------------------------------------------------------------- dequant

// INT4: 8 codes in one 32-bit word (code i = nibble i = element k0 + i) are
// unpacked to four half2 holding the exact small integers, paired (0,4) (1,5)
// (2,6) (3,7). With u = nibble ^ 8 = code + 8 in 0..15, the fp16 with bits
// 0x6400 | u is 1024 + u, so subtracting 1032 gives the signed code; the
// nibbles at bits 4..7 land as 1024 + 16u and are rescaled by an exact fma.
// Same unpack without scaling, in PTX: the sign flip is folded into each LOP3
// constant ((x & m) ^ c, c = 0x6400.. | 0x0008..), the fp16 constants live in
// registers (1032 and the (1/16, -72) rescale of the high nibbles).
// Every constant is a register operand (a LOP3 takes one immediate at most;
// a second one would cost a move per use), so the compiler keeps them in
// registers across the unrolled loops.
LW_DEV void unpack_int4_word(uint32_t q, uint32_t (&o)[4]) {
  const uint32_t k1032 = 0x64086408u, k1_16 = 0x2C002C00u, km72 = 0xD480D480u;
  const uint32_t mlo = 0x000F000Fu, mhi = 0x00F000F0u, xlo = 0x64086408u, xhi = 0x64806480u;
  asm("{\n"
      " .reg .b32 y, a, b, c, d;\n"
      " shr.u32 y, %4, 8;\n"
      " lop3.b32 a, %4, %8, %10, 0x6a;\n"
      " lop3.b32 b, %4, %9, %11, 0x6a;\n"
      " lop3.b32 c, y, %8, %10, 0x6a;\n"
      " lop3.b32 d, y, %9, %11, 0x6a;\n"
      " sub.f16x2 %0, a, %5;\n"
      " fma.rn.f16x2 %1, b, %6, %7;\n"
      " sub.f16x2 %2, c, %5;\n"
      " fma.rn.f16x2 %3, d, %6, %7;\n"
      "}\n"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(q), "r"(k1032), "r"(k1_16), "r"(km72), "r"(mlo), "r"(mhi), "r"(xlo), "r"(xhi));
}

// fp16x2 product, round to nearest (one rounding of the exact product).
LW_DEV uint32_t hmul2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// 4 INT8 codes (bytes 0..3 = elements k0..k0+3) to two half2 (0,1) (2,3).
// u = byte ^ 0x80 = code + 128; fp16 bits 0x64uu = 1024 + u; minus 1152.
LW_DEV void dequant_int8_word(uint32_t q, uint32_t (&o)[2]) {
  const uint32_t k1152 = 0x64806480u, magic = 0x64646464u, sign = 0x80808080u;
  asm("{\n"
      " .reg .b32 x, a, b;\n"
      " xor.b32 x, %2, %5;\n"
      " prmt.b32 a, x, %4, 0x4140;\n"
      " prmt.b32 b, x, %4, 0x4342;\n"
      " sub.f16x2 %0, a, %3;\n"
      " sub.f16x2 %1, b, %3;\n"
      "}\n"
      : "=r"(o[0]), "=r"(o[1])
      : "r"(q), "r"(k1152), "r"(magic), "r"(sign));
}

// Permute 8 halves (h0..h7) to (h0,h4)(h1,h5)(h2,h6)(h3,h7): the element
// pairing that unpack_int4_word produces.
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

// Host: read and clear this translation unit's device error flag on the
// current device (synchronous). LW_OK when nothing was recorded.
static inline int lw_tu_take_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, lw::lw_tu_error, sizeof(int)) != cudaSuccess) return LW_ERR_LAUNCH;
  if (v) {
    const int z = 0;
    if (cudaMemcpyToSymbol(lw::lw_tu_error, &z, sizeof(int)) != cudaSuccess) return LW_ERR_LAUNCH;
  }
  return v;
}

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
