// Dequant GEMV for M <= 8 whose weight stream runs through a CTA-wide shared
// memory ring fed by TMA tile copies (sm_100a).
//
// Same arithmetic, prologues and epilogues as gemv_stream_kernel
// (gemv_core.cuh): out[m, n] = sum_k act[m, k] * W[n, k] with every weight
// dequantized exactly (fp16(code * scale), liteweight/quantize.py:30-43,
// :102-128), fp32 tensor-core sums, one fp16 rounding.
//
// Work. A unit is one 16-row tile of the weight matrix over all of K. Its
// bytes stream in stages of 16 rows x 1024 bytes (16 KB: one 3-D TMA box of
// 8 chunks x 16 rows x 128 bytes - eight 16-row x 128-byte 2-D boxes when the
// row bytes are not whole 128-byte chunks - 128-byte swizzle), `spr` stages
// per unit; its fp16 scales (16 consecutive rows of the scale matrix, one
// contiguous block) arrive with one bulk copy into one of four unit buffers.
// CTA b takes units b, b + grid, b + 2 grid, ...: no CTA waits on another or
// on a global counter (claiming units through one atomic counter was measured
// slower: under a full weight stream each claim's round trip stalls the
// producer). A tile is never split between CTAs: no partial sum leaves the SM.
//
// Roles (one CTA per SM, 18 warps):
//   warp 16    one lane copies each unit's scales into the next free unit
//              buffer and issues each stage's weight copy into the next free
//              ring slot, writing the stage's unit id into the slot's header.
//              It starts before griddepcontrol.wait: weights do not depend on
//              the previous kernel, so up to `stages` x 16 KB per SM stream in
//              while that kernel finishes (unless weights_after_wait: the
//              drop-in ops, whose weights a previous kernel may have written,
//              only overlap the launch and the barrier setup).
//   warps 0-15 warp w owns chunk w (64 bytes of each row) of every stage: per
//              stage each lane reads 16 bytes of two rows, unpacks and scales
//              them, and feeds mma.sync m16n8k16 with the staged activation
//              as operand B, spreading the MMAs over four accumulators (a
//              dependent mma.sync waits for the previous result); it takes
//              its scales for the whole unit from the unit buffer at the
//              unit's start. At the end of a unit every warp writes its
//              partial tile into one of four shared-memory buffers and goes
//              on to the next unit.
//   warp 17    the reducer: sums each unit's 16 partial tiles in warp order
//              (the same sums on every run) and applies the epilogue, off the
//              consumers' path.
// Lane (g, t) holds tile rows pi(g) and pi(g) + 8, pi(g) = (g >> 1) |
// ((g & 1) << 2): with the 128-byte swizzle (16-byte piece j of row r at
// piece j ^ (r & 7)) the 8 lanes of each quarter warp then read 8 distinct
// bank groups. The epilogues take pi(g) as the lane's row.
//
// Every wait is bounded: on expiry the kernel records LW_ERR_TIMEOUT (device
// error flag), the roles stop at their next wait, and the producer waits
// (bounded) for the copies it issued before the CTA exits.
#pragma once

#include <cuda.h>   // CUtensorMap

#include "gemv_core.cuh"

namespace lw {

constexpr int kRingConsumerWarps = 16;
constexpr int kRingConsumers = kRingConsumerWarps * 32;
constexpr int kRingProducerWarp = kRingConsumerWarps;       // warp 16
constexpr int kRingReducerWarp = kRingConsumerWarps + 1;    // warp 17
constexpr int kRingThreads = kRingConsumers + 64;
constexpr int kRingCombBufs = 4;                            // partial-tile buffers (units in flight to the reducer)
constexpr int kRingStageRowBytes = 1024;               // bytes of each tile row per stage
constexpr int kRingBoxes = kRingStageRowBytes / 128;   // 16-row x 128-byte TMA boxes per stage
constexpr int kRingStageBytes = 16 * kRingStageRowBytes;
constexpr int kRingMaxStages = 13;
constexpr int kRingMaxUnit = 8;                        // stages of a unit with scales (row bytes <= 8 KB)
constexpr int kRingScaleBufs = 4;                      // unit scale buffers
constexpr int kRingMaxScaleBytes = 4096;               // one buffer: 16 rows x up to 128 groups x 2 bytes
constexpr int kRingHeadBytes = 1024;                   // barriers + headers
constexpr int kRingCombBytes = kRingCombBufs * kRingConsumerWarps * 32 * 16;   // partial tiles
// shared memory a launch needs besides its ring and staged activation (the
// ring starts on a 1024-byte boundary, hence the slack)
constexpr int kRingFixedBytes = kRingHeadBytes + kRingCombBytes + kRingScaleBufs * kRingMaxScaleBytes + 1024;
constexpr long long kRingWaitNs = 2000000000;          // 2 s: far beyond any copy or hand-off
// The producer's wait for a free slot also spans the consumers' wait for the
// previous kernel (programmatic dependent launch) and their wait for other
// ranks (PRO_PEER_RESID_NORM, up to in_timeout_ns): its bound is this much
// longer than the latter.
constexpr long long kRingProducerWaitNs = 60000000000LL;

struct RingParams {
  StreamParams p;          // matmul, prologue, epilogue (p.kchunks = 16 * spr, p.cp staged row stride)
  CUtensorMap tm_w;        // weight rows [N][K * BITS / 8 bytes] u8, 128-byte swizzle (see map3d)
  int spr;                 // stages per unit (ceil(row bytes / 1024))
  int boxes_last;          // 2-D boxes of a unit's last stage that start inside the row
  int units;               // ceil(N / 16)
  int stages;              // ring slots
  int map3d;               // 1: tm_w is the 3-D view {128 bytes, rows, row bytes / 128}, one box per stage
  int weights_after_wait;  // 1: weights and scales are read after griddepcontrol.wait too (they may be
                           // the previous kernel's output: the drop-in ops launched with PDL)
};

LW_DEV void tma_load_box(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
LW_DEV void tma_load_box3(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}
LW_DEV void mbar_arrive_local(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
LW_DEV void named_sync(int id, int nthreads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory"); }

// The lane's lower tile row (see the file comment).
LW_DEV int ring_row(int g) { return (g >> 1) | ((g & 1) << 2); }

// gemv_piece (exact dequant) for one row pair, its MMAs spread over four
// accumulators: a dependent mma.sync waits for its predecessor's result, so
// one accumulator per warp would make each stage a chain of 8 MMAs.
template <int BITS>
LW_DEV void ring_piece(float (&acc)[4][4], const uint4& qa, const uint4& qb, uint32_t sa, uint32_t sb,
                       const __half* arow, int off) {
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
      const uint4 av = *reinterpret_cast<const uint4*>(arow + off + w * 32);
      mma16816(acc[(2 * w) & 3], A[0], B[0], A[1], B[1], av.x, av.y);
      mma16816(acc[(2 * w + 1) & 3], A[2], B[2], A[3], B[3], av.z, av.w);
    }
  } else if constexpr (BITS == 8) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 av = *reinterpret_cast<const uint4*>(arow + off + j * 32);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t A[2], B[2];
        dequant_int8_word(a32[2 * j + h], A);
        dequant_int8_word(b32[2 * j + h], B);
        A[0] = hmul2_rn(A[0], sa);
        A[1] = hmul2_rn(A[1], sa);
        B[0] = hmul2_rn(B[0], sb);
        B[1] = hmul2_rn(B[1], sb);
        mma16816(acc[2 * j + h], A[0], B[0], A[1], B[1], h ? av.z : av.x, h ? av.w : av.y);
      }
    }
  } else {
    const uint4 av = *reinterpret_cast<const uint4*>(arow + off);
    mma16816(acc[0], qa.x, qb.x, qa.y, qb.y, av.x, av.y);
    mma16816(acc[1], qa.z, qb.z, qa.w, qb.w, av.z, av.w);
  }
}

// ---- codes variant (FOLD): scales applied per chunk in fp32
// Each code enters the tensor core as an exact fp16 subnormal: (code + 8) *
// 2^-24 for INT4 (the nibble XOR 8 in the low bits of a half; a nibble four
// bits up is 16 times that and is summed apart) and (code + 128) * 2^-24 for
// INT8 (the byte XOR 0x80). For a 64-byte chunk of a row (one scale group) the
// fp32 sum d of those products gives
//   sum_k code_k * a_k = 2^24 * d - OFF * sum_k a_k      (OFF = 8 or 128)
// with sum_k a_k the chunk's activation sum, staged once per launch; the
// result is scaled by the group's scale in fp32. The weights are not rounded
// to fp16(code * scale) first, so this is an opt-in (fold_scales), not the
// numerics of liteweight's dequantize.
LW_DEV void codes_int4_word(uint32_t q, uint32_t (&o)[4]) {
  const uint32_t mlo = 0x000F000Fu, mhi = 0x00F000F0u, xlo = 0x00080008u, xhi = 0x00800080u;
  asm("{\n"
      " .reg .b32 y;\n"
      " shr.u32 y, %4, 8;\n"
      " lop3.b32 %0, %4, %5, %7, 0x6a;\n"
      " lop3.b32 %1, %4, %6, %8, 0x6a;\n"
      " lop3.b32 %2, y, %5, %7, 0x6a;\n"
      " lop3.b32 %3, y, %6, %8, 0x6a;\n"
      "}\n"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(q), "r"(mlo), "r"(mhi), "r"(xlo), "r"(xhi));
}

// bytes 0, 1 (o[0]) and 2, 3 (o[1]) as (code + 128) * 2^-24
LW_DEV void codes_int8_word(uint32_t q, uint32_t (&o)[2]) {
  const uint32_t x = q ^ 0x80808080u;
  o[0] = __byte_perm(x, 0u, 0x4140);
  o[1] = __byte_perm(x, 0u, 0x4342);
}

// d = a * b (no accumulator input)
LW_DEV void mma16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// The lane's 16-byte pieces of rows gr (qa) and gr + 8 (qb) in one chunk:
// d (INT4: the low nibbles into dlo, the high ones into dhi; two chains of
// each) starts from zero. Same activation pairing as gemv_piece
// (perm_int4_pairs for INT4).
template <int BITS>
LW_DEV void ring_codes_piece(float (&dlo)[2][4], float (&dhi)[2][4], const uint4& qa, const uint4& qb,
                             const __half* arow, int off) {
  const uint32_t* a32 = reinterpret_cast<const uint32_t*>(&qa);
  const uint32_t* b32 = reinterpret_cast<const uint32_t*>(&qb);
  if constexpr (BITS == 4) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t A[4], B[4];
      codes_int4_word(a32[w], A);
      codes_int4_word(b32[w], B);
      const uint4 av = *reinterpret_cast<const uint4*>(arow + off + w * 32);
      if (w < 2) {
        mma16816_z(dlo[w & 1], A[0], B[0], A[2], B[2], av.x, av.z);
        mma16816_z(dhi[w & 1], A[1], B[1], A[3], B[3], av.y, av.w);
      } else {
        mma16816(dlo[w & 1], A[0], B[0], A[2], B[2], av.x, av.z);
        mma16816(dhi[w & 1], A[1], B[1], A[3], B[3], av.y, av.w);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 av = *reinterpret_cast<const uint4*>(arow + off + j * 32);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t A[2], B[2];
        codes_int8_word(a32[2 * j + h], A);
        codes_int8_word(b32[2 * j + h], B);
        if (j == 0)
          mma16816_z(dlo[h], A[0], B[0], A[1], B[1], h ? av.z : av.x, h ? av.w : av.y);
        else
          mma16816(dlo[h], A[0], B[0], A[1], B[1], h ? av.z : av.x, h ? av.w : av.y);
      }
    }
  }
}

// acc += scale * (2^24 d - OFF * asum) for the lane's rows (lo, hi: the two
// fp16 scales in s2) and columns 2t, 2t + 1 (asum: that chunk's activation sums).
template <int BITS>
LW_DEV void ring_codes_finish(float (&acc)[4], const float (&dlo)[2][4], const float (&dhi)[2][4], uint32_t s2,
                              float2 asum) {
  constexpr float kOff = BITS == 4 ? 8.f : 128.f;
  const float slo = __half2float(__ushort_as_half((unsigned short)(s2 & 0xFFFFu)));
  const float shi = __half2float(__ushort_as_half((unsigned short)(s2 >> 16)));
  const float s24[2] = {slo * 16777216.f, shi * 16777216.f};   // exact: a power of two
  const float soff[2] = {-kOff * slo, -kOff * shi};            // exact likewise
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = dlo[0][i] + dlo[1][i];
    const float d = BITS == 4 ? fmaf(dhi[0][i] + dhi[1][i], 0.0625f, lo) : lo;
    acc[i] = fmaf(d, s24[i >> 1], fmaf(soff[i >> 1], (i & 1) ? asum.y : asum.x, acc[i]));
  }
}

// Shared memory of the per-chunk activation sums of the codes variant: [chunk][8 columns] fp32.
__host__ __device__ constexpr int ring_asum_bytes(int spr) { return 16 * spr * 8 * 4; }

template <int BITS, int PRO, int EPI, bool FOLD = false>
__global__ void __launch_bounds__(kRingThreads, 1) gemv_ring_kernel(const __grid_constant__ RingParams rp) {
  constexpr int MT = 1;
  constexpr int E = WT<BITS>::E;
  constexpr int KC = 4 * E;
  constexpr bool SCALED = BITS < 16;
  const StreamParams& p = rp.p;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ float ssq[kMaxM * kRingConsumerWarps];
  __shared__ volatile int abort_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = rp.stages;
  const int ngroups = SCALED ? p.K / p.G : 1;
  // layout: [ring barriers, headers, partial-tile and scale-buffer barriers |
  // partial tiles | unit scale buffers | ring (1024-aligned: the swizzle
  // pattern follows address bits 4-9) | staged activation, gamma]
  const uint32_t base = smem_u32(smem_raw);
  const uint32_t full0 = base, empty0 = base + 8u * kRingMaxStages;
  int* hdr = reinterpret_cast<int*>(smem_raw + 16 * kRingMaxStages);   // [S][2]: unit
  const uint32_t cfull0 = base + 512, cempty0 = base + 544;           // [partial-tile buffer]
  const uint32_t sfull0 = base + 576, sempty0 = base + 608;           // [scale buffer]
  int* cunit = reinterpret_cast<int*>(smem_raw + 640);                // [partial-tile buffer]: its unit, -1 = end
  float* comb = reinterpret_cast<float*>(smem_raw + kRingHeadBytes);   // [buffer][warp][lane][4]
  const uint32_t sbuf_off = (uint32_t)(kRingHeadBytes + kRingCombBytes);
  const uint32_t ring_addr =
      (base + sbuf_off + (uint32_t)(kRingScaleBufs * kRingMaxScaleBytes) + 1023u) & ~1023u;
  uint8_t* ring = smem_raw + (ring_addr - base);
  __half* act_s = reinterpret_cast<__half*>(ring + (size_t)S * kRingStageBytes);
  __half* gam_s = act_s + (size_t)p.M * p.cp;
  // (codes variant) per-chunk activation sums, after the activation and gamma
  float* asum_s = reinterpret_cast<float*>(
      reinterpret_cast<uint8_t*>(act_s) +
      (((size_t)p.M * p.cp * 2 + (PRO == PRO_PLAIN ? 0 : (size_t)(p.K + 7) / 8 * 16) + 15) & ~(size_t)15));

  // the weight map's descriptor is fetched while the barriers are set up
  if (tid == kRingProducerWarp * 32)
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&rp.tm_w)) : "memory");
  // barriers: one per lane of warp 0 (lane s < 16: ring slot s; 16 + h: partial-tile
  // buffer h; 20 + j: scale buffer j), each lane fencing its own inits
  static_assert(kRingMaxStages <= 16 && kRingCombBufs <= 4 && kRingScaleBufs <= 4, "one barrier pair per lane");
  if (warp == 0) {
    bool did = false;
    if (lane < S) {
      mbar_init(full0 + 8u * lane, 1);
      mbar_init(empty0 + 8u * lane, kRingConsumerWarps);
      did = true;
    } else if (lane >= 16 && lane < 16 + kRingCombBufs) {
      mbar_init(cfull0 + 8u * (lane - 16), kRingConsumerWarps);
      mbar_init(cempty0 + 8u * (lane - 16), 1);
      did = true;
    } else if (lane >= 20 && lane < 20 + kRingScaleBufs) {
      mbar_init(sfull0 + 8u * (lane - 20), 1);
      mbar_init(sempty0 + 8u * (lane - 20), kRingConsumerWarps);
      did = true;
    }
    if (lane == 31) abort_s = 0;
    if (did) fence_mbar_init();
  }
  __syncthreads();

  auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_s) return false;
    if (mbar_wait_bounded(bar, parity, kRingWaitNs)) return true;
    abort_s = 1;
    return false;
  };

  if (warp == kRingProducerWarp) {
    // ------------------------------------------------------------ producer
    const int units = rp.units;
    const int grid = (int)gridDim.x;
    // the free-slot wait: long bound, gives up at once when a consumer aborted
    auto wait_free = [&](uint32_t bar, uint32_t parity) -> bool {
      if (mbar_try_wait(bar, parity)) return true;
      const long long limit = kRingProducerWaitNs + (PRO == PRO_PEER_RESID_NORM ? p.in_timeout_ns : 0);
      const unsigned long long t0 = globaltimer_ns();
      for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if (abort_s) return false;
        if ((it & 255u) == 0u && (long long)(globaltimer_ns() - t0) > limit) break;
      }
      lw_record_error(LW_ERR_TIMEOUT);
      abort_s = 1;
      return false;
    };
    if (rp.weights_after_wait) pdl_wait();
    // units b, b + grid, b + 2 grid, ...
    int u = (int)blockIdx.x;
    int slot = 0, nunit = 0;
    uint32_t phase = 0;               // parity of the ring's current lap
    uint32_t issued = 0;              // bit s: slot s has held a copy
    bool live = true;
    while (live && u < units) {
      if constexpr (SCALED) {
        // the unit's scales: rows u*16 .. u*16+15 are one contiguous block
        const int j = nunit & (kRingScaleBufs - 1);
        if (!wait_free(sempty0 + 8u * j, ((nunit / kRingScaleBufs) & 1) ^ 1u)) {
          live = false;
          break;
        }
        if (lane == 0) {
          const uint32_t bytes = (uint32_t)(min(16, p.N - u * 16) * ngroups * 2);
          mbar_arrive_expect_tx(sfull0 + 8u * j, bytes);
          bulk_g2s(base + sbuf_off + (uint32_t)j * kRingMaxScaleBytes, p.scales + (size_t)u * 16 * ngroups, bytes,
                   sfull0 + 8u * j);
        }
      }
      ++nunit;
      for (int st = 0; st < rp.spr; ++st) {
        // the slot's previous contents have been read by all consumer warps
        if (!wait_free(empty0 + 8u * slot, phase ^ 1u)) {
          live = false;
          break;
        }
        if (lane == 0) {
          hdr[2 * slot] = u;
          const uint32_t dst = ring_addr + (uint32_t)slot * kRingStageBytes;
          if (rp.map3d) {
            // one copy: chunks past the row end are filled with zeros (and counted)
            mbar_arrive_expect_tx(full0 + 8u * slot, (uint32_t)kRingStageBytes);
            tma_load_box3(dst, &rp.tm_w, 0, u * 16, st * kRingBoxes, full0 + 8u * slot);
          } else {
            const int nb = st + 1 < rp.spr ? kRingBoxes : rp.boxes_last;
            mbar_arrive_expect_tx(full0 + 8u * slot, (uint32_t)(nb * 16 * 128));
            for (int b = 0; b < nb; ++b)
              tma_load_box(dst + (uint32_t)b * 2048u, &rp.tm_w, st * kRingStageRowBytes + b * 128, u * 16,
                           full0 + 8u * slot);
          }
        }
        issued |= 1u << slot;
        if (++slot == S) {
          slot = 0;
          phase ^= 1u;
        }
      }
      u += grid;
    }
    if (live) {
      // end of work: an empty stage with header -1
      if (wait_free(empty0 + 8u * slot, phase ^ 1u)) {
        if (lane == 0) {
          hdr[2 * slot] = -1;
          mbar_arrive_local(full0 + 8u * slot);
        }
        // this slot's last copy was consumed (hence landed) before it was
        // released, and its barrier has now completed one phase more: no wait
        issued &= ~(1u << slot);
      } else {
        live = false;
      }
    }
    // No copy may land after the CTA has exited: wait (bounded) for each
    // slot's newest copy - this lap's for the slots before `slot`, the last
    // lap's for the others - and for each scale buffer's newest copy. In a
    // healthy run they have all landed.
    for (int s = 0; s < S; ++s) {
      if (!((issued >> s) & 1u)) continue;
      mbar_wait_bounded(full0 + 8u * s, (s < slot) ? phase : (phase ^ 1u), kRingWaitNs);
    }
    if constexpr (SCALED) {
      for (int k = max(0, nunit - kRingScaleBufs); k < nunit; ++k)
        mbar_wait_bounded(sfull0 + 8u * (k & (kRingScaleBufs - 1)), (k / kRingScaleBufs) & 1, kRingWaitNs);
    }
    return;
  }

  const int g = lane >> 2, t = lane & 3;
  const int gr = ring_row(g);

  if (warp == kRingReducerWarp) {
    // ------------------------------------------------------------ reducer
    pdl_wait();
    uint32_t out_flag = 0;
    if constexpr (kPeerEpi<EPI>) out_flag = exchange_flag(*p.out_step, p.out_tag, p.out_tags);
    for (int k = 0;; ++k) {
      const int b = k & (kRingCombBufs - 1);
      if (!wait(cfull0 + 8u * b, (k / kRingCombBufs) & 1)) break;
      const int u = cunit[b];
      if (u < 0) break;
      const float* cb = comb + (size_t)b * kRingConsumerWarps * 32 * 4;
      float sum[MT][4] = {{0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int w = 0; w < kRingConsumerWarps; ++w) {
        const float4 f = *reinterpret_cast<const float4*>(cb + ((size_t)w * 32 + lane) * 4);
        sum[0][0] += f.x;
        sum[0][1] += f.y;
        sum[0][2] += f.z;
        sum[0][3] += f.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_local(cempty0 + 8u * b);
      finish_tile<MT, EPI>(p, u, sum, lane, out_flag, gr);
    }
    if constexpr (EPI == EPI_PEER_ARGMAX) {
      // The last CTA to finish (every CTA's atomicMax is then in the local
      // keys) sends this rank's keys to every rank as flagged words.
      int last = 0;
      if (lane == 0) {
        __threadfence();
        last = atomicAdd(p.out_arrivals, 1) == (int)gridDim.x - 1;
      }
      if (__shfl_sync(0xffffffffu, last, 0)) {
        __threadfence();
        const unsigned long long f16 = (unsigned long long)exchange_flag16(out_flag) << 48;
        for (int m = lane; m < p.M; m += 32) {
          const unsigned long long word = (__ldcg(p.argmax_keys + m) & 0xFFFFFFFFFFFFull) | f16;
#pragma unroll
          for (int d = 0; d < kMaxRanks; ++d)
            if (d < p.out_world) st_relaxed_sys_u64(p.out_dst[d] + (size_t)p.out_rank * p.M + m, word);
        }
        if (lane == 0) *p.out_arrivals = 0;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // this lane's 16-byte piece of a stage: box warp / 2, its half warp % 2, rows gr and gr + 8
  const uint32_t piece_off = (uint32_t)((warp >> 1) * 2048 + gr * 128 + (((4 * (warp & 1) + t) ^ gr) << 4));
  // scale group of this lane's piece in stage st (the same for every unit)
  int goff[kRingMaxUnit];
#pragma unroll
  for (int st = 0; st < kRingMaxUnit; ++st) goff[st] = min(((st * 16 + warp) * KC + t * E) >> p.gshift, ngroups - 1);

  stage_gamma<PRO, kRingConsumers>(p, gam_s);
  pdl_wait();
  pdl_launch_dependents();
  uint32_t in_flag = 0;
  if constexpr (PRO == PRO_PEER_RESID_NORM) in_flag = exchange_flag(*p.in_step, p.in_tag, p.in_tags);
  WaitBudget wb;
  stage_activation<BITS, PRO, kRingConsumers, 1>(p, act_s, gam_s, ssq, in_flag, wb);
  if constexpr (FOLD) {
    // each chunk's activation sum per column (columns past M: zero)
    for (int c = warp; c < p.kchunks; c += kRingConsumerWarps) {
      for (int m = 0; m < 8; ++m) {
        float sum = 0.f;
        if (m < p.M) {
          for (int e = lane; e < KC; e += 32) sum += __half2float(act_s[(size_t)m * p.cp + c * KC + e]);
          sum = warp_sum(sum);
        }
        if (lane == 0) asum_s[c * 8 + m] = sum;
      }
    }
    stage_sync<1, kRingConsumers>();
  }

  const __half* arow[MT] = {act_s + (size_t)min(g, p.M - 1) * p.cp + t * 8};
  int slot = 0;
  uint32_t phase = 0;
  int nunit = 0;   // units done: partial-tile buffer and scale buffer nunit % 4
  // this warp's partial tile of unit u (-1: the end) into buffer nunit % 4,
  // once the reducer has read that buffer's previous unit
  auto hand_off = [&](int u, const float (&acc)[MT][4]) -> bool {
    const int b = nunit & (kRingCombBufs - 1);
    const uint32_t use = (uint32_t)(nunit / kRingCombBufs);
    if (use > 0 && !wait(cempty0 + 8u * b, (use - 1) & 1u)) return false;
    float* cb = comb + (size_t)b * kRingConsumerWarps * 32 * 4;
    *reinterpret_cast<float4*>(cb + ((size_t)warp * 32 + lane) * 4) =
        make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
    if (warp == 0 && lane == 0) cunit[b] = u;
    __syncwarp();
    if (lane == 0) mbar_arrive_local(cfull0 + 8u * b);
    return true;
  };
  for (;;) {
    if (!wait(full0 + 8u * slot, phase)) break;
    const int u = hdr[2 * slot];
    if (u < 0) break;
    // the unit's scales, one fp16 per stage for each of the lane's two rows
    // (lo = row gr, hi = row gr + 8; rows past N read row N - 1)
    uint32_t sv[kRingMaxUnit];
    if constexpr (SCALED) {
      const int j = nunit & (kRingScaleBufs - 1);
      if (!wait(sfull0 + 8u * j, (nunit / kRingScaleBufs) & 1)) break;
      const unsigned short* sb =
          reinterpret_cast<const unsigned short*>(smem_raw + sbuf_off + j * kRingMaxScaleBytes);
      const int last = p.N - 1 - u * 16;
      const unsigned short* s0 = sb + min(gr, last) * ngroups;
      const unsigned short* s1 = sb + min(gr + 8, last) * ngroups;
#pragma unroll
      for (int st = 0; st < kRingMaxUnit; ++st) {
        if (st >= rp.spr) break;
        sv[st] = (uint32_t)s0[goff[st]] | ((uint32_t)s1[goff[st]] << 16);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_local(sempty0 + 8u * j);
    }
    float acc[MT][4] = {{0.f, 0.f, 0.f, 0.f}};   // codes variant: the unit's sum
    float acc4[4][4] = {};                        // exact: four chains, summed at the unit's end
    bool ok = true;
    auto one = [&](int st, uint32_t s2) {
      const uint8_t* sp = ring + (size_t)slot * kRingStageBytes + piece_off;
      const uint4 qa = lds128(sp), qb = lds128(sp + 8 * 128);
      const int off = (st * 16 + warp) * KC;
      if constexpr (FOLD) {
        float dlo[2][4], dhi[2][4];
        ring_codes_piece<BITS>(dlo, dhi, qa, qb, arow[0], off);
        const float2 as = *reinterpret_cast<const float2*>(asum_s + (st * 16 + warp) * 8 + 2 * t);
        ring_codes_finish<BITS>(acc[0], dlo, dhi, s2, as);
      } else {
        const uint32_t sa = __byte_perm(s2, 0, 0x1010), sb = __byte_perm(s2, 0, 0x3232);
        ring_piece<BITS>(acc4, qa, qb, sa, sb, arow[0], off);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_local(empty0 + 8u * slot);
      if (++slot == S) {
        slot = 0;
        phase ^= 1u;
      }
    };
    if constexpr (SCALED) {
#pragma unroll
      for (int st = 0; st < kRingMaxUnit; ++st) {
        if (st >= rp.spr) break;
        if (st > 0 && !wait(full0 + 8u * slot, phase)) {
          ok = false;
          break;
        }
        one(st, sv[st]);
      }
    } else {
#pragma unroll 1
      for (int st = 0; st < rp.spr; ++st) {
        if (st > 0 && !wait(full0 + 8u * slot, phase)) {
          ok = false;
          break;
        }
        one(st, 0u);
      }
    }
    if (!ok) break;
    if constexpr (!FOLD) {
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[0][i] = (acc4[0][i] + acc4[1][i]) + (acc4[2][i] + acc4[3][i]);
    }
    // ---- the unit's partial tile goes to the reducer
    if (!hand_off(u, acc)) break;
    ++nunit;
  }
  // end of work: an empty hand-off with unit -1 lets the reducer finish
  if (!abort_s) {
    float zero[MT][4] = {{0.f, 0.f, 0.f, 0.f}};
    hand_off(-1, zero);
  }
}

}  // namespace lw
