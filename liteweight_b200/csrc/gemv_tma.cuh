// Persistent dequant GEMV whose weight stream runs through shared memory.
//
// Same work split, arithmetic, prologues and epilogues as gemv_stream_kernel
// (gemv_core.cuh) with one CTA of kTmaWarps warps per SM, for M <= 8 (one n8
// batch tile) and INT4 / INT8 weights. The difference is how weights reach
// the tensor cores: each warp owns a ring of S slots in shared memory; a slot
// holds one batch (kTmaU chunks of 64 bytes of each of the 16 rows of a tile),
// brought in by 16 bulk asynchronous copies (cp.async.bulk, one per row,
// issued by 16 lanes) whose bytes complete the slot's mbarrier. The warp keeps
// S - 1 batches in flight while it computes one, without holding them in
// registers: ~100-160 KB of weights in flight per SM, against ~64 KB for the
// register double buffer, and one copy instruction per 256-byte row segment
// instead of one load per 16 bytes per lane. The first S batches are issued
// before griddepcontrol.wait, so they stream during the previous kernel.
//
// Slot layout: row r of the tile at r * kTmaRowStride; the 64-byte pad puts
// rows g and g + 1 64 bytes apart modulo 128, so the 8 lanes of a quarter
// warp (rows g, g+1 x pieces t = 0..3) read 8 distinct 16-byte bank groups.
#pragma once

#include "gemv_core.cuh"

namespace lw {

constexpr int kTmaWarps = 8;
constexpr int kTmaThreads = kTmaWarps * 32;
constexpr int kTmaU = 4;                               // chunks per batch
constexpr int kTmaRowStride = kTmaU * 64 + 64;         // bytes
constexpr int kTmaSlotBytes = 16 * kTmaRowStride;      // 5 KB
constexpr int kTmaMaxSlots = 6;
constexpr int kTmaBarBytes = 1024;                     // mbarriers: kTmaWarps * kTmaMaxSlots * 8 B, padded
constexpr long long kTmaWaitNs = 200000000;            // 200 ms: a bulk copy never takes this long

template <int BITS, int PRO, int EPI, bool FOLD>
__global__ void __launch_bounds__(kTmaThreads, 1) gemv_tma_kernel(const StreamParams p) {
  static_assert(BITS == 4 || BITS == 8, "bulk-copy GEMV: INT4 / INT8 weights");
  static_assert(EPI != EPI_PEER_ARGMAX, "the argmax exchange runs on the fp16 lm_head only");
  constexpr int MT = 1;
  constexpr int U = kTmaU;
  constexpr int E = WT<BITS>::E;
  constexpr int KC = 4 * E;
  extern __shared__ __align__(16) uint8_t smem[];   // bulk-copy destinations need 16 B, mbarriers 8 B
  __shared__ float ssq[kMaxM * (kTmaThreads / 32)];

  const int S = p.ring_slots;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int wid = blockIdx.x * kTmaWarps + warp;
  const int C = p.kchunks;
  const int total = p.tiles * C;
  const int g0 = min(total, wid * p.per), g1 = min(total, g0 + p.per);
  const size_t rowbytes = (size_t)p.K * BITS / 8;
  const int ngroups = p.K / p.G;

  uint8_t* ring = smem + kTmaBarBytes + (size_t)warp * S * kTmaSlotBytes;
  __half* act_s = reinterpret_cast<__half*>(smem + kTmaBarBytes + (size_t)kTmaWarps * S * kTmaSlotBytes);
  __half* gam_s = act_s + (size_t)p.M * p.cp;
  const uint32_t bars = smem_u32(smem) + 8u * (uint32_t)(warp * S);
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(bars + 8u * s, 1);
    fence_mbar_init();
  }
  __syncwarp();

  // issue cursor (copies) and compute cursor over the same run of work
  RunCursor is{g0 / max(C, 1), g0 - (g0 / max(C, 1)) * C, g1 - g0};
  RunCursor cs = is;
  uint32_t pending = 0;   // slots with copies not yet waited for
  uint32_t phase = 0;     // bit s: parity of slot s's next completion

  // Next batch of the issue cursor into `slot` (warp-uniform). Rows past N
  // are clamped to N - 1 (computed, never stored); the last chunk of a row may
  // be short (the staged activation is zero there and any byte is a finite code).
  auto issue = [&](int slot) {
    const int bt = is.t, bc = is.c;
    const int n = is.take(U, C);
    if (!n) return;
    const uint32_t bytes = (uint32_t)min((size_t)n * 64, rowbytes - (size_t)bc * 64);
    const uint32_t bar = bars + 8u * slot;
    if (lane == 0) mbar_arrive_expect_tx(bar, 16u * bytes);
    __syncwarp();
    if (lane < 16) {
      const int row = min(bt * 16 + lane, p.N - 1);
      fence_proxy_async_smem();
      bulk_g2s(smem_u32(ring + (size_t)slot * kTmaSlotBytes + lane * kTmaRowStride),
               p.w + (size_t)row * rowbytes + (size_t)bc * 64, bytes, bar);
    }
    pending |= 1u << slot;
  };

  auto load_scales = [&](int bt, int bc, int bn, uint32_t(&sa)[U], uint32_t(&sb)[U]) {
    const int r0 = min(bt * 16 + g, p.N - 1), r1 = min(bt * 16 + g + 8, p.N - 1);
    const unsigned short* s0 = reinterpret_cast<const unsigned short*>(p.scales) + (size_t)r0 * ngroups;
    const unsigned short* s1 = reinterpret_cast<const unsigned short*>(p.scales) + (size_t)r1 * ngroups;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (u < bn) {
        const int grp = min(((bc + u) * KC + (FOLD ? 0 : t * E)) >> p.gshift, ngroups - 1);
        const uint32_t h0 = __ldg(s0 + grp), h1 = __ldg(s1 + grp);
        if constexpr (FOLD) {
          sa[u] = __float_as_uint(__half2float(__ushort_as_half((unsigned short)h0)));
          sb[u] = __float_as_uint(__half2float(__ushort_as_half((unsigned short)h1)));
        } else {
          sa[u] = h0 | (h0 << 16);
          sb[u] = h1 | (h1 << 16);
        }
      }
    }
  };

  // Weights do not depend on the previous kernel: fill the ring first.
  for (int s = 0; s < S; ++s) issue(s);
  uint32_t saA[U], sbA[U], saB[U], sbB[U];
  int tA = cs.t, cA = cs.c, nA = cs.take(U, C);
  if (nA) load_scales(tA, cA, nA, saA, sbA);

  stage_gamma<PRO, kTmaThreads>(p, gam_s);
  pdl_wait();
  pdl_launch_dependents();   // the next kernel's CTAs may fill the SM slots freed here

  uint32_t in_flag = 0, out_flag = 0;
  if constexpr (PRO == PRO_PEER_RESID_NORM) in_flag = exchange_flag(*p.in_step, p.in_tag, p.in_tags);
  if constexpr (kPeerEpi<EPI>) out_flag = exchange_flag(*p.out_step, p.out_tag, p.out_tags);
  WaitBudget wb;
  stage_activation<BITS, PRO, kTmaThreads>(p, act_s, gam_s, ssq, in_flag, wb);

  float acc[MT][4] = {{0.f, 0.f, 0.f, 0.f}};
  int seg_c0 = g0 - (g0 / max(C, 1)) * C;
  const __half* arow[MT] = {act_s + (size_t)min(g, p.M - 1) * p.cp + t * 8};
  bool live = true;   // false once a copy was given up on: stop computing, keep the split-tile protocol
  int slot = 0;

  auto step = [&](int bt, int bc, int bn, const uint32_t(&sa)[U], const uint32_t(&sb)[U]) {
    if (live) {
      live = mbar_wait_bounded(bars + 8u * slot, (phase >> slot) & 1u, kTmaWaitNs);
      if (live) {
        pending &= ~(1u << slot);
        phase ^= 1u << slot;
      }
    }
    if (live) {
      const uint8_t* sl = ring + (size_t)slot * kTmaSlotBytes + t * 16;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (u < bn) {
          const uint4 qa = lds128(sl + g * kTmaRowStride + u * 64);
          const uint4 qb = lds128(sl + (g + 8) * kTmaRowStride + u * 64);
          const int off = (bc + u) * KC;
          if constexpr (FOLD) {
            float dc[MT][4] = {{0.f, 0.f, 0.f, 0.f}};
            gemv_piece_codes<BITS, MT>(dc, qa, qb, arow, off);
            const float s0f = __uint_as_float(sa[u]), s1f = __uint_as_float(sb[u]);
            acc[0][0] = fmaf(dc[0][0], s0f, acc[0][0]);
            acc[0][1] = fmaf(dc[0][1], s0f, acc[0][1]);
            acc[0][2] = fmaf(dc[0][2], s1f, acc[0][2]);
            acc[0][3] = fmaf(dc[0][3], s1f, acc[0][3]);
          } else {
            gemv_piece<BITS, MT>(acc, qa, qb, sa[u], sb[u], arow, off);
          }
        }
      }
      __syncwarp();   // every lane is done with the slot before it is refilled
      issue(slot);
    }
    slot = slot + 1 == S ? 0 : slot + 1;
    const int end_c = bc + bn;
    if (end_c == C || bt * C + end_c == g1) {
      flush_tile<MT, EPI>(p, bt, seg_c0, end_c, wid, acc, lane, out_flag);
      acc[0][0] = acc[0][1] = acc[0][2] = acc[0][3] = 0.f;
      seg_c0 = 0;
    }
  };

  while (nA) {
    int tB = cs.t, cB = cs.c, nB = cs.take(U, C);
    if (nB) load_scales(tB, cB, nB, saB, sbB);
    step(tA, cA, nA, saA, sbA);
    if (!nB) break;
    tA = cs.t;
    cA = cs.c;
    nA = cs.take(U, C);
    if (nA) load_scales(tA, cA, nA, saA, sbA);
    step(tB, cB, nB, saB, sbB);
  }

  // Copies are only ever left in flight after a wait gave up: wait for them
  // (bounded again) so none lands after the CTA has exited.
  if (pending) {
    for (int s = 0; s < S; ++s)
      if ((pending >> s) & 1u) mbar_wait_bounded(bars + 8u * s, (phase >> s) & 1u, kTmaWaitNs);
  }

}

}  // namespace lw
