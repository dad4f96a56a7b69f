// Host-side planning and launch of the persistent stream-K GEMV kernel.
#pragma once

#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "gemv_core.cuh"
#include "gemv_ring.cuh"
#include "gemv_tma.cuh"
#include "tma_host.cuh"

namespace lw {

constexpr int kStageBudget = 220 * 1024;   // dynamic shared memory for the staged activation
constexpr int kBatch = 2;                  // 16-byte chunks per row per register buffer
// fp16 weights carry no dequant temporaries, so their register buffers hold 4
// chunks (more bytes in flight per warp; the fp16 lm_head measured 5 % faster).
template <int BITS>
constexpr int kBatchOf = BITS == 16 ? 4 : kBatch;
// Workspace layout: a fixed region of per-tile counters (kept zero between
// calls, so any later call of any shape finds its counters zero), then the
// fp32 slots, which are fully rewritten before they are read.
constexpr size_t kCounterBytes = 64 * 1024;
constexpr int kMaxSplitTiles = (int)(kCounterBytes / 4);

inline int device_sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct StreamPlan {
  int tiles, kchunks, cp, per, grid, max_slots, mt;
  size_t smem, ws_bytes;  // ws_bytes = 0 when no tile is split
  int ring_slots;         // > 0: the bulk-copy kernel (gemv_tma_kernel) with this many slots per warp
};

// The bulk-copy GEMV (gemv_tma.cuh) serves M <= 8 with INT4 / INT8 weights
// when the environment sets LW_B200_GEMV=bulk; by default every launch uses
// the register-pipeline kernel, which measures faster on B200 (the per-lane
// bulk copies are issued one lane at a time through uniform registers).
inline bool tma_enabled() {
  static const bool on = [] {
    const char* v = getenv("LW_B200_GEMV");
    return v && strcmp(v, "bulk") == 0;
  }();
  return on;
}

constexpr size_t kTmaSmemBudget = 232448 - 512;   // opt-in dynamic shared memory per CTA, less static

// Shared memory for the RMSNorm weight of the norm prologues (K halves, whole 16-byte groups).
inline size_t gamma_bytes(int pro, int K) { return pro == PRO_PLAIN ? 0 : (size_t)(K + 7) / 8 * 16; }

// Plan of the bulk-copy kernel; false when its ring (>= 3 slots per warp) and
// the staged activation do not fit in shared memory.
template <int BITS, int PRO>
bool plan_tma(int M, int N, int K, bool allow_split, StreamPlan* pl) {
  constexpr int KC = 4 * WT<BITS>::E;
  if (BITS == 16 || M > 8) return false;
  pl->mt = 1;
  pl->tiles = (N + 15) / 16;
  pl->kchunks = (K + KC - 1) / KC;
  const int kpad = pl->kchunks * KC;
  pl->cp = ((size_t)M * (kpad + 32) * 2 <= (size_t)kStageBudget) ? kpad + 32 : kpad;
  const size_t act = align_up((size_t)M * pl->cp * 2 + gamma_bytes(PRO, K), 128);
  if (act + kTmaBarBytes >= kTmaSmemBudget) return false;
  const int slots = (int)std::min<size_t>(kTmaMaxSlots, (kTmaSmemBudget - kTmaBarBytes - act) /
                                                            ((size_t)kTmaWarps * kTmaSlotBytes));
  if (slots < 3) return false;
  pl->ring_slots = slots;
  pl->smem = kTmaBarBytes + (size_t)kTmaWarps * slots * kTmaSlotBytes + act;
  const long long warps_max = (long long)device_sm_count() * kTmaWarps;
  const long long total = (long long)pl->tiles * pl->kchunks;
  long long per = std::max<long long>(kTmaU, (total + warps_max - 1) / warps_max);
  if (!allow_split || pl->tiles > kMaxSplitTiles) per = (per + pl->kchunks - 1) / pl->kchunks * pl->kchunks;
  pl->per = (int)per;
  const long long warps = (total + per - 1) / per;
  pl->grid = (int)((warps + kTmaWarps - 1) / kTmaWarps);
  const bool split = (per % pl->kchunks) != 0;
  pl->max_slots = split ? (pl->kchunks - 1) / pl->per + 2 : 0;
  pl->ws_bytes = split ? kCounterBytes + (size_t)pl->tiles * pl->max_slots * 32 * 4 * 4 : 0;
  return true;
}

inline int mt_for(int M) { return M <= 8 ? 1 : (M <= 16 ? 2 : 4); }

// Largest activation row block one launch can stage.
template <int BITS>
int stage_rows(int K) {
  constexpr int KC = 4 * WT<BITS>::E;
  const int kpad = ((K + KC - 1) / KC) * KC;
  return std::max(1, std::min(kMaxM, kStageBudget / (kpad * 2)));
}

// Scale-group shift: element k is in group k >> gshift. -1 when the group size
// is neither a power of two nor K (the stream kernel does not take it).
inline int group_shift(int K, int G) {
  if (G == K) return 31;
  if (G <= 0 || (G & (G - 1))) return -1;
  int s = 0;
  while ((1 << s) < G) ++s;
  return s;
}

// Every 4-lane chunk inside one scale group: the codes may be summed unscaled and
// each chunk sum scaled once in fp32. This skips the fp16 rounding of code *
// scale that liteweight's dequantize (and its Triton kernels) apply, so it is an
// opt-in: the drop-in matmul entry points always dequantize exactly.
template <int BITS>
inline bool fold_scales(int K, int G) {
  constexpr int KC = 4 * WT<BITS>::E;
  return BITS < 16 && (G == K || G % KC == 0);
}

template <int BITS, int MT, int PRO, int EPI>
cudaError_t plan_for(int M, int N, int K, bool allow_split, StreamPlan* pl) {
  constexpr int KC = 4 * WT<BITS>::E;
  pl->mt = MT;
  pl->tiles = (N + 15) / 16;
  pl->kchunks = (K + KC - 1) / KC;
  const int kpad = pl->kchunks * KC;
  pl->cp = ((size_t)M * (kpad + 32) * 2 + gamma_bytes(PRO, K) <= (size_t)kStageBudget) ? kpad + 32 : kpad;
  pl->smem = (size_t)M * pl->cp * 2 + gamma_bytes(PRO, K);
  auto kern = gemv_stream_kernel<BITS, MT, kBatchOf<BITS>, PRO, EPI, BITS < 16>;
  cudaError_t e = cudaSuccess;
  if (pl->smem > 48 * 1024) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl->smem);
  if (e != cudaSuccess) return e;
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kStreamThreads, pl->smem);
  if (e != cudaSuccess) return e;
  occ = std::max(1, occ);
  const long long warps_max = (long long)device_sm_count() * occ * (kStreamThreads / 32);
  const long long total = (long long)pl->tiles * pl->kchunks;
  long long per = std::max<long long>(kBatchOf<BITS>, (total + warps_max - 1) / warps_max);
  if (!allow_split || pl->tiles > kMaxSplitTiles) per = (per + pl->kchunks - 1) / pl->kchunks * pl->kchunks;
  pl->per = (int)per;
  const long long warps = (total + per - 1) / per;
  pl->grid = (int)((warps + kStreamThreads / 32 - 1) / (kStreamThreads / 32));
  const bool split = (per % pl->kchunks) != 0;
  pl->max_slots = split ? (pl->kchunks - 1) / pl->per + 2 : 0;
  pl->ws_bytes = split ? kCounterBytes + (size_t)pl->tiles * pl->max_slots * 32 * 4 * MT * 4 : 0;
  pl->ring_slots = 0;
  return cudaSuccess;
}

// ------------------------------------------------------------------ ring GEMV
// The TMA-ring kernel (gemv_ring.cuh) serves M <= 8 whenever its weight rows
// can be a tensor map (row bytes a multiple of 16, weight 16-byte aligned) and
// at least kRingMinStages ring slots fit beside the staged activation. Set
// LW_B200_GEMV=stream to use the register-pipeline kernel instead.
constexpr int kRingMinStages = 4;
constexpr size_t kRingSmemMax = 232448;   // opt-in dynamic shared memory per CTA on sm_100
constexpr size_t kRingStaticBytes = 4096; // the kernel's static shared memory, rounded up

inline bool ring_enabled() {
  static const bool on = [] {
    const char* v = getenv("LW_B200_GEMV");
    return !(v && (strcmp(v, "stream") == 0 || strcmp(v, "bulk") == 0));
  }();
  return on;
}

// LW_B200_RING_3D=0 issues the eight 2-D boxes per stage even when the 3-D view applies.
inline bool ring_3d_enabled() {
  static const bool on = [] {
    const char* v = getenv("LW_B200_RING_3D");
    return !(v && strcmp(v, "0") == 0);
  }();
  return on;
}

struct RingPlan {
  int spr, boxes_last, units, stages, grid, cp, kchunks;
  size_t smem, ws_bytes;
};

// scales: the unit copy needs 16-byte aligned blocks of whole 16-byte multiples
// (16 rows x groups x 2 bytes; for the last tile, (N mod 16) rows) that fit a
// unit buffer; a null `scales` (sizing only) skips the alignment check.
// fold: the codes variant (fold_scales<BITS>(K, G) must hold), which also
// stages per-chunk activation sums.
template <int BITS, int PRO>
bool plan_ring(int M, int N, int K, int G, const void* w, const void* scales, RingPlan* pl, bool fold = false) {
  constexpr int KC = 4 * WT<BITS>::E;
  if (!ring_enabled() || M < 1 || M > 8 || N < 16) return false;
  if (BITS < 16) {
    const long long ngroups = G > 0 ? K / G : 0;
    if (ngroups < 1 || ngroups * 32 > kRingMaxScaleBytes || ((long long)N * ngroups) % 8 ||
        (scales && reinterpret_cast<uintptr_t>(scales) % 16))
      return false;
  }
  const size_t rowbytes = (size_t)K * BITS / 8;
  if (rowbytes % 16 || rowbytes < 128 || (w && (reinterpret_cast<uintptr_t>(w) % 16))) return false;
  pl->spr = (int)((rowbytes + kRingStageRowBytes - 1) / kRingStageRowBytes);
  // a unit's scales ride in registers for up to kRingMaxUnit stages; fp16 rows
  // are whole stages (a box left unissued keeps stale bytes, harmless only
  // for integer codes, which are finite whatever they are)
  if (BITS < 16 ? pl->spr > kRingMaxUnit
                : rowbytes % (ring_3d_enabled() ? 128 : kRingStageRowBytes) != 0)   // (3-D copies fill zeros)
    return false;
  pl->boxes_last = (int)((rowbytes - (size_t)(pl->spr - 1) * kRingStageRowBytes + 127) / 128);
  pl->kchunks = 16 * pl->spr;
  const int kpad = pl->kchunks * KC;
  pl->cp = ((size_t)M * (kpad + 32) * 2 + gamma_bytes(PRO, K) <= (size_t)kStageBudget) ? kpad + 32 : kpad;
  const size_t act = align_up((size_t)M * pl->cp * 2 + gamma_bytes(PRO, K), 16) + (fold ? ring_asum_bytes(pl->spr) : 0);
  const size_t fixed = (size_t)kRingFixedBytes + act + kRingStaticBytes;
  if (fixed + (size_t)kRingMinStages * kRingStageBytes > kRingSmemMax) return false;
  pl->stages = (int)std::min<size_t>(kRingMaxStages, (kRingSmemMax - fixed) / kRingStageBytes);
  pl->smem = (size_t)kRingFixedBytes + (size_t)pl->stages * kRingStageBytes + act;
  pl->units = (N + 15) / 16;
  pl->grid = std::min(device_sm_count(), pl->units);
  pl->ws_bytes = 0;               // static schedule, whole tiles: no workspace
  return true;
}

template <int BITS, int PRO, int EPI, bool FOLD = false>
cudaError_t launch_ring(StreamParams p, const RingPlan& pl, cudaStream_t s, bool pdl, bool weights_after_wait = false) {
  RingParams rp;
  memset(&rp, 0, sizeof(rp));
  const size_t rowbytes = (size_t)p.K * BITS / 8;
  // whole 128-byte chunks: the 3-D view, one copy per stage; else 2-D boxes
  rp.map3d = rowbytes % 128 == 0 && ring_3d_enabled();
  const bool ok = rp.map3d ? encode_3d(&rp.tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.w, 128, (uint64_t)p.N,
                                       rowbytes / 128, rowbytes, 128, 128, 16, kRingBoxes, CU_TENSOR_MAP_SWIZZLE_128B)
                           : encode_2d(&rp.tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.w, rowbytes, (uint64_t)p.N,
                                       rowbytes, 128, 16, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok) return cudaErrorInvalidValue;
  p.kchunks = pl.kchunks;
  p.cp = pl.cp;
  p.tiles = pl.units;
  p.gshift = BITS < 16 ? group_shift(p.K, p.G) : 31;
  rp.p = p;
  rp.spr = pl.spr;
  rp.boxes_last = pl.boxes_last;
  rp.units = pl.units;
  rp.stages = pl.stages;
  rp.weights_after_wait = weights_after_wait;
  auto kern = gemv_ring_kernel<BITS, PRO, EPI, FOLD>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
  if (e != cudaSuccess) return e;
  return lw_launch(kern, dim3(pl.grid), dim3(kRingThreads), pl.smem, s, pdl, rp);
}

// Which plan a launch of these sizes uses: the bulk-copy kernel when it
// applies (its tiles kept whole if the workspace is too small to split),
// else the register-pipeline kernel.
template <int BITS, int PRO>
bool choose_tma(int M, int N, int K, size_t ws_bytes, StreamPlan* pl) {
  if (!tma_enabled() || !plan_tma<BITS, PRO>(M, N, K, true, pl)) return false;
  if (pl->ws_bytes > ws_bytes) return plan_tma<BITS, PRO>(M, N, K, false, pl);
  return true;
}

template <int BITS, int PRO, int EPI, bool FOLD>
cudaError_t launch_tma(StreamParams p, const StreamPlan& pl, void* ws, cudaStream_t s, bool pdl) {
  auto kern = gemv_tma_kernel<BITS, PRO, EPI, FOLD>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
  if (e != cudaSuccess) return e;
  p.tiles = pl.tiles;
  p.kchunks = pl.kchunks;
  p.cp = pl.cp;
  p.per = pl.per;
  p.max_slots = pl.max_slots;
  p.ring_slots = pl.ring_slots;
  p.counters = pl.ws_bytes ? static_cast<int*>(ws) : nullptr;
  p.slots = pl.ws_bytes ? reinterpret_cast<float*>(static_cast<char*>(ws) + kCounterBytes) : nullptr;
  p.gshift = group_shift(p.K, p.G);
  return lw_launch(kern, dim3(pl.grid), dim3(kTmaThreads), pl.smem, s, pdl, p);
}

// Launch one row block (M <= 32). The workspace (counters first, zeroed before
// first use, then slots) is used only when the plan splits tiles; without a
// large enough workspace the plan keeps tiles whole.
template <int BITS, int PRO, int EPI>
cudaError_t launch_stream_block(StreamParams p, void* ws, size_t ws_bytes, cudaStream_t s, bool pdl,
                                bool allow_fold = false, bool allow_ring = true, bool ring_safe_pdl = false) {
  if (allow_ring) {
    const bool fold = allow_fold && fold_scales<BITS>(p.K, p.G);
    RingPlan rpl;
    if (plan_ring<BITS, PRO>(p.M, p.N, p.K, p.G, p.w, p.scales, &rpl, fold)) {
      if constexpr (BITS < 16) {
        if (fold) return launch_ring<BITS, PRO, EPI, true>(p, rpl, s, pdl || ring_safe_pdl, ring_safe_pdl);
      }
      // ring_safe_pdl: programmatic dependent launch with every global read after the wait
      return launch_ring<BITS, PRO, EPI>(p, rpl, s, pdl || ring_safe_pdl, ring_safe_pdl);
    }
  }
  StreamPlan pl;
  if constexpr (BITS != 16 && EPI != EPI_PEER_ARGMAX) {
    if (choose_tma<BITS, PRO>(p.M, p.N, p.K, ws_bytes, &pl)) {
      if (allow_fold && fold_scales<BITS>(p.K, p.G)) return launch_tma<BITS, PRO, EPI, true>(p, pl, ws, s, pdl);
      return launch_tma<BITS, PRO, EPI, false>(p, pl, ws, s, pdl);
    }
  }
  cudaError_t e;
  const int mt = mt_for(p.M);
#define LW_PLAN(MT_)                                                                    \
  e = plan_for<BITS, MT_, PRO, EPI>(p.M, p.N, p.K, true, &pl);                          \
  if (e == cudaSuccess && pl.ws_bytes > ws_bytes)                                       \
    e = plan_for<BITS, MT_, PRO, EPI>(p.M, p.N, p.K, false, &pl);
  if (mt == 1) {
    LW_PLAN(1)
  } else if (mt == 2) {
    LW_PLAN(2)
  } else {
    LW_PLAN(4)
  }
#undef LW_PLAN
  if (e != cudaSuccess) return e;
  p.tiles = pl.tiles;
  p.kchunks = pl.kchunks;
  p.cp = pl.cp;
  p.per = pl.per;
  p.max_slots = pl.max_slots;
  if (pl.ws_bytes) {
    p.counters = static_cast<int*>(ws);
    p.slots = reinterpret_cast<float*>(static_cast<char*>(ws) + kCounterBytes);
  } else {
    p.counters = nullptr;
    p.slots = nullptr;
  }
  p.gshift = BITS < 16 ? group_shift(p.K, p.G) : 31;
  dim3 grid(pl.grid), block(kStreamThreads);
  const bool fold = allow_fold && fold_scales<BITS>(p.K, p.G);
  if (pl.smem > 48 * 1024) {   // the variant launched may differ from the one planned with
    cudaError_t ea = cudaSuccess;
    if (mt == 1) ea = cudaFuncSetAttribute(fold ? gemv_stream_kernel<BITS, 1, kBatchOf<BITS>, PRO, EPI, true>
                                                : gemv_stream_kernel<BITS, 1, kBatchOf<BITS>, PRO, EPI, false>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
    else if (mt == 2) ea = cudaFuncSetAttribute(fold ? gemv_stream_kernel<BITS, 2, kBatchOf<BITS>, PRO, EPI, true>
                                                     : gemv_stream_kernel<BITS, 2, kBatchOf<BITS>, PRO, EPI, false>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
    else ea = cudaFuncSetAttribute(fold ? gemv_stream_kernel<BITS, 4, kBatchOf<BITS>, PRO, EPI, true>
                                        : gemv_stream_kernel<BITS, 4, kBatchOf<BITS>, PRO, EPI, false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
    if (ea != cudaSuccess) return ea;
  }
#define LW_GO(MT_)                                                                                          \
  return fold ? lw_launch(gemv_stream_kernel<BITS, MT_, kBatchOf<BITS>, PRO, EPI, true>, grid, block, pl.smem, s, pdl, p) \
              : lw_launch(gemv_stream_kernel<BITS, MT_, kBatchOf<BITS>, PRO, EPI, false>, grid, block, pl.smem, s, pdl, p);
  if (mt == 1) { LW_GO(1) }
  if (mt == 2) { LW_GO(2) }
  LW_GO(4)
#undef LW_GO
}

// Workspace bytes a launch of these sizes can use to split tiles.
template <int BITS, int PRO, int EPI>
size_t stream_workspace(int M, int N, int K) {
  size_t need = 0;
  const int rows = stage_rows<BITS>(K);
  for (int m0 = 0; m0 < M; m0 += rows) {
    const int mb = std::min(rows, M - m0);
    // (the ring kernel needs none; the split-tile kernel is its fallback)
    StreamPlan pl;
    if (BITS != 16 && EPI != EPI_PEER_ARGMAX && tma_enabled() && plan_tma<BITS, PRO>(mb, N, K, true, &pl)) {
      need = std::max(need, pl.ws_bytes);
      continue;
    }
    cudaError_t e;
    const int mt = mt_for(mb);
    if (mt == 1)
      e = plan_for<BITS, 1, PRO, EPI>(mb, N, K, true, &pl);
    else if (mt == 2)
      e = plan_for<BITS, 2, PRO, EPI>(mb, N, K, true, &pl);
    else
      e = plan_for<BITS, 4, PRO, EPI>(mb, N, K, true, &pl);
    if (e == cudaSuccess) need = std::max(need, pl.ws_bytes);
  }
  return need;
}

}  // namespace lw
