// Fused-GEMV variants of the tensor-parallel decode step whose all-reduces go
// through peer memory instead of NCCL.
//
// Per layer the step runs, on every rank r of `world`:
//   q|k|v (this rank's heads)      PRO_PEER_RESID_NORM (exchange of the last down_proj) + EPI_ROPE_KV
//   attention (this rank's heads)
//   o_proj (this rank's K columns) EPI_PEER_F32: fp32 partial -> every rank's slot r
//   gate|up (this rank's rows)     PRO_PEER_RESID_NORM (exchange of o_proj) + EPI_SWIGLU
//   down_proj (this rank's K cols) EPI_PEER_F32
// then lm_head (this rank's vocabulary rows) PRO_PEER_RESID_NORM +
// EPI_PEER_ARGMAX, and the sampling kernel, which waits for every rank's keys.
//
// The all-reduce is one-shot: each producing kernel stores its partial
// straight into every rank's receive buffer while its tiles finish, and the
// consuming kernel sums the world partials in rank order, so every rank gets
// the same bits (and, for two ranks, the same bits as an NCCL sum). No kernel
// waits for a kernel of its own GPU that has not been launched before it, so
// no pair of waiting kernels ever has to be co-resident on one GPU.
#include "fused_host.cuh"

#define LW_FUSED_TP_TABLE(X)                                \
  X(4, lw::PRO_PEER_RESID_NORM, lw::EPI_ROPE_KV)            \
  X(8, lw::PRO_PEER_RESID_NORM, lw::EPI_ROPE_KV)            \
  X(4, lw::PRO_PEER_RESID_NORM, lw::EPI_SWIGLU)             \
  X(8, lw::PRO_PEER_RESID_NORM, lw::EPI_SWIGLU)             \
  X(4, lw::PRO_PLAIN, lw::EPI_PEER_F32)                     \
  X(8, lw::PRO_PLAIN, lw::EPI_PEER_F32)                     \
  X(16, lw::PRO_PEER_RESID_NORM, lw::EPI_PEER_ARGMAX)      \
  X(16, lw::PRO_NORM, lw::EPI_PEER_ARGMAX)                  \
  X(4, lw::PRO_PEER_RESID_NORM, lw::EPI_PEER_ARGMAX)        \
  X(8, lw::PRO_PEER_RESID_NORM, lw::EPI_PEER_ARGMAX)        \
  X(4, lw::PRO_NORM, lw::EPI_PEER_ARGMAX)                   \
  X(8, lw::PRO_NORM, lw::EPI_PEER_ARGMAX)

namespace lw {

bool tp_fused_launch(const lw_fused_gemv_args* a, cudaStream_t s, cudaError_t* e) {
#define X(B_, P_, E_)                                                    \
  if (a->bits == B_ && a->prologue == P_ && a->epilogue == E_) {       \
    *e = fused_launch<B_, P_, E_>(a, s);                               \
    return true;                                                       \
  }
  LW_FUSED_TP_TABLE(X)
#undef X
  return false;
}

bool tp_fused_ws(const lw_fused_gemv_args* a, size_t* bytes) {
#define X(B_, P_, E_)                                                    \
  if (a->bits == B_ && a->prologue == P_ && a->epilogue == E_) {       \
    *bytes = fused_ws<B_, P_, E_>(a);                                  \
    return true;                                                       \
  }
  LW_FUSED_TP_TABLE(X)
#undef X
  return false;
}

}  // namespace lw

int lw_decode_tp_take_error() { return lw_tu_take_error(); }
