// Host side of lw_fused_gemv: argument translation and the typed launch,
// shared by the translation units that instantiate the kernel variants.
#pragma once

#include "gemv_host.cuh"

namespace lw {

inline StreamParams to_stream(const lw_fused_gemv_args* a) {
  StreamParams p = {};
  p.act = static_cast<const __half*>(a->act);
  p.w = static_cast<const uint8_t*>(a->weight);
  p.scales = static_cast<const __half*>(a->scales);
  p.bias = static_cast<const __half*>(a->bias);
  p.residual = static_cast<const __half*>(a->residual);
  p.out = static_cast<__half*>(a->out);
  p.lda = a->lda;
  p.ldo = a->ldo;
  p.M = a->M;
  p.N = a->N;
  p.K = a->K;
  p.G = a->bits == 16 ? a->K : a->group_size;
  p.gamma = static_cast<const __half*>(a->gamma);
  p.eps = a->eps;
  p.psum = a->psum;
  p.x_out = static_cast<__half*>(a->x_out);
  p.rope_cos = static_cast<const __half*>(a->rope_cos);
  p.rope_sin = static_cast<const __half*>(a->rope_sin);
  p.pos = a->pos;
  p.head_dim = a->head_dim;
  p.n_q_heads = a->n_q_heads;
  p.n_kv_heads = a->n_kv_heads;
  p.max_seq = a->max_seq;
  p.q_out = static_cast<__half*>(a->q_out);
  p.k_cache = static_cast<__half*>(a->k_cache);
  p.v_cache = static_cast<__half*>(a->v_cache);
  p.out_f32 = a->out_f32;
  p.argmax_keys = a->argmax_keys;
  p.argmax_offset = a->argmax_offset;
  p.seq = a->prefill_seq;
  if (a->prologue == LW_PRO_PEER_RESID_NORM && a->xin) {
    p.in_world = a->xin->world;
    p.in_tag = a->xin->tag;
    p.in_tags = a->xin->tags_per_step;
    p.in_src = static_cast<const unsigned long long*>(a->xin->src);
    p.in_step = a->xin->step;
    p.in_error = a->xin->error;
    p.in_timeout_ns = a->xin->timeout_ns;
    p.in_slice_flags = a->xin->slice_flags;
  }
  if ((a->epilogue == LW_EPI_PEER_F32 || a->epilogue == LW_EPI_PEER_ARGMAX) && a->xout) {
    p.out_world = a->xout->world;
    p.out_rank = a->xout->rank;
    p.out_tag = a->xout->tag;
    p.out_tags = a->xout->tags_per_step;
    p.out_step = a->xout->step;
    for (int d = 0; d < a->xout->world && d < kMaxRanks; ++d)
      p.out_dst[d] = static_cast<unsigned long long*>(a->xout->dst[d]);
    p.out_arrivals = a->xout->arrivals;
  }
  return p;
}

template <int BITS, int PRO, int EPI>
cudaError_t fused_launch(const lw_fused_gemv_args* a, cudaStream_t s) {
  return launch_stream_block<BITS, PRO, EPI>(to_stream(a), a->workspace, a->workspace_bytes, s, a->pdl != 0,
                                             a->fold_scales != 0, a->kernel != 1);
}

template <int BITS, int PRO, int EPI>
size_t fused_ws(const lw_fused_gemv_args* a) {
  return stream_workspace<BITS, PRO, EPI>(a->M, a->N, a->K);
}

// The tensor-parallel exchange variants (decode_tp.cu): launch / workspace of
// a->bits, a->prologue, a->epilogue if that combination is one of them.
bool tp_fused_launch(const lw_fused_gemv_args* a, cudaStream_t s, cudaError_t* e);
bool tp_fused_ws(const lw_fused_gemv_args* a, size_t* bytes);

}  // namespace lw
