"""Native decode engine for Llama-family models on B200.

Replaces the per-token loop of liteweight/generate.py:97-124 (HF forward with
DynamicCache, ~10 eager ops + 7 QuantLinear calls per layer, a host sync per
token) with one CUDA graph per decode step built from the library's fused
kernels (include/liteweight_b200.h, decode step section):

  per layer: [RMSNorm + q|k|v GEMV + RoPE + KV append] -> [split-KV GQA
  attention] -> [o GEMV + residual] -> [RMSNorm + gate|up GEMV + SwiGLU] ->
  [down GEMV + residual];  then [RMSNorm + lm_head GEMV + argmax] -> [pick /
  embed next token, advance position].

The position lives on the device, so the same graph replays every step; the
prompt is consumed by the same step (its tokens are "forced" in the token
table), so prefill and decode share one code path. KV cache: preallocated
fp16 [B, n_kv, max_seq, head_dim] per layer (the layout of the reference's
KVCache, generate.py:22-25).

Tensor parallelism (``tp_size > 1``, one process per GPU): q/k/v and gate/up
are split by output rows (heads / intermediate), o and down by input
columns, the lm_head by vocabulary rows. The o/down fp32 partial sums and
the per-rank argmax keys are all-reduced, by default through peer memory
inside the kernels (``exchange="peer"``: the producing GEMV stores its
partial into every rank's receive buffer over NVLink, the next norm prologue
waits for all of them and sums them in rank order; include/liteweight_b200.h,
tensor-parallel exchange), or by NCCL all-reduces between the kernels
(``exchange="nccl"``).
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch

from liteweight_b200 import _native as nat

c_int, c_void_p, c_float, c_size_t = ctypes.c_int, ctypes.c_void_p, ctypes.c_float, ctypes.c_size_t

PRO_PLAIN, PRO_NORM, PRO_RESID_NORM, PRO_PEER_RESID_NORM = 0, 1, 2, 3
EPI_PLAIN, EPI_ROPE_KV, EPI_SWIGLU, EPI_F32, EPI_ARGMAX, EPI_PEER_F32, EPI_PEER_ARGMAX = 0, 1, 2, 3, 4, 5, 6
MAX_RANKS = 8


class ExchangeOut(ctypes.Structure):
    """Mirror of lw_exchange_out (include/liteweight_b200.h)."""
    _fields_ = [("world", c_int), ("rank", c_int), ("dst", c_void_p * MAX_RANKS), ("step", c_void_p),
                ("tag", c_int), ("tags_per_step", c_int), ("arrivals", c_void_p)]


class ExchangeIn(ctypes.Structure):
    """Mirror of lw_exchange_in (include/liteweight_b200.h)."""
    _fields_ = [("world", c_int), ("tag", c_int), ("tags_per_step", c_int), ("src", c_void_p), ("step", c_void_p),
                ("error", c_void_p), ("timeout_ns", ctypes.c_longlong), ("slice_flags", c_void_p)]


SLICE_FLAGS = 1024   # per slot set: one flag per CTA of a cooperatively reducing GEMV (kSliceFlagsMax)


def exchange_flag(step: int, tag: int, tags_per_step: int) -> int:
    """Flag word of exchange `tag` at step `step` (as the kernels compute it)."""
    f = (step * tags_per_step + tag + 1) & 0xFFFFFFFF
    return f or 1


class FusedGemvArgs(ctypes.Structure):
    """Mirror of lw_fused_gemv_args (include/liteweight_b200.h)."""
    _fields_ = [
        ("bits", c_int), ("prologue", c_int), ("epilogue", c_int), ("pdl", c_int), ("fold_scales", c_int),
        ("M", c_int), ("N", c_int), ("K", c_int), ("group_size", c_int), ("lda", c_int), ("ldo", c_int),
        ("act", c_void_p), ("weight", c_void_p), ("scales", c_void_p), ("bias", c_void_p), ("residual", c_void_p),
        ("out", c_void_p), ("gamma", c_void_p), ("psum", c_void_p), ("x_out", c_void_p),
        ("eps", c_float), ("head_dim", c_int), ("n_q_heads", c_int), ("n_kv_heads", c_int), ("max_seq", c_int),
        ("argmax_offset", c_int),
        ("rope_cos", c_void_p), ("rope_sin", c_void_p), ("pos", c_void_p),
        ("q_out", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p),
        ("out_f32", c_void_p), ("argmax_keys", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("xin", c_void_p), ("xout", c_void_p), ("prefill_seq", c_void_p), ("sched_set", c_int),
        ("kernel", c_int),
    ]


class PrefillGemmArgs(ctypes.Structure):
    """Mirror of lw_prefill_gemm_args (include/liteweight_b200.h)."""
    _fields_ = [
        ("bits", c_int), ("epilogue", c_int), ("pdl", c_int), ("M", c_int), ("N", c_int), ("K", c_int),
        ("group_size", c_int), ("lda", c_int), ("ldo", c_int),
        ("act", c_void_p), ("weight", c_void_p), ("scales", c_void_p), ("out", c_void_p), ("residual", c_void_p),
        ("head_dim", c_int), ("n_q_heads", c_int), ("n_kv_heads", c_int), ("max_seq", c_int),
        ("rope_cos", c_void_p), ("rope_sin", c_void_p), ("pos", c_void_p), ("seq", c_void_p),
        ("q_out", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p),
        ("argmax_keys", c_void_p), ("argmax_offset", c_int),
    ]


TC_EPI_RESID, TC_EPI_SWIGLU, TC_EPI_ROPE_KV, TC_EPI_F32, TC_EPI_ARGMAX = 0, 1, 2, 3, 4
TC_ROWS = 256   # prompt-chunk rows on the tensor-core path (the GEMM's largest M)


def tc_decode_min_batch() -> int:
    """Smallest decode batch whose linears run on the tensor-core GEMM (it reads
    each weight once for all rows; the GEMVs stage at most 26 rows of a K = 4096
    activation per launch and re-read the weights per row block).
    LW_B200_TC_DECODE_MIN overrides it; 0 keeps every batch on the GEMVs."""
    v = os.environ.get("LW_B200_TC_DECODE_MIN")
    return int(v) if v not in (None, "") else 24


class AttentionArgs(ctypes.Structure):
    """Mirror of lw_attention_args (include/liteweight_b200.h)."""
    _fields_ = [
        ("q", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p), ("out", c_void_p), ("pos", c_void_p),
        ("batch", c_int), ("n_q_heads", c_int), ("n_kv_heads", c_int), ("head_dim", c_int), ("max_seq", c_int),
        ("pdl", c_int), ("prefill_seq", c_void_p),
    ]


nat.register("lw_fused_gemv", [ctypes.POINTER(FusedGemvArgs), c_void_p])
nat.register("lw_fused_gemv_workspace_size", [ctypes.POINTER(FusedGemvArgs)], c_size_t)
nat.register("lw_attention_decode", [ctypes.POINTER(AttentionArgs), c_void_p])
nat.register("lw_embed_tokens", [c_void_p] * 4 + [c_int] * 3 + [c_void_p])
nat.register("lw_sample_tokens", [c_void_p] * 8 + [c_int] * 3 + [c_void_p])
nat.register("lw_struct_size", [c_int], c_size_t)
nat.register("lw_prefill_embed", [c_void_p] * 5 + [c_int] * 4 + [c_void_p])
nat.register("lw_prefill_advance", [c_void_p] * 2 + [c_int] * 2 + [c_void_p])
nat.register("lw_prefill_sample", [c_void_p] * 8 + [c_int] * 4 + [c_void_p])
nat.register("lw_prefill_gemm", [ctypes.POINTER(PrefillGemmArgs), c_void_p])
nat.register("lw_rmsnorm_rows", [c_void_p] * 3 + [c_int] * 2 + [c_float, c_int, c_void_p])
nat.register("lw_resid_rmsnorm_rows", [c_void_p] * 4 + [c_int] * 2 + [c_float, c_int, c_void_p])
nat.register("lw_peer_alloc", [c_size_t, ctypes.POINTER(c_void_p)])
nat.register("lw_peer_free", [c_void_p])
nat.register("lw_peer_handle_size", [], c_size_t)
nat.register("lw_peer_export", [c_void_p, c_void_p])
nat.register("lw_peer_import", [c_void_p, ctypes.POINTER(c_void_p)])
nat.register("lw_peer_close", [c_void_p])


def check_abi() -> None:
    """The ctypes mirrors must have the library's struct sizes."""
    lib = nat.lib()
    for which, cls in ((0, FusedGemvArgs), (1, AttentionArgs), (2, ExchangeOut), (3, ExchangeIn),
                       (4, PrefillGemmArgs)):
        got = int(lib.lw_struct_size(which))
        if got != ctypes.sizeof(cls):
            raise RuntimeError(f"{cls.__name__}: ctypes size {ctypes.sizeof(cls)} != library size {got}")


# ------------------------------------------------------------------ model spec / weights

@dataclass
class LlamaSpec:
    hidden: int
    inter: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    bits: int = 4
    group_size: int = 128
    eps: float = 1e-5
    rope_theta: float = 500000.0

    def linear_shapes(self):
        """(name, out_features, in_features) of the quantized linears of one layer."""
        h, i, hd = self.hidden, self.inter, self.head_dim
        return [("q", self.n_heads * hd, h), ("k", self.n_kv_heads * hd, h), ("v", self.n_kv_heads * hd, h),
                ("o", h, self.n_heads * hd), ("gate", i, h), ("up", i, h), ("down", h, i)]

    def weight_bytes_per_token(self, include_lm_head: bool = True, lm_head_bits: int = 16) -> int:
        """Bytes one decode step must read: packed weights + fp16 scales (+ lm_head, norms).
        lm_head_bits 16: the fp16 lm_head (liteweight keeps it unquantized); 8 / 4:
        a quantized one with this spec's group size."""
        per_layer = sum(n * k * self.bits // 8 + 2 * n * (k // self.group_size) for _, n, k in self.linear_shapes())
        total = self.n_layers * (per_layer + 4 * self.hidden)
        if include_lm_head:
            v, h = self.vocab, self.hidden
            total += (v * h * 2 if lm_head_bits == 16
                      else v * h * lm_head_bits // 8 + 2 * v * (h // self.group_size)) + 2 * h
        return total

    def kv_bytes_per_position(self) -> int:
        return self.n_layers * 2 * self.n_kv_heads * self.head_dim * 2


LLAMA_3_2_1B = dict(hidden=2048, inter=8192, n_layers=16, n_heads=32, n_kv_heads=8, head_dim=64, vocab=128256)
LLAMA_3_8B = dict(hidden=4096, inter=14336, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128, vocab=128256)
LLAMA_3_70B = dict(hidden=8192, inter=28672, n_layers=80, n_heads=64, n_kv_heads=8, head_dim=128, vocab=128256)


@dataclass
class LayerWeights:
    """One layer's quantized linears in liteweight's format, unsharded, natural row order."""
    q: tuple
    k: tuple
    v: tuple
    o: tuple
    gate: tuple
    up: tuple
    down: tuple
    in_norm: torch.Tensor
    post_norm: torch.Tensor


def rope_pair_order(n_heads: int, head_dim: int, device) -> torch.Tensor:
    """Row permutation that puts head dims d and d + hd/2 in rows g and g+8 of
    each 16-row tile: tile j of a head holds dims 8j..8j+7 and hd/2+8j..+7."""
    hd, half = head_dim, head_dim // 2
    per_head = []
    for j in range(hd // 16):
        per_head += list(range(8 * j, 8 * j + 8)) + list(range(half + 8 * j, half + 8 * j + 8))
    idx = torch.tensor(per_head, dtype=torch.long)
    return torch.cat([idx + h * hd for h in range(n_heads)]).to(device)


def interleave8(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Rows a[8t:8t+8], b[8t:8t+8] alternately (gate/up pairs in one 16-row tile)."""
    n = a.shape[0]
    return torch.stack([a.reshape(n // 8, 8, -1), b.reshape(n // 8, 8, -1)], dim=1).reshape(2 * n, -1).contiguous()


def shard_rows(t: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    n = t.shape[0] // size
    return t[rank * n:(rank + 1) * n]


def shard_cols(t: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    n = t.shape[1] // size
    return t[:, rank * n:(rank + 1) * n]


class PackedLayer:
    """Device buffers of one layer in the engine's layout (this rank's shard)."""

    def __init__(self, lw: LayerWeights, spec: LlamaSpec, rank: int, size: int, device):
        hd = spec.head_dim
        nq, nkv = spec.n_heads // size, spec.n_kv_heads // size

        def rows(pair):
            q, s = pair
            return shard_rows(q, rank, size), shard_rows(s, rank, size)

        qw, qs = rows(lw.q)
        kw, ks = rows(lw.k)
        vw, vs = rows(lw.v)
        perm_q = rope_pair_order(nq, hd, qw.device)
        perm_kv = rope_pair_order(nkv, hd, qw.device)
        self.qkv_w = torch.cat([qw[perm_q], kw[perm_kv], vw[perm_kv]]).contiguous().to(device)
        self.qkv_s = torch.cat([qs[perm_q], ks[perm_kv], vs[perm_kv]]).contiguous().to(device)
        gw, gs = rows(lw.gate)
        uw, us = rows(lw.up)
        self.gu_w = interleave8(gw, uw).to(device)
        self.gu_s = interleave8(gs, us).to(device)
        # o / down: split the input columns (K); packed INT4 columns are K/2 bytes
        ow, os_ = lw.o
        dw, ds = lw.down
        self.o_w = shard_cols(ow, rank, size).contiguous().to(device)
        self.o_s = shard_cols(os_, rank, size).contiguous().to(device)
        self.d_w = shard_cols(dw, rank, size).contiguous().to(device)
        self.d_s = shard_cols(ds, rank, size).contiguous().to(device)
        self.in_norm = lw.in_norm.to(device=device, dtype=torch.float16).contiguous()
        self.post_norm = lw.post_norm.to(device=device, dtype=torch.float16).contiguous()


def rope_tables(inv_freq: torch.Tensor, max_seq: int, scaling: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_seq, head_dim] fp16, computed like modeling_llama.py:124-136."""
    inv = inv_freq.to(device=device, dtype=torch.float32)
    pos = torch.arange(max_seq, device=device, dtype=torch.float32)
    freqs = (inv[None, :, None] @ pos[None, None, :]).transpose(1, 2)[0]
    emb = torch.cat([freqs, freqs], dim=-1)
    return (emb.cos() * scaling).half().contiguous(), (emb.sin() * scaling).half().contiguous()


def default_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """modeling_llama.py:119-121 (default RoPE)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))


# ------------------------------------------------------------------ engine

def _stage_rows(K: int, bits: int, norm: bool) -> int:
    """Activation rows one fused GEMV launch can stage in shared memory (rows x
    K padded to whole chunks, fp16, plus the RMSNorm weight for the norm
    prologues, within the 220 KiB the kernels budget)."""
    kc = {4: 128, 8: 64, 16: 32}[bits]
    kpad = -(-K // kc) * kc
    return (220 * 1024 - (((K + 7) // 8) * 16 if norm else 0)) // (2 * kpad)


def down_rows(spec: LlamaSpec, tp_size: int = 1) -> int:
    """Rows one down_proj launch can stage (its K, the intermediate size, is the largest)."""
    return max(1, _stage_rows(spec.inter // tp_size, spec.bits, False))


def peer_batch_limit(spec: LlamaSpec, tp_size: int, lm_head_bits: int = 16) -> int:
    """Largest decode batch the in-kernel peer exchange takes: every GEMV of
    the step must stage the whole batch in one launch (larger batches run in
    row blocks, with exchange='nccl' under tensor parallelism)."""
    H, hd = spec.hidden, spec.head_dim
    return min(32, _stage_rows(H, spec.bits, True), _stage_rows(spec.n_heads // tp_size * hd, spec.bits, False),
               _stage_rows(spec.inter // tp_size, spec.bits, False), _stage_rows(H, lm_head_bits, True))


def prefill_rows(spec: LlamaSpec, tp_size: int = 1, limit: int = 32) -> int:
    """Positions per prompt chunk: the most rows the q|k|v, o, gate|up and
    lm_head launches can stage, at most `limit`. With one rank the down_proj
    runs in row blocks of down_rows() (its weights are re-read per block); with
    tensor parallelism the chunk also fits the down_proj, whose partial sums go
    to the other ranks in one exchange per chunk."""
    H, hd = spec.hidden, spec.head_dim
    rows = min(_stage_rows(H, spec.bits, True), _stage_rows(spec.n_heads // tp_size * hd, spec.bits, False),
               _stage_rows(H, 16, True))
    if tp_size > 1:
        rows = min(rows, down_rows(spec, tp_size))
    return max(1, min(limit, rows))


def tc_supported(spec: LlamaSpec, tp_size: int = 1) -> bool:
    """The tensor-core prompt GEMM takes every linear of a rank's layer shard:
    weight rows in whole 128-row tiles, K in whole 64-element blocks."""
    hd, nq, nkv, inter = spec.head_dim, spec.n_heads // tp_size, spec.n_kv_heads // tp_size, spec.inter // tp_size
    ns = [(nq + 2 * nkv) * hd, spec.hidden, 2 * inter]
    ks = [spec.hidden, nq * hd, inter]
    return (spec.bits in (4, 8) and spec.group_size >= 32 and all(n % 128 == 0 for n in ns)
            and all(k % 64 == 0 for k in ks))


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


class PeerExchange:
    """Receive buffers of every exchange of one rank's decode step, in one
    block of device memory that the other ranks map (CUDA IPC), plus this
    rank's mappings of their blocks.

    Values travel as flagged 8-byte words (include/liteweight_b200.h,
    tensor-parallel exchange). Block layout (bytes): keys [world][rows] words
    | two slot sets, each [world][rows][hidden] words, for up to `batch` rows
    (a launch of M rows uses the first world * M rows of a set). Partial-sum exchange e
    (o_proj of layer e // 2, or its down_proj) uses slot set e % 2: a rank can
    only be one exchange ahead of another (it cannot produce exchange e + 1
    before it has consumed e, which needs every rank's e), so a set is never
    overwritten while a rank still reads it, and the flags tell a word of
    exchange e from one of e - 2. The keys exchange is the last tag.
    """

    def __init__(self, group, rank: int, world: int, batch: int, hidden: int, n_partial: int, device,
                 timeout_s: float = 10.0):
        assert 1 <= world <= MAX_RANKS
        self.rank, self.world, self.group, self.device = rank, world, group, torch.device(device)
        self.n_partial = n_partial
        self.rows = batch
        self.tags = n_partial + 1
        self.slot_off = _align(8 * world * batch, 256)
        self.set_bytes = _align(8 * world * batch * hidden, 256)
        self.part_bytes = 8 * batch * hidden
        self.total = self.slot_off + 2 * self.set_bytes
        lib = nat.lib()
        with torch.cuda.device(self.device):
            ptr = c_void_p()
            nat.check("lw_peer_alloc", lib.lw_peer_alloc(self.total, ctypes.byref(ptr)))
            self.base = ptr.value
            handle = (ctypes.c_ubyte * int(lib.lw_peer_handle_size()))()
            nat.check("lw_peer_export", lib.lw_peer_export(self.base, handle))
            handles = [None] * world
            torch.distributed.all_gather_object(handles, bytes(handle), group=group)
            self.peers = []
            for d in range(world):
                if d == rank:
                    self.peers.append(self.base)
                    continue
                q = c_void_p()
                nat.check("lw_peer_import", lib.lw_peer_import(handles[d], ctypes.byref(q)))
                self.peers.append(q.value)
        self.step = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.error = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.arrivals = torch.zeros(1, dtype=torch.int32, device=self.device)
        # LW_B200_EXCHANGE_SPLIT=1: the consuming GEMV reduces the partials
        # cooperatively (each CTA one slice of K, a flag per CTA, one flag array
        # per slot set) instead of every CTA reading every rank's partials for
        # the whole K. Same bits; measured slower at two ranks (569.5 vs 721.4
        # tokens/s: each CTA then waits for the grid's last one), so off by default.
        self.split = os.environ.get("LW_B200_EXCHANGE_SPLIT") == "1"
        self.slice_flags = torch.zeros(2 * SLICE_FLAGS, dtype=torch.int32, device=self.device)
        self.outs, self.ins = [], []
        for e in range(self.tags):
            out = ExchangeOut(world=world, rank=rank, step=self.step.data_ptr(), tag=e, tags_per_step=self.tags,
                              arrivals=self.arrivals.data_ptr())
            for d in range(world):
                out.dst[d] = self.peers[d] + self._recv_offset(e)   # the kernel adds rank * rows
            self.outs.append(out)
            flags = (self.slice_flags.data_ptr() + 4 * SLICE_FLAGS * (e % 2)
                     if self.split and e < n_partial else None)
            self.ins.append(ExchangeIn(world=world, tag=e, tags_per_step=self.tags,
                                       src=self.base + self._recv_offset(e), step=self.step.data_ptr(),
                                       error=self.error.data_ptr(), timeout_ns=int(timeout_s * 1e9),
                                       slice_flags=flags))
        self.closed = False

    def _recv_offset(self, e: int) -> int:
        return self.slot_off + (e % 2) * self.set_bytes if e < self.n_partial else 0

    def out_ptr(self, e: int) -> int:
        return ctypes.addressof(self.outs[e])

    def in_ptr(self, e: int) -> int:
        return ctypes.addressof(self.ins[e])

    def check(self) -> None:
        """Raise if a device-side wait of an exchange gave up (a rank stopped producing)."""
        err = int(self.error.item())
        if err:
            raise nat.LiteweightError("peer exchange", err, "a wait for another rank timed out")

    def close(self) -> None:
        """Unmap the other ranks' blocks and free this one. Collective: every
        rank calls it after its last step (barriers keep a block alive until no
        rank can still write into it)."""
        if self.closed:
            return
        lib = nat.lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            torch.distributed.barrier(group=self.group)
            for d, p in enumerate(self.peers):
                if d != self.rank:
                    nat.check("lw_peer_close", lib.lw_peer_close(p))
            torch.distributed.barrier(group=self.group)
            nat.check("lw_peer_free", lib.lw_peer_free(self.base))
        self.closed = True


class DecodeEngine:
    """Batched greedy decode of a Llama model on one GPU (or one tensor-parallel rank)."""

    def __init__(self, spec: LlamaSpec, layers: list, embed: torch.Tensor, final_norm: torch.Tensor,
                 lm_head: torch.Tensor | None, rope_cos: torch.Tensor, rope_sin: torch.Tensor, batch: int,
                 max_seq: int, device=None, tp_rank: int = 0, tp_size: int = 1, tp_group=None, pdl: bool = True,
                 fold_scales: bool = False, exchange: str = "peer", exchange_timeout_s: float = 10.0,
                 lm_head_quant: tuple | None = None, tune_kernels: bool = True):
        assert exchange in ("peer", "nccl")
        self.spec, self.B, self.S = spec, batch, max_seq
        self.fold = int(fold_scales)
        self.device = torch.device(device) if device is not None else embed.device
        self.tp_rank, self.tp_size, self.tp_group = tp_rank, tp_size, tp_group
        assert spec.n_heads % tp_size == 0 and spec.n_kv_heads % tp_size == 0, "heads must split evenly"
        assert spec.inter % (8 * tp_size) == 0 and spec.vocab % tp_size == 0
        assert batch >= 1   # batches past what one GEMV launch stages run as row blocks
        self.nq, self.nkv = spec.n_heads // tp_size, spec.n_kv_heads // tp_size
        self.inter = spec.inter // tp_size
        self.vshard = spec.vocab // tp_size
        self.pdl = int(pdl)
        check_abi()
        dev, H, hd = self.device, spec.hidden, spec.head_dim
        self.layers = layers
        self.embed = embed.to(device=dev, dtype=torch.float16).contiguous()
        # lm_head: fp16 [V, H] (liteweight keeps it unquantized; tied to the embedding when None),
        # or lm_head_quant = (qweight, scales, bits, group_size) in liteweight's format (what
        # swap_linears makes of it when it is not skipped)
        self.lm_bits, self.lm_group, self.lm_scales = 16, spec.hidden, None
        if lm_head_quant is not None:
            q, sc, bits, grp = lm_head_quant
            assert bits in (4, 8) and spec.hidden % grp == 0
            self.lm_bits, self.lm_group = bits, grp
            self.lm_head = shard_rows(q.to(dev).contiguous(), tp_rank, tp_size).contiguous()
            self.lm_scales = shard_rows(sc.to(device=dev, dtype=torch.float16).contiguous(), tp_rank,
                                        tp_size).contiguous()
        else:
            head = self.embed if lm_head is None else lm_head.to(device=dev, dtype=torch.float16).contiguous()
            self.lm_head = shard_rows(head, tp_rank, tp_size)
        self.final_norm = final_norm.to(device=dev, dtype=torch.float16).contiguous()
        self.rope_cos = rope_cos.to(dev).contiguous()
        self.rope_sin = rope_sin.to(dev).contiguous()
        assert self.rope_cos.shape[0] >= max_seq
        f16 = dict(dtype=torch.float16, device=dev)
        self.k_cache = [torch.zeros(batch, self.nkv, max_seq, hd, **f16) for _ in layers]
        self.v_cache = [torch.zeros(batch, self.nkv, max_seq, hd, **f16) for _ in layers]
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.seq = torch.zeros(1, dtype=torch.int32, device=dev)   # sequence of the prompt chunk in flight
        self.tokens = torch.full((max_seq + 1, batch), -1, dtype=torch.int32, device=dev)
        self.step_count = torch.zeros(1, dtype=torch.int32, device=dev)
        # decode buffers (row = sequence) and prompt-chunk buffers (row = position). Prompt
        # chunks of TC_ROWS positions run their linears on the tensor cores (lw_prefill_gemm;
        # with tensor parallelism the row-split linears' fp32 partials are all-reduced by NCCL
        # between the GEMMs); shapes the GEMM does not tile run the fused GEMVs and exchanges.
        self.use_tc = tc_supported(spec, tp_size)
        n = tc_decode_min_batch()
        self.tc_decode = self.use_tc and n > 0 and n <= batch <= TC_ROWS
        self.prefill_rows = TC_ROWS if self.use_tc else prefill_rows(spec, tp_size)
        self.dec = self._buffers(batch)
        self.pf = self._buffers(self.prefill_rows)
        self.x, self.x2, self.q, self.attn = self.dec.x, self.dec.x2, self.dec.q, self.dec.attn
        self.act, self.logits, self.psum, self.keys = self.dec.act, self.dec.logits, self.dec.psum, self.dec.keys
        self.exchange = None
        if tp_size > 1 and exchange == "peer":
            self.exchange = PeerExchange(tp_group, tp_rank, tp_size,
                                         max(batch, prefill_rows(spec, tp_size) if self.use_tc else self.prefill_rows), H,
                                         2 * len(layers), dev, exchange_timeout_s)
            self.step_count = self.exchange.step
        self._build_calls()
        self.graph = None
        self.prefill_graphs = {}
        self.host_pos = 0
        self.kernel_choice = {}
        if tune_kernels:
            self.tune_kernels()

    def _buffers(self, rows: int):
        """Activations of one launch shape (rows = sequences of a decode step or
        positions of a prompt chunk)."""
        dev, H, hd = self.device, self.spec.hidden, self.spec.head_dim
        f16 = dict(dtype=torch.float16, device=dev)

        class Bufs:
            pass
        b = Bufs()
        b.rows = rows
        b.x, b.x2 = torch.zeros(rows, H, **f16), torch.zeros(rows, H, **f16)
        b.q = torch.zeros(rows, self.nq * hd, **f16)
        b.attn = torch.zeros(rows, self.nq * hd, **f16)
        b.act = torch.zeros(rows, self.inter, **f16)
        b.logits = torch.zeros(rows, self.vshard, **f16)
        b.psum = torch.zeros(rows, H, dtype=torch.float32, device=dev)
        b.keys = torch.zeros(rows, dtype=torch.int64, device=dev)
        b.h = torch.zeros(rows, H, **f16)   # RMSNorm output (tensor-core prompt chunks)
        return b

    # -------------------------------------------------------------- call table
    def _gemv(self, rows: int, **kw) -> FusedGemvArgs:
        a = FusedGemvArgs()
        a.pdl, a.M, a.eps, a.fold_scales = self.pdl, rows, self.spec.eps, self.fold
        for k, v in kw.items():
            setattr(a, k, v.data_ptr() if isinstance(v, torch.Tensor) else v)
        return a

    def _make_calls(self, bufs, prefill: bool, final: bool = True):
        """The kernels of one decode step (prefill=False: row b = sequence b at
        *pos) or of one prompt chunk (prefill=True: row m = position *pos + m
        of sequence *seq; `final` adds the lm_head and the pick of the next
        token, else the chunk ends by advancing the position)."""
        sp, H, hd, rows = self.spec, self.spec.hidden, self.spec.head_dim, bufs.rows
        tp = self.tp_size > 1
        ex = self.exchange
        seq = self.seq.data_ptr() if prefill else None
        calls = []
        xs = [bufs.x, bufs.x2]
        cur = 0           # index of the buffer holding the residual stream
        pending = None    # exchange whose all-reduced partial waits to be added to the residual
        gemv_args = []

        def norm_pro():
            nonlocal cur, pending
            if pending is not None:
                d = dict(prologue=PRO_RESID_NORM, act=xs[cur], psum=bufs.psum, x_out=xs[1 - cur], lda=H)
                if ex is not None:
                    d.update(prologue=PRO_PEER_RESID_NORM, xin=ex.in_ptr(pending))
                cur = 1 - cur
                pending = None
            else:
                d = dict(prologue=PRO_NORM, act=xs[cur], lda=H)
            return d

        def partial_epi(e):
            if not tp:
                return dict(epilogue=EPI_PLAIN, out=xs[cur], residual=xs[cur])
            if ex is not None:
                return dict(epilogue=EPI_PEER_F32, xout=ex.out_ptr(e))
            return dict(epilogue=EPI_F32, out_f32=bufs.psum)

        # bytes per row of every per-row pointer a decode GEMV takes (row m = sequence m)
        row_bytes = dict(psum=4 * H, q_out=2 * self.nq * hd, k_cache=2 * self.nkv * self.S * hd,
                         v_cache=2 * self.nkv * self.S * hd, argmax_keys=8, out_f32=4 * H)

        def gemv_blocks(name, K, bits, kw):
            """One decode GEMV as row blocks of at most what one launch can
            stage (every block re-reads the weights); a single call when the
            rows fit. The peer exchange addresses whole [M][K] blocks, so it
            takes only batches that fit."""
            fit = min(32, max(1, _stage_rows(K, bits, kw.get("prologue", PRO_NORM) != PRO_PLAIN)))
            if prefill or rows <= fit:
                a = self._gemv(rows, bits=bits, K=K, **kw)
                calls.append(("gemv", a, name))
                gemv_args.append(a)
                return
            if ex is not None:
                raise ValueError(f"batch {rows} exceeds the {fit} rows one {name} launch stages; the peer "
                                 "exchange takes whole batches: use exchange='nccl'")
            ld = dict(act=kw.get("lda", 0), x_out=kw.get("lda", 0), out=kw.get("ldo", 0), residual=kw.get("ldo", 0))
            for r0 in range(0, rows, fit):
                d = dict(kw)
                for k, v in kw.items():
                    per = row_bytes.get(k, 2 * ld[k] if k in ld else None)
                    if per is None or v is None:
                        continue
                    d[k] = (v.data_ptr() if isinstance(v, torch.Tensor) else v) + r0 * per
                a = self._gemv(min(fit, rows - r0), bits=bits, K=K, **d)
                calls.append(("gemv", a, name))
                gemv_args.append(a)

        if prefill:
            calls.append(("prefill_embed", bufs, "embed"))
        for li, L in enumerate(self.layers):
            pro = norm_pro()
            gemv_blocks("qkv", H, sp.bits, dict(
                epilogue=EPI_ROPE_KV, N=(self.nq + 2 * self.nkv) * hd, group_size=sp.group_size, weight=L.qkv_w,
                scales=L.qkv_s, gamma=L.in_norm, head_dim=hd, n_q_heads=self.nq, n_kv_heads=self.nkv,
                max_seq=self.S, rope_cos=self.rope_cos, rope_sin=self.rope_sin, pos=self.pos, q_out=bufs.q,
                k_cache=self.k_cache[li], v_cache=self.v_cache[li], prefill_seq=seq, **pro))
            at = AttentionArgs(q=bufs.q.data_ptr(), k_cache=self.k_cache[li].data_ptr(),
                               v_cache=self.v_cache[li].data_ptr(), out=bufs.attn.data_ptr(), pos=self.pos.data_ptr(),
                               batch=rows, n_q_heads=self.nq, n_kv_heads=self.nkv, head_dim=hd, max_seq=self.S,
                               pdl=self.pdl, prefill_seq=seq)
            calls.append(("attn", at, "attn"))
            gemv_blocks("o", self.nq * hd, sp.bits, dict(
                prologue=PRO_PLAIN, N=H, group_size=sp.group_size, weight=L.o_w, scales=L.o_s, act=bufs.attn,
                lda=self.nq * hd, ldo=H, **partial_epi(2 * li)))
            if tp:
                if ex is None:
                    calls.append(("allreduce", bufs.psum, "allreduce"))
                pending = 2 * li
            pro = norm_pro()
            gemv_blocks("gu", H, sp.bits, dict(
                epilogue=EPI_SWIGLU, N=2 * self.inter, group_size=sp.group_size, weight=L.gu_w, scales=L.gu_s,
                gamma=L.post_norm, out=bufs.act, ldo=self.inter, **pro))
            blk = rows if (tp and ex is not None) else min(rows, down_rows(sp, self.tp_size), 32)
            for r0 in range(0, rows, blk):   # row blocks when the chunk exceeds what the down_proj can stage
                nr = min(blk, rows - r0)
                epi = partial_epi(2 * li + 1)
                if not tp:
                    epi.update(out=xs[cur].data_ptr() + 2 * r0 * H, residual=xs[cur].data_ptr() + 2 * r0 * H)
                elif ex is None:
                    epi.update(out_f32=bufs.psum.data_ptr() + 4 * r0 * H)
                a = self._gemv(nr, bits=sp.bits, prologue=PRO_PLAIN, N=H, K=self.inter, group_size=sp.group_size,
                               weight=L.d_w, scales=L.d_s, act=bufs.act.data_ptr() + 2 * r0 * self.inter,
                               lda=self.inter, ldo=H, **epi)
                calls.append(("gemv", a, "down"))
                gemv_args.append(a)
            if tp:
                if ex is None:
                    calls.append(("allreduce", bufs.psum, "allreduce"))
                pending = 2 * li + 1
        if not final:
            # the residual stream of the chunk is not needed further: only the KV cache
            calls.append(("prefill_advance", rows, "advance"))
            return calls, gemv_args
        pro = norm_pro()
        head = dict(epilogue=EPI_ARGMAX, argmax_keys=bufs.keys)
        if ex is not None:
            head.update(epilogue=EPI_PEER_ARGMAX, xout=ex.out_ptr(2 * len(self.layers)))
        gemv_blocks("lm_head", H, self.lm_bits, dict(
            N=self.vshard, group_size=self.lm_group, weight=self.lm_head, scales=self.lm_scales,
            gamma=self.final_norm, out=bufs.logits, ldo=self.vshard, argmax_offset=self.tp_rank * self.vshard,
            **head, **pro))
        if tp and ex is None:
            calls.append(("allreduce_max", bufs.keys, "allreduce"))
        calls.append(("prefill_sample" if prefill else "sample", bufs, "sample"))
        return calls, gemv_args

    def _make_tc_calls(self, bufs, final: bool, decode: bool = False):
        """A prompt chunk on the tensor cores: per layer RMSNorm rows, the q|k|v
        GEMM (RoPE + KV append), attention, the o GEMM (+ residual, in place),
        RMSNorm, the gate|up GEMM (SwiGLU), the down GEMM (+ residual); the last
        chunk then runs the lm_head GEMV on its last row only. With tensor
        parallelism the o and down GEMMs write this rank's fp32 partial sums,
        NCCL all-reduces them, and lw_resid_rmsnorm_rows adds them to the
        residual before the next norm; the lm_head's vocabulary-shard argmax keys
        are max-reduced the same way, so prefill_sample reads local keys.
        decode=True: the same layers for one decode step of a large batch (row
        m = sequence m at *pos), then the lm_head GEMV over every row (in row
        blocks of what one launch stages) and the sampler."""
        sp, H, hd, rows = self.spec, self.spec.hidden, self.spec.head_dim, bufs.rows
        seq = None if decode else self.seq.data_ptr()
        tp = self.tp_size > 1
        bufs.sample_xin = None
        calls = [] if decode else [("prefill_embed", bufs, "embed")]

        def tc(epi, N, K, w, s_, act, lda, out, ldo, name="tc", bits=None, group_size=None, **kw):
            a = PrefillGemmArgs(bits=sp.bits if bits is None else bits, epilogue=epi, pdl=self.pdl, M=rows, N=N,
                                K=K, group_size=sp.group_size if group_size is None else group_size, lda=lda,
                                ldo=ldo, act=act.data_ptr(), weight=w.data_ptr(),
                                scales=s_.data_ptr() if s_ is not None else None,
                                out=out.data_ptr() if out is not None else None)
            for k, v in kw.items():
                setattr(a, k, v.data_ptr() if isinstance(v, torch.Tensor) else v)
            return ("tcgemm", a, name)

        def norm(gamma, pending):
            if pending:
                return ("resid_rmsnorm", (bufs.x, bufs.psum, gamma, bufs.h, rows), "norm")
            return ("rmsnorm", (bufs.x, gamma, bufs.h, rows), "norm")

        def row_split(w, s_, act, K, name):
            if not tp:
                return [tc(TC_EPI_RESID, H, K, w, s_, act, K, bufs.x, H, name=name, residual=bufs.x)]
            return [tc(TC_EPI_F32, H, K, w, s_, act, K, bufs.psum, H, name=name), ("allreduce", bufs.psum, "allreduce")]

        for li, L in enumerate(self.layers):
            calls.append(norm(L.in_norm, tp and li > 0))
            calls.append(tc(TC_EPI_ROPE_KV, (self.nq + 2 * self.nkv) * hd, H, L.qkv_w, L.qkv_s, bufs.h, H, bufs.q,
                            self.nq * hd, name="qkv", head_dim=hd, n_q_heads=self.nq, n_kv_heads=self.nkv,
                            max_seq=self.S, rope_cos=self.rope_cos, rope_sin=self.rope_sin, pos=self.pos, seq=seq,
                            q_out=bufs.q, k_cache=self.k_cache[li], v_cache=self.v_cache[li]))
            at = AttentionArgs(q=bufs.q.data_ptr(), k_cache=self.k_cache[li].data_ptr(),
                               v_cache=self.v_cache[li].data_ptr(), out=bufs.attn.data_ptr(), pos=self.pos.data_ptr(),
                               batch=rows, n_q_heads=self.nq, n_kv_heads=self.nkv, head_dim=hd, max_seq=self.S,
                               pdl=self.pdl, prefill_seq=seq)
            calls.append(("attn", at, "attn"))
            calls += row_split(L.o_w, L.o_s, bufs.attn, self.nq * hd, "o")
            calls.append(norm(L.post_norm, tp))
            calls.append(tc(TC_EPI_SWIGLU, 2 * self.inter, H, L.gu_w, L.gu_s, bufs.h, H, bufs.act, self.inter,
                            name="gu"))
            calls += row_split(L.d_w, L.d_s, bufs.act, self.inter, "down")
        if not final:
            calls.append(("prefill_advance", rows, "advance"))
            return calls, []
        if tp:   # the last down partial joins the residual stream (h is not used)
            calls.append(norm(self.final_norm, True))
        if decode and self.vshard % 128 == 0 and (self.lm_bits == 16 or self.lm_group >= 32):
            # every row's logits and argmax key on the tensor cores: the head's
            # weights are read once for the whole batch
            if not tp:
                calls.append(norm(self.final_norm, False))
            calls.append(tc(TC_EPI_ARGMAX, self.vshard, H, self.lm_head, self.lm_scales, bufs.h, H, bufs.logits,
                            self.vshard, name="lm_head", bits=self.lm_bits,
                            group_size=H if self.lm_bits == 16 else self.lm_group, argmax_keys=bufs.keys,
                            argmax_offset=self.tp_rank * self.vshard))
            if tp:
                calls.append(("allreduce_max", bufs.keys, "allreduce"))
            calls.append(("sample", bufs, "sample"))
            return calls, []
        if decode:
            # every row's logits and argmax key, in row blocks of what one GEMV launch stages
            fit = min(32, max(1, _stage_rows(H, self.lm_bits, True)))
            gemv_args = []
            for r0 in range(0, rows, fit):
                a = self._gemv(min(fit, rows - r0), bits=self.lm_bits, prologue=PRO_NORM, epilogue=EPI_ARGMAX,
                               N=self.vshard, K=H, group_size=self.lm_group, weight=self.lm_head,
                               scales=self.lm_scales, gamma=self.final_norm, act=bufs.x.data_ptr() + 2 * r0 * H,
                               lda=H, out=bufs.logits.data_ptr() + 2 * r0 * self.vshard, ldo=self.vshard,
                               argmax_keys=bufs.keys.data_ptr() + 8 * r0, argmax_offset=self.tp_rank * self.vshard)
                calls.append(("gemv", a, "lm_head"))
                gemv_args.append(a)
            if tp:
                calls.append(("allreduce_max", bufs.keys, "allreduce"))
            calls.append(("sample", bufs, "sample"))
            return calls, gemv_args
        last = bufs.x.data_ptr() + 2 * (rows - 1) * H
        a = self._gemv(1, bits=self.lm_bits, prologue=PRO_NORM, epilogue=EPI_ARGMAX, N=self.vshard, K=H,
                       group_size=self.lm_group, weight=self.lm_head, scales=self.lm_scales,
                       gamma=self.final_norm, act=last, lda=H,
                       out=bufs.logits.data_ptr() + 2 * (rows - 1) * self.vshard, ldo=self.vshard,
                       argmax_keys=bufs.keys.data_ptr() + 8 * (rows - 1), argmax_offset=self.tp_rank * self.vshard)
        calls.append(("gemv", a, "lm_head"))
        if tp:
            calls.append(("allreduce_max", bufs.keys, "allreduce"))
        calls.append(("prefill_sample", bufs, "sample"))
        return calls, [a]

    def _attach_workspace(self, gemv_args):
        """One workspace shared by the sequential GEMVs of every call list."""
        need = max([int(nat.lib().lw_fused_gemv_workspace_size(ctypes.byref(a))) for a in gemv_args] + [256])
        if getattr(self, "workspace", None) is None or self.workspace.numel() < need:
            if getattr(self, "workspace", None) is not None:
                # a graph captured before may still write there: never hand it back
                self._retired_workspaces = getattr(self, "_retired_workspaces", []) + [self.workspace]
            self.workspace = torch.zeros(max(need, 256), dtype=torch.uint8, device=self.device)
            for a in getattr(self, "_all_gemv_args", []):
                a.workspace, a.workspace_bytes = self.workspace.data_ptr(), self.workspace.numel()
        self._all_gemv_args = getattr(self, "_all_gemv_args", []) + list(gemv_args)
        for a in gemv_args:
            a.workspace, a.workspace_bytes = self.workspace.data_ptr(), self.workspace.numel()

    def _build_calls(self):
        self.workspace = None
        if self.tc_decode:   # large batches: the step's linears on the tensor cores (NCCL under TP)
            self.calls, gemv_args = self._make_tc_calls(self.dec, final=True, decode=True)
        else:
            self.calls, gemv_args = self._make_calls(self.dec, prefill=False)
        self._attach_workspace(gemv_args)
        self.stat_args = {id(a): self._stat_variant(a) for a in gemv_args}
        self.x_in = self.x   # layer 0 reads the residual stream from self.x; sample writes it there
        self.sample_xin = (self.exchange.in_ptr(2 * len(self.layers))
                           if self.exchange is not None and not self.tc_decode else None)
        self.prefill_calls = {}

    def _stat_variant(self, a: FusedGemvArgs) -> FusedGemvArgs:
        """The same GEMV with its exchange replaced by local buffers, for timing
        one kernel class alone (a lone exchange would never be answered)."""
        b = FusedGemvArgs.from_buffer_copy(a)
        if b.prologue == PRO_PEER_RESID_NORM:
            b.prologue, b.psum, b.xin = PRO_RESID_NORM, self.psum.data_ptr(), None
        if b.epilogue == EPI_PEER_F32:
            b.epilogue, b.out_f32, b.xout = EPI_F32, self.psum.data_ptr(), None
        elif b.epilogue == EPI_PEER_ARGMAX:
            b.epilogue, b.xout = EPI_ARGMAX, None
        return b

    # -------------------------------------------------------------- execution
    def _enqueue_step(self, sample: bool = True):
        self._enqueue(self.calls, sample)

    def _enqueue(self, calls, sample: bool = True):
        lib = nat.lib()
        s = torch.cuda.current_stream(self.device).cuda_stream
        for kind, a, _name in calls:
            if kind == "sample" and not sample:
                continue
            if kind == "gemv":
                nat.check("lw_fused_gemv", lib.lw_fused_gemv(ctypes.byref(a), s))
            elif kind == "attn":
                nat.check("lw_attention_decode", lib.lw_attention_decode(ctypes.byref(a), s))
            elif kind == "allreduce":
                torch.distributed.all_reduce(a, group=self.tp_group)
            elif kind == "allreduce_max":
                torch.distributed.all_reduce(a, op=torch.distributed.ReduceOp.MAX, group=self.tp_group)
            elif kind == "sample":
                self._sample(s)
            elif kind == "tcgemm":
                nat.check("lw_prefill_gemm", lib.lw_prefill_gemm(ctypes.byref(a), s))
            elif kind == "rmsnorm":
                x, gamma, h, rows = a
                nat.check("lw_rmsnorm_rows", lib.lw_rmsnorm_rows(x.data_ptr(), gamma.data_ptr(), h.data_ptr(), rows,
                                                                 self.spec.hidden, self.spec.eps, self.pdl, s))
            elif kind == "resid_rmsnorm":
                x, psum, gamma, h, rows = a
                nat.check("lw_resid_rmsnorm_rows", lib.lw_resid_rmsnorm_rows(
                    x.data_ptr(), psum.data_ptr(), gamma.data_ptr(), h.data_ptr(), rows, self.spec.hidden,
                    self.spec.eps, self.pdl, s))
            elif kind == "prefill_embed":
                nat.check("lw_prefill_embed", lib.lw_prefill_embed(
                    self.tokens.data_ptr(), self.embed.data_ptr(), a.x.data_ptr(), self.pos.data_ptr(),
                    self.seq.data_ptr(), a.rows, self.B, self.spec.hidden, self.pdl, s))
            elif kind == "prefill_advance":
                nat.check("lw_prefill_advance", lib.lw_prefill_advance(
                    self.pos.data_ptr(), self.step_count.data_ptr(), a, self.pdl, s))
            elif kind == "prefill_sample":
                nat.check("lw_prefill_sample", lib.lw_prefill_sample(
                    self.tokens.data_ptr(), a.keys.data_ptr(), self.embed.data_ptr(), self.x_in.data_ptr(),
                    self.pos.data_ptr(), self.step_count.data_ptr(), self.seq.data_ptr(),
                    getattr(a, "sample_xin", self.sample_xin), a.rows,
                    self.B, self.spec.hidden, self.pdl, s))

    def _sample(self, s):
        nat.check("lw_sample_tokens", nat.lib().lw_sample_tokens(
            self.tokens.data_ptr(), self.keys.data_ptr(), self.embed.data_ptr(), self.x_in.data_ptr(),
            self.pos.data_ptr(), self.done.data_ptr(), self.step_count.data_ptr(), self.sample_xin, self.B,
            self.spec.hidden, self.pdl, s))

    def kernels_per_step(self) -> int:
        return sum(1 for k, _, _n in self.calls if k in ("gemv", "attn", "sample", "tcgemm", "rmsnorm",
                                                          "resid_rmsnorm"))

    def tune_kernels(self, reps: int = 5, margin: float = 0.03) -> dict:
        """Per projection class of the decode step (qkv, o, gu, down, lm_head),
        time its launches alone (a CUDA graph replayed `reps` times, CUDA
        events) with the shared-memory ring GEMV and with the register-pipeline
        GEMV, and keep the ring unless the other is faster by more than
        `margin`. Runs on the engine's scratch state (before start())."""
        classes = []
        for kind, _a, n in self.calls:
            if kind == "gemv" and n not in classes:
                classes.append(n)
        dev = self.device
        for name in classes:
            ms = {}
            for kern in (0, 1):
                for kind, a, n in self.calls:
                    if kind == "gemv" and n == name:
                        a.kernel = kern
                        self.stat_args[id(a)].kernel = kern
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):
                    self.enqueue_only(name)
                torch.cuda.synchronize(dev)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=side):
                    self.enqueue_only(name)
                g.replay()
                torch.cuda.synchronize(dev)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    g.replay()
                e1.record()
                torch.cuda.synchronize(dev)
                ms[kern] = e0.elapsed_time(e1) / reps
                del g
            pick = 1 if ms[1] < ms[0] * (1.0 - margin) else 0
            for kind, a, n in self.calls:
                if kind == "gemv" and n == name:
                    a.kernel = pick
                    self.stat_args[id(a)].kernel = pick
            self.kernel_choice[name] = {"kernel": "ring" if pick == 0 else "register-pipeline",
                                        "ring_us": round(ms[0] * 1e3, 2), "pipeline_us": round(ms[1] * 1e3, 2)}
        self.check()
        return self.kernel_choice

    def enqueue_only(self, name: str):
        """Enqueue just the kernels of one class (qkv, attn, o, gu, down, lm_head)
        of a step, for per-kernel timing; the outputs are scratch."""
        lib = nat.lib()
        s = torch.cuda.current_stream(self.device).cuda_stream
        for kind, a, n in self.calls:
            if n != name:
                continue
            if kind == "gemv":
                nat.check("lw_fused_gemv", lib.lw_fused_gemv(ctypes.byref(self.stat_args[id(a)]), s))
            elif kind == "attn":
                nat.check("lw_attention_decode", lib.lw_attention_decode(ctypes.byref(a), s))
            elif kind == "tcgemm":
                nat.check("lw_prefill_gemm", lib.lw_prefill_gemm(ctypes.byref(a), s))

    def generate(self, input_ids: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
        """Greedy continuation of input_ids [B, P] (host or device); returns the
        new tokens [B, max_new_tokens] on the host. The prompt runs in chunks
        (prefill), then one graph replay per new token, one device->host copy
        at the end."""
        self.start(input_ids)
        self.prefill()
        self.capture()
        self.step(max_new_tokens - 1)
        out = self.generated(max_new_tokens).to("cpu")
        self.check()
        return out

    # -------------------------------------------------------------- prefill
    def _prefill_calls(self, rows: int, final: bool):
        key = (rows, final)
        if self.exchange is not None and not self.use_tc:
            assert rows <= self.exchange.rows, "prompt chunk larger than the exchange buffers"
        if key not in self.prefill_calls:
            bufs = self.pf if rows == self.pf.rows else self._buffers(rows)
            if self.use_tc:
                calls, gemv_args = self._make_tc_calls(bufs, final)
            else:
                calls, gemv_args = self._make_calls(bufs, prefill=True, final=final)
            self._attach_workspace(gemv_args)
            self.prefill_calls[key] = calls
        return self.prefill_calls[key]

    def _capture_graph(self, calls):
        """CUDA graph of a call list, after one eager run whose effects on the
        decode state (tokens, position, residual stream, keys) are undone; the
        exchange step count is not, so every rank stays in step."""
        saved = (self.tokens.clone(), self.pos.clone(), self.x_in.clone(), self.keys.clone())
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._enqueue(calls)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            self._enqueue(calls)
        torch.cuda.synchronize(self.device)
        self.tokens.copy_(saved[0])
        self.pos.copy_(saved[1])
        self.x_in.copy_(saved[2])
        self.keys.copy_(saved[3])
        return g

    def _prefill_graph(self, rows: int, final: bool):
        key = (rows, final)
        if key not in self.prefill_graphs:
            self.prefill_graphs[key] = self._capture_graph(self._prefill_calls(rows, final))
        return self.prefill_graphs[key]

    def prefill(self, graph: bool = True):
        """Run every sequence's prompt (loaded by start()) through the model in
        chunks of up to prefill_rows positions: the KV cache holds positions
        0..P-1, the first new token of each sequence is picked and embedded,
        and the position is P. One chunk reads every weight once."""
        P, R = self.prompt_len, self.prefill_rows
        n = (P + R - 1) // R
        last = P - (n - 1) * R
        plan = [(R, False)] * (n - 1) + [(last, True)]
        for b in range(self.B):
            self.seq.fill_(b)
            self.pos.zero_()
            for rows, final in plan:
                if graph:
                    self._prefill_graph(rows, final).replay()
                else:
                    self._enqueue(self._prefill_calls(rows, final))
        self.host_pos = P

    def check(self) -> None:
        """Raise if a tensor-parallel exchange wait gave up (reads a device flag: syncs)."""
        if self.exchange is not None:
            self.exchange.check()

    def close(self) -> None:
        """Release the graph and, with a peer exchange, the shared block
        (collective over the tensor-parallel group)."""
        self.graph = None
        self.prefill_graphs = {}
        if self.exchange is not None:
            self.exchange.close()

    def start(self, prompt: torch.Tensor, forced: torch.Tensor | None = None):
        """Load a prompt (int [B, P]) and optional further forced tokens; position 0."""
        B, P = prompt.shape
        assert B == self.B
        self.tokens.fill_(-1)
        self.tokens[:P] = prompt.T.to(device=self.device, dtype=torch.int32)
        if forced is not None:
            self.tokens[P:P + forced.shape[1]] = forced.T.to(device=self.device, dtype=torch.int32)
        self.pos.zero_()
        self.keys.zero_()
        s = torch.cuda.current_stream(self.device).cuda_stream
        nat.call("lw_embed_tokens", self.tokens.data_ptr(), self.embed.data_ptr(), self.x_in.data_ptr(),
                 self.pos.data_ptr(), self.B, self.spec.hidden, 0, s)
        self.host_pos = 0
        self.prompt_len = P

    def capture(self):
        """Capture one decode step as a CUDA graph (after one eager step to warm up)."""
        if self.graph is None:
            self.graph = self._capture_graph(self.calls)

    def step(self, n: int = 1, graph: bool = True):
        for _ in range(n):
            if graph and self.graph is not None:
                self.graph.replay()
            else:
                self._enqueue_step()
            self.host_pos += 1

    def step_logits(self):
        """Eager step up to the logits (no token pick); pick_next() finishes it."""
        self._enqueue_step(sample=False)

    def pick_next(self):
        """Pick the next token (forced table entry or argmax), embed it, advance."""
        self._sample(torch.cuda.current_stream(self.device).cuda_stream)
        self.host_pos += 1

    def generated(self, new_tokens: int) -> torch.Tensor:
        P = self.prompt_len
        return self.tokens[P:P + new_tokens].T


# ------------------------------------------------------------------ HF model glue

def supports(model) -> bool:
    """True for LlamaForCausalLM-style models whose linears are liteweight QuantLinear."""
    from liteweight_b200.quantlinear import QuantLinear
    try:
        inner = model.model
        layer = inner.layers[0]
        qls = [layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj, layer.self_attn.o_proj,
               layer.mlp.gate_proj, layer.mlp.up_proj, layer.mlp.down_proj]
    except (AttributeError, IndexError, TypeError):
        return False
    if not all(isinstance(m, QuantLinear) and m.bias is None for m in qls):
        return False
    head = getattr(model, "lm_head", None)
    if isinstance(head, QuantLinear) and head.bias is not None:
        return False
    cfg = getattr(model, "config", None)
    return cfg is not None and getattr(cfg, "hidden_act", "silu") == "silu" and torch.cuda.is_available() \
        and next(model.parameters()).is_cuda


def spec_from_hf(model) -> LlamaSpec:
    cfg = model.config
    layer = model.model.layers[0]
    q = layer.self_attn.q_proj
    hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    return LlamaSpec(hidden=cfg.hidden_size, inter=cfg.intermediate_size, n_layers=cfg.num_hidden_layers,
                     n_heads=cfg.num_attention_heads, n_kv_heads=cfg.num_key_value_heads, head_dim=hd,
                     vocab=cfg.vocab_size, bits=q.bits, group_size=q.group_size, eps=cfg.rms_norm_eps)


def layers_from_hf(model) -> list:
    out = []
    for layer in model.model.layers:
        a, m = layer.self_attn, layer.mlp
        out.append(LayerWeights(
            q=(a.q_proj.qweight, a.q_proj.scales), k=(a.k_proj.qweight, a.k_proj.scales),
            v=(a.v_proj.qweight, a.v_proj.scales), o=(a.o_proj.qweight, a.o_proj.scales),
            gate=(m.gate_proj.qweight, m.gate_proj.scales), up=(m.up_proj.qweight, m.up_proj.scales),
            down=(m.down_proj.qweight, m.down_proj.scales),
            in_norm=layer.input_layernorm.weight.data, post_norm=layer.post_attention_layernorm.weight.data))
    return out


def engine_from_hf(model, batch: int, max_seq: int, tp_rank: int = 0, tp_size: int = 1, tp_group=None,
                   pdl: bool = True) -> DecodeEngine:
    spec = spec_from_hf(model)
    dev = next(model.parameters()).device
    packed = [PackedLayer(lw, spec, tp_rank, tp_size, dev) for lw in layers_from_hf(model)]
    # the model's own rotary embedding: exact HF cos/sin (default or llama3 scaled)
    rot = model.model.rotary_emb
    x = torch.zeros(1, 1, spec.hidden, dtype=torch.float16, device=dev)
    with torch.no_grad():
        cos, sin = rot(x, torch.arange(max_seq, device=dev)[None])
    from liteweight_b200.quantlinear import QuantLinear
    head = model.lm_head
    lm_w, lm_q = None, None
    if isinstance(head, QuantLinear):
        # swap_linears without skip=("lm_head",): the head is quantized too
        assert head.bias is None, "a biased lm_head is not supported"
        lm_q = (head.qweight, head.scales, head.bits, head.group_size)
    elif head.weight.data.data_ptr() != model.model.embed_tokens.weight.data.data_ptr():
        lm_w = head.weight.data
    return DecodeEngine(spec, packed, model.model.embed_tokens.weight.data, model.model.norm.weight.data,
                        lm_w, cos[0], sin[0], batch, max_seq, dev, tp_rank, tp_size, tp_group, pdl,
                        lm_head_quant=lm_q)


def build_engine(spec: LlamaSpec, layers: list, embed: torch.Tensor, final_norm: torch.Tensor,
                 lm_head: torch.Tensor | None, inv_freq: torch.Tensor, batch: int, max_seq: int, device,
                 attention_scaling: float = 1.0, tp_rank: int = 0, tp_size: int = 1, tp_group=None,
                 pdl: bool = True, fold_scales: bool = False, exchange: str = "peer",
                 lm_head_quant: tuple | None = None, tune_kernels: bool = True) -> DecodeEngine:
    """Engine from unsharded LayerWeights (liteweight-format tensors, any device).
    tune_kernels=False keeps the default GEMV choice (the ring kernel wherever
    it applies) instead of timing both, so two engines give the same bits."""
    packed = [PackedLayer(lw, spec, tp_rank, tp_size, device) for lw in layers]
    cos, sin = rope_tables(inv_freq, max_seq, attention_scaling, device)
    return DecodeEngine(spec, packed, embed, final_norm, lm_head, cos, sin, batch, max_seq, device, tp_rank,
                        tp_size, tp_group, pdl, fold_scales, exchange, lm_head_quant=lm_head_quant,
                        tune_kernels=tune_kernels)


def synthetic_layers(spec: LlamaSpec, device, seed: int = 0, std: float = 0.02) -> list:
    """Random-init layers (W ~ N(0, std) quantized with liteweight's RTN on the
    device, one linear at a time), norms 1 + N(0, 0.1): stands in for a
    checkpoint of the given architecture."""
    from liteweight_b200.quantize import quantize_int4, quantize_int8
    quant = quantize_int4 if spec.bits == 4 else quantize_int8
    g = torch.Generator(device=device).manual_seed(seed)
    layers = []
    for _ in range(spec.n_layers):
        lin = {}
        for name, n, k in spec.linear_shapes():
            w = torch.randn(n, k, device=device, generator=g, dtype=torch.float32).mul_(std).half()
            lin[name] = quant(w, spec.group_size)
            del w
        norms = [(1.0 + 0.1 * torch.randn(spec.hidden, device=device, generator=g)).half() for _ in range(2)]
        layers.append(LayerWeights(in_norm=norms[0], post_norm=norms[1], **lin))
    return layers


_ENGINES: dict = {}


def generate_ids(model, input_ids: torch.Tensor, max_new_tokens: int, temperature: float = 0.0,
                 top_k: int | None = None, eos_ids: set | None = None) -> list:
    """Greedy (or sampled) continuation of input_ids [B, P]; returns a list of
    token lists (each cut before its first EOS), as liteweight/generate.py:106-124."""
    from liteweight_b200.generate import _sample
    B, P = input_ids.shape
    need = P + max_new_tokens
    key = (id(model), B)
    eng = _ENGINES.get(key)
    if eng is None or eng.S < need:
        eng = engine_from_hf(model, batch=B, max_seq=max(need, 256))
        _ENGINES[key] = eng
    if temperature == 0.0:
        out = eng.generate(input_ids, max_new_tokens)
    else:
        eng.start(input_ids)
        # sampling (generate.py:54-59): same kernels; each new token is drawn by
        # torch on the device from the logits and forced into the token table
        for p in range(P + max_new_tokens - 1):
            eng.step_logits()
            if p >= P - 1:
                eng.tokens[p + 1] = _sample(eng.logits.float(), temperature, top_k).to(torch.int32)
            eng.pick_next()
        out = eng.generated(max_new_tokens).cpu()
    res = []
    for row in out.tolist():
        seq = []
        for t in row:
            if eos_ids and t in eos_ids:
                break
            seq.append(t)
        res.append(seq)
    return res
