"""Benchmark of liteweight_b200's hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|gemv] [--model 8b|1b|70b] [--batch B]

Prints ONE JSON line (rank 0). Workloads:

* ``decode`` (default) - greedy decode of a random-init Llama-3-8B
  architecture, INT4 group-128 weight-only (the reference's format), batch 1,
  512 uniform-random prompt ids, fp16 KV cache, tensor parallel over the N
  ranks (one process per GPU; the all-reduces run inside the GEMV kernels
  over NVLink peer memory, or as NCCL all-reduces with ``--exchange nccl``).
  One step = one decode token
  for the batch (graph replay of the fused decode step). Metric: decode
  tokens/s of the whole job (``scaling: strong``: the model and batch are
  fixed as N grows). ``--model 1b`` (INT8, prompt 128) and ``--model 70b``
  (INT4, context 2048) select the other decode configurations.
* ``gemv`` - the dequant GEMV of the Llama-3.2-1B linear shapes (K x N =
  2048x2048, 2048x512, 2048x8192, 8192x2048), INT4 and INT8 with group size
  128, M = 1: one step = those 8 GEMVs, each on its own weight copy from a
  rotating set larger than twice the L2. Metric: algorithmic GB/s (weights +
  fp16 scales + activation + output over time). Multi-GPU: independent
  replicas (``scaling: weak``). A per-M sweep (M = 1..256) is reported beside it.

``--impl reference`` times the reference's CPU path for the same workload
(dequantize the packed weights, fp32 matmul, fp16 result - restated by the
numpy oracle) on the host cores, rank 0 only, on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

GEMV_SHAPES = [(2048, 2048), (2048, 512), (2048, 8192), (8192, 2048)]   # (K, N)
GROUP = 128
L2_BYTES = 126 * 1024 * 1024


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: str):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def __enter__(self):
        try:
            import tempfile
            self.out = tempfile.NamedTemporaryFile("w", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.out is not None:
            self.out.close()

    def summary(self) -> dict | None:
        if self.proc is None or self.out is None:
            return None
        try:
            lines = [ln.strip() for ln in Path(self.out.name).read_text().splitlines() if ln.strip()]
        except OSError:
            return None
        finally:
            try:
                os.unlink(self.out.name)
            except OSError:
                pass
        sms, maxs, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxs.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxs), "reasons": sorted(reasons),
                "samples": len(sms)}


# ----------------------------------------------------------------- distributed

class Dist:
    def __init__(self):
        self.world = env_int("WORLD_SIZE", 1)
        self.rank = env_int("RANK", 0)
        self.local_rank = env_int("LOCAL_RANK", 0)
        self.pg = None

    def init(self, backend: str):
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120))
            self.pg = dist

    def barrier(self, device=None):
        if self.pg is not None:
            if device is not None:
                self.pg.barrier(device_ids=[device.index])
            else:
                self.pg.barrier()

    def max(self, v: float, device) -> float:
        if self.pg is None:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device=device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float, device) -> float:
        if self.pg is None:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device=device)
        self.pg.all_reduce(t)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


# ----------------------------------------------------------------- GEMV workload

def gemv_bytes(M: int, K: int, N: int, bits: int) -> int:
    from liteweight_b200.perf import quant_matmul_workload
    return quant_matmul_workload(M, K, N, bits, GROUP).bytes_moved


def capture_graph(fn):
    """CUDA graph of fn() captured on a side stream (after one eager warm-up there)."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn()
    torch.cuda.synchronize()
    return g


def time_graph(g, reps: int) -> float:
    """Average ms of one replay, CUDA events on the launching stream."""
    import torch
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


class GemvWorkload:
    name = "gemv"
    metric = "dequant-GEMV HBM GB/s (M=1, Llama-3.2-1B linear shapes, INT4+INT8 G128)"
    unit = "GB/s"

    def __init__(self, device, seed: int = 0):
        import torch
        from liteweight_b200 import _native as nat
        self.torch, self.nat, self.dev = torch, nat, device
        self.M = 1
        gen = torch.Generator(device=device).manual_seed(seed)
        self.items = [(bits, K, N) for bits in (4, 8) for K, N in GEMV_SHAPES]   # (bits, K, N)
        step_w = sum(N * K * b // 8 for b, K, N in self.items)
        # weight copies: one rotation is more than twice the L2
        self.R = max(3, -(-2 * L2_BYTES // step_w))
        self.weights = []   # [copy][item] -> (q, s)
        for _ in range(self.R):
            per = []
            for bits, K, N in self.items:
                if bits == 4:
                    q = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=device, generator=gen)
                else:
                    q = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=device, generator=gen)
                s = (torch.rand(N, K // GROUP, device=device, generator=gen) * 2e-3 + 1e-4).half()
                per.append((q, s))
            self.weights.append(per)
        self.acts = {K: torch.randn(256, K, dtype=torch.float16, device=device, generator=gen)
                     for K in {K for _, K, _ in self.items}}
        self.outs = {N: torch.empty(256, N, dtype=torch.float16, device=device)
                     for N in {N for _, _, N in self.items}}
        self.bytes_per_step = sum(gemv_bytes(self.M, K, N, b) for b, K, N in self.items)
        n0 = nat.launch_count()
        self.step_graphs = [capture_graph(lambda r=r: self._step(r)) for r in range(self.R)]
        # capture_graph runs fn twice (eager warm-up + capture): launches of one step
        self.launches_per_step = (nat.launch_count() - n0) // (2 * self.R)

    def _call(self, i: int, copy: int, M: int):
        bits, K, N = self.items[i]
        q, s = self.weights[copy][i]
        act, out = self.acts[K], self.outs[N]
        stream = self.torch.cuda.current_stream().cuda_stream
        ws, ws_bytes = self.nat.matmul_workspace(bits, M, N, K, self.dev, stream)
        fn = "lw_gemm_w4a16" if bits == 4 else "lw_gemm_w8a16"
        self.nat.call(fn, act.data_ptr(), q.data_ptr(), s.data_ptr(), None, out.data_ptr(), M, N, K, GROUP,
                      ws, ws_bytes, stream)

    def _step(self, copy: int):
        for i in range(len(self.items)):
            self._call(i, copy, self.M)

    def step(self, it: int):
        self.step_graphs[it % self.R].replay()

    def kernel_stats(self) -> dict:
        """Per kernel family: algorithmic bytes and device time of its launches in
        one step, each launch timed in a graph of R back-to-back launches over the
        rotating weight copies (CUDA events around the replays)."""
        fam = {}
        for i, (bits, K, N) in enumerate(self.items):
            g = capture_graph(lambda i=i: [self._call(i, r, self.M) for r in range(self.R)])
            ms = time_graph(g, 20) / self.R
            d = fam.setdefault(f"gemv_w{bits}a16", {"bytes": 0, "ms": 0.0, "launches": 0, "shapes": {}})
            d["bytes"] += gemv_bytes(self.M, K, N, bits)
            d["ms"] += ms
            d["launches"] += 1
            d["shapes"][f"{K}x{N}"] = {"us": round(ms * 1e3, 3),
                                       "GB/s": round(gemv_bytes(self.M, K, N, bits) / (ms * 1e-3) / 1e9, 1)}
        return fam

    def e2e(self, steps: int) -> dict:
        """Same GEMVs through the public drop-in ops with host buffers: pinned
        activation copied in and the result copied out every call."""
        torch = self.torch
        from liteweight_b200 import kernels
        host_act = {K: a[:self.M].cpu().pin_memory() for K, a in self.acts.items()}
        host_out = [torch.empty(self.M, N, dtype=torch.float16).pin_memory() for _, _, N in self.items]
        h2d = sum(self.M * K * 2 for _, K, _ in self.items)
        d2h = sum(self.M * N * 2 for _, _, N in self.items)

        def one(it):
            copy = it % self.R
            for i, (bits, K, N) in enumerate(self.items):
                a = host_act[K].to(self.dev, non_blocking=True)
                q, s = self.weights[copy][i]
                fn = kernels.matmul_int4 if bits == 4 else kernels.matmul_int8
                host_out[i].copy_(fn(a, q, s, GROUP), non_blocking=True)

        for it in range(3):
            one(it)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for it in range(steps):
            one(it)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        return {"value": round(self.bytes_per_step / (ms * 1e-3) / 1e9, 2), "unit": self.unit,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 4),
                "path": "liteweight_b200.kernels.matmul_int4/int8 per call (ctypes), pinned host in/out"}

    def sweep(self) -> dict:
        """Algorithmic GB/s vs M for both bit widths over the four shapes (graph-timed)."""
        out = {}
        for bits in (4, 8):
            for M in (1, 2, 4, 8, 16, 32, 64, 128, 256):
                idx = [self.items.index((bits, K, N)) for K, N in GEMV_SHAPES]
                g = capture_graph(lambda: [self._call(i, r, M) for r in range(self.R) for i in idx])
                ms = time_graph(g, 5) / self.R
                tot_b = sum(gemv_bytes(M, K, N, bits) for K, N in GEMV_SHAPES)
                out[f"w{bits}_M{M}"] = round(tot_b / (ms * 1e-3) / 1e9, 1)
        return out


# ----------------------------------------------------------------- decode workload

MODELS = {
    "8b": dict(arch="LLAMA_3_8B", bits=4, prompt=512, new=256, name="Llama-3-8B"),
    "1b": dict(arch="LLAMA_3_2_1B", bits=8, prompt=128, new=256, name="Llama-3.2-1B"),
    "70b": dict(arch="LLAMA_3_70B", bits=4, prompt=2048, new=256, name="Llama-3-70B"),
}


class DecodeWorkload:
    unit = "tokens/s"

    def __init__(self, device, dist: "Dist", model: str, batch: int, extra_steps: int, fold: bool = False,
                 exchange: str = "peer", prompt: int | None = None, new: int | None = None,
                 layers: int | None = None):
        import torch
        from liteweight_b200 import engine as E
        cfg = MODELS[model]
        self.torch, self.E, self.dev, self.cfg = torch, E, device, cfg
        arch = dict(getattr(E, cfg["arch"]))
        if layers:
            arch["n_layers"] = layers
        self.spec = E.LlamaSpec(**arch, bits=cfg["bits"], group_size=GROUP)
        self.B, self.P, self.T = batch, prompt or cfg["prompt"], new or cfg["new"]
        self.tp, self.rank = dist.world, dist.rank
        self.metric = (f"decode tokens/s ({cfg['name']} INT{cfg['bits']} G{GROUP} weight-only, batch {batch}, "
                       f"prompt {self.P}, greedy, TP{self.tp})")
        max_seq = self.P + max(self.T, extra_steps) + 1
        g = torch.Generator(device=device).manual_seed(20251201)
        spec = self.spec
        packed = []
        for li in range(spec.n_layers):
            # identical full layer on every rank (same seed), then this rank's shard
            lw = E.synthetic_layers(E.LlamaSpec(**{**spec.__dict__, "n_layers": 1}), device, seed=1000 + li)[0]
            packed.append(E.PackedLayer(lw, spec, self.rank, self.tp, device))
            del lw
        embed = (torch.randn(spec.vocab, spec.hidden, device=device, generator=g) * 0.02).half()
        norm = (1.0 + 0.1 * torch.randn(spec.hidden, device=device, generator=g)).half()
        cos, sin = E.rope_tables(E.default_inv_freq(spec.head_dim, spec.rope_theta), max_seq, 1.0, device)
        group = None
        if self.tp > 1:
            import torch.distributed as tdist
            group = tdist.group.WORLD
        self.eng = E.DecodeEngine(spec, packed, embed, norm, None, cos, sin, batch, max_seq, device, self.rank,
                                  self.tp, group, fold_scales=fold, exchange=exchange)
        gp = torch.Generator().manual_seed(7)
        self.prompt = torch.randint(0, spec.vocab, (batch, self.P), generator=gp)
        torch.cuda.synchronize()

    def prefill(self):
        """Load the prompt and run it through the model in chunks (the engine's
        prefill), up to the first decode step."""
        self.eng.start(self.prompt)
        self.eng.prefill()
        self.eng.capture()

    def step(self, it: int):
        self.eng.step(1)

    def context(self) -> int:
        return self.eng.host_pos + 1

    def bytes_per_step(self, ctx: int) -> int:
        """Weight bytes (this rank's shard, incl. fp16 lm_head shard) + KV bytes read."""
        sp = self.spec
        return sp.weight_bytes_per_token() // self.tp + self.B * sp.kv_bytes_per_position() * ctx // self.tp

    def kernel_stats(self, ctx: int) -> dict:
        """Per kernel class: one step's launches captured alone in a graph,
        replayed and timed with CUDA events (avg duration per launch)."""
        torch, sp, eng = self.torch, self.spec, self.eng
        H, I, hd = sp.hidden, sp.inter // self.tp, sp.head_dim
        nq, nkv = sp.n_heads // self.tp, sp.n_kv_heads // self.tp

        def wbytes(n, k):
            return n * k * sp.bits // 8 + 2 * n * (k // GROUP)
        per_launch = {
            "qkv": wbytes((nq + 2 * nkv) * hd, H) + 2 * self.B * H,
            "attn": self.B * 2 * nkv * ctx * hd * 2,
            "o": wbytes(H, nq * hd) + 2 * self.B * nq * hd,
            "gu": wbytes(2 * I, H) + 2 * self.B * H,
            "down": wbytes(H, I) + 2 * self.B * I,
            "lm_head": (sp.vocab // self.tp) * H * 2 + 2 * self.B * H,
        }
        out = {}
        for name, b in per_launch.items():
            launches = sum(1 for _, _, n in eng.calls if n == name)
            g = capture_graph(lambda name=name: eng.enqueue_only(name))
            ms = time_graph(g, 10) / launches
            out[name] = {"launches": launches, "bytes": b, "us": round(ms * 1e3, 3),
                         "GB/s": round(b / (ms * 1e-3) / 1e9, 1)}
            del g
        return out

    def e2e(self) -> dict:
        """The public decode call with host buffers: prompt ids from pinned host
        memory, prefill + T greedy tokens, generated ids copied back."""
        torch = self.torch
        host_ids = self.prompt.to(torch.int32).pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        ids = self.eng.generate(host_ids, self.T)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        return {"ms": ms, "tokens": self.B * self.T, "h2d_bytes_per_step": host_ids.numel() * 4,
                "d2h_bytes_per_step": ids.numel() * 4, "ids": ids}


class CpuDecode:
    """The reference's CPU path for one decode step, on a bounded sample: the
    oracle's QuantLinear arithmetic (dequantize the packed weights every call,
    fp32 matmul; liteweight/quantize.py:30-60, :102-135) for the seven linears
    of one layer at batch 1, split by output rows over the host cores, plus
    the fp16 lm_head; per-token time = layers x layer time + lm_head time
    (norms, RoPE and attention at batch 1 are <1% of the arithmetic and left
    out)."""

    def __init__(self, model: str, batch: int = 1):
        from liteweight_b200 import engine as E
        from oracle import quant as oq
        cfg = MODELS[model]
        self.spec = E.LlamaSpec(**getattr(E, cfg["arch"]), bits=cfg["bits"], group_size=GROUP)
        self.oq, self.B = oq, batch
        rng = np.random.default_rng(3)
        self.lin = []
        for name, n, k in self.spec.linear_shapes():
            if self.spec.bits == 4:
                q = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
            else:
                q = rng.integers(-127, 128, (n, k), dtype=np.int8)
            s = (rng.random((n, k // GROUP)) * 2e-3 + 1e-4).astype(np.float16)
            self.lin.append((name, q, s, rng.standard_normal((batch, k)).astype(np.float16)))
        self.cores = os.cpu_count() or 1
        self.pool = ThreadPoolExecutor(self.cores)
        self.lm_rows = 8192
        self.lm = (rng.standard_normal((self.lm_rows, self.spec.hidden)) * 0.02).astype(np.float16)
        self.h = rng.standard_normal((batch, self.spec.hidden)).astype(np.float16)

    def _rows(self, fn, n):
        blocks = np.array_split(np.arange(n), self.cores)
        return np.concatenate(list(self.pool.map(fn, blocks)), axis=1)

    def linear(self, i: int) -> float:
        name, q, s, act = self.lin[i]
        t = time.perf_counter()
        self._rows(lambda r: self.oq.packed_matmul(act, q[r], s[r], GROUP, self.spec.bits), q.shape[0])
        return time.perf_counter() - t

    def lm_head_seconds(self) -> float:
        t = time.perf_counter()
        self._rows(lambda r: (self.h.astype(np.float32) @ self.lm[r].astype(np.float32).T).astype(np.float16),
                   self.lm_rows)
        return (time.perf_counter() - t) * self.spec.vocab / self.lm_rows

    def measure(self, min_seconds: float = 10.0) -> dict:
        t0 = time.perf_counter()
        sums = [0.0] * len(self.lin)
        n = 0
        while n == 0 or time.perf_counter() - t0 < min_seconds:
            for i in range(len(self.lin)):
                sums[i] += self.linear(i)
            n += 1
        layer = sum(sums) / n
        lm = self.lm_head_seconds()
        tok_s = self.B / (self.spec.n_layers * layer + lm)
        return {"value": round(tok_s, 5), "unit": "tokens/s", "cores": self.cores, "kind": "port",
                "layer_seconds": round(layer, 3), "lm_head_seconds": round(lm, 3),
                "sample": f"{n} pass(es) over the 7 quantized linears of one layer (dequantize + fp32 matmul, "
                          f"rows split over {self.cores} threads) + the fp16 lm_head on {self.lm_rows} vocab rows "
                          f"scaled to {self.spec.vocab}; per token = {self.spec.n_layers} layers + lm_head"}


# ----------------------------------------------------------------- CPU baseline (reference path)

class CpuGemv:
    """The reference's CPU path for the same GEMVs: dequantize the packed weights
    and fp32-matmul (liteweight/quantize.py:30-60, :102-135), as restated by the
    oracle, split by output rows over the host cores."""

    def __init__(self, seed: int = 0):
        from oracle import quant as oq
        self.oq = oq
        rng = np.random.default_rng(seed)
        self.items = []
        for bits in (4, 8):
            for K, N in GEMV_SHAPES:
                if bits == 4:
                    q = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
                else:
                    q = rng.integers(-127, 128, (N, K), dtype=np.int8)
                s = (rng.random((N, K // GROUP)) * 2e-3 + 1e-4).astype(np.float16)
                act = rng.standard_normal((1, K)).astype(np.float16)
                self.items.append((bits, K, N, q, s, act))
        self.cores = os.cpu_count() or 1
        self.pool = ThreadPoolExecutor(self.cores)
        self.bytes_per_step = sum(gemv_bytes(1, K, N, b) for b, K, N, *_ in self.items)

    def _gemv(self, bits, q, s, act):
        n = q.shape[0]
        blocks = np.array_split(np.arange(n), self.cores)
        parts = list(self.pool.map(lambda r: self.oq.packed_matmul(act, q[r], s[r], GROUP, bits), blocks))
        return np.concatenate(parts, axis=1)

    def step(self):
        for bits, K, N, q, s, act in self.items:
            self._gemv(bits, q, s, act)

    def measure(self, min_seconds: float = 10.0, max_steps: int = 30) -> dict:
        self.step()
        t0 = time.perf_counter()
        n = 0
        while n < max_steps and (n == 0 or time.perf_counter() - t0 < min_seconds):
            self.step()
            n += 1
        dt = (time.perf_counter() - t0) / n
        return {"value": round(self.bytes_per_step / dt / 1e9, 3), "unit": "GB/s", "cores": self.cores,
                "kind": "port", "ms_per_step": round(dt * 1e3, 2),
                "sample": f"{n} passes over the 8 M=1 GEMVs (INT4+INT8, 1B shapes), numpy dequantize + fp32 "
                          f"matmul split by output rows over {self.cores} threads"}


# ----------------------------------------------------------------- main

def traffic_for(kernel_key: str) -> int | None:
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(kernel_key)
    except (OSError, ValueError):
        return None


def smi_gpu_id(local_rank: int) -> str:
    """nvidia-smi id of this rank's GPU (CUDA_VISIBLE_DEVICES entries are physical ids)."""
    vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    return vis[local_rank] if local_rank < len(vis) else str(local_rank)


def run_reference_gemv(args, dist: Dist):
    if dist.rank != 0:
        return
    cpu = CpuGemv()
    for _ in range(args.warmup):
        cpu.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu.step()
    dt = (time.perf_counter() - t0) / args.steps
    value = cpu.bytes_per_step / dt / 1e9
    line = {"impl": "reference", "metric": GemvWorkload.metric, "value": round(value, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8/int8 codes, fp32 acc",
            "data": "synthetic", "config": {"workload": "gemv M=1 Llama-3.2-1B shapes INT4+INT8 G128"},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cpu.cores, "kind": "port",
                             "sample": "every step = the 8 M=1 GEMVs, numpy dequantize + fp32 matmul"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_gemv(args, dist: Dist):
    import torch
    from liteweight_b200 import _native as nat
    from liteweight_b200 import build as lwbuild
    from liteweight_b200.perf import b200_measured

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the product has no CPU path)")
    dev = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(dev)
    dist.init("nccl")
    lwbuild.build()
    nat.lib()
    wl = GemvWorkload(dev, seed=1234 + dist.rank)
    for it in range(args.warmup):
        wl.step(it)
    torch.cuda.synchronize()
    dist.barrier(dev)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(smi_gpu_id(dist.local_rank)) as clk:
        e0.record()
        for it in range(args.steps):
            wl.step(args.warmup + it)
        e1.record()
        torch.cuda.synchronize()
    launches = args.steps * wl.launches_per_step   # kernels inside the replayed step graphs
    dist.barrier(dev)
    ms = e0.elapsed_time(e1)
    ms_max = dist.max(ms, dev)
    total_bytes = dist.sum(wl.bytes_per_step * args.steps, dev)
    value = total_bytes / (ms_max * 1e-3) / 1e9
    fam = wl.kernel_stats()
    e2e = wl.e2e(max(10, args.steps))
    sweep = wl.sweep() if (dist.world == 1 and not args.no_sweep) else None
    peak, peak_src = b200_measured(ROOT / "MEASURED_PEAKS.json")
    dom = max(fam, key=lambda k: fam[k]["ms"])
    d = fam[dom]
    achieved = d["bytes"] / (d["ms"] * 1e-3) / 1e9
    per_launch_bytes = d["bytes"] / d["launches"]
    roofline = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1),
                "peak": peak.peak_mem_bandwidth_gbs, "peak_source": peak_src, "unit": "GB/s",
                "frac": round(achieved / peak.peak_mem_bandwidth_gbs, 4),
                "algorithmic_bytes_per_launch": int(per_launch_bytes),
                "avg_launch_us": round(d["ms"] / d["launches"] * 1e3, 3),
                "traffic": traffic_for(dom)}
    clocks = clk.summary()
    if dist.rank != 0:
        dist.close()
        return
    cpu = CpuGemv().measure() if dist.world == 1 else None
    line = {"metric": wl.metric, "value": round(value, 2), "unit": wl.unit, "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8/int8 codes x fp16, fp32 acc",
            "data": "synthetic",
            "config": {"workload": "gemv M=1 Llama-3.2-1B shapes (KxN 2048x2048, 2048x512, 2048x8192, 8192x2048) "
                                   "INT4+INT8 G128", "parallelism": f"replicas x{dist.world}",
                       "l2": f"rotating {wl.R} weight copies ({wl.R * sum(N * K * b // 8 for b, K, N in wl.items) >> 20}"
                             " MiB) > L2"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
            "kernels": {k: {"launches_per_step": v["launches"],
                            "GB/s": round(v["bytes"] / (v["ms"] * 1e-3) / 1e9, 1), "shapes": v["shapes"]}
                        for k, v in fam.items()},
            "clocks": clocks}
    if sweep is not None:
        line["gbs_vs_m"] = sweep
    print(json.dumps(line), flush=True)
    dist.close()


def run_decode(args, dist: Dist):
    import torch
    from liteweight_b200 import _native as nat
    from liteweight_b200 import build as lwbuild
    from liteweight_b200.perf import b200_measured

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the product has no CPU path)")
    dev = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(dev)
    dist.init("nccl")
    lwbuild.build()
    nat.lib()
    wl = DecodeWorkload(dev, dist, args.model, args.batch, args.warmup + args.steps, fold=args.fold,
                        exchange=args.exchange, prompt=args.prompt, new=args.new, layers=args.layers)
    if dist.world > 1:   # NCCL communicator up before graph capture
        t = torch.zeros(1, device=dev)
        dist.pg.all_reduce(t)
        torch.cuda.synchronize()
    wl.prefill()
    for it in range(args.warmup):
        wl.step(it)
    torch.cuda.synchronize()
    dist.barrier(dev)
    torch.cuda.synchronize()
    ctx0 = wl.context()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(smi_gpu_id(dist.local_rank)) as clk:
        e0.record()
        for it in range(args.steps):
            wl.step(it)
        e1.record()
        torch.cuda.synchronize()
    dist.barrier(dev)
    wl.eng.check()
    ms = e0.elapsed_time(e1)
    ms_max = dist.max(ms, dev)
    ctx_mid = ctx0 + args.steps // 2
    value = wl.B * args.steps / (ms_max * 1e-3)
    step_ms = ms_max / args.steps
    peak, peak_src = b200_measured(ROOT / "MEASURED_PEAKS.json")
    # per-kernel timing (kernel classes replayed alone), then the end-to-end call
    kstats = wl.kernel_stats(ctx_mid)
    dom = max(kstats, key=lambda k: kstats[k]["us"] * kstats[k]["launches"])
    d = kstats[dom]
    achieved = d["GB/s"]
    roofline = {"bound": "hbm", "kernel": f"fused GEMV {dom}" if dom != "attn" else "attention",
                "achieved": achieved, "peak": peak.peak_mem_bandwidth_gbs, "peak_source": peak_src, "unit": "GB/s",
                "frac": round(achieved / peak.peak_mem_bandwidth_gbs, 4), "algorithmic_bytes_per_launch": d["bytes"],
                "avg_launch_us": d["us"], "traffic": traffic_for(f"decode_{args.model}_tp{dist.world}_{dom}")}
    bstep = wl.bytes_per_step(ctx_mid)
    decode_roofline = {"bytes_per_step_per_gpu": bstep, "achieved_GBs_per_gpu": round(bstep / (step_ms * 1e-3) / 1e9, 1),
                       "frac": round(bstep / (step_ms * 1e-3) / 1e9 / peak.peak_mem_bandwidth_gbs, 4),
                       "roofline_tokens_per_s": round(wl.B * peak.peak_mem_bandwidth_gbs * 1e9 / bstep, 1),
                       "context_mid": ctx_mid}
    e = wl.e2e()
    e2e_ms = dist.max(e["ms"], dev)
    e2e = {"value": round(e["tokens"] / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
           "h2d_bytes_per_step": e["h2d_bytes_per_step"], "d2h_bytes_per_step": e["d2h_bytes_per_step"],
           "step": f"one call = prompt {wl.P} ids in, chunked prefill ({wl.eng.prefill_rows} positions per "
                   f"chunk) + {wl.T} greedy tokens, ids out",
           "ms_per_call": round(e2e_ms, 3)}
    clocks = clk.summary()
    launches = args.steps * wl.eng.kernels_per_step()
    if dist.rank != 0:
        wl.eng.close()
        dist.close()
        return
    cpu = CpuDecode(args.model, wl.B).measure() if dist.world == 1 else None
    line = {"metric": wl.metric, "value": round(value, 2), "unit": "tokens/s", "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": f"int{wl.spec.bits} weights x fp16, fp32 acc",
            "data": "synthetic (random-init weights, uniform random prompt ids)",
            "config": {"workload": f"decode {MODELS[args.model]['name']} INT{wl.spec.bits} G{GROUP}",
                       "model": MODELS[args.model]["name"], "global_batch": wl.B, "prompt": wl.P,
                       "new_tokens": wl.T, "seq_len": wl.P + wl.T, "parallelism": f"tp{dist.world}",
                       "dequant": "per-chunk fp32 scale" if args.fold else "exact fp16(code*scale)",
                       "all_reduce": ("none" if dist.world == 1 else
                                      "in-kernel peer-memory exchange over NVLink" if args.exchange == "peer"
                                      else "NCCL all_reduce in the step graph"),
                       "l2": f"inputs larger than L2 ({wl.spec.weight_bytes_per_token() / dist.world / 1e9:.2f} GB "
                             "of weights per GPU per step)"},
            "roofline": roofline, "decode_roofline": decode_roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": int(launches), "kernels": {k: {kk: v[kk] for kk in ("launches", "us", "GB/s")}
                                                       for k, v in kstats.items()},
            "clocks": clocks}
    print(json.dumps(line), flush=True)
    wl.eng.close()
    dist.close()


def run_reference_decode(args, dist: Dist):
    """The reference's CPU path on the box's cores: every step is one of the 7
    quantized linears of a layer (rotating), dequantized and matmul'd as the
    reference does; tokens/s = batch / (layers x summed linear times + lm_head)."""
    if dist.rank != 0:
        return
    cpu = CpuDecode(args.model, args.batch)
    for i in range(min(args.warmup, 7)):
        cpu.linear(i % 7)
    times = [[] for _ in range(7)]
    t0 = time.perf_counter()
    for it in range(args.steps):
        times[it % 7].append(cpu.linear(it % 7))
    wall = time.perf_counter() - t0
    layer = sum(sum(t) / len(t) for t in times if t) * (7 / max(1, sum(1 for t in times if t)))
    lm = cpu.lm_head_seconds()
    tok_s = args.batch / (cpu.spec.n_layers * layer + lm)
    cfg = MODELS[args.model]
    line = {"impl": "reference", "metric": (f"decode tokens/s ({cfg['name']} INT{cfg['bits']} G{GROUP} weight-only, "
                                            f"batch {args.batch}, prompt {cfg['prompt']}, greedy, TP{args.gpus})"),
            "value": round(tok_s, 5), "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": f"int{cfg['bits']} codes, fp32 acc",
            "data": "synthetic",
            "config": {"workload": f"decode {cfg['name']} INT{cfg['bits']} G{GROUP}", "global_batch": args.batch},
            "cpu_baseline": {"value": round(tok_s, 5), "unit": "tokens/s", "cores": cpu.cores, "kind": "port",
                             "sample": f"{args.steps} linears (rotating over a layer's 7) + fp16 lm_head sample, "
                                       f"extrapolated to {cpu.spec.n_layers} layers"},
            "e2e": {"value": round(tok_s, 5), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "gemv"], default="decode")
    ap.add_argument("--model", choices=sorted(MODELS), default="8b")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--fold", action="store_true",
                    help="decode GEMVs scale each chunk sum in fp32 instead of dequantizing exactly")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="tensor-parallel all-reduce: in-kernel through peer memory, or NCCL between kernels")
    ap.add_argument("--prompt", type=int, default=None, help="prompt length (profiling runs; default: the config's)")
    ap.add_argument("--new", type=int, default=None, help="new tokens of the e2e call (profiling runs)")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder layers (small profiling cases only: the line is then not the config's number)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 200 if args.impl == "ours" else 21
    if args.warmup is None:
        args.warmup = 10 if args.impl == "ours" else 3
    args.warmup = max(args.warmup, 3)
    dist = Dist()
    if args.workload == "decode":
        (run_reference_decode if args.impl == "reference" else run_decode)(args, dist)
    else:
        (run_reference_gemv if args.impl == "reference" else run_gemv)(args, dist)


if __name__ == "__main__":
    main()
