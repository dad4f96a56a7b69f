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

The default decode line also carries (one GPU) a ``gemv`` object with the
same M = 1 figures, the single-QuantLinear W8A16 case (K = 2048, N = 8192,
per-output-channel scales, M = 1 and 16), the 8B gate|up shape and the
GB/s-vs-M sweep, and a ``parity`` object: the greedy ids of the timed
configuration and the first decode steps' logits checked against a
teacher-forced fp32 torch restatement of the same packed weights.

``--impl reference`` times the reference's CPU path for the same workload
(dequantize the packed weights, fp32 matmul, fp16 result - restated with
torch tensor ops by oracle/torch_cpu.py) on the host cores, rank 0 only.
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
CONFIG1 = (8, 2048, 8192, 2048)   # bits, K, N, G: one W8A16 QuantLinear with per-output-channel scales
GATE_UP_8B = (4, 4096, 28672, 128)
L2_BYTES = 126 * 1024 * 1024


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running.
    Entering waits (up to 3 s) for the first sample, so a short timed region
    still has samples from its start; leaving waits one interval more."""

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
            import shutil
            line_buffered = ["stdbuf", "-oL"] if shutil.which("stdbuf") else []   # a line per sample, as taken
            self.proc = subprocess.Popen(
                line_buffered + ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.out, stderr=subprocess.DEVNULL)
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < 3.0 and self.proc.poll() is None:
                if os.path.getsize(self.out.name) > 0:
                    break
                time.sleep(0.01)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.06)   # one more sample after the region
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
            dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=300))
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

def gemv_bytes(M: int, K: int, N: int, bits: int, group: int = GROUP) -> int:
    from liteweight_b200.perf import quant_matmul_workload
    return quant_matmul_workload(M, K, N, bits, group).bytes_moved


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

    def __init__(self, device, seed: int = 0, extras: bool = True):
        import torch
        from liteweight_b200 import _native as nat
        self.torch, self.nat, self.dev = torch, nat, device
        self.M = 1
        gen = torch.Generator(device=device).manual_seed(seed)
        # (bits, K, N, G): the step's 8 GEMVs, then the extra cases timed beside it
        self.items = [(bits, K, N, GROUP) for bits in (4, 8) for K, N in GEMV_SHAPES]
        self.n_step = len(self.items)
        if extras:
            self.items += [CONFIG1, GATE_UP_8B]
        step_w = sum(N * K * b // 8 for b, K, N, _ in self.items[:self.n_step])
        # weight copies of the step's GEMVs: one rotation is more than twice the L2
        self.R = max(3, -(-2 * L2_BYTES // step_w))
        self.weights = []   # [item][copy] -> (q, s)
        for i, (bits, K, N, G) in enumerate(self.items):
            per = []
            for r in range(self.copies_for(i)):
                if bits == 4:
                    q = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=device, generator=gen)
                else:
                    q = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=device, generator=gen)
                s = (torch.rand(N, K // G, device=device, generator=gen) * 2e-3 + 1e-4).half()
                per.append((q, s))
            self.weights.append(per)
        self.acts = {K: torch.randn(256, K, dtype=torch.float16, device=device, generator=gen)
                     for K in {it[1] for it in self.items}}
        self.outs = {N: torch.empty(256, N, dtype=torch.float16, device=device)
                     for N in {it[2] for it in self.items}}
        self.bytes_per_step = sum(gemv_bytes(self.M, K, N, b, G) for b, K, N, G in self.items[:self.n_step])
        n0 = nat.launch_count()
        self.step_graphs = [capture_graph(lambda r=r: self._step(r)) for r in range(self.R)]
        # capture_graph runs fn twice (eager warm-up + capture): launches of one step
        self.launches_per_step = (nat.launch_count() - n0) // (2 * self.R)

    def copies_for(self, i: int) -> int:
        """Weight copies of item i: the step's GEMVs rotate together (R copies,
        more than twice the L2 per rotation); an extra case alone needs more
        than twice the L2 of its own copies."""
        if i < self.n_step:
            return self.R
        bits, K, N, _ = self.items[i]
        return max(2, -(-2 * L2_BYTES // (N * K * bits // 8)))

    def _call(self, i: int, copy: int, M: int):
        bits, K, N, G = self.items[i]
        q, s = self.weights[i][copy]
        act, out = self.acts[K], self.outs[N]
        stream = self.torch.cuda.current_stream().cuda_stream
        ws, ws_bytes = self.nat.matmul_workspace(bits, M, N, K, self.dev, stream)
        fn = "lw_gemm_w4a16" if bits == 4 else "lw_gemm_w8a16"
        self.nat.call(fn, act.data_ptr(), q.data_ptr(), s.data_ptr(), None, out.data_ptr(), M, N, K, G,
                      ws, ws_bytes, stream)

    def _step(self, copy: int):
        for i in range(self.n_step):
            self._call(i, copy, self.M)

    def step(self, it: int):
        self.step_graphs[it % self.R].replay()

    def time_item(self, i: int, M: int, reps: int = 20) -> float:
        """ms of one launch of item i at M rows: a graph of back-to-back launches
        over the rotating weight copies (more than twice the L2), CUDA events
        around its replays."""
        n = self.copies_for(i)
        g = capture_graph(lambda: [self._call(i, r, M) for r in range(n)])
        ms = time_graph(g, reps) / n
        del g
        return ms

    def kernel_stats(self) -> dict:
        """Per kernel family: algorithmic bytes and device time of its launches in
        one step (time_item per launch)."""
        fam = {}
        for i, (bits, K, N, G) in enumerate(self.items[:self.n_step]):
            ms = self.time_item(i, self.M)
            d = fam.setdefault(f"gemv_w{bits}a16", {"bytes": 0, "ms": 0.0, "launches": 0, "shapes": {}})
            b = gemv_bytes(self.M, K, N, bits, G)
            d["bytes"] += b
            d["ms"] += ms
            d["launches"] += 1
            d["shapes"][f"{K}x{N}"] = {"us": round(ms * 1e3, 3), "GB/s": round(b / (ms * 1e-3) / 1e9, 1)}
        return fam

    def extra_stats(self, peak_gbs: float, peak_tflops: float | None = None) -> dict:
        """The single W8A16 QuantLinear with per-output-channel scales (K=2048,
        N=8192; M = 1 and 16) and the 8B gate|up shape (INT4, K=4096, N=28672;
        M = 1, and M = 256 - the tcgen05 route of the drop-in op - in TFLOP/s
        against the measured bf16 burst peak)."""
        out = {}
        for i in range(self.n_step, len(self.items)):
            bits, K, N, G = self.items[i]
            name = (f"config1_w8a16_perchannel_K{K}_N{N}" if (bits, K, N, G) == CONFIG1
                    else f"w4a16_gate_up_8b_K{K}_N{N}_G{G}")
            for M in ((1, 16) if (bits, K, N, G) == CONFIG1 else (1, 256)):
                ms = self.time_item(i, M)
                gbs = gemv_bytes(M, K, N, bits, G) / (ms * 1e-3) / 1e9
                point = {"us": round(ms * 1e3, 3), "GB/s": round(gbs, 1), "frac": round(gbs / peak_gbs, 4)}
                if M > 32 and peak_tflops:
                    tf = 2 * M * N * K / (ms * 1e-3) / 1e12
                    point.update({"TFLOP/s": round(tf, 1), "tensor_frac": round(tf / peak_tflops, 4)})
                out.setdefault(name, {})[f"M{M}"] = point
        return out

    def e2e(self, steps: int) -> dict:
        """Same GEMVs through the public drop-in ops with host buffers: pinned
        activation copied in and the result copied out every call."""
        torch = self.torch
        from liteweight_b200 import kernels
        host_act = {K: a[:self.M].cpu().pin_memory() for K, a in self.acts.items()}
        host_out = [torch.empty(self.M, N, dtype=torch.float16).pin_memory() for _, _, N, _ in self.items]
        h2d = sum(self.M * K * 2 for _, K, _, _ in self.items[:self.n_step])
        d2h = sum(self.M * N * 2 for _, _, N, _ in self.items[:self.n_step])

        def one(it):
            copy = it % self.R
            for i, (bits, K, N, G) in enumerate(self.items[:self.n_step]):
                a = host_act[K].to(self.dev, non_blocking=True)
                q, s = self.weights[i][copy]
                fn = kernels.matmul_int4 if bits == 4 else kernels.matmul_int8
                host_out[i].copy_(fn(a, q, s, G), non_blocking=True)

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
            idx = [self.items.index((bits, K, N, GROUP)) for K, N in GEMV_SHAPES]
            for M in (1, 2, 4, 8, 16, 32, 64, 128, 256):
                g = capture_graph(lambda: [self._call(i, r, M) for r in range(self.R) for i in idx])
                ms = time_graph(g, 5) / self.R
                del g
                tot_b = sum(gemv_bytes(M, K, N, bits) for K, N in GEMV_SHAPES)
                out[f"w{bits}_M{M}"] = round(tot_b / (ms * 1e-3) / 1e9, 1)
        return out

    def summary(self, peak_gbs: float, sweep: bool = True, peak_tflops: float | None = None) -> dict:
        """The GEMV half of the headline metric, for the default line."""
        fam = self.kernel_stats()
        m1 = {}
        for k, v in fam.items():
            gbs = v["bytes"] / (v["ms"] * 1e-3) / 1e9
            m1[k] = {"GB/s": round(gbs, 1), "frac": round(gbs / peak_gbs, 4), "shapes": v["shapes"]}
        out = {"M1_llama_3_2_1b_shapes_G128": m1, **self.extra_stats(peak_gbs, peak_tflops),
               "timing": "graph of back-to-back launches over rotating weight copies > 2x L2, CUDA events",
               "peak_gbs": peak_gbs}
        if sweep:
            out["gbs_vs_m"] = self.sweep()
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
                 layers: int | None = None, lm_head_bits: int = 16):
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
        self.lm_bits = lm_head_bits
        self.metric = decode_metric(model, batch, self.P, self.tp, lm_head_bits)
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
        self.embed, self.norm, self.cos, self.sin = embed, norm, cos, sin
        # the lm_head is the tied embedding: fp16 as liteweight keeps it, or quantized
        # like swap_linears does when the head is not skipped
        self.lm_quant = None
        if lm_head_bits != 16:
            from liteweight_b200.quantize import quantize_int4, quantize_int8
            q, sc = (quantize_int4 if lm_head_bits == 4 else quantize_int8)(embed, GROUP)
            self.lm_quant = (q, sc, lm_head_bits, GROUP)
        group = None
        if self.tp > 1:
            import torch.distributed as tdist
            group = tdist.group.WORLD
        self.packed, self.max_seq, self.group, self.fold, self.exchange = packed, max_seq, group, fold, exchange
        self.eng = E.DecodeEngine(spec, packed, embed, norm, None, cos, sin, batch, max_seq, device, self.rank,
                                  self.tp, group, fold_scales=fold, exchange=exchange, lm_head_quant=self.lm_quant)
        gp = torch.Generator().manual_seed(7)
        self.prompt = torch.randint(0, spec.vocab, (batch, self.P), generator=gp)
        torch.cuda.synchronize()

    def side_engine(self, batch: int, layers: int | None = None, exchange: str | None = None):
        """Another engine over the same packed layers (the first `layers` of
        them), embedding, norm and head: a batch point or the shallow check."""
        E = self.E
        exchange = self.exchange if exchange is None else exchange
        spec = self.spec if layers is None else E.LlamaSpec(**{**self.spec.__dict__, "n_layers": layers})
        packed = self.packed if layers is None else self.packed[:layers]
        return E.DecodeEngine(spec, packed, self.embed, self.norm, None, self.cos, self.sin, batch, self.max_seq,
                              self.dev, self.rank, self.tp, self.group, fold_scales=self.fold,
                              exchange=exchange, lm_head_quant=self.lm_quant)

    def layer_weights(self, li: int):
        """Layer li's unsharded weights, regenerated from its seed (the same
        tensors every rank sharded when the engine was built)."""
        E = self.E
        return E.synthetic_layers(E.LlamaSpec(**{**self.spec.__dict__, "n_layers": 1}), self.dev, seed=1000 + li)[0]

    def teacher_forced_logits(self, ids, steps: int, eng=None, prompt=None):
        """The engine's logits [steps, B, V/TP] (this rank's vocabulary shard)
        of decode steps 1..steps with the given generated ids forced: step j
        predicts ids[:, j]."""
        torch = self.torch
        eng = self.eng if eng is None else eng
        eng.start(self.prompt if prompt is None else prompt, forced=ids)
        eng.prefill()
        eng.capture()
        out = []
        for _ in range(steps):
            eng.step(1)
            out.append(eng.logits.float().clone())
        torch.cuda.synchronize()
        eng.check()
        return torch.stack(out, 0)

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
        return (sp.weight_bytes_per_token(lm_head_bits=self.lm_bits) // self.tp
                + self.B * sp.kv_bytes_per_position() * ctx // self.tp)

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
            "lm_head": ((sp.vocab // self.tp) * H * 2 if self.lm_bits == 16 else
                        wbytes(sp.vocab // self.tp, H) * self.lm_bits // sp.bits) + 2 * self.B * H,
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


class TorchDecodeReference:
    """Checker of the decode line's parity (never timed): a teacher-forced
    torch computation, on the device, of the same packed weights through the
    reference's arithmetic - every QuantLinear dequantizes exactly
    (liteweight/quantize.py:30-43, :102-128) and multiplies in fp32 with an
    fp16 result (:60) - and of the HF Llama layers around them as the fp16 HF
    model computes them on a GPU (transformers 5.5.0 modeling_llama.py:
    RMSNorm with rsqrt :63-68, RoPE :138-167, SwiGLU :171-184, fp16 residual
    adds :320-335, and attention through torch's scaled_dot_product_attention
    on fp16 tensors, the "sdpa" implementation HF selects by default)."""

    def __init__(self, wl: DecodeWorkload, split_k: int = 1, layers: int | None = None):
        # split_k > 1: every fp32 matmul sums K in that many slices (another,
        # equally valid, accumulation order: the spread it causes is the noise
        # floor any implementation faces at this depth)
        self.wl, self.torch, self.split_k = wl, wl.torch, split_k
        self.layers = wl.spec.n_layers if layers is None else layers   # the first `layers` layers only

    def _dequant(self, q, s, bits, G):
        torch = self.torch
        n = q.shape[0]
        if bits == 4:
            b = q.view(torch.int8)
            codes = torch.stack(((b << 4) >> 4, b >> 4), dim=-1).view(n, -1)
        else:
            codes = q
        k = codes.shape[1]
        w = codes.float().view(n, k // G, G) * s.float().unsqueeze(-1)
        return w.view(n, k).half().float()

    def _lin(self, x16, pair, bits, G):
        q, s = pair
        w = self._dequant(q, s, bits, G)
        if self.split_k == 1:
            return (x16.float() @ w.t()).half()
        xs, ws = x16.float().chunk(self.split_k, dim=-1), w.chunk(self.split_k, dim=-1)
        acc = xs[0] @ ws[0].t()
        for xa, wa in zip(xs[1:], ws[1:]):
            acc = acc + xa @ wa.t()
        return acc.half()

    @staticmethod
    def _rmsnorm(x16, w, eps):
        import torch
        xf = x16.float()
        var = xf.pow(2).mean(-1, keepdim=True)
        return (w * (xf * torch.rsqrt(var + eps)).half())

    @staticmethod
    def _rope(x16, cos, sin):
        h = x16.shape[-1] // 2
        rot = x16.new_empty(x16.shape)
        rot[..., :h] = -x16[..., h:]
        rot[..., h:] = x16[..., :h]
        return ((x16.float() * cos.float()).half().float() + (rot.float() * sin.float()).half().float()).half()

    def logits(self, tokens, first: int, count: int):
        """fp32 logits [B, count, V] at positions first .. first+count-1 of the
        int64 token rows [B, T] (each position sees tokens[:, :pos+1])."""
        torch, wl = self.torch, self.wl
        sp, dev = wl.spec, wl.dev
        hd, nh, nkv = sp.head_dim, sp.n_heads, sp.n_kv_heads
        B, T = tokens.shape
        prev_tf32 = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            x = wl.embed[tokens.to(dev)].half()                               # [B, T, H]
            cos, sin = wl.cos[:T][:, None, :], wl.sin[:T][:, None, :]         # [T, 1, hd]
            for li in range(self.layers):
                L = wl.layer_weights(li)
                for b in range(B):
                    xb = x[b]
                    h = self._rmsnorm(xb, L.in_norm, sp.eps)
                    q = self._rope(self._lin(h, L.q, sp.bits, sp.group_size).view(T, nh, hd), cos, sin)
                    k = self._rope(self._lin(h, L.k, sp.bits, sp.group_size).view(T, nkv, hd), cos, sin)
                    v = self._lin(h, L.v, sp.bits, sp.group_size).view(T, nkv, hd)
                    rep = nh // nkv
                    kx = k.repeat_interleave(rep, dim=1).transpose(0, 1)          # repeat_kv: [nh, T, hd]
                    vx = v.repeat_interleave(rep, dim=1).transpose(0, 1)
                    a = torch.nn.functional.scaled_dot_product_attention(
                        q.transpose(0, 1)[None], kx[None], vx[None], is_causal=True, scale=hd ** -0.5)
                    a = a[0].transpose(0, 1).reshape(T, nh * hd)
                    del kx, vx
                    xb = (xb.float() + self._lin(a, L.o, sp.bits, sp.group_size).float()).half()
                    h = self._rmsnorm(xb, L.post_norm, sp.eps)
                    g = self._lin(h, L.gate, sp.bits, sp.group_size).float()
                    u = self._lin(h, L.up, sp.bits, sp.group_size).float()
                    act = ((g / (1.0 + torch.exp(-g))).half().float() * u).half()
                    x[b] = (xb.float() + self._lin(act, L.down, sp.bits, sp.group_size).float()).half()
                del L
            h = self._rmsnorm(x[:, first:first + count], wl.norm, sp.eps)      # [B, count, H]
            if wl.lm_quant is not None:
                q, sc, bits, grp = wl.lm_quant
                head = self._dequant(q, sc, bits, grp)
            else:
                head = wl.embed.float()
            return h.float() @ head.t()
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev_tf32


def decode_parity(wl: DecodeWorkload, ids_host, rank: int, steps: int = 32) -> dict | None:
    """Greedy match rate of the timed configuration's generated ids and the
    max err / row tolerance of the first `steps` decode steps' logits, both
    against TorchDecodeReference (rank 0 computes it; every rank runs the
    engine's teacher-forced pass, a collective under tensor parallelism)."""
    torch = wl.torch
    steps = max(1, min(steps, wl.T - 1))
    ids = ids_host.to(torch.int64)
    got = wl.teacher_forced_logits(ids, steps)                      # [steps, B, Vs]
    if rank != 0:
        return None
    toks = torch.cat([wl.prompt.to(torch.int64), ids], dim=1)        # [B, P + T]
    P, T = wl.P, wl.T
    ref = TorchDecodeReference(wl)
    # positions P-1 .. P+T-2 predict ids[:, 0 .. T-1]; only T-1 of them need the full model
    lg = ref.logits(toks[:, :P + T - 1], P - 1, T)                   # [B, T, V]
    ref_ids = lg.argmax(-1).cpu()
    match = float((ref_ids == ids).float().mean())
    miss = (ref_ids != ids).nonzero()
    first_mismatch = int(miss[:, 1].min()) if miss.numel() else None
    vs = got.shape[-1]
    r = lg[:, 1:1 + steps].transpose(0, 1)                           # [steps, B, V]
    tol = 1e-2 * r.double().pow(2).sum(-1, keepdim=True).sqrt() / (r.shape[-1] ** 0.5)
    err = (got.double() - r[..., :vs].double()).abs()
    ratio = float((err / tol).max())
    # the same reference with every matmul summed in two K halves: the spread
    # between two valid fp32 accumulation orders through the whole depth
    alt = TorchDecodeReference(wl, split_k=2).logits(toks[:, :P + steps], P, steps).transpose(0, 1)
    floor = float(((alt.double() - r.double()).abs() / tol).max())
    del alt
    return {"match_rate": round(match, 4), "tokens_compared": int(ids.numel()),
            "first_mismatch_step": first_mismatch, "logits_err_over_tol": round(ratio, 4),
            "reference_vs_itself_err_over_tol": round(floor, 4),
            "reference_vs_itself_note": "the reference with each fp32 matmul summed in two K halves vs as one "
                                        "sum, same steps: the accumulation-order noise floor at this depth",
            "logits_steps_compared": steps, "logits_columns": f"vocab shard 0 of {wl.tp} ({vs} of {r.shape[-1]})",
            "tolerance": "max-abs err <= 1e-2 * ||ref row||_2 / sqrt(V), per (step, sequence)",
            "reference": "teacher-forced torch on the device: the same packed weights dequantized exactly with fp32 "
                         "matmuls, the HF fp16 Llama layers with sdpa attention, full depth"}


def shallow_parity(wl: DecodeWorkload, dist: "Dist", layers: int = 2, steps: int = 16) -> dict | None:
    """The decode line's logits check where fp32 summation order cannot
    dominate: an engine over the first `layers` layers of the same packed
    model (same embedding and head), greedy tokens from its own run,
    teacher-forced logits of `steps` steps against TorchDecodeReference over
    the same layers."""
    torch = wl.torch
    eng = wl.side_engine(wl.B, layers=layers)
    ids = eng.generate(wl.prompt, steps + 1).to(torch.int64)
    got = wl.teacher_forced_logits(ids, steps, eng=eng)
    eng.close()
    del eng
    if dist.rank != 0:
        return None
    toks = torch.cat([wl.prompt.to(torch.int64), ids], dim=1)
    r = TorchDecodeReference(wl, layers=layers).logits(toks[:, :wl.P + steps], wl.P, steps).transpose(0, 1)
    tol = 1e-2 * r.double().pow(2).sum(-1, keepdim=True).sqrt() / (r.shape[-1] ** 0.5)
    vs = got.shape[-1]
    ratio = float(((got.double() - r[..., :vs].double()).abs() / tol).max())
    return {"layers": layers, "logits_steps_compared": steps, "logits_err_over_tol": round(ratio, 4)}


def batch_sweep(wl: DecodeWorkload, dist: "Dist", batches, warmup: int, steps: int, peak_gbs: float,
                parity_seqs: int = 4, parity_tokens: int = 16) -> list:
    """The same model at other batch sizes (an engine per batch over the same
    packed weights): tokens/s of the whole job (max over ranks), the step's
    roofline fraction, and the greedy match of the first `parity_seqs`
    sequences' first `parity_tokens` generated tokens against the
    teacher-forced TorchDecodeReference."""
    torch, dev = wl.torch, wl.dev
    out = []
    for B in batches:
        # the peer exchange takes batches one launch stages whole; larger ones
        # run in row blocks with NCCL all-reduces between the kernels
        xchg = wl.exchange
        if wl.tp > 1 and xchg == "peer" and B > wl.E.peer_batch_limit(wl.spec, wl.tp, wl.lm_bits):
            xchg = "nccl"
        eng = wl.side_engine(B, exchange=xchg)
        prompt = torch.randint(0, wl.spec.vocab, (B, wl.P), generator=torch.Generator().manual_seed(100 + B))
        eng.start(prompt)
        eng.prefill()
        eng.capture()
        for _ in range(warmup):
            eng.step(1)
        torch.cuda.synchronize()
        dist.barrier(dev)
        torch.cuda.synchronize()
        ctx0 = eng.host_pos + 1
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            eng.step(1)
        e1.record()
        torch.cuda.synchronize()
        dist.barrier(dev)
        eng.check()
        ms = dist.max(e0.elapsed_time(e1), dev)
        n = min(parity_tokens, warmup + steps)
        ids = eng.generated(n + 1).to("cpu", torch.int64)[:parity_seqs]
        # per class of the step: its launches alone in a graph, CUDA events
        kus = {}
        for name in dict.fromkeys(nm for kind, _a, nm in eng.calls if kind in ("gemv", "attn", "tcgemm")):
            launches = sum(1 for kind, _a, nm in eng.calls if nm == name and kind in ("gemv", "attn", "tcgemm"))
            g = capture_graph(lambda name=name: eng.enqueue_only(name))
            kus[name] = {"launches": launches, "us": round(time_graph(g, 5) / launches * 1e3, 2),
                         "path": "tcgemm" if any(kind == "tcgemm" and nm == name for kind, _a, nm in eng.calls)
                         else "gemv" if name != "attn" else "attention"}
            del g
        eng.close()
        del eng
        step_ms = ms / steps
        bstep = (wl.spec.weight_bytes_per_token(lm_head_bits=wl.lm_bits) // wl.tp
                 + B * wl.spec.kv_bytes_per_position() * (ctx0 + steps // 2) // wl.tp)
        point = {"batch": B, "tokens_per_s": round(B * steps / (ms * 1e-3), 1), "ms_per_step": round(step_ms, 4),
                 "decode_roofline_frac": round(bstep / (step_ms * 1e-3) / 1e9 / peak_gbs, 4), "kernels": kus}
        if wl.tp > 1:
            point["all_reduce"] = "in-kernel peer exchange" if xchg == "peer" else "NCCL in the step graph"
        if dist.rank == 0 and parity_seqs > 0:
            toks = torch.cat([prompt[:parity_seqs].to(torch.int64), ids], dim=1)
            lg = TorchDecodeReference(wl).logits(toks[:, :wl.P + n], wl.P - 1, n + 1)
            ref_ids = lg.argmax(-1).cpu()
            point["match_rate"] = round(float((ref_ids == ids).float().mean()), 4)
            point["match_compared"] = f"first {n + 1} tokens of sequences 0..{parity_seqs - 1}"
            del lg
        out.append(point)
        torch.cuda.empty_cache()
    return out


def decode_config(model: str, batch: int, prompt: int, new: int, world: int, fold: bool, exchange: str,
                  lm_head_bits: int = 16) -> dict:
    """The `config` object of a decode line (both arms print the same one)."""
    cfg = MODELS[model]
    from liteweight_b200 import engine as E
    spec = E.LlamaSpec(**getattr(E, cfg["arch"]), bits=cfg["bits"], group_size=GROUP)
    return {"workload": f"decode {cfg['name']} INT{cfg['bits']} G{GROUP}", "model": cfg["name"],
            "lm_head": ("fp16 (liteweight skips it)" if lm_head_bits == 16
                        else f"INT{lm_head_bits} G{GROUP} (swap_linears without the skip)"),
            "global_batch": batch, "prompt": prompt, "new_tokens": new, "seq_len": prompt + new,
            "parallelism": f"tp{world}",
            "dequant": "per-chunk fp32 scale" if fold else "exact fp16(code*scale)",
            "all_reduce": ("none" if world == 1 else
                           "in-kernel peer-memory exchange over NVLink" if exchange == "peer"
                           else "NCCL all_reduce in the step graph"),
            "l2": f"inputs larger than L2 ({spec.weight_bytes_per_token(lm_head_bits=lm_head_bits) / world / 1e9:.2f}"
                  " GB of weights per GPU per step)"}


def decode_metric(model: str, batch: int, prompt: int, world: int, lm_head_bits: int = 16) -> str:
    cfg = MODELS[model]
    head = "" if lm_head_bits == 16 else f", INT{lm_head_bits} lm_head"
    return (f"decode tokens/s ({cfg['name']} INT{cfg['bits']} G{GROUP} weight-only{head}, batch {batch}, "
            f"prompt {prompt}, greedy, TP{world})")


class CpuDecode:
    """The reference's CPU path for one decode token: every quantized linear
    of every layer dequantized and fp32-multiplied as liteweight's oracle does
    (liteweight/quantize.py:30-60, :102-135; restated with torch ops by
    oracle/torch_cpu.py), plus the fp16 lm_head through the same fp32 matmul,
    at the configuration's batch; one BLAS call per linear over all host
    threads (torch.set_num_threads(os.cpu_count())). Norms, RoPE and attention
    at this batch are <1% of the arithmetic and left out. Weight codes are
    random bytes (the work does not depend on the values); `distinct` layer
    sets are cycled through the L layer positions."""

    def __init__(self, model: str, batch: int = 1, distinct: int = 4, lm_head_bits: int = 16):
        import torch
        from liteweight_b200 import engine as E
        from oracle import torch_cpu
        self.torch, self.tc = torch, torch_cpu
        self.lm_bits = lm_head_bits
        self.cores = os.cpu_count() or 1
        torch.set_num_threads(self.cores)
        cfg = MODELS[model]
        self.spec = E.LlamaSpec(**getattr(E, cfg["arch"]), bits=cfg["bits"], group_size=GROUP)
        self.B = batch
        g = torch.Generator().manual_seed(3)
        sp = self.spec

        def rows(n, make):   # n rows: a random 1024-row block repeated (generating all of them is slow)
            blk = make(min(n, 1024))
            return blk.repeat(-(-n // blk.shape[0]), 1)[:n].contiguous()
        self.layers = []
        for _ in range(min(distinct, sp.n_layers)):
            lin = []
            for _name, n, k in sp.linear_shapes():
                if sp.bits == 4:
                    q = rows(n, lambda r: torch.randint(0, 256, (r, k // 2), dtype=torch.uint8, generator=g))
                else:
                    q = rows(n, lambda r: torch.randint(-127, 128, (r, k), dtype=torch.int8, generator=g))
                s = rows(n, lambda r: (torch.rand(r, k // GROUP, generator=g) * 2e-3 + 1e-4).half())
                lin.append((q, s, k))
            self.layers.append(lin)
        self.acts = {k: torch.randn(batch, k, generator=g).half() for _n, _o, k in sp.linear_shapes()}
        self.lm = rows(sp.vocab, lambda r: (torch.rand(r, sp.hidden, generator=g) * 0.04 - 0.02).half())
        if lm_head_bits != 16:   # a quantized head runs as one more QuantLinear
            self.lm = rows(sp.vocab, lambda r: torch.randint(0, 256, (r, sp.hidden * lm_head_bits // 8),
                                                             dtype=torch.uint8, generator=g)
                           if lm_head_bits == 4 else
                           torch.randint(-127, 128, (r, sp.hidden), dtype=torch.int8, generator=g))
            self.lm_s = rows(sp.vocab, lambda r: (torch.rand(r, sp.hidden // GROUP, generator=g) * 2e-3).half())
        self.h = torch.randn(batch, sp.hidden, generator=g).half()

    def layer(self, li: int) -> float:
        t = time.perf_counter()
        for q, s, k in self.layers[li % len(self.layers)]:
            self.tc.quant_linear(self.acts[k], q, s, GROUP, self.spec.bits)
        return time.perf_counter() - t

    def lm_head(self) -> float:
        t = time.perf_counter()
        if self.lm_bits == 16:
            self.tc.fp16_linear(self.h, self.lm)
        else:
            self.tc.quant_linear(self.h, self.lm, self.lm_s, GROUP, self.lm_bits)
        return time.perf_counter() - t

    def token(self, budget_s: float = 90.0) -> dict:
        """One whole token (all L layers + lm_head) unless that would take more
        than budget_s: then the layers timed so far are extrapolated to L."""
        L = self.spec.n_layers
        t0 = time.perf_counter()
        times = []
        for li in range(L):
            times.append(self.layer(li))
            if time.perf_counter() - t0 > budget_s:
                break
        lm = self.lm_head()
        head = "fp16" if self.lm_bits == 16 else f"INT{self.lm_bits}"
        layer_mean = sum(times) / len(times)
        tok_s = self.B / (layer_mean * L + lm)
        whole = len(times) == L
        return {"value": round(tok_s, 5), "unit": "tokens/s", "cores": self.cores, "kind": "port",
                "seconds_per_token": round(layer_mean * L + lm, 3), "layer_seconds": round(layer_mean, 4),
                "lm_head_seconds": round(lm, 4),
                "sample": (f"one whole token: {L} layers x 7 quantized linears + the {head} lm_head; "
                           if whole else f"{len(times)} of {L} layers (x 7 linears) + the {head} lm_head, "
                                         f"extrapolated to {L} layers; ")
                          + f"batch {self.B}, torch dequantize + fp32 matmul (oracle/torch_cpu.py), "
                            f"torch.set_num_threads({self.cores})"}


class CpuGemv:
    """The reference's CPU path for the GEMV step: the 8 M=1 QuantLinear calls
    of the 1B shapes, dequantized and fp32-multiplied with torch ops
    (oracle/torch_cpu.py) over all host threads."""

    def __init__(self, seed: int = 0):
        import torch
        from oracle import torch_cpu
        self.torch, self.tc = torch, torch_cpu
        self.cores = os.cpu_count() or 1
        torch.set_num_threads(self.cores)
        g = torch.Generator().manual_seed(seed)
        self.items = []
        for bits in (4, 8):
            for K, N in GEMV_SHAPES:
                if bits == 4:
                    q = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g)
                else:
                    q = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=g)
                s = (torch.rand(N, K // GROUP, generator=g) * 2e-3 + 1e-4).half()
                act = torch.randn(1, K, generator=g).half()
                self.items.append((bits, K, N, q, s, act))
        self.bytes_per_step = sum(gemv_bytes(1, K, N, b) for b, K, N, *_ in self.items)

    def step(self):
        for bits, K, N, q, s, act in self.items:
            self.tc.quant_linear(act, q, s, GROUP, bits)

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
                "sample": f"{n} passes over the 8 M=1 GEMVs (INT4+INT8, 1B shapes), torch dequantize + fp32 "
                          f"matmul (oracle/torch_cpu.py), torch.set_num_threads({self.cores})"}


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


def gemv_config(world: int) -> dict:
    return {"workload": "gemv M=1 Llama-3.2-1B shapes (KxN 2048x2048, 2048x512, 2048x8192, 8192x2048) INT4+INT8 G128",
            "parallelism": f"replicas x{world}",
            "l2": "rotating weight copies, more than twice the L2 per rotation"}


def run_reference_gemv(args, dist: Dist):
    if dist.rank != 0:
        return
    cpu = CpuGemv()
    for _ in range(min(args.warmup, 3)):
        cpu.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu.step()
    dt = (time.perf_counter() - t0) / args.steps
    value = cpu.bytes_per_step / dt / 1e9
    line = {"impl": "reference", "metric": GemvWorkload.metric, "value": round(value, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8/int8 codes, fp32 acc",
            "data": "synthetic", "config": gemv_config(args.gpus),
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cpu.cores, "kind": "port",
                             "sample": "every step = the 8 M=1 GEMVs, torch dequantize + fp32 matmul "
                                       f"(oracle/torch_cpu.py), torch.set_num_threads({cpu.cores})"},
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
    wl = GemvWorkload(dev, seed=1234 + dist.rank, extras=False)
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
            "config": {**gemv_config(dist.world),
                       "l2": f"rotating {wl.R} weight copies "
                             f"({wl.R * sum(N * K * b // 8 for b, K, N, _ in wl.items[:wl.n_step]) >> 20} MiB) > L2"},
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
                        exchange=args.exchange, prompt=args.prompt, new=args.new, layers=args.layers,
                        lm_head_bits=args.lm_head_bits)
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
        torch.cuda.nvtx.range_push("decode_timed")   # the profiling recipes filter on this range
        e0.record()
        for it in range(args.steps):
            wl.step(it)
        e1.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
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
    parity = None if args.no_parity else decode_parity(wl, e["ids"], dist.rank)
    shallow = None if args.no_parity else shallow_parity(wl, dist)
    if parity is not None:
        parity["shallow"] = shallow
    spec_b = args.batch_sweep if args.batch_sweep is not None else ("8,32,64" if args.model == "8b" and wl.B == 1
                                                                    else "")
    sweep_b = [int(b) for b in spec_b.split(",") if b]
    bsweep = (batch_sweep(wl, dist, sweep_b, args.warmup, min(args.steps, 50), peak.peak_mem_bandwidth_gbs,
                          parity_seqs=0 if args.no_parity else 4) if sweep_b else None)
    gemv = None
    if dist.world == 1 and not args.no_gemv:
        gw = GemvWorkload(dev, seed=1234)
        gemv = gw.summary(peak.peak_mem_bandwidth_gbs, sweep=not args.no_sweep, peak_tflops=peak.peak_bf16_tflops)
        del gw
    if dist.rank != 0:
        wl.eng.close()
        dist.close()
        return
    cpu = (CpuDecode(args.model, wl.B, lm_head_bits=args.lm_head_bits).token()
           if (dist.world == 1 and not args.no_cpu) else None)
    line = {"metric": decode_metric(args.model, wl.B, wl.P, dist.world, args.lm_head_bits), "value": round(value, 2),
            "unit": "tokens/s", "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": f"int{wl.spec.bits} weights x fp16, fp32 acc",
            "data": "synthetic (random-init weights, uniform random prompt ids)",
            "config": decode_config(args.model, wl.B, wl.P, wl.T, dist.world, args.fold, args.exchange,
                                    args.lm_head_bits),
            "roofline": roofline, "decode_roofline": decode_roofline, "parity": parity, "gemv": gemv,
            "batch_sweep": bsweep, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": int(launches),
            "kernels": {k: {**{kk: v[kk] for kk in ("launches", "us", "GB/s")},
                            **({"gemv": wl.eng.kernel_choice[k]} if k in wl.eng.kernel_choice else {})}
                        for k, v in kstats.items()},
            "clocks": clocks}
    if args.layers:
        line["config"]["layers"] = args.layers
    print(json.dumps(line), flush=True)
    wl.eng.close()
    dist.close()


def run_reference_decode(args, dist: Dist):
    """The reference's CPU path on the box's host cores (rank 0 only; the other
    ranks exit): one whole decode token - every quantized linear of every
    layer dequantized and fp32-multiplied as the reference's oracle does, plus
    the fp16 lm_head (CpuDecode) - after `warmup` (at most 3) warm-up layers.
    The line reports tokens/s of that token; `steps` and `warmup` echo the
    arguments, the sample is described in cpu_baseline."""
    if dist.rank != 0:
        return
    cfg = MODELS[args.model]
    P, T = args.prompt or cfg["prompt"], args.new or cfg["new"]
    cpu = CpuDecode(args.model, args.batch, lm_head_bits=args.lm_head_bits)
    for i in range(min(args.warmup, 3)):
        cpu.layer(i)
    t0 = time.perf_counter()
    tok = cpu.token()
    wall = time.perf_counter() - t0
    line = {"impl": "reference", "metric": decode_metric(args.model, args.batch, P, args.gpus, args.lm_head_bits),
            "value": tok["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(wall * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": f"int{cfg['bits']} codes, fp32 acc",
            "data": "synthetic (random codes and scales of the configuration's shapes)",
            "config": decode_config(args.model, args.batch, P, T, args.gpus, args.fold, args.exchange,
                                    args.lm_head_bits),
            "cpu_baseline": tok,
            "e2e": {"value": tok["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
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
    ap.add_argument("--no-parity", action="store_true", help="skip the decode line's parity check (profiling runs)")
    ap.add_argument("--batch-sweep", default=None,
                    help="comma-separated batch sizes timed beside the line (default 8,32,64 for 8B batch 1; '' none)")
    ap.add_argument("--no-gemv", action="store_true", help="skip the decode line's GEMV figures (profiling runs)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (profiling runs)")
    ap.add_argument("--lm-head-bits", type=int, choices=[16, 8, 4], default=16,
                    help="16: fp16 lm_head as liteweight keeps it (default); 8 / 4: quantized (opt-in)")
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
