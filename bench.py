"""Benchmark of liteweight_b200's hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload gemv]

Prints ONE JSON line (rank 0). Workloads:

* ``gemv`` - the dequant GEMV of the Llama-3.2-1B linear shapes (K x N =
  2048x2048, 2048x512, 2048x8192, 8192x2048), INT4 and INT8 with group size
  128, one activation row (M = 1): one step = those 8 GEMVs, each on its own
  weight copy from a rotating set larger than L2 (so every step reads its
  weights from HBM). Metric: algorithmic GB/s (weights + fp16 scales +
  activation + output, divided by time). Multi-GPU: independent replicas
  (``scaling: weak``). A per-M sweep (M = 1..256) is reported beside it.

``--impl reference`` times the reference's CPU path for the same workload
(dequantize the packed weights, fp32 matmul, fp16 result - restated by the
numpy oracle) on the host cores, rank 0 only.
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
            self.out = open(ROOT / "gpurun_out" / f".clocks_{os.getpid()}.csv", "w") \
                if (ROOT / "gpurun_out").exists() else None
            if self.out is None:
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


def run_reference(args, dist: Dist):
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


def run_ours(args, dist: Dist):
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["gemv"], default="gemv")
    ap.add_argument("--no-sweep", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
    else:
        run_ours(args, dist)


if __name__ == "__main__":
    main()
