"""Roofline arithmetic for the dequant matmul and the decode step on B200.

Mirrors liteweight/device.py:4-41 (DeviceSpec) and liteweight/perf_model.py:5-37
(Workload, quant_matmul_workload, predict), with two differences: the B200
entry takes its bandwidth / tensor peaks from the measured figures when a
``MEASURED_PEAKS.json`` is given, and the byte count includes the fp16 scales
(2 * N * K / G bytes), which the reference's model leaves out
(perf_model.py:13-17); ``include_scales=False`` reproduces the reference figure.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path


@dataclass(frozen=True)
class DeviceSpec:
    name: str
    peak_mem_bandwidth_gbs: float
    peak_bf16_tflops: float
    sm_count: int
    shared_mem_per_sm_kb: float
    measured_mem_bandwidth_gbs: float | None = None

    @property
    def peak_bw_bytes_s(self) -> float:
        return self.peak_mem_bandwidth_gbs * 1e9

    @property
    def peak_flops(self) -> float:
        return self.peak_bf16_tflops * 1e12

    @property
    def ridge_point(self) -> float:
        return self.peak_flops / self.peak_bw_bytes_s

    @property
    def effective_bw_bytes_s(self) -> float:
        return (self.measured_mem_bandwidth_gbs or self.peak_mem_bandwidth_gbs) * 1e9


# Nominal B200 (HGX): 7.7 TB/s HBM3e, 2.25 PFLOP/s dense fp16/bf16, 148 SMs, 228 KB smem/SM.
B200 = DeviceSpec(name="NVIDIA B200 (sm_100a)", peak_mem_bandwidth_gbs=7700.0, peak_bf16_tflops=2250.0,
                  sm_count=148, shared_mem_per_sm_kb=228.0)

# Used when no measured peaks file is available (an earlier measurement on B200s).
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def load_measured_peaks(path: str | Path | None = None) -> dict | None:
    p = Path(path) if path else Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text())
    except (OSError, ValueError):
        return None


def b200_measured(path: str | Path | None = None) -> tuple[DeviceSpec, str]:
    """B200 spec whose roofline denominators are the measured peaks; returns (spec, source)."""
    peaks = load_measured_peaks(path)
    if peaks and peaks.get("hbm_gbs") and peaks.get("bf16_tflops"):
        return (DeviceSpec(name=B200.name, peak_mem_bandwidth_gbs=float(peaks["hbm_gbs"]),
                           peak_bf16_tflops=float(peaks["bf16_tflops"]), sm_count=148,
                           shared_mem_per_sm_kb=228.0, measured_mem_bandwidth_gbs=float(peaks["hbm_gbs"])),
                "measured")
    return (DeviceSpec(name=B200.name, peak_mem_bandwidth_gbs=FALLBACK_HBM_GBS,
                       peak_bf16_tflops=FALLBACK_BF16_TFLOPS, sm_count=148, shared_mem_per_sm_kb=228.0),
            "fallback")


@dataclass
class Workload:
    name: str
    flops: int
    bytes_moved: int


def quant_matmul_workload(M: int, K: int, N: int, weight_bits: int, group_size: int | None = 128,
                          include_scales: bool = True) -> Workload:
    """Algorithmic bytes of one dequant matmul: weights + scales + activation + output."""
    flops = 2 * M * K * N
    weight_bytes = K * N * weight_bits // 8
    scale_bytes = 2 * N * (K // group_size) if (include_scales and weight_bits < 16 and group_size) else 0
    bytes_moved = weight_bytes + scale_bytes + 2 * M * K + 2 * M * N
    return Workload(name=f"matmul_M{M}_K{K}_N{N}_w{weight_bits}", flops=flops, bytes_moved=bytes_moved)


def predict(w: Workload, dev: DeviceSpec) -> dict:
    t_mem = w.bytes_moved / dev.effective_bw_bytes_s
    t_compute = w.flops / dev.peak_flops
    return {"arithmetic_intensity": w.flops / w.bytes_moved, "bound": "memory" if t_mem >= t_compute else "compute",
            "predicted_time": max(t_mem, t_compute), "t_mem": t_mem, "t_compute": t_compute}
