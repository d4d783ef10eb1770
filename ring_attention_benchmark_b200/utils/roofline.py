"""Roofline denominators and the fused-kernel roofline.

Peaks come from ``MEASURED_PEAKS.json`` at the repository root when present (a
STREAM-style copy and a cuBLAS bf16 GEMM measured on the B200s this code runs
on); otherwise from the fallback figures of the same measurement: 6.65 TB/s and
1.59 PFLOP/s.  NVLink: 770 GB/s per direction per GPU measured peer copy (900
nominal).

For attention the tensor-core peak depends on the precision: bf16 runs at the
bf16 rate; fp32 runs as three tf32 products (3xTF32) at half the bf16 rate, so
its effective peak is bf16 / 6.

The fused ring kernel's roofline time is the slower of its FLOPs at that peak
and the K/V bytes that must cross NVLink at link bandwidth.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
NVLINK_GBPS = 770.0
NVLINK_NOMINAL_GBPS = 900.0


@dataclass
class Peaks:
    hbm_gbs: float
    bf16_tflops: float
    bf16_tflops_sustained: float
    source: str


def load_peaks() -> Peaks:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return Peaks(float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                     float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    except (OSError, KeyError, ValueError):
        return Peaks(6650.0, 1590.0, 1400.0, "fallback")


def tensor_peak_tflops(prec: str, peaks: Peaks = None, sustained: bool = False) -> float:
    p = peaks or load_peaks()
    bf16 = p.bf16_tflops_sustained if sustained else p.bf16_tflops
    return bf16 if prec == "bf16" else bf16 / 6.0


def attention_roofline_ms(flops: float, nvlink_bytes: float, prec: str,
                          peaks: Peaks = None, sustained: bool = False) -> float:
    t_math = flops / (tensor_peak_tflops(prec, peaks, sustained) * 1e12)
    t_link = nvlink_bytes / (NVLINK_GBPS * 1e9)
    return max(t_math, t_link) * 1e3
