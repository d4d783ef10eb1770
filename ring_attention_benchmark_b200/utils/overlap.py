"""Summary of the fused kernel's overlap trace.

With tracing on (`RingAttention.overlap_trace`), the TMA thread of every CTA
records `%globaltimer` stamps: when its role started and ended, and for each
ring block s >= 1 when it first had to wait for the block (copied over NVLink
by the copy warps of all CTAs) and when the block was present.  A TMA thread
that waits stops feeding the tensor cores once its shared-memory stages run
dry, so the waits bound how long the transfer can have stalled the math.
"""
from __future__ import annotations

from typing import Dict

import torch


def summarize(stamps: torch.Tensor, world: int) -> Dict[str, object]:
    """stamps: [grid, slots, 2] int64 globaltimer ns (FusedRing.read_trace)."""
    s = stamps.to(torch.float64)
    start, end = s[:, 0, 0], s[:, 0, 1]
    live = start > 0
    if not bool(live.any()):
        return {"ctas": 0}
    t0 = float(start[live].min())
    span = float(end[live].max()) - t0
    role = (end - start)[live]
    out: Dict[str, object] = {"ctas": int(live.sum()), "kernel_tma_span_us": round(span / 1e3, 2),
                              "blocks": []}
    stall = torch.zeros_like(start)
    for b in range(1, world):
        w0, w1 = s[:, b, 0], s[:, b, 1]
        waited = live & (w0 > 0)
        if not bool(waited.any()):
            out["blocks"].append({"block": b, "ctas_waited": 0})
            continue
        wait = (w1 - w0)[waited]
        stall[waited] += (w1 - w0)[waited]
        ready = (w1 - t0)[waited]
        out["blocks"].append({
            "block": b, "ctas_waited": int(waited.sum()),
            "wait_us_median": round(float(wait.median()) / 1e3, 3),
            "wait_us_max": round(float(wait.max()) / 1e3, 3),
            "present_at_us_median": round(float(ready.median()) / 1e3, 2),
            "present_at_us_max": round(float(ready.max()) / 1e3, 2),
        })
    frac = stall[live] / role.clamp(min=1.0)
    out["tma_wait_fraction_median"] = round(float(frac.median()), 5)
    out["tma_wait_fraction_max"] = round(float(frac.max()), 5)
    return out
