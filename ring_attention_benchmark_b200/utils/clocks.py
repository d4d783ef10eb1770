"""Clock and throttle sampling with nvidia-smi during a timed region.

Reads the clocks and the throttle reasons only; no GPU setting is changed.
"""
from __future__ import annotations

import csv
import io
import shutil
import statistics
import subprocess
from typing import Dict, List, Optional

QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, period_ms: int = 50, gpus: Optional[List[int]] = None):
        self.period_ms = period_ms
        self.gpus = gpus
        self.proc = None

    def start(self) -> "ClockSampler":
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        cmd = [exe, f"--query-gpu={QUERY}", "--format=csv,noheader,nounits",
               "-lms", str(self.period_ms)]
        if self.gpus is not None:
            cmd.append("--id=" + ",".join(str(g) for g in self.gpus))
        self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                     text=True)
        return self

    def stop(self) -> Dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        return summarize(out)


def _active(v: str) -> bool:
    v = v.strip().lower()
    return v in ("active", "1", "yes") or v.startswith("active")


def summarize(text: str) -> Dict:
    sm, smax, power = [], [], []
    reasons = set()
    for row in csv.reader(io.StringIO(text)):
        if len(row) < 9:
            continue
        try:
            sm.append(float(row[1]))
            smax.append(float(row[2]))
            power.append(float(row[3]))
        except ValueError:
            continue
        for name, val in zip(REASONS, row[5:9]):
            if _active(val):
                reasons.add(name)
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
    top = max(sm)
    loaded = [s for s, p in zip(sm, power) if p > 0.5 * max(power)] or sm
    return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax),
            "sm_peak_seen_mhz": top, "samples": len(sm), "reasons": sorted(reasons),
            "power_w_max": max(power)}
