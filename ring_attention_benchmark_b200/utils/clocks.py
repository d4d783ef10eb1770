"""Clock and throttle-reason sampling during a timed region.

A background thread polls NVML (the library behind nvidia-smi) every few
milliseconds, so even a timed loop of a few tens of milliseconds gets samples;
without NVML it falls back to an `nvidia-smi --query-gpu ... -lms` subprocess.
Only reads clocks, power and throttle reasons; no GPU setting is changed.
"""
from __future__ import annotations

import csv
import io
import shutil
import statistics
import subprocess
import threading
import time
from typing import Dict, List, Optional

QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
# NVML clocks-event-reason masks, by pynvml's constant names (value fallback)
_NVML_NAMES = {
    "sw_power_cap": ("nvmlClocksThrottleReasonSwPowerCap", 0x4),
    "hw_slowdown": ("nvmlClocksThrottleReasonHwSlowdown", 0x8),
    "sw_thermal_slowdown": ("nvmlClocksThrottleReasonSwThermalSlowdown", 0x20),
    "hw_thermal_slowdown": ("nvmlClocksThrottleReasonHwThermalSlowdown", 0x40),
    "applications_clocks_setting": ("nvmlClocksThrottleReasonApplicationsClocksSetting", 0x2),
}


class ClockSampler:
    def __init__(self, period_ms: float = 5.0, gpus: Optional[List[int]] = None):
        self.period_s = period_ms / 1e3
        self.gpus = gpus
        self.samples = []  # (sm_mhz, max_mhz, power_w, reasons)
        self._stop = threading.Event()
        self._thread = None
        self._proc = None
        self._nvml = None

    # ---------------- NVML path ----------------
    def _init_nvml(self) -> bool:
        try:
            import pynvml

            pynvml.nvmlInit()
            n = pynvml.nvmlDeviceGetCount()
            idx = self.gpus if self.gpus is not None else list(range(n))
            self._handles = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in idx]
            self._bits = {k: int(getattr(pynvml, n, v)) for k, (n, v) in _NVML_NAMES.items()}
            self._nvml = pynvml
            return True
        except Exception:
            return False

    def _poll(self):
        nv = self._nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or getattr(
            nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
        while not self._stop.is_set():
            for h in self._handles:
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                    pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                    bits = get_reasons(h)
                    rs = [k for k, b in self._bits.items() if bits & b]
                    self.samples.append((float(sm), float(mx), pw, rs))
                except Exception:
                    pass
            time.sleep(self.period_s)

    def start(self) -> "ClockSampler":
        if self._init_nvml():
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
            time.sleep(2 * self.period_s)  # first samples before the timed region
            return self
        exe = shutil.which("nvidia-smi")
        if exe is not None:
            cmd = [exe, f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", "-lms", "20"]
            if self.gpus is not None:
                cmd.append("--id=" + ",".join(str(g) for g in self.gpus))
            self._proc = subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                          stderr=subprocess.DEVNULL, text=True)
        return self

    def stop(self) -> Dict:
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass
            return summarize_samples(self.samples, "nvml")
        if self._proc is not None:
            self._proc.terminate()
            try:
                out, _ = self._proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
                out, _ = self._proc.communicate()
            return summarize(out)
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"]}


def summarize_samples(samples, source: str) -> Dict:
    if not samples:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "source": source}
    power = [s[2] for s in samples]
    pmax = max(power)
    loaded = [s for s in samples if s[2] > 0.5 * pmax] or samples
    reasons = sorted({r for s in samples for r in s[3]})
    return {"sm_mhz": statistics.median(s[0] for s in loaded),
            "sm_max_mhz": max(s[1] for s in samples),
            "sm_min_mhz": min(s[0] for s in loaded),
            "samples": len(samples), "reasons": reasons, "power_w_max": round(pmax, 1),
            "source": source}


def _active(v: str) -> bool:
    v = v.strip().lower()
    return v in ("active", "1", "yes") or v.startswith("active")


def summarize(text: str) -> Dict:
    samples = []
    for row in csv.reader(io.StringIO(text)):
        if len(row) < 9:
            continue
        try:
            sm, mx, pw = float(row[1]), float(row[2]), float(row[3])
        except ValueError:
            continue
        rs = [name for name, val in zip(REASONS, row[5:9]) if _active(val)]
        samples.append((sm, mx, pw, rs))
    return summarize_samples(samples, "nvidia-smi")
