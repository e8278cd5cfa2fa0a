"""Sample GPU clocks and throttle reasons with ``nvidia-smi`` while a timed region runs (read-only queries)."""
from __future__ import annotations

import os
import shutil
import statistics
import subprocess
import tempfile
from typing import Dict, List, Optional

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_indices: Optional[List[int]] = None, period_ms: int = 200):
        self.gpus = gpu_indices
        self.period_ms = period_ms
        self.proc = None
        self.path = None

    def start(self) -> "ClockSampler":
        if shutil.which("nvidia-smi") is None:
            return self
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        self._fh = open(self.path, "w")
        self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits",
                                      f"-lms", str(self.period_ms)], stdout=self._fh, stderr=subprocess.DEVNULL)
        return self

    def stop(self) -> Dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._fh.close()
        try:
            with open(self.path) as f:
                lines = f.read().splitlines()
        finally:
            os.unlink(self.path)
        return summarize(lines, self.gpus)


def visible_gpu_indices(n: int) -> List[int]:
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    if cvd:
        try:
            return [int(x) for x in cvd.split(",")[:n]]
        except ValueError:
            pass
    return list(range(n))


def summarize(lines: List[str], gpus: Optional[List[int]] = None) -> Dict:
    sm, smax, power = [], [], []
    reasons = set()
    for ln in lines:
        parts = [p.strip() for p in ln.split(",")]
        if len(parts) < 9:
            continue
        try:
            idx = int(parts[0])
        except ValueError:
            continue
        if gpus is not None and idx not in gpus:
            continue
        try:
            sm.append(float(parts[1]))
            smax.append(float(parts[2]))
            power.append(float(parts[3]))
        except ValueError:
            continue
        for name, v in zip(REASONS, parts[5:9]):
            if v.lower() == "active":
                reasons.add(name)
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
    # "under load" = samples in the upper half of the observed power range
    pmax = max(power)
    loaded = [s for s, p in zip(sm, power) if p >= 0.5 * pmax] or sm
    return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
            "samples": len(sm), "power_w_max": pmax}
