"""Online power-limit (TDP) governor driven by the serving stack's live decode rate.

Behaviour follows the reference governor (``adaptive_tdp_governor.py:134-218`` token-file parsing,
``:253-296`` per-workload profile, ``:308-528`` probe loop): while decode throughput is stable, lower one GPU's power
limit by ``step_w`` (round robin, never below ``max(floor_w, min_w)`` nor at/below a limit that already failed), let it
settle, measure, restore, measure again, and keep the lower limit only if the probed rate is within
``allowed_loss_frac`` of the mean of the rates before and after.  Prefill runs at the workload's prefill limits
(the maximum); idle or a workload change aborts a probe and restores the limit.

Safety: writing power limits is OFF by default.  The governor runs in observe mode (it computes and logs the limits it
would set) unless it is constructed with ``apply=True``; the CLI additionally requires ``--apply`` and the
environment variable ``HRM_TDP_ALLOW_WRITE=1``.  Power control goes through a small backend interface so the whole
state machine is testable on a CPU host against a fake (``tests/test_tdp_governor.py``); ``NvmlBackend`` is the real
one (NVML via ``nvidia_ml_py``).  The design differs from the reference in that the loop is a pure ``step(now,
reading)`` method (no sleeps, no global state), the probe schedule is an explicit enum, and the profile keeps its own
schema tag.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Protocol

SCHEMA = "hrm-b200-tdp-governor/v1"


# ------------------------------------------------------------------------------------------------ readings
@dataclass
class Reading:
    phase: str                      # "decode" | "prefill" | "idle"
    tps: float                      # effective decode tokens/s (0 when unknown)
    workload: str = "default"
    inter_token_ms: Optional[float] = None
    raw: dict = field(default_factory=dict)


_PHASES = {
    "decode": ("decode", "decoding", "generate", "generating", "inference"),
    "prefill": ("prefill", "prompt", "prompting", "loading"),
    "idle": ("idle", "none", "waiting"),
}


def _phase_name(x) -> str:
    s = str(x or "").strip().lower()
    for name, words in _PHASES.items():
        if s in words:
            return name
    return ""


def _first_float(obj: dict, keys) -> Optional[float]:
    for k in keys:
        if k in obj:
            try:
                return float(obj[k])
            except (TypeError, ValueError):
                continue
    return None


def parse_reading(text: str, min_live_tps: float = 1.0) -> Reading:
    """Parse the live token-rate file: a bare number (tokens/s) or a JSON object with ``phase``/``state``,
    ``decode_tps``/``tps``/``tokens_per_second``/``current_tps``/``tok_s``, ``inter_token_ms`` (or ``token_gap_ms``,
    ``avg_token_ms``, ``it_gap_ms``) and ``workload_key``/``model_key``/``model``/``profile``."""
    text = (text or "").strip()
    if not text:
        return Reading("idle", 0.0)
    try:
        v = float(text)
        return Reading("decode" if v >= min_live_tps else "idle", v, raw={"decode_tps": v})
    except ValueError:
        pass
    obj = json.loads(text)
    if not isinstance(obj, dict):
        raise ValueError("token file must hold a number or a JSON object")
    phase = _phase_name(obj.get("phase")) or _phase_name(obj.get("state"))
    if not phase and any(obj.get(k) for k in ("prefill", "prefill_active", "prompt_active")):
        phase = "prefill"
    if not phase and any(obj.get(k) for k in ("decode", "decode_active", "generating", "generation_active")):
        phase = "decode"
    tps = _first_float(obj, ("decode_tps", "tps", "tokens_per_second", "current_tps", "tok_s"))
    gap = _first_float(obj, ("inter_token_ms", "token_gap_ms", "avg_token_ms", "it_gap_ms"))
    if tps is None or tps <= 0:
        tps = 1000.0 / gap if gap and gap > 0 else 0.0
    if not phase:
        phase = "decode" if tps >= min_live_tps else "idle"
    wl = str(obj.get("workload_key") or obj.get("model_key") or obj.get("model") or obj.get("profile")
             or "default").strip() or "default"
    return Reading(phase, float(tps), wl, gap, obj)


def read_token_file(path: str, min_live_tps: float = 1.0) -> Reading:
    try:
        with open(path, "r", encoding="utf-8") as f:
            return parse_reading(f.read(), min_live_tps)
    except (OSError, ValueError):
        return Reading("idle", 0.0)


# ------------------------------------------------------------------------------------------------ backends
@dataclass
class GpuPower:
    index: int
    name: str
    limit_w: int
    min_w: int
    max_w: int
    draw_w: float = -1.0


class PowerBackend(Protocol):
    def query(self) -> List[GpuPower]: ...
    def set_limit(self, index: int, watts: int) -> None: ...


class NvmlBackend:
    """NVML power queries / limits (``nvidia_ml_py``).  Setting a limit needs root; it is only ever called when the
    governor runs with ``apply=True``."""

    def __init__(self, indices: Optional[List[int]] = None):
        import pynvml
        self._nv = pynvml
        pynvml.nvmlInit()
        n = pynvml.nvmlDeviceGetCount()
        self.indices = indices if indices is not None else list(range(n))
        self._h = {i: pynvml.nvmlDeviceGetHandleByIndex(i) for i in self.indices}

    def query(self) -> List[GpuPower]:
        nv, out = self._nv, []
        for i, h in self._h.items():
            name = nv.nvmlDeviceGetName(h)
            name = name.decode() if isinstance(name, bytes) else name
            lo, hi = nv.nvmlDeviceGetPowerManagementLimitConstraints(h)
            lim = nv.nvmlDeviceGetPowerManagementLimit(h)
            try:
                draw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
            except Exception:
                draw = -1.0
            out.append(GpuPower(i, name, int(round(lim / 1000)), int(round(lo / 1000)), int(round(hi / 1000)), draw))
        return out

    def set_limit(self, index: int, watts: int) -> None:
        self._nv.nvmlDeviceSetPowerManagementLimit(self._h[index], int(watts) * 1000)


# ------------------------------------------------------------------------------------------------ governor
@dataclass
class Settings:
    step_w: int = 10
    floor_w: int = 110
    stable_samples: int = 10
    stable_cv: float = 0.04
    min_live_tps: float = 1.0
    allowed_loss_frac: float = 0.025
    probe_settle_s: float = 1.2
    probe_window_s: float = 2.2
    recover_settle_s: float = 1.0
    recover_window_s: float = 1.8
    cooldown_s: float = 5.0


class Stage:
    SETTLE_PROBE = "settle_probe"
    COLLECT_PROBE = "collect_probe"
    SETTLE_RECOVER = "settle_recover"
    COLLECT_RECOVER = "collect_recover"


def _cv(xs: List[float]) -> float:
    if len(xs) < 2:
        return float("inf")
    m = sum(xs) / len(xs)
    return statistics.pstdev(xs) / m if m > 0 else float("inf")


def _median(xs) -> float:
    xs = list(xs)
    return statistics.median(xs) if xs else 0.0


class Governor:
    def __init__(self, backend: PowerBackend, settings: Settings = Settings(), apply: bool = False,
                 profile: Optional[dict] = None, log=None):
        self.b, self.s, self.apply = backend, settings, apply
        self.gpus = backend.query()
        if not self.gpus:
            raise RuntimeError("no GPUs to govern")
        self.profile = profile if (profile or {}).get("schema") == SCHEMA else self._empty_profile()
        self.applied: Dict[str, int] = {str(g.index): g.limit_w for g in self.gpus}
        self.recent = deque(maxlen=max(3, settings.stable_samples))
        self.probe: Optional[dict] = None
        self.rr = 0
        self.last_probe_end = float("-inf")
        self.writes: List[tuple] = []   # (index, watts) requested, applied or not
        self.log = log or (lambda msg: None)

    # -- profile
    def _empty_profile(self) -> dict:
        return {"schema": SCHEMA, "gpus": [{"index": g.index, "name": g.name, "min_w": g.min_w, "max_w": g.max_w}
                                           for g in self.gpus],
                "settings": vars(self.s).copy(), "workloads": {}, "current": {}}

    def workload(self, key: str) -> dict:
        wls = self.profile.setdefault("workloads", {})
        if key not in wls:
            wls[key] = {"decode_w": {str(g.index): g.max_w for g in self.gpus},
                        "prefill_w": {str(g.index): g.max_w for g in self.gpus},
                        "meta": {str(g.index): {"last_good_w": g.max_w, "last_bad_w": None, "accepted": 0,
                                                "rejected": 0} for g in self.gpus},
                        "reference_tps": None, "baseline_tps": None}
        return wls[key]

    # -- limit writes (observe mode records only)
    def _set(self, index: int, watts: int) -> None:
        key = str(index)
        if self.applied.get(key) == int(watts):
            return
        self.writes.append((index, int(watts)))
        self.log(f"{'set' if self.apply else 'would set'} GPU {index} power limit -> {int(watts)} W")
        if self.apply:
            self.b.set_limit(index, int(watts))
        self.applied[key] = int(watts)

    def _set_all(self, limits: Dict[str, int]) -> None:
        for k, w in limits.items():
            self._set(int(k), int(w))

    def _end_probe(self, now: float, restore: bool = True) -> None:
        if self.probe is not None and restore:
            self._set(self.probe["gpu"], self.probe["orig_w"])
        self.probe = None
        self.last_probe_end = now

    def _next_target(self, wl: dict):
        n = len(self.gpus)
        for off in range(n):
            g = self.gpus[(self.rr + off) % n]
            key = str(g.index)
            cand = int(wl["decode_w"][key]) - self.s.step_w
            bad = wl["meta"][key]["last_bad_w"]
            if cand < max(self.s.floor_w, g.min_w) or (bad is not None and cand <= bad):
                continue
            self.rr = (self.rr + off + 1) % n
            return g, cand
        return None, None

    # -- one control step
    def step(self, now: float, r: Reading) -> None:
        wl = self.workload(r.workload)
        if r.phase == "decode":
            self.recent.append(r.tps)
            wl["baseline_tps"] = round(_median(self.recent), 6)
        else:
            self.recent.clear()

        if r.phase == "prefill":
            if self.probe is not None:
                self._end_probe(now)
            self._set_all(wl["prefill_w"])
        elif r.phase == "decode":
            if self.probe is not None and r.workload != self.probe["workload"]:
                self._end_probe(now)
            if self.probe is None:
                self._set_all(wl["decode_w"])
                stable = (len(self.recent) >= self.s.stable_samples and _cv(list(self.recent)) <= self.s.stable_cv
                          and _median(self.recent) >= self.s.min_live_tps)
                if stable and now - self.last_probe_end >= self.s.cooldown_s:
                    g, cand = self._next_target(wl)
                    if g is not None:
                        self.probe = {"gpu": g.index, "workload": r.workload, "orig_w": int(wl["decode_w"][str(g.index)]),
                                      "cand_w": int(cand), "before_tps": _median(self.recent), "probe": [],
                                      "after": [], "stage": Stage.SETTLE_PROBE, "t0": now}
                        self._set(g.index, cand)
            else:
                self._advance_probe(now, r, wl)
        else:
            if self.probe is not None:
                self._end_probe(now)

        self.profile["current"] = {"phase": r.phase, "workload": r.workload, "applied_w": dict(self.applied),
                                   "recent_tps": round(_median(self.recent), 6), "probe": self.probe,
                                   "apply": self.apply}

    def _advance_probe(self, now: float, r: Reading, wl: dict) -> None:
        p, s = self.probe, self.s
        el = now - p["t0"]
        if p["stage"] == Stage.SETTLE_PROBE and el >= s.probe_settle_s:
            p["stage"], p["t0"] = Stage.COLLECT_PROBE, now
        elif p["stage"] == Stage.COLLECT_PROBE:
            if r.tps >= s.min_live_tps:
                p["probe"].append(r.tps)
            if el >= s.probe_window_s:
                p["probe_tps"] = _median(p["probe"])
                self._set(p["gpu"], p["orig_w"])
                p["stage"], p["t0"] = Stage.SETTLE_RECOVER, now
        elif p["stage"] == Stage.SETTLE_RECOVER and el >= s.recover_settle_s:
            p["stage"], p["t0"] = Stage.COLLECT_RECOVER, now
        elif p["stage"] == Stage.COLLECT_RECOVER:
            if r.tps >= s.min_live_tps:
                p["after"].append(r.tps)
            if el >= s.recover_window_s:
                ref = (p["before_tps"] + _median(p["after"])) / 2.0
                ratio = p.get("probe_tps", 0.0) / ref if ref > 0 else 0.0
                key = str(p["gpu"])
                meta = wl["meta"][key]
                if ratio >= 1.0 - s.allowed_loss_frac:
                    wl["decode_w"][key] = p["cand_w"]
                    meta["last_good_w"] = p["cand_w"]
                    meta["accepted"] += 1
                    self._set(p["gpu"], p["cand_w"])
                    self.log(f"GPU {p['gpu']}: accepted {p['cand_w']} W (ratio {ratio:.3f})")
                else:
                    meta["last_bad_w"] = p["cand_w"]
                    meta["rejected"] += 1
                    self.log(f"GPU {p['gpu']}: rejected {p['cand_w']} W (ratio {ratio:.3f})")
                wl["reference_tps"] = round(ref, 6)
                self._end_probe(now, restore=False)


def atomic_write_json(path: str, obj: dict) -> None:
    tmp = f"{path}.tmp"
    with open(tmp, "w", encoding="utf-8") as f:
        json.dump(obj, f, indent=2)
    os.replace(tmp, path)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-tdp-governor",
                                 description="adaptive GPU power-limit governor (observe mode unless --apply)")
    ap.add_argument("--token-file", default="adaptive_tdp_live.json")
    ap.add_argument("--output", default="adaptive_tdp_profile.json")
    ap.add_argument("--gpus", default=None, help="comma-separated GPU indices")
    ap.add_argument("--poll-ms", type=int, default=500)
    ap.add_argument("--iterations", type=int, default=0, help="stop after N polls (0 = run forever)")
    ap.add_argument("--apply", action="store_true",
                    help="really write power limits (also needs HRM_TDP_ALLOW_WRITE=1 and root)")
    for f in Settings.__dataclass_fields__.values():
        ap.add_argument("--" + f.name.replace("_", "-"), type=type(f.default), default=f.default)
    a = ap.parse_args(argv)
    apply = bool(a.apply and os.environ.get("HRM_TDP_ALLOW_WRITE") == "1")
    if a.apply and not apply:
        print("--apply ignored: set HRM_TDP_ALLOW_WRITE=1 to allow power-limit writes", file=sys.stderr)
    settings = Settings(**{k: getattr(a, k) for k in Settings.__dataclass_fields__})
    sel = [int(x) for x in a.gpus.split(",")] if a.gpus else None
    prof = None
    if os.path.exists(a.output):
        try:
            prof = json.load(open(a.output))
        except Exception:
            prof = None
    gov = Governor(NvmlBackend(sel), settings, apply=apply, profile=prof, log=lambda m: print(m, flush=True))
    n = 0
    while a.iterations <= 0 or n < a.iterations:
        gov.step(time.time(), read_token_file(a.token_file, settings.min_live_tps))
        atomic_write_json(a.output, gov.profile)
        n += 1
        time.sleep(a.poll_ms / 1000.0)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
