"""Adaptive TDP governor against a fake power backend (no GPU, no NVML, no power-limit writes)."""
import json

from hrm_flashrenderer_b200.utils.tdp_governor import (GpuPower, Governor, Reading, Settings, parse_reading,
                                                      read_token_file, main as gov_main)


class FakeBackend:
    def __init__(self, n=2, limit=1000, lo=200, hi=1000):
        self.gpus = [GpuPower(i, "B200", limit, lo, hi) for i in range(n)]
        self.calls = []

    def query(self):
        return list(self.gpus)

    def set_limit(self, index, watts):
        self.calls.append((index, watts))
        self.gpus[index].limit_w = watts


FAST = Settings(step_w=50, floor_w=300, stable_samples=3, stable_cv=0.05, probe_settle_s=1, probe_window_s=2,
                recover_settle_s=1, recover_window_s=2, cooldown_s=0)


def _run(gov, tps_fn, seconds, phase="decode", wl="default", t0=0.0):
    t = t0
    while t < t0 + seconds:
        gov.step(t, Reading(phase, tps_fn(gov, t), wl))
        t += 0.5
    return t


def test_parse_reading_formats():
    assert parse_reading("") .phase == "idle"
    r = parse_reading("42.5")
    assert (r.phase, r.tps) == ("decode", 42.5)
    assert parse_reading("0.2").phase == "idle"
    r = parse_reading(json.dumps({"state": "generating", "tok_s": 10, "model": "llama70b"}))
    assert (r.phase, r.tps, r.workload) == ("decode", 10.0, "llama70b")
    r = parse_reading(json.dumps({"prefill_active": True, "inter_token_ms": 20}))
    assert (r.phase, r.tps) == ("prefill", 50.0)
    r = parse_reading(json.dumps({"avg_token_ms": 4}))
    assert (r.phase, r.tps) == ("decode", 250.0)


def test_unreadable_token_file_is_idle(tmp_path):
    assert read_token_file(str(tmp_path / "missing.json")).phase == "idle"
    p = tmp_path / "bad.json"
    p.write_text("{not json")
    assert read_token_file(str(p)).phase == "idle"


def test_observe_mode_never_writes():
    be = FakeBackend()
    gov = Governor(be, FAST, apply=False)
    _run(gov, lambda g, t: 100.0, 40)
    assert be.calls == []                 # nothing reached the backend
    assert gov.writes                     # but the governor did plan probes


def test_probe_accepts_when_rate_holds_and_walks_down_round_robin():
    be = FakeBackend(n=2)
    gov = Governor(be, FAST, apply=True)
    _run(gov, lambda g, t: 100.0, 60)
    wl = gov.profile["workloads"]["default"]
    assert wl["meta"]["0"]["accepted"] >= 2 and wl["meta"]["1"]["accepted"] >= 2
    assert wl["decode_w"]["0"] < 1000 and wl["decode_w"]["1"] < 1000
    assert all(w >= 300 for _, w in be.calls)   # floor respected


def test_probe_rejects_when_rate_drops_and_remembers_bad_limit():
    be = FakeBackend(n=1)
    gov = Governor(be, FAST, apply=True)
    # throughput collapses whenever the limit is below 900 W
    _run(gov, lambda g, t: 100.0 if be.gpus[0].limit_w >= 900 else 50.0, 120)
    wl = gov.profile["workloads"]["default"]
    assert wl["decode_w"]["0"] == 900
    assert wl["meta"]["0"]["last_bad_w"] == 850
    assert min(w for _, w in be.calls) == 850        # never probed below the known-bad limit again
    assert be.gpus[0].limit_w == 900


def test_prefill_and_idle_restore_limits():
    be = FakeBackend(n=1)
    gov = Governor(be, FAST, apply=True)
    t = _run(gov, lambda g, t: 100.0, 4)       # stable -> a probe has started at a lower limit
    assert gov.probe is not None and be.gpus[0].limit_w == 950
    gov.step(t, Reading("prefill", 0.0))
    assert gov.probe is None and be.gpus[0].limit_w == 1000
    t = _run(gov, lambda g, t: 100.0, 4, t0=t + 1)
    assert gov.probe is not None
    gov.step(t, Reading("idle", 0.0))
    assert gov.probe is None and be.gpus[0].limit_w == 1000


def test_workloads_are_profiled_separately():
    be = FakeBackend(n=1)
    gov = Governor(be, FAST, apply=True)
    _run(gov, lambda g, t: 100.0, 30, wl="a")
    _run(gov, lambda g, t: 100.0, 6, wl="b", t0=100)
    wls = gov.profile["workloads"]
    assert wls["a"]["decode_w"]["0"] < 1000
    assert "b" in wls and wls["b"]["meta"]["0"]["accepted"] == 0


def test_cli_apply_needs_env(monkeypatch, tmp_path, capsys):
    import hrm_flashrenderer_b200.utils.tdp_governor as mod
    be = FakeBackend(n=1)
    monkeypatch.setattr(mod, "NvmlBackend", lambda sel: be)
    monkeypatch.delenv("HRM_TDP_ALLOW_WRITE", raising=False)
    tok = tmp_path / "live.json"
    tok.write_text("100")
    out = tmp_path / "profile.json"
    rc = gov_main(["--token-file", str(tok), "--output", str(out), "--poll-ms", "0", "--iterations", "40",
                   "--apply", "--stable-samples", "3", "--cooldown-s", "0"])
    assert rc == 0 and be.calls == []
    assert "--apply ignored" in capsys.readouterr().err
    prof = json.loads(out.read_text())
    assert prof["schema"].startswith("hrm-b200-tdp-governor") and prof["current"]["apply"] is False
