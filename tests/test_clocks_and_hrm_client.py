"""Clock sampling summary (no GPU: synthetic nvidia-smi CSV, fake nvidia-smi) and the HRM query client's two paths
(in-process C ABI and the ``hrm`` CLI subprocess) against a real index, plus its timeout and error paths."""
import os
import stat
import subprocess
import sys
import time

import pytest

from hrm_flashrenderer_b200.utils import clocks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CORE = os.path.join(ROOT, "hrm_core")
HRM = os.path.join(CORE, "build", "hrm")
sys.path.insert(0, os.path.join(ROOT, "tests", "fixtures"))


# ------------------------------------------------------------------------------------------------ clocks
def _row(idx, sm, smax, power, hw="Not Active", therm="Not Active", swt="Not Active", cap="Not Active"):
    return f"{idx}, {sm}, {smax}, {power}, 0x0, {hw}, {therm}, {swt}, {cap}"


def test_summary_median_under_load_and_reasons():
    lines = [_row(0, 1965, 1965, 120.0)] + [_row(0, 1800 + i, 1965, 990.0, cap="Active") for i in range(5)]
    lines += [_row(1, 500, 1965, 1000.0, hw="Active")]        # another GPU, filtered out below
    lines += ["garbage", "0, n/a, 1965, 10, 0x0, a, b, c, d"]
    s = clocks.summarize(lines, gpus=[0])
    assert s["sm_mhz"] == 1802 and s["sm_max_mhz"] == 1965 and s["samples"] == 6
    assert s["reasons"] == ["sw_power_cap"]
    s_all = clocks.summarize(lines)
    assert "hw_slowdown" in s_all["reasons"] and s_all["samples"] == 7


def test_summary_empty():
    assert clocks.summarize([]) == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_visible_gpu_indices(monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5,7")
    assert clocks.visible_gpu_indices(2) == [3, 5]
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-abc")
    assert clocks.visible_gpu_indices(2) == [0, 1]


def test_sampler_with_fake_nvidia_smi(tmp_path, monkeypatch):
    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/bin/sh\nwhile true; do echo '0, 1900, 1965, 800, 0x0, Not Active, Not Active, Not Active, "
                    "Active'; sleep 0.05; done\n")
    fake.chmod(fake.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    before = set(os.listdir(os.environ.get("TMPDIR", "/tmp")))
    s = clocks.ClockSampler([0], period_ms=50).start()
    time.sleep(0.4)
    r = s.stop()
    assert r["samples"] >= 1 and r["sm_mhz"] == 1900 and r["reasons"] == ["sw_power_cap"]
    assert not os.path.exists(s.path)                       # the sample file is removed
    assert s.proc.poll() is not None                        # the sampler process is gone
    after = set(os.listdir(os.environ.get("TMPDIR", "/tmp")))
    assert not [f for f in after - before if f.startswith("clocks_")]


def test_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    r = clocks.ClockSampler().start().stop()
    assert r["samples"] == 0 and r["reasons"] == ["nvidia-smi unavailable"]


# ------------------------------------------------------------------------------------------------ HRM client
@pytest.fixture(scope="module")
def model(tmp_path_factory):
    subprocess.run(["make", "-C", CORE, "-j4", "all"], check=True, capture_output=True)
    from hrm_corpus import corpus
    d = tmp_path_factory.mktemp("hrmc")
    (d / "corpus.txt").write_text(corpus())
    subprocess.run([HRM, "prep", "--input", str(d / "corpus.txt"), "--out", str(d / "p.jsonl"), "--cluster-size", "40"],
                   check=True, capture_output=True)
    subprocess.run([HRM, "build", "--payloads", str(d / "p.jsonl"), "--outdir", str(d / "m")], check=True,
                   capture_output=True)
    return d / "m"


def test_api_and_subprocess_paths_agree(model):
    from hrm_flashrenderer_b200.serving.hrm_client import run_hrm_query
    from pathlib import Path
    prompt = "how does the router pick a lane for a long prompt"
    a = run_hrm_query(Path(HRM), model, prompt, top_k=5, top_m=400, k=8, prefer_api=True, repo_root=Path(ROOT))
    b = run_hrm_query(Path(HRM), model, prompt, top_k=5, top_m=400, k=8, prefer_api=False, repo_root=Path(ROOT))
    # the CLI re-joins stdin lines with a trailing newline, as the reference's `hrm query --prompt-stdin` does
    # (hrm_core/src/cli/main.cpp:36-43); whitespace does not change the signature, so the retrieval is the same
    assert a.raw["prompt"] == prompt and b.raw["prompt"] == prompt + "\n"
    strip = lambda r: {k: v for k, v in r.items() if k != "prompt"}
    assert strip(a.raw) == strip(b.raw)
    assert a.raw.get("chosen"), a.raw


def test_missing_index_and_binary(model, tmp_path):
    from hrm_flashrenderer_b200.serving.hrm_client import run_hrm_query
    from pathlib import Path
    with pytest.raises(FileNotFoundError):
        run_hrm_query(Path(HRM), tmp_path, "q", prefer_api=True, repo_root=Path(ROOT))
    with pytest.raises(FileNotFoundError):
        run_hrm_query(tmp_path / "no-hrm", model, "q", prefer_api=False, repo_root=Path(ROOT))


def test_subprocess_timeout(model, tmp_path):
    from hrm_flashrenderer_b200.serving.hrm_client import run_hrm_query
    from pathlib import Path
    slow = tmp_path / "hrm"
    slow.write_text("#!/bin/sh\nsleep 5\n")
    slow.chmod(slow.stat().st_mode | stat.S_IEXEC)
    t0 = time.monotonic()
    with pytest.raises(RuntimeError, match="timed out"):
        run_hrm_query(slow, model, "q", prefer_api=False, repo_root=Path(ROOT), timeout_s=0.3)
    assert time.monotonic() - t0 < 3.0
