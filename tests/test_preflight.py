"""Preflight with a fake nvidia-smi (no GPU): the happy path, a GPU-count failure and a missing-index failure, as the
reference's ``scripts/test_prod_preflight.sh:27-110`` checks them."""
import os

from hrm_flashrenderer_b200.launcher import hw, preflight

FAKE = os.path.join(os.path.dirname(__file__), "fixtures", "fake_nvidia_smi.py")


def _index(tmp_path, files=("router_index.bin", "index.sqlite")):
    d = tmp_path / "model_index"
    d.mkdir()
    for f in files:
        (d / f).write_bytes(b"x")
    return str(d)


def _select(tmp_path, monkeypatch, n=8):
    p = hw.write_selection(hw.HWSelection(b200_count=n), tmp_path / "hw.env")
    monkeypatch.setenv("HW_SELECTION_FILE", str(p))


def _by_name(res):
    return {name: (ok, msg) for name, ok, msg in res}


def test_happy_path_pool_and_index(tmp_path, monkeypatch):
    _select(tmp_path, monkeypatch)
    monkeypatch.setenv("FAKE_GPU_MEM", ",".join(["183359"] * 8))
    monkeypatch.setenv("FAKE_LINK", "NV18")
    r = _by_name(preflight.run_preflight(_index(tmp_path), smi=FAKE))
    assert r["hardware pool"][0], r["hardware pool"]
    assert "lanes" in r["hardware pool"][1]
    assert r["hrm index"][0], r["hrm index"]
    assert r["python"][0] and r["python deps"][0]
    assert r["scripts"][0], r["scripts"]


def test_gpu_count_failure(tmp_path, monkeypatch, capsys):
    _select(tmp_path, monkeypatch, n=8)
    monkeypatch.setenv("FAKE_GPU_MEM", ",".join(["183359"] * 4))
    monkeypatch.setenv("FAKE_LINK", "NV18")
    idx = _index(tmp_path)
    r = _by_name(preflight.run_preflight(idx, smi=FAKE))
    assert not r["hardware pool"][0]
    assert preflight.main(["--hrm_model", idx, "--smi", FAKE]) == 1
    assert "[FAIL] hardware pool" in capsys.readouterr().out


def test_missing_index_failure(tmp_path, monkeypatch, capsys):
    _select(tmp_path, monkeypatch)
    monkeypatch.setenv("FAKE_GPU_MEM", ",".join(["183359"] * 8))
    idx = _index(tmp_path, files=("router_index.bin",))
    r = _by_name(preflight.run_preflight(idx, smi=FAKE))
    assert not r["hrm index"][0] and "index.sqlite" in r["hrm index"][1]
    assert r["hardware pool"][0]
    assert preflight.main(["--hrm_model", idx, "--smi", FAKE]) == 1
    assert "[FAIL] hrm index" in capsys.readouterr().out


def test_no_gpu_mode_skips_device_checks(tmp_path, monkeypatch):
    _select(tmp_path, monkeypatch)
    r = _by_name(preflight.run_preflight("", smi=str(tmp_path / "no-such-smi"), need_gpu=False))
    assert r["hardware pool"][0] and "skipped" in r["hardware pool"][1]
    assert r["hrm index"][0] and "skipped" in r["hrm index"][1]


def test_bad_selection_file_fails_pool(tmp_path, monkeypatch):
    bad = tmp_path / "bad.env"
    bad.write_text("HW_POOL_VERSION=2\n")
    monkeypatch.setenv("HW_SELECTION_FILE", str(bad))
    r = _by_name(preflight.run_preflight("", smi=FAKE, need_gpu=False))
    assert not r["hardware pool"][0]
