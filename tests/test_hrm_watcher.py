"""HRM watcher: change detection, debounce, atomic index swap, failure keeps the old index (CPU, real hrm CLI)."""
import json
import subprocess
from pathlib import Path

import pytest

from hrm_flashrenderer_b200.serving.hrm_watcher import Watcher, rebuild_index, snapshot, write_corpus
from hrm_flashrenderer_b200.serving.utils import find_hrm_binary

HRM = find_hrm_binary()
needs_hrm = pytest.mark.skipif(not Path(HRM).is_file(), reason="hrm core not built (make -C hrm_core)")


def _src(tmp_path):
    d = tmp_path / "code"
    (d / "pkg").mkdir(parents=True)
    (d / "pkg" / "a.py").write_text("def silver_bridge():\n    return 'the silver bridge spans the river'\n")
    (d / "run.sh").write_text("echo 'winter tower lights'\n")
    (d / ".git").mkdir()
    (d / ".git" / "x.py").write_text("ignored = True\n")
    (d / "pkg" / "b.pyc").write_bytes(b"\0")
    return d


def test_corpus_and_snapshot_skip_ignored(tmp_path):
    d = _src(tmp_path)
    n = write_corpus([d], tmp_path / "c.txt")
    text = (tmp_path / "c.txt").read_text()
    assert n == 2 and "# FILE: " in text and "silver bridge" in text and "ignored" not in text
    assert len(snapshot([d])) == 2


@needs_hrm
def test_rebuild_is_queryable_and_atomic(tmp_path):
    d = _src(tmp_path)
    idx = tmp_path / "live_index"
    rebuild_index([d], idx, str(HRM), cluster_size=2)
    assert (idx / "router_index.bin").is_file() and (idx / "index.sqlite").is_file()
    out = subprocess.run([str(HRM), "query", "--model", str(idx), "--format", "json", "--prompt", "silver bridge"],
                         capture_output=True, text=True, check=True).stdout
    assert "silver" in json.dumps(json.loads(out))
    assert not list(tmp_path.glob(".hrm_watch_*"))   # staging dirs cleaned up


@needs_hrm
def test_watcher_debounces_and_rebuilds_once(tmp_path):
    d = _src(tmp_path)
    idx = tmp_path / "idx"
    logs = []
    w = Watcher([d], idx, str(HRM), cluster_size=2, debounce_s=1.0, log=logs.append)
    assert w.poll(now=0.0) is False                        # nothing changed
    (d / "pkg" / "c.py").write_text("merchant_promise = 'the river stone'\n")
    assert w.poll(now=1.0) is False                        # change seen, debounce starts
    (d / "pkg" / "a.py").write_text("def silver_bridge():\n    return 'rebuilt'\n")
    assert w.poll(now=1.5) is False                        # another change restarts the window
    assert w.poll(now=2.0) is False
    assert w.poll(now=2.6) is True and w.rebuilds == 1
    assert w.poll(now=10.0) is False and w.rebuilds == 1   # quiet: no more rebuilds
    assert (idx / "router_index.bin").is_file()


def test_failed_rebuild_keeps_previous_index(tmp_path):
    d = _src(tmp_path)
    idx = tmp_path / "idx"
    idx.mkdir()
    (idx / "router_index.bin").write_bytes(b"old")
    w = Watcher([d], idx, hrm_bin=str(tmp_path / "no_such_hrm"), debounce_s=0.0, log=lambda m: None)
    (d / "new.py").write_text("x = 1\n")
    w.poll(now=0.0)
    assert w.poll(now=1.0) is False and w.failures == 1
    assert (idx / "router_index.bin").read_bytes() == b"old"
