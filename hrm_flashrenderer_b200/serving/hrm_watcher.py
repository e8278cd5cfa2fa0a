"""Live HRM index rebuild on source changes.

Reference behaviour (``hrm_watcher.py:19-69``): watch a set of directories; on any change (directories, ``.git`` and
``.pyc`` ignored) concatenate every ``*.py`` / ``*.sh`` file under them into one corpus (each file preceded by a
``# FILE: <path>`` line), then run ``hrm prep --cluster-size 300`` and ``hrm build`` into the live index directory.

This version needs no file-system notification library (none is available on the serving image): it polls a
snapshot of (path, mtime, size) for the watched extensions, debounces bursts of changes (an editor save writes several
files), and builds the new index into a sibling directory that is swapped in with ``os.replace`` once complete, so a
lane reading the index never sees a half-written ``router_index.bin`` / ``index.sqlite`` pair.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import tempfile
import time
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Tuple

from .utils import find_hrm_binary

DEFAULT_EXTS = (".py", ".sh")
IGNORED_PARTS = {".git", "__pycache__"}

Snapshot = Dict[str, Tuple[float, int]]


def _walk(dirs: Iterable[Path], exts: Tuple[str, ...]) -> List[Path]:
    out = []
    for d in dirs:
        d = Path(d)
        if not d.is_dir():
            continue
        for ext in exts:
            for p in d.rglob("*" + ext):
                if p.is_file() and not (IGNORED_PARTS & set(p.parts)):
                    out.append(p)
    return sorted(set(out))


def snapshot(dirs: Iterable[Path], exts: Tuple[str, ...] = DEFAULT_EXTS) -> Snapshot:
    snap: Snapshot = {}
    for p in _walk(dirs, exts):
        try:
            st = p.stat()
        except OSError:
            continue
        snap[str(p)] = (st.st_mtime, st.st_size)
    return snap


def write_corpus(dirs: Iterable[Path], corpus: Path, exts: Tuple[str, ...] = DEFAULT_EXTS) -> int:
    """Concatenate the watched files (extension by extension per directory, as the reference does)."""
    n = 0
    with open(corpus, "w", encoding="utf-8") as f:
        for d in dirs:
            d = Path(d)
            if not d.is_dir():
                continue
            for ext in exts:
                for p in sorted(d.rglob("*" + ext)):
                    if not p.is_file() or (IGNORED_PARTS & set(p.parts)):
                        continue
                    try:
                        text = p.read_text(encoding="utf-8", errors="ignore")
                    except OSError:
                        continue
                    f.write(f"# FILE: {p}\n")
                    f.write(text + "\n\n")
                    n += 1
    return n


def rebuild_index(dirs: Iterable[Path], index_dir: Path, hrm_bin: Optional[str] = None, cluster_size: int = 300,
                  exts: Tuple[str, ...] = DEFAULT_EXTS) -> Path:
    """corpus -> payloads (``hrm prep``) -> index (``hrm build``) in a temp dir, then atomically swap it in."""
    hrm = str(find_hrm_binary(explicit=hrm_bin))
    index_dir = Path(index_dir).resolve()
    index_dir.parent.mkdir(parents=True, exist_ok=True)
    work = Path(tempfile.mkdtemp(prefix=".hrm_watch_", dir=index_dir.parent))
    try:
        corpus, payloads, staged = work / "corpus.txt", work / "payloads.jsonl", work / "index"
        if write_corpus(dirs, corpus, exts) == 0:
            raise RuntimeError("no source files to index")
        subprocess.run([hrm, "prep", "--input", str(corpus), "--out", str(payloads),
                        "--cluster-size", str(cluster_size)], check=True, capture_output=True)
        subprocess.run([hrm, "build", "--payloads", str(payloads), "--outdir", str(staged)],
                       check=True, capture_output=True)
        old = None
        if index_dir.exists():
            old = work / "previous"
            os.replace(index_dir, old)
        os.replace(staged, index_dir)
        return index_dir
    finally:
        shutil.rmtree(work, ignore_errors=True)


class Watcher:
    def __init__(self, dirs: List[Path], index_dir: Path, hrm_bin: Optional[str] = None, cluster_size: int = 300,
                 debounce_s: float = 1.0, exts: Tuple[str, ...] = DEFAULT_EXTS, log=print):
        self.dirs = [Path(d).expanduser() for d in dirs]
        self.index_dir, self.hrm_bin, self.cluster_size = Path(index_dir), hrm_bin, cluster_size
        self.debounce_s, self.exts, self.log = debounce_s, exts, log
        self.snap = snapshot(self.dirs, exts)
        self.pending_since: Optional[float] = None
        self.rebuilds = 0
        self.failures = 0

    def poll(self, now: Optional[float] = None) -> bool:
        """One polling step; returns True when a rebuild ran.  A change starts the debounce window; the rebuild runs
        once no further change was seen for ``debounce_s``."""
        now = time.monotonic() if now is None else now
        cur = snapshot(self.dirs, self.exts)
        if cur != self.snap:
            changed = sorted(set(cur.items()) ^ set(self.snap.items()))
            self.log(f"change detected ({len(changed)} entries, e.g. {changed[0][0]}); rebuilding after quiet period")
            self.snap = cur
            self.pending_since = now
            return False
        if self.pending_since is not None and now - self.pending_since >= self.debounce_s:
            self.pending_since = None
            try:
                rebuild_index(self.dirs, self.index_dir, self.hrm_bin, self.cluster_size, self.exts)
                self.rebuilds += 1
                self.log(f"HRM index updated: {self.index_dir}")
                return True
            except Exception as e:   # keep watching; the previous index stays in place
                self.failures += 1
                self.log(f"rebuild failed: {e}")
        return False


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-watch", description="rebuild an HRM index when sources change")
    ap.add_argument("--dir", action="append", dest="dirs", default=None,
                    help="directory to watch (repeatable; default: ~/code ~/projects ~/scripts)")
    ap.add_argument("--index_dir", default="./model_coding")
    ap.add_argument("--hrm_bin", default=None)
    ap.add_argument("--cluster_size", type=int, default=300)
    ap.add_argument("--interval", type=float, default=1.0)
    ap.add_argument("--debounce", type=float, default=1.0)
    ap.add_argument("--ext", action="append", default=None, help="file extension to index (default .py .sh)")
    ap.add_argument("--once", action="store_true", help="build the index once and exit")
    a = ap.parse_args(argv)
    dirs = a.dirs or [str(Path.home() / d) for d in ("code", "projects", "scripts")]
    exts = tuple(a.ext) if a.ext else DEFAULT_EXTS
    if a.once:
        rebuild_index([Path(d) for d in dirs], Path(a.index_dir), a.hrm_bin, a.cluster_size, exts)
        return 0
    w = Watcher([Path(d) for d in dirs], Path(a.index_dir), a.hrm_bin, a.cluster_size, a.debounce, exts)
    print(f"watching {', '.join(str(d) for d in w.dirs)} -> {a.index_dir}", flush=True)
    try:
        while True:
            w.poll()
            time.sleep(a.interval)
    except KeyboardInterrupt:
        return 0


if __name__ == "__main__":
    raise SystemExit(main())
