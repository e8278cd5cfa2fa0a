"""Production preflight: every check the lane launcher relies on, reported before anything starts.

Reference: ``scripts/prod_preflight.sh:44-193`` (commands present, Python 3.10-3.12, HRM backend, index files, GPU
count, selected pool vs live VRAM tiers, python deps, CLI entry points, ``bash -n`` of scripts, topology self-test).
Retargeted: B200 pool from ``.hw_selection.env`` vs ``nvidia-smi`` (>= 150 GB per GPU, NVLink between lane GPUs),
the in-tree sm_100a extension and HRM core library, and the engine's Python dependencies.  Checks that need a GPU
read ``nvidia-smi`` only (no CUDA context is created), so preflight also runs on a machine whose GPUs are busy.
"""
import argparse
import importlib
import os
import shutil
import subprocess
import sys
from pathlib import Path
from typing import Callable, List, Tuple

from .hw import derive, load_selection
from .topology import detect_layout, plan_lanes

REPO_ROOT = Path(__file__).resolve().parents[2]


def _check(name: str, fn: Callable[[], str], results: List[Tuple[str, bool, str]]) -> None:
    try:
        msg = fn() or "ok"
        results.append((name, True, msg))
    except Exception as e:
        results.append((name, False, str(e)))


def run_preflight(hrm_model: str = "", smi: str = "nvidia-smi", need_gpu: bool = True) -> List[Tuple[str, bool, str]]:
    res: List[Tuple[str, bool, str]] = []

    def py_version():
        v = sys.version_info
        if not (3, 10) <= (v.major, v.minor) <= (3, 13):
            raise RuntimeError(f"python {v.major}.{v.minor} unsupported (3.10-3.13)")
        return f"python {v.major}.{v.minor}"

    def deps():
        missing = [m for m in ("torch", "numpy", "fastapi", "uvicorn", "pydantic") if importlib.util.find_spec(m) is None]
        if missing:
            raise RuntimeError("missing python packages: " + ", ".join(missing))
        return "deps ok"

    def extension():
        so = list((REPO_ROOT / "hrm_flashrenderer_b200").glob("_C*.so"))
        if not so:
            raise RuntimeError("CUDA extension not built: python setup.py build_ext --inplace")
        return so[0].name

    def hrm_core():
        lib = REPO_ROOT / "hrm_core" / "build" / "libhrm_api.so"
        cli = REPO_ROOT / "hrm_core" / "build" / "hrm"
        if not lib.is_file() or not cli.is_file():
            raise RuntimeError("HRM core not built: make -C hrm_core")
        return "libhrm_api.so + hrm"

    def hrm_index():
        if not hrm_model:
            return "skipped (no --hrm_model)"
        d = Path(hrm_model)
        for f in ("router_index.bin", "index.sqlite"):
            if not (d / f).is_file():
                raise RuntimeError(f"{d / f} missing")
        return str(d)

    def commands():
        missing = [c for c in ("nvcc", "make", "g++") if shutil.which(c) is None]
        if need_gpu and shutil.which(smi) is None and not os.path.isfile(smi):
            missing.append(smi)
        if missing:
            raise RuntimeError("missing commands: " + ", ".join(missing))
        return "nvcc make g++" + (" nvidia-smi" if need_gpu else "")

    def pool():
        sel = load_selection()
        d = derive(sel)
        if not need_gpu:
            return f"selection ok (lanes {d.lanes}); GPU checks skipped"
        plan = plan_lanes(detect_layout(smi), d)
        return f"lanes {plan.lanes} links {plan.link}"

    def shell_syntax():
        bad = []
        for sh in sorted((REPO_ROOT / "hrm_flashrenderer_b200" / "launcher").glob("*.sh")):
            if subprocess.run(["bash", "-n", str(sh)], capture_output=True).returncode != 0:
                bad.append(sh.name)
        if bad:
            raise RuntimeError("bash -n failed: " + ", ".join(bad))
        return "launcher scripts parse"

    for name, fn in (("python", py_version), ("python deps", deps), ("commands", commands),
                     ("cuda extension", extension), ("hrm core", hrm_core), ("hrm index", hrm_index),
                     ("hardware pool", pool), ("scripts", shell_syntax)):
        _check(name, fn, res)
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-preflight")
    ap.add_argument("--hrm_model", default="")
    ap.add_argument("--smi", default=os.environ.get("NVIDIA_SMI", "nvidia-smi"))
    ap.add_argument("--no_gpu", action="store_true")
    a = ap.parse_args(argv)
    res = run_preflight(a.hrm_model, a.smi, not a.no_gpu)
    ok = True
    for name, passed, msg in res:
        print(f"[{'ok' if passed else 'FAIL'}] {name}: {msg}")
        ok &= passed
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
