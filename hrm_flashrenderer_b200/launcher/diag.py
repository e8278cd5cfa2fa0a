"""GPU subsystem diagnostic (counterpart of the reference's ``scripts/diag_gpu.py``): versions, visible devices, a
tiny allocation on each, peer access between every pair, the sm_100a extension (SM count, a 1-token GEMM on the
first device) and NCCL's version.  Prints one line per check and a JSON summary; exit status 1 when a check that
applies fails.  Reads device state only; changes no GPU setting.

    python -m hrm_flashrenderer_b200.launcher.diag
"""
from __future__ import annotations

import json
import sys
import time
from typing import Callable, Dict


def run(log: Callable[[str], None] = print) -> Dict:
    import torch
    rep: Dict = {"torch": torch.__version__, "cuda_available": torch.cuda.is_available(), "devices": [],
                 "peer_access": {}, "failures": []}

    def check(name: str, fn):
        t0 = time.perf_counter()
        try:
            out = fn()
            log(f"[diag] {name}: ok {out if out is not None else ''} ({(time.perf_counter() - t0) * 1e3:.1f} ms)")
            return out
        except Exception as e:
            rep["failures"].append(f"{name}: {type(e).__name__}: {e}")
            log(f"[diag] {name}: FAILED {type(e).__name__}: {e}")
            return None

    log(f"[diag] python {sys.version.split()[0]}, torch {torch.__version__}, CUDA available: "
        f"{torch.cuda.is_available()}")
    if not torch.cuda.is_available():
        return rep
    rep["cuda_runtime"] = torch.version.cuda
    try:
        rep["nccl"] = ".".join(map(str, torch.cuda.nccl.version()))
    except Exception:
        rep["nccl"] = None
    n = torch.cuda.device_count()
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        rep["devices"].append({"index": i, "name": p.name, "sm_count": p.multi_processor_count,
                               "memory_gb": round(p.total_memory / 2**30, 1), "cc": f"{p.major}.{p.minor}"})
        check(f"alloc cuda:{i}", lambda i=i: float(torch.ones(1, device=f"cuda:{i}").sum().item()))
    for i in range(n):
        for j in range(n):
            if i != j:
                rep["peer_access"][f"{i}->{j}"] = bool(torch.cuda.can_device_access_peer(i, j))

    def ext_gemm():
        from .. import ops
        C = ops.ext()
        x = torch.randn(1, 256, device="cuda:0").half()
        w = ops.tile_w8(torch.randint(-127, 128, (256, 256), dtype=torch.int8, device="cuda:0"))
        s = torch.full((256,), 1e-3, device="cuda:0")
        y = ops.w8a16_linear(x, w, s, out_dtype=torch.float32)
        ops.check_status()
        return {"sm_count": C.sm_count(), "gemm_finite": bool(torch.isfinite(y).all().item())}
    rep["extension"] = check("sm_100a extension", ext_gemm)
    return rep


def main(argv=None) -> int:
    import argparse
    ap = argparse.ArgumentParser(prog="hrm-flash-diag", description=__doc__.split("\n")[0])
    ap.parse_args(argv)
    rep = run()
    print(json.dumps(rep))
    return 1 if rep["failures"] else 0


if __name__ == "__main__":
    raise SystemExit(main())
