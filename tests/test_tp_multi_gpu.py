"""Multi-GPU tensor parallelism (needs >= 2 GPUs; skipped otherwise): fused GEMM + peer-memory all-reduce kernel
and the TP engine, run as one process per GPU (see tests/mgpu_worker.py)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("n", [2, 4, 8])
def test_tp_fused_allreduce_and_engine(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs >= {n} GPUs")
    env = dict(os.environ, PYTHONPATH=str(ROOT), NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(29621 + n),
           str(ROOT / "tests" / "mgpu_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=660)
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    rec = json.loads(lines[-1]) if lines else None
    print("mgpu record:", rec)   # visible with -s / in the failure report
    if r.returncode != 0:
        print("mgpu stderr tail:\n" + r.stderr[-6000:])
    assert r.returncode == 0 and rec is not None, (rec, r.stderr[-3000:])
    assert rec["world"] == n and rec["ok"] and rec["fused_ar_max_err"] < 1e-2, rec
    assert min(rec["tp_vs_tp1_70b_first_divergence"]) >= 16, rec
    assert rec["fused_ar_70b_max_abs_err"] < 1e-2, rec
