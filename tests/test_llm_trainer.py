"""Experiments-plane trainer / chat CLI on CPU: training reduces the loss, checkpoints resume, chat decodes,
data-parallel ranks (gloo) stay in lock-step.  A GPU variant checks the fused optimizer kernels."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "fixtures"))
from hrm_corpus import corpus  # noqa: E402

from hrm_flashrenderer_b200.experiments.llm import Optimizer, split_batch  # noqa: E402

try:
    from hrm_flashrenderer_b200.experiments import pairindex as _pi
    _pi.lib()
    HAVE_PI = True
except Exception:
    HAVE_PI = False
needs_pi = pytest.mark.skipif(not HAVE_PI, reason="libhrm_pairindex.so not built")

SMALL = ["--k1", "64", "--k2", "32", "--dmodel", "32", "--heads", "2", "--layers", "2", "--ffn", "48", "--tmax", "64",
         "--seq", "16", "--device", "cpu", "--lr", "3e-3"]


def _run(args, **kw):
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    return subprocess.run([sys.executable, "-m", "hrm_flashrenderer_b200.experiments.llm"] + args, capture_output=True,
                          text=True, env=env, timeout=300, **kw)


def test_split_batch_by_memory():
    assert split_batch(64, [180, 180]) == [32, 32]
    assert sum(split_batch(10, [24, 11, 11])) == 10 and split_batch(10, [24, 11, 11])[0] >= 4
    assert split_batch(3, [1, 1, 1, 1]) == [1, 1, 1, 1]   # every device keeps >= 1 sample
    assert all(x >= 1 for x in split_batch(5, [100, 1]))


def test_optimizer_cpu_matches_adamw_formula():
    torch.manual_seed(0)
    w = torch.nn.Parameter(torch.randn(1000))
    w0 = w.data.clone()
    g = torch.randn(1000) * 10
    opt = Optimizer(w, lr=1e-2, wd=0.1, clip=1.0)
    opt.step(g)
    cs = 1.0 / float(g.norm())
    gg = g * cs
    m, v = 0.1 * gg, 0.001 * gg * gg
    want = w0 - 1e-2 * ((m / 0.1) / (torch.sqrt(v / 0.001) + 1e-8) + 0.1 * w0)
    torch.testing.assert_close(w.data, want, rtol=1e-5, atol=1e-6)
    assert int(opt.step_t) == 2


@needs_pi
def test_train_resume_and_chat(tmp_path):
    data = tmp_path / "c.txt"
    data.write_text(corpus(500, seed=1))
    ck = tmp_path / "ck.bin"
    r = _run(["--train", "--data", str(data), "--ckpt", str(ck), "--index", str(tmp_path / "none.bin"),
              "--steps", "40", "--batch", "8", "--log_every", "10", "--save_every", "0"] + SMALL)
    assert r.returncode == 0, r.stderr
    losses = [float(l.split("loss=")[1].split()[0]) for l in r.stdout.splitlines() if "loss=" in l]
    assert len(losses) == 4 and losses[-1] < losses[0]
    assert ck.is_file()
    r2 = _run(["--train", "--data", str(data), "--ckpt", str(ck), "--steps", "10", "--batch", "8", "--log_every",
               "10", "--save_every", "0"] + SMALL)
    assert r2.returncode == 0, r2.stderr
    resumed = float([l for l in r2.stdout.splitlines() if "loss=" in l][0].split("loss=")[1].split()[0])
    assert resumed < losses[0]                     # continued from the trained weights
    r3 = _run(["--chat", "--ckpt", str(ck), "--measure", "--chat_prompt", "KING LEAR:"] + SMALL,
              input="who guards the bridge\n/reset\nthe river\n/quit\n")
    assert r3.returncode == 0, r3.stderr
    assert "[chat] commands" in r3.stderr and "tok/s" in r3.stderr


@needs_pi
def test_data_parallel_gloo_two_ranks(tmp_path):
    data = tmp_path / "c.txt"
    data.write_text(corpus(300, seed=2))
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", "--master-port", "29611", "-m", "hrm_flashrenderer_b200.experiments.llm", "--train", "--data",
           str(data), "--ckpt", str(tmp_path / "dp.bin"), "--steps", "6", "--batch", "4", "--log_every", "3",
           "--save_every", "0"] + SMALL
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    assert "gpus=2 batch=4 [2, 2]" in r.stdout and (tmp_path / "dp.bin").is_file()


@pytest.mark.gpu
def test_fused_optimizer_kernels_match_cpu():
    torch.manual_seed(0)
    n = 3_000_001
    w = torch.randn(n)
    g = torch.randn(n) * 3
    g[17] = float("nan")
    cpu = Optimizer(torch.nn.Parameter(w.clone()), lr=1e-3, wd=0.01, clip=1.0)
    gpu = Optimizer(torch.nn.Parameter(w.clone().cuda()), lr=1e-3, wd=0.01, clip=1.0)
    for _ in range(3):
        cpu.step(g)
        gpu.step(g.cuda())
    torch.testing.assert_close(gpu.flat.data.cpu(), cpu.flat.data, rtol=1e-4, atol=1e-6)
    assert int(gpu.step_t) == 4


@pytest.mark.gpu
@needs_pi
def test_gpu_training_with_graph(tmp_path):
    data = tmp_path / "c.txt"
    data.write_text(corpus(500, seed=1))
    args = [a if a != "cpu" else "cuda" for a in SMALL]
    r = _run(["--train", "--data", str(data), "--ckpt", str(tmp_path / "g.bin"), "--steps", "30", "--batch", "8",
              "--log_every", "10", "--save_every", "0", "--measure"] + args)
    assert r.returncode == 0, r.stderr
    assert "graph capture unavailable" not in r.stderr
    losses = [float(l.split("loss=")[1].split()[0]) for l in r.stdout.splitlines() if "loss=" in l]
    assert losses[-1] < losses[0]
