"""TP lane daemon on CPU/gloo (world 2): RPC ping/generate/shutdown; tokens equal the unsharded engine's."""
import os
import subprocess
import sys
import time

import pytest
import torch

sys.path.insert(0, os.path.dirname(__file__))
from _http import free_port  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_tokens(prompts, n, sampling=None):
    from hrm_flashrenderer_b200.config import TINY, EngineConfig
    from hrm_flashrenderer_b200.models.llama import LlamaW8
    from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
    m = LlamaW8.synthesize(TINY, device="cpu", max_pos=512 + 16)
    eng = InferenceEngine(m, EngineConfig(max_seq_len=512, max_batch=8, use_cuda_graphs=False), num_blocks=256)
    return eng.generate(prompts, n, stop_on_eos=False, sampling=sampling)


def test_daemon_world2_rpc(tmp_path):
    from hrm_flashrenderer_b200.serving.daemon import DaemonAddr, client_ping, client_generate, client_shutdown
    ready = tmp_path / "ready"
    env = dict(os.environ, OMP_NUM_THREADS="2")
    p = subprocess.Popen([sys.executable, "-m", "hrm_flashrenderer_b200.serving.daemon", "--model", "synthetic:tiny",
                          "--world", "2", "--device", "cpu", "--max_seq_len", "512", "--max_batch", "8",
                          "--ready_file", str(ready), "--master_port", str(free_port()), "--num_kv_blocks", "256"],
                         cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    try:
        t0 = time.time()
        while not ready.exists():
            assert p.poll() is None, p.stdout.read().decode()[-3000:]
            assert time.time() - t0 < 180, "daemon did not start"
            time.sleep(0.2)
        host, port = ready.read_text().strip().rsplit(":", 1)
        addr = DaemonAddr(host, int(port), b"hrmflash")
        assert client_ping(addr)
        g = torch.Generator().manual_seed(3)
        prompts = [torch.randint(0, 1024, (12,), generator=g).tolist() for _ in range(2)]
        outs = [client_generate(addr, input_ids=pr, max_new_tokens=10, stop_on_eos=False)["tokens"] for pr in prompts]
        assert outs == _reference_tokens(prompts, 10)
        # a sampled request: the TP = 2 lane draws what one unsharded engine draws with the same seed
        from hrm_flashrenderer_b200.runtime.sampling import SamplingParams
        got = client_generate(addr, input_ids=prompts[0], max_new_tokens=10, stop_on_eos=False, temperature=0.9,
                              top_k=30, seed=77)["tokens"]
        assert got == _reference_tokens(prompts[:1], 10, SamplingParams(0.9, 30, 77))[0]
        assert got != outs[0]
        client_shutdown(addr)
        p.wait(timeout=120)
        assert p.returncode == 0
    finally:
        if p.poll() is None:
            p.kill()


@pytest.mark.parametrize("fused", [True, False])
def test_build_engine_enables_fused_collectives(monkeypatch, fused):
    """The lane builds its shard with the in-kernel NVLink collectives unless told to use NCCL calls (the call is
    a no-op at TP = 1 and on the CPU, so here it is only counted)."""
    from hrm_flashrenderer_b200.models.llama import LlamaW8
    from hrm_flashrenderer_b200.serving.daemon import LaneArgs, build_engine
    calls = []
    monkeypatch.setattr(LlamaW8, "enable_fused_collectives", lambda self, group=None: calls.append(group))
    a = LaneArgs("synthetic:tiny", 1, max_seq_len=256, max_batch=2, device="cpu", num_kv_blocks=64,
                 fused_collectives=fused)
    eng = build_engine(a, 0, 1, None)
    assert calls == ([None] if fused else [])
    assert len(eng.generate([[1, 2, 3]], 2, stop_on_eos=False)[0]) == 2


def test_daemon_world2_prefix_cache(tmp_path):
    """TP = 2 lane with the prefix cache: prefix matching and publication are mirrored to the follower, so both
    ranks share the same blocks, and requests sharing a prefix still get the unsharded engine's tokens."""
    from hrm_flashrenderer_b200.serving.daemon import DaemonAddr, client_generate, client_metrics, client_shutdown
    ready = tmp_path / "ready"
    env = dict(os.environ, OMP_NUM_THREADS="2")
    p = subprocess.Popen([sys.executable, "-m", "hrm_flashrenderer_b200.serving.daemon", "--model", "synthetic:tiny",
                          "--world", "2", "--device", "cpu", "--max_seq_len", "512", "--max_batch", "8",
                          "--ready_file", str(ready), "--master_port", str(free_port()), "--num_kv_blocks", "256"],
                         cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    try:
        t0 = time.time()
        while not ready.exists():
            assert p.poll() is None, p.stdout.read().decode()[-3000:]
            assert time.time() - t0 < 180, "daemon did not start"
            time.sleep(0.2)
        host, port = ready.read_text().strip().rsplit(":", 1)
        addr = DaemonAddr(host, int(port), b"hrmflash")
        g = torch.Generator().manual_seed(8)
        system = torch.randint(0, 1024, (40,), generator=g).tolist()
        prompts = [system + torch.randint(0, 1024, (5 + 3 * i,), generator=g).tolist() for i in range(3)]
        outs = [client_generate(addr, input_ids=pr, max_new_tokens=8, stop_on_eos=False)["tokens"] for pr in prompts]
        assert outs == _reference_tokens(prompts, 8)
        assert client_metrics(addr)["prefix_cache_hit_blocks"] >= 4
        client_shutdown(addr)
        p.wait(timeout=120)
        assert p.returncode == 0
    finally:
        if p.poll() is None:
            p.kill()
