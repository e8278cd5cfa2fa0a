"""Multi-phase decode GEMM chain (o_proj -> gate/up -> down -> next QKV in one launch).

CPU: the model's chained decode path (ops run phase by phase) gives the same tokens as the per-GEMM path.
GPU: the cooperative multi-phase kernel against the single-GEMM kernels.  The GPU tests run when HRM_TEST_CHAIN=1:
the f16 pair matched the single launches bitwise at M = 1 and 16 on a B200; the decode-layer sequence has not run
on a GPU yet, and M 33..64 (BN = 64) is rejected after a timeout on its first run."""
import os

import pytest
import torch

from hrm_flashrenderer_b200 import ops
from hrm_flashrenderer_b200.config import TINY, EngineConfig
from hrm_flashrenderer_b200.models.llama import LlamaW8
from hrm_flashrenderer_b200.models.weights import synth_weights
from hrm_flashrenderer_b200.runtime.engine import InferenceEngine

RUN_GPU = os.environ.get("HRM_TEST_CHAIN", "0") == "1"


def _prompts(n, L, vocab, seed=1):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (L,), generator=g).tolist() for _ in range(n)]


def _generate(cfg, w, chain, device="cpu", graphs=False):
    model = LlamaW8.from_weights(cfg, w, device=device, max_pos=256)
    eng = InferenceEngine(model, EngineConfig(max_seq_len=128, max_batch=4, use_cuda_graphs=graphs,
                                              chain_layers=chain), num_blocks=32)
    return eng.generate(_prompts(3, 20, cfg.vocab), 12, stop_on_eos=False)


def test_cpu_chained_decode_matches_per_gemm_path():
    w = synth_weights(TINY, seed=0)
    assert _generate(TINY, w, True) == _generate(TINY, w, False)


@pytest.mark.gpu
@pytest.mark.skipif(not RUN_GPU, reason="set HRM_TEST_CHAIN=1 to run the multi-phase kernel")
@pytest.mark.parametrize("M", [1, 16, 32])
def test_gpu_chain_f16_pair_matches_two_launches(M):
    dev = "cuda"
    g = torch.Generator(device="cpu").manual_seed(M)
    K1, N1, N2 = 4096, 2048, 3072
    w1 = torch.randint(-127, 128, (N1, K1), generator=g, dtype=torch.int8).to(dev)
    w2 = torch.randint(-127, 128, (N2, N1), generator=g, dtype=torch.int8).to(dev)
    s1 = (torch.rand(N1, generator=g) * 1e-3).to(dev)
    s2 = (torch.rand(N2, generator=g) * 1e-3).to(dev)
    x = torch.randn(M, K1, generator=g).half().to(dev)
    t1, t2 = ops.tile_w8(w1), ops.tile_w8(w2)
    y1 = torch.empty(M, N1, dtype=torch.float16, device=dev)
    y2 = torch.empty(M, N2, dtype=torch.float16, device=dev)
    r1 = torch.empty_like(y1)
    r2 = torch.empty_like(y2)
    ops.w8a16_linear_out(x, t1, s1, r1)
    ops.w8a16_linear_out(r1, t2, s2, r2)
    for _ in range(3):   # repeated launches: barrier counters re-armed
        ops.w8a16_chain([("f16", x, t1, s1, y1, None, 1.0, 0.0), ("f16", y1, t2, s2, y2, None, 1.0, 0.0)])
        ops.check_status()
        assert torch.equal(y1, r1) and torch.equal(y2, r2)


@pytest.mark.gpu
@pytest.mark.skipif(not RUN_GPU, reason="set HRM_TEST_CHAIN=1 to run the multi-phase kernel")
@pytest.mark.parametrize("graphs", [False, True])
def test_gpu_chained_decode_matches_per_gemm_path(graphs):
    from hrm_flashrenderer_b200.config import ModelConfig, RopeScaling
    cfg = ModelConfig(name="gpu-small", hidden=1024, layers=3, heads=8, kv_heads=2, head_dim=128, intermediate=2816,
                      vocab=4096, rms_eps=1e-5, rope_theta=500000.0, rope_scaling=RopeScaling(8.0, 1.0, 4.0, 8192),
                      max_position_embeddings=8192)
    w = synth_weights(cfg, seed=2)
    a = _generate(cfg, w, True, "cuda", graphs)
    ops.check_status()
    assert a == _generate(cfg, w, False, "cuda", graphs)
