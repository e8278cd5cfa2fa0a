"""End-to-end GPU model vs the CPU fp32 oracle, CUDA-graph decode vs eager decode."""
from dataclasses import replace

import pytest
import torch

from hrm_flashrenderer_b200.config import ModelConfig, EngineConfig, RopeScaling
from hrm_flashrenderer_b200.models.oracle import OracleLlama
from hrm_flashrenderer_b200.models.weights import synth_weights
from hrm_flashrenderer_b200.models.llama import LlamaW8
from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
from hrm_flashrenderer_b200 import ops

pytestmark = pytest.mark.gpu

# Production head_dim / GQA / llama3-RoPE features at a size the CPU oracle handles quickly.
SMALL = ModelConfig(name="gpu-small", hidden=1024, layers=2, heads=8, kv_heads=2, head_dim=128, intermediate=2816,
                    vocab=4096, rms_eps=1e-5, rope_theta=500000.0, rope_scaling=RopeScaling(8.0, 1.0, 4.0, 8192),
                    max_position_embeddings=8192)
SMALL_QWEN = replace(SMALL, name="gpu-small-qwen", qkv_bias=True, heads=10, kv_heads=2, rope_scaling=None,
                     rope_theta=1e6, hidden=1280)


def _prompts(n, L, vocab, seed=1):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (L,), generator=g).tolist() for _ in range(n)]


@pytest.mark.parametrize("cfg", [SMALL, SMALL_QWEN], ids=lambda c: c.name)
@pytest.mark.parametrize("graphs", [True, False])
def test_gpu_engine_matches_oracle(cfg, graphs):
    w = synth_weights(cfg, seed=0, norm_jitter=0.1)
    prompts = _prompts(3, 40, cfg.vocab)
    ref = OracleLlama(cfg, w, max_pos=512).generate(prompts, 12)
    model = LlamaW8.from_weights(cfg, w, device="cuda", max_pos=512)
    eng = InferenceEngine(model, EngineConfig(max_seq_len=256, max_batch=4, use_cuda_graphs=graphs), num_blocks=128)
    got = eng.generate(prompts, 12, stop_on_eos=False)
    # greedy tokens must agree with the fp32 oracle (f16 GEMM operands / bf16 KV: allow a late divergence only)
    for a, b in zip(got, ref):
        n = next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), len(a))
        assert n >= 8, (a, b)


def test_gpu_engine_deterministic_and_graph_equals_eager():
    cfg = SMALL
    w = synth_weights(cfg, seed=1)
    prompts = _prompts(5, 33, cfg.vocab, seed=2)
    outs = []
    for graphs in (True, True, False):
        model = LlamaW8.from_weights(cfg, w, device="cuda", max_pos=512)
        eng = InferenceEngine(model, EngineConfig(max_seq_len=256, max_batch=8, use_cuda_graphs=graphs),
                              num_blocks=128)
        outs.append(eng.generate(prompts, 16, stop_on_eos=False))
    assert outs[0] == outs[1] == outs[2]


def test_prefill_logits_identical_across_engine_instances():
    """Two engines built one after the other in one process produce bitwise-identical prefill tokens and decode."""
    cfg = SMALL
    w = synth_weights(cfg, seed=1)
    prompts = _prompts(5, 33, cfg.vocab, seed=2)
    firsts = []
    for _ in range(3):
        model = LlamaW8.from_weights(cfg, w, device="cuda", max_pos=512)
        eng = InferenceEngine(model, EngineConfig(max_seq_len=256, max_batch=8, use_cuda_graphs=False),
                              num_blocks=128)
        sids = [eng.new_seq() for _ in prompts]
        firsts.append(eng.prefill(list(zip(sids, prompts))))
        from hrm_flashrenderer_b200 import ops
        ops.check_status()
    assert firsts[0] == firsts[1] == firsts[2]


def test_synthesize_on_device_shapes():
    cfg = replace(SMALL, layers=1)
    m = LlamaW8.synthesize(cfg, device="cuda")
    L = m.layers[0]
    # GPU weights are pre-tiled: [N/128, K/64, 8192]
    assert ops.weight_nk(L.w_qkv, L.s_qkv) == (cfg.q_dim + 2 * cfg.kv_dim, cfg.hidden)
    assert ops.weight_nk(L.w_gu, L.s_gu) == (2 * cfg.intermediate, cfg.hidden)
    assert L.w_qkv.shape == ((cfg.q_dim + 2 * cfg.kv_dim) // 128, cfg.hidden // 64, 8192)
    assert m.weight_bytes() > 0


@pytest.mark.parametrize("graphs", [True, False])
def test_programmatic_dependent_launch_on_off_identical(graphs):
    """Decode with programmatic dependent launch (early weight / KV prefetch before the previous grid ends) gives the
    same tokens as plain stream order; contexts span several 128-key tiles so attention runs split and prefetches."""
    cfg = SMALL
    w = synth_weights(cfg, seed=3)
    prompts = _prompts(4, 300, cfg.vocab, seed=5)
    outs = []
    try:
        for on in (False, True, True):
            ops.ext().set_pdl(on)
            model = LlamaW8.from_weights(cfg, w, device="cuda", max_pos=1024)
            eng = InferenceEngine(model, EngineConfig(max_seq_len=512, max_batch=4, use_cuda_graphs=graphs),
                                  num_blocks=160)
            outs.append(eng.generate(prompts, 24, stop_on_eos=False))
            ops.check_status()
    finally:
        ops.ext().set_pdl(True)
    assert outs[0] == outs[1] == outs[2]
