"""Prefix cache on the GPU: requests that share a system prefix reuse its KV blocks (prefill starts after them, the
prefill attention reads the shared blocks through the block table) and continue like runs without the cache."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_prefix_cache_matches_isolated_runs_on_gpu():
    from hrm_flashrenderer_b200 import ops
    from hrm_flashrenderer_b200.config import EngineConfig, ModelConfig
    from hrm_flashrenderer_b200.models.llama import LlamaW8
    from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
    cfg = ModelConfig(name="gpu-prefix", hidden=1024, layers=2, heads=8, kv_heads=2, head_dim=128,
                      intermediate=2816, vocab=4096, rms_eps=1e-5, rope_theta=500000.0)
    g = torch.Generator().manual_seed(4)
    system = torch.randint(0, 4096, (160,), generator=g).tolist()
    prompts = [system + torch.randint(0, 4096, (n,), generator=g).tolist() for n in (9, 33, 70)]
    model = LlamaW8.synthesize(cfg, device="cuda", max_pos=512 + 16)
    outs = {}
    for pc in (False, True):
        eng = InferenceEngine(model, EngineConfig(max_seq_len=512, max_batch=4, prefix_cache=pc), num_blocks=128)
        outs[pc] = [eng.generate([p], 12, stop_on_eos=False)[0] for p in prompts]
        if pc:
            assert eng.bm.prefix_hits >= 2 * 10
    ops.check_status()
    # the shared blocks were computed in another batch (another GEMM split of the prompt rows), so late greedy
    # near-ties may flip; a wrong block table or stale KV would change the first tokens
    for a, b in zip(outs[True], outs[False]):
        same = next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), len(a))
        assert same >= 6, (a, b)
