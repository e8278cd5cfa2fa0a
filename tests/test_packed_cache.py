"""Packed-shard cache: a DSI8 export loads once, later loads come from the per-rank cache with identical results."""
from dataclasses import replace

import torch

from hrm_flashrenderer_b200.config import TINY, EngineConfig, ModelConfig
from hrm_flashrenderer_b200.formats.dsi8 import write_dsi8
from hrm_flashrenderer_b200.models.llama import LlamaW8
from hrm_flashrenderer_b200.models.packed_cache import cache_path
from hrm_flashrenderer_b200.models.weights import synth_weights
from hrm_flashrenderer_b200.runtime.engine import InferenceEngine


def _gen(model):
    eng = InferenceEngine(model, EngineConfig(max_seq_len=64, max_batch=2, use_cuda_graphs=False), num_blocks=16)
    return eng.generate([[5, 9, 200, 31], [7, 7, 7]], 6, stop_on_eos=False)


def test_cache_round_trip(tmp_path, monkeypatch):
    cfg = replace(TINY, qkv_bias=True)
    src = tmp_path / "m.bin"
    write_dsi8(src, cfg, synth_weights(cfg, seed=3))
    cache = tmp_path / "cache"
    a = LlamaW8.from_dsi8(str(src), device="cpu", max_pos=128, cache_dir=str(cache))
    cp = cache_path(str(cache), str(src), 0, 1, "cpu")
    assert cp.is_file()
    # the second load must not read the export
    import hrm_flashrenderer_b200.formats.dsi8 as dsi8
    monkeypatch.setattr(dsi8, "read_dsi8", lambda *a, **k: (_ for _ in ()).throw(AssertionError("export read")))
    b = LlamaW8.from_dsi8(str(src), device="cpu", max_pos=128, cache_dir=str(cache))
    assert b.cfg == a.cfg and b.plan == a.plan
    assert torch.equal(b.layers[1].w_gu, a.layers[1].w_gu) and torch.equal(b.layers[0].b_qkv, a.layers[0].b_qkv)
    assert _gen(a) == _gen(b)


def test_cache_key_tracks_source_and_layout(tmp_path):
    src = tmp_path / "m.bin"
    write_dsi8(src, TINY, synth_weights(TINY, seed=0))
    k = {cache_path(str(tmp_path), str(src), r, w, "cpu") for r, w in ((0, 1), (0, 2), (1, 2))}
    assert len(k) == 3
    assert cache_path(str(tmp_path), str(src), 0, 1, "cpu") != cache_path(str(tmp_path), str(src), 0, 1, "cuda")
    before = cache_path(str(tmp_path), str(src), 0, 1, "cpu")
    write_dsi8(src, TINY, synth_weights(TINY, seed=1))   # a new export at the same path
    assert cache_path(str(tmp_path), str(src), 0, 1, "cpu") != before


def test_config_dict_round_trip():
    from hrm_flashrenderer_b200.config import LLAMA31_70B
    assert ModelConfig.from_dict(LLAMA31_70B.to_dict()) == LLAMA31_70B
