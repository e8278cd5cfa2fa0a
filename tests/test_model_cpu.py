"""CPU numerics: quantisation rule, DSI8 round trip, the engine's CPU path vs the fp32 oracle."""
import numpy as np
import torch

from hrm_flashrenderer_b200.config import TINY, LLAMA31_70B, rope_inv_freq
from hrm_flashrenderer_b200.formats.dsi8 import write_dsi8, read_dsi8
from hrm_flashrenderer_b200.models.oracle import OracleLlama
from hrm_flashrenderer_b200.models.weights import quantize_rows, synth_weights, QTensor
from hrm_flashrenderer_b200.models.llama import LlamaW8
from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
from hrm_flashrenderer_b200.config import EngineConfig


def test_quantize_rule_matches_exporter_semantics():
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, size=(7, 33)).astype(np.float32)
    w[3] = 0.0                                           # all-zero row -> absmax clamp 1e-8
    absmax = np.maximum(np.abs(w).max(axis=-1), 1e-8)
    scale = absmax / 127.0
    q_ref = np.clip(np.round(w / scale[:, None]), -128, 127).astype(np.int8)
    qt = quantize_rows(torch.from_numpy(w))
    assert np.array_equal(qt.q.numpy(), q_ref)
    assert np.allclose(qt.scale.numpy(), scale.astype(np.float32))


def test_dsi8_roundtrip(tmp_path):
    cfg = TINY.with_layers(2)
    w = synth_weights(cfg, seed=3)
    p = write_dsi8(tmp_path / "m.bin", cfg, w)
    cfg2, w2 = read_dsi8(p)
    assert (cfg2.hidden, cfg2.layers, cfg2.heads, cfg2.kv_heads, cfg2.head_dim, cfg2.intermediate, cfg2.vocab) == \
        (cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab)
    assert set(w2) == set(w)
    for k, v in w.items():
        if isinstance(v, QTensor):
            assert torch.equal(v.q, w2[k].q) and torch.equal(v.scale, w2[k].scale)
        else:
            assert torch.equal(v, w2[k])
    # header is the reference layout: magic, version, 8 x u32, f64, f32, 2 x u32
    raw = open(p, "rb").read(60)
    assert raw[:4] == b"DSI8"
    assert np.frombuffer(raw[8:40], dtype=np.uint32).tolist() == [256, 8, 2, 32, 688, 1024, 2, cfg.max_position_embeddings]


def test_llama3_rope_scaling_bands():
    inv = rope_inv_freq(LLAMA31_70B)
    base = [1.0 / (500000.0 ** (2 * i / 128)) for i in range(64)]
    assert inv[0] == base[0]                      # high frequency: unchanged
    assert abs(inv[-1] - base[-1] / 8.0) < 1e-18  # low frequency: divided by factor


def _engine(cfg, w, **kw):
    model = LlamaW8.from_weights(cfg, w, device="cpu", max_pos=256)
    return InferenceEngine(model, EngineConfig(max_seq_len=128, max_batch=4, use_cuda_graphs=False, **kw),
                           num_blocks=64)


def test_cpu_engine_matches_oracle_tokens():
    cfg = TINY.with_layers(2)
    w = synth_weights(cfg, seed=0, norm_jitter=0.1)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab, (12,), generator=g).tolist() for _ in range(2)]
    ref = OracleLlama(cfg, w, max_pos=256).generate(prompts, 8)
    got = _engine(cfg, w).generate(prompts, 8, stop_on_eos=False)
    assert got == ref


def test_chunked_prefill_equals_single_chunk():
    cfg = TINY.with_layers(2)
    w = synth_weights(cfg, seed=5)
    prompts = [list(range(3, 40)), list(range(100, 121))]
    a = _engine(cfg, w, prefill_chunk=7).generate(prompts, 5, stop_on_eos=False)
    b = _engine(cfg, w, prefill_chunk=4096).generate(prompts, 5, stop_on_eos=False)
    assert a == b


def test_eos_stops_generation():
    cfg = TINY.with_layers(1)
    w = synth_weights(cfg, seed=2)
    eng = _engine(cfg, w)
    free = eng.generate([[5, 6, 7]], 6, stop_on_eos=False)[0]
    stop = eng.generate([[5, 6, 7]], 6, stop_on_eos=True, eos_ids=[free[2]])[0]
    assert stop == free[:3]


def test_tile_w8_roundtrip_and_layout():
    from hrm_flashrenderer_b200 import ops
    g = torch.Generator().manual_seed(0)
    q = torch.randint(-128, 128, (300, 192), dtype=torch.int8, generator=g)
    t = ops.tile_w8(q)
    assert t.shape == (3, 3, 8192)
    assert torch.equal(ops.untile_w8(t, 300), q)
    # block (n=1, k=2) is chunk-major: [chunk c][row r][16 bytes]
    blk = t[1, 2].view(4, 128, 16)
    for c in range(4):
        assert torch.equal(blk[c, 5], q[128 + 5, 128 + 16 * c:128 + 16 * c + 16])
    assert int(t[2, 0].view(4, 128, 16)[:, 300 - 256:].abs().sum()) == 0   # padded rows are zero
