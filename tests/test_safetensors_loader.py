"""Sharded safetensors reader (the reference loader interface): index and single-file checkpoints, every dtype the
checkpoints use, zero-copy views and slices, header validation, and loading the engine through it."""
import json

import pytest
import torch

from hrm_flashrenderer_b200.formats.safetensors import SafetensorsFile, WeightLoader, write_safetensors


def _tensors():
    g = torch.Generator().manual_seed(0)
    return {"a.f32": torch.randn(5, 7, generator=g),
            "b.f16": torch.randn(4, 6, generator=g).half(),
            "c.bf16": torch.randn(8, 3, generator=g).bfloat16(),
            "d.i8": torch.randint(-128, 127, (3, 9), generator=g, dtype=torch.int8),
            "e.vec": torch.randn(11, generator=g),
            "f.empty": torch.zeros(0, 4)}


def test_single_file_roundtrip_and_slices(tmp_path):
    ts = _tensors()
    write_safetensors(tmp_path / "model.safetensors", ts, metadata={"format": "pt"})
    with WeightLoader(tmp_path) as L:
        assert sorted(L.keys()) == sorted(ts)
        for k, t in ts.items():
            got = L.get(k)
            assert got.dtype == t.dtype and torch.equal(got, t), k
        assert torch.equal(L.rows("a.f32", 1, 4), ts["a.f32"][1:4])
        assert torch.equal(L.cols("c.bf16", 1, 3), ts["c.bf16"][:, 1:3])
        assert torch.equal(L.get_slice("b.f16", (slice(0, 2), slice(3, 6))), ts["b.f16"][:2, 3:])
        # views into one mapping: the same key twice shares its memory, a row slice starts inside it
        a1, a2 = L.get("a.f32"), L.get("a.f32")
        assert a1.data_ptr() == a2.data_ptr()
        assert L.rows("a.f32", 2, 3).data_ptr() == a1.data_ptr() + 2 * 7 * 4
        with pytest.raises(KeyError):
            L.get("nope")
    # a view outlives close(): the mapping goes with its last view
    keep = L.get("c.bf16")
    L.close()
    assert torch.equal(keep, ts["c.bf16"])


def test_index_over_two_shards(tmp_path):
    ts = _tensors()
    names = sorted(ts)
    write_safetensors(tmp_path / "model-00001-of-00002.safetensors", {k: ts[k] for k in names[:3]})
    write_safetensors(tmp_path / "model-00002-of-00002.safetensors", {k: ts[k] for k in names[3:]})
    wm = {k: ("model-00001-of-00002.safetensors" if k in names[:3] else "model-00002-of-00002.safetensors")
          for k in names}
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    L = WeightLoader(tmp_path)
    for k, t in ts.items():
        assert torch.equal(L.get(k), t)
    assert len(L._files) == 2
    L.close()


def test_bad_files(tmp_path):
    with pytest.raises(FileNotFoundError):
        WeightLoader(tmp_path)
    p = write_safetensors(tmp_path / "x.safetensors", {"w": torch.ones(4, 4)})
    raw = p.read_bytes()
    (tmp_path / "short.safetensors").write_bytes(raw[:-8])
    with pytest.raises(ValueError, match="do not fit"):
        SafetensorsFile(tmp_path / "short.safetensors")
    (tmp_path / "tiny.safetensors").write_bytes(b"\x01\x02")
    with pytest.raises(ValueError):
        SafetensorsFile(tmp_path / "tiny.safetensors")


def test_engine_loads_through_the_loader(tmp_path):
    """compat.llama_tp over a safetensors checkpoint gives the same tokens as loading the same weights directly."""
    from hrm_flashrenderer_b200.compat import llama_tp as lt
    from hrm_flashrenderer_b200.config import TINY
    from hrm_flashrenderer_b200.models.weights import QTensor, synth_weights
    w = synth_weights(TINY, seed=0)
    fw = {k: (v.dequant() if isinstance(v, QTensor) else v) for k, v in w.items()}
    write_safetensors(tmp_path / "model.safetensors", {k: v.to(torch.bfloat16) if v.dim() == 2 else v
                                                       for k, v in fw.items()})
    hf = {"hidden_size": 256, "num_attention_heads": 8, "num_key_value_heads": 2, "num_hidden_layers": 4,
          "intermediate_size": 688, "vocab_size": 1024, "rms_norm_eps": 1e-5, "rope_theta": 10000.0,
          "eos_token_id": 2}
    ids = torch.randint(3, 1024, (2, 10), generator=torch.Generator().manual_seed(2))
    with WeightLoader(tmp_path) as L:
        a = lt.TPLlamaForCausalLM(hf, 64, device="cpu").load_from_loader(L)
        out_a = lt.generate_tp(a, ids, 6, eos_token_id=None)
    bf = {k: (v.to(torch.bfloat16).float() if v.dim() == 2 else v) for k, v in fw.items()}
    b = lt.TPLlamaForCausalLM(hf, 64, device="cpu").load_weights(bf)
    assert torch.equal(out_a, lt.generate_tp(b, ids, 6, eos_token_id=None))


def test_from_pretrained(tmp_path):
    from hrm_flashrenderer_b200.compat import llama_tp as lt
    from hrm_flashrenderer_b200.config import TINY
    from hrm_flashrenderer_b200.models.oracle import OracleLlama
    from hrm_flashrenderer_b200.models.weights import QTensor, synth_weights
    w = synth_weights(TINY, seed=0)
    fw = {k: (v.dequant() if isinstance(v, QTensor) else v) for k, v in w.items()}
    write_safetensors(tmp_path / "model.safetensors", fw)
    (tmp_path / "config.json").write_text(json.dumps({
        "hidden_size": 256, "num_attention_heads": 8, "num_key_value_heads": 2, "num_hidden_layers": 4,
        "intermediate_size": 688, "vocab_size": 1024, "rms_norm_eps": 1e-5, "rope_theta": 10000.0,
        "eos_token_id": 2}))
    m = lt.TPLlamaForCausalLM.from_pretrained(tmp_path, 64, device="cpu")
    ids = torch.randint(3, 1024, (2, 10), generator=torch.Generator().manual_seed(2))
    out = lt.generate_tp(m, ids, 6, eos_token_id=None)
    assert out[:, 10:].tolist() == OracleLlama(TINY, w, max_pos=128).generate(ids.tolist(), 6)
