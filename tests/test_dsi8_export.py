"""HF checkpoint -> DSI8 export (streamed from safetensors shards): Llama-style with a separate lm_head and bf16
weights over two shards, Qwen2-style with q/k/v biases, tied embeddings; every record equals the per-row int8
quantisation of the source tensor, and the engine built from the export matches the oracle of the same weights."""
import json

import pytest
import torch

from hrm_flashrenderer_b200.config import TINY
from hrm_flashrenderer_b200.formats.dsi8 import DSI8File, export_dsi8, read_dsi8
from hrm_flashrenderer_b200.formats.safetensors import write_safetensors
from hrm_flashrenderer_b200.models.weights import QTensor, layer_names, quantize_rows, synth_weights

HF = {"hidden_size": 256, "num_attention_heads": 8, "num_key_value_heads": 2, "num_hidden_layers": 2,
      "intermediate_size": 688, "vocab_size": 1024, "rms_norm_eps": 1e-5, "rope_theta": 10000.0,
      "eos_token_id": [2, 5], "bos_token_id": 1, "max_position_embeddings": 2048,
      "architectures": ["LlamaForCausalLM"], "model_type": "llama"}


def _float(cfg, seed=0, bias=False):
    w = synth_weights(cfg, seed=seed)
    out = {k: (v.dequant() if isinstance(v, QTensor) else v) for k, v in w.items()}
    if bias:
        g = torch.Generator().manual_seed(9)
        for l in range(cfg.layers):
            n = layer_names(l)
            out[n["bq"]] = torch.randn(cfg.q_dim, generator=g)
            out[n["bk"]] = torch.randn(cfg.kv_dim, generator=g)
            out[n["bv"]] = torch.randn(cfg.kv_dim, generator=g)
    return out


def _hf_dir(tmp_path, hf, tensors, shards=1, dtype=torch.bfloat16):
    d = tmp_path / "hf"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hf))
    names = sorted(tensors)
    for i in range(shards):
        part = {k: (tensors[k].to(dtype) if tensors[k].dim() == 2 else tensors[k]) for k in names[i::shards]}
        write_safetensors(d / f"model-{i + 1:05d}-of-{shards:05d}.safetensors", part)
    return d


def _check(path, src, dtype=torch.bfloat16):
    with DSI8File(path) as f:
        f.check()
        for k, v in src.items():
            got = f.get(k)
            if v.dim() == 2:
                ref = quantize_rows(v.to(dtype).float())
                assert torch.equal(got.q, ref.q) and torch.equal(got.scale, ref.scale), k
            else:
                assert torch.equal(got, v.float()), k


def test_llama_two_shards_bf16(tmp_path):
    cfg = TINY.with_layers(2)
    src = _float(cfg)
    d = _hf_dir(tmp_path, HF, src, shards=2)
    p = export_dsi8(d, tmp_path / "m.bin")
    _check(p, src)
    c2, _ = read_dsi8(p)
    assert c2.eos_token_ids == (2, 5) and c2.max_position_embeddings == 2048 and not c2.tie_embeddings


def test_qwen_biases_and_tied_embeddings(tmp_path):
    hf = dict(HF, architectures=["Qwen2ForCausalLM"], model_type="qwen2", tie_word_embeddings=True)
    from dataclasses import replace
    cfg = replace(TINY.with_layers(2), qkv_bias=True, tie_embeddings=True)
    src = _float(cfg, bias=True)
    src.pop("lm_head.weight", None)
    d = _hf_dir(tmp_path, hf, src, dtype=torch.float16)
    p = export_dsi8(d, tmp_path / "q.bin")
    _check(p, src, dtype=torch.float16)
    c2, w2 = read_dsi8(p)
    assert c2.qkv_bias and c2.tie_embeddings and "lm_head.weight" not in w2


def test_engine_from_export_matches_oracle(tmp_path):
    from hrm_flashrenderer_b200.models.llama import LlamaW8
    from hrm_flashrenderer_b200.models.oracle import OracleLlama
    from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
    from hrm_flashrenderer_b200.config import EngineConfig
    cfg = TINY.with_layers(2)
    src = _float(cfg)
    p = export_dsi8(_hf_dir(tmp_path, HF, src, dtype=torch.float32), tmp_path / "m.bin")
    model = LlamaW8.from_dsi8(str(p), device="cpu", max_pos=128)
    eng = InferenceEngine(model, EngineConfig(max_seq_len=96, max_batch=2, use_cuda_graphs=False), num_blocks=16)
    prompts = [[5, 9, 100, 7, 3], [44, 2, 900]]
    ref = OracleLlama(model.cfg, read_dsi8(p)[1], max_pos=128).generate(prompts, 6)
    assert eng.generate(prompts, 6, stop_on_eos=False) == ref


def test_rejects_q4_and_empty_dirs(tmp_path):
    d = tmp_path / "e"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(HF))
    with pytest.raises(ValueError):
        export_dsi8(d, tmp_path / "x.bin", quant="q4")
    with pytest.raises(RuntimeError, match="no safetensors"):
        export_dsi8(d, tmp_path / "x.bin")
