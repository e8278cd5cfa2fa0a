"""Service helpers: locating the ``hrm`` binary and validating models for the native TP engine.

Reference: ``hrm_flash/utils.py:12-207`` (``find_hrm_binary``, ``validate_tp_world``,
``validate_native_model_config``, ``validate_native_weight_layout``).
"""
from __future__ import annotations

import json
import os
import shutil
from pathlib import Path
from typing import Any, Optional

REPO_ROOT = Path(__file__).resolve().parents[2]


def find_hrm_binary(repo_root: Optional[Path] = None, explicit: Optional[str] = None) -> Path:
    """explicit -> $HRM_BIN -> PATH -> <repo>/hrm_core/build/hrm -> ./hrm_core/build/hrm -> ../hrm_core/build/hrm."""
    if explicit:
        return Path(explicit).expanduser().resolve()
    if os.environ.get("HRM_BIN"):
        return Path(os.environ["HRM_BIN"]).expanduser().resolve()
    w = shutil.which("hrm")
    if w:
        return Path(w).resolve()
    for root in (repo_root, REPO_ROOT, Path.cwd(), Path.cwd().parent):
        if root is not None:
            c = Path(root) / "hrm_core" / "build" / "hrm"
            if c.is_file():
                return c.resolve()
    return Path("hrm")


def _get(cfg: Any, name: str, default=None):
    if isinstance(cfg, dict):
        return cfg.get(name, default)
    return getattr(cfg, name, default)


def validate_tp_world(config: Any, world: int) -> None:
    hidden = int(_get(config, "hidden_size"))
    heads = int(_get(config, "num_attention_heads"))
    inter = int(_get(config, "intermediate_size", hidden * 4))
    vocab = int(_get(config, "vocab_size"))
    for name, v in (("hidden_size", hidden), ("num_attention_heads", heads), ("intermediate_size", inter),
                    ("vocab_size", vocab)):
        if v % world:
            raise ValueError(f"TP world={world} invalid: {name}={v} not divisible by world")


def validate_native_model_config(config: Any) -> None:
    """Dense Llama/Qwen2 decoders with head_dim 64 or 128 only; MoE / DeepSeek-V3 are rejected."""
    hidden = int(_get(config, "hidden_size"))
    heads = int(_get(config, "num_attention_heads"))
    head_dim = int(_get(config, "head_dim", 0) or 0) or (hidden // heads if hidden % heads == 0 else 0)
    if not head_dim:
        raise ValueError(f"Invalid model config: hidden_size={hidden} not divisible by num_attention_heads={heads}")
    if head_dim not in (64, 128):
        raise ValueError(f"Unsupported head_dim={head_dim}: the attention kernels support head_dim 64 or 128 only.")
    archs = [str(a).lower() for a in (_get(config, "architectures") or [])]
    if any("moe" in a for a in archs):
        raise ValueError("MoE architecture detected: only dense models are supported.")
    if any("deepseekv3" in a or "deepseek_v3" in a for a in archs):
        raise ValueError("DeepSeek-V3 (MoE) architecture detected: only dense distill variants are supported.")
    for name in ("num_local_experts", "n_routed_experts", "num_experts"):
        v = _get(config, name)
        try:
            if v is not None and int(v) > 1:
                raise ValueError(f"MoE config detected via {name}={int(v)}: only dense models are supported.")
        except (TypeError, ValueError) as e:
            if "MoE" in str(e):
                raise


REQUIRED_KEYS = [
    "model.embed_tokens.weight",
    "model.layers.0.self_attn.q_proj.weight", "model.layers.0.self_attn.k_proj.weight",
    "model.layers.0.self_attn.v_proj.weight", "model.layers.0.self_attn.o_proj.weight",
    "model.layers.0.mlp.gate_proj.weight", "model.layers.0.mlp.up_proj.weight",
    "model.layers.0.mlp.down_proj.weight", "model.layers.0.input_layernorm.weight",
    "model.layers.0.post_attention_layernorm.weight", "model.norm.weight",
]


def validate_native_weight_layout(model_dir) -> None:
    model_dir = Path(model_dir).resolve()
    idx, single = model_dir / "model.safetensors.index.json", model_dir / "model.safetensors"
    if idx.is_file():
        keys = set((json.loads(idx.read_text()).get("weight_map") or {}).keys())
    elif single.is_file():
        import struct
        with single.open("rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            keys = set(json.loads(f.read(n)).keys())
    else:
        raise ValueError("No safetensors weights found (model.safetensors or model.safetensors.index.json).")
    missing = [k for k in REQUIRED_KEYS if k not in keys]
    if missing:
        raise ValueError(f"Weights are not a dense Llama/Qwen layout; first missing key: {missing[0]}")
