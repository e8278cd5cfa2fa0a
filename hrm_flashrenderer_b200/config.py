"""Typed model / engine configuration with the architecture presets this framework is benchmarked on.

One dataclass replaces the scattered ``getattr(config, ...)`` reads of the reference torch path
(``engine/llama_tp.py:246-258``) and the fixed header fields of the DSI8 exporter
(``hrm_flash/deepseek_export.py:130-141``).  Unlike the exporter, ``max_position_embeddings`` and EOS
lists are taken from the HF config instead of being hard-coded (reference quirk: ``Tmax=4096`` and
``eos_token_id`` assumed to be an int, ``deepseek_export.py:135,139``).
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, field, asdict, replace
from pathlib import Path
from typing import Optional, Sequence


@dataclass(frozen=True)
class RopeScaling:
    """Llama-3 style frequency-dependent RoPE scaling (``rope_type == "llama3"``)."""

    factor: float = 8.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 4.0
    original_max_position_embeddings: int = 8192


@dataclass(frozen=True)
class ModelConfig:
    """Dense Llama / Qwen2 decoder description.

    ``qkv_bias`` is the Qwen2 q/k/v bias (the reference torch path drops it, ``engine/llama_tp.py:127-143``).
    ``head_dim`` is explicit so that configs with ``hidden != heads * head_dim`` are representable.
    """

    name: str = "tiny"
    hidden: int = 256
    layers: int = 4
    heads: int = 8
    kv_heads: int = 2
    head_dim: int = 32
    intermediate: int = 688
    vocab: int = 1024
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_scaling: Optional[RopeScaling] = None
    qkv_bias: bool = False
    tie_embeddings: bool = False
    max_position_embeddings: int = 4096
    bos_token_id: int = 1
    eos_token_ids: tuple = (2,)

    # ---- derived -------------------------------------------------------------------------------
    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def group(self) -> int:
        return self.heads // self.kv_heads

    def param_count(self) -> int:
        per_layer = (self.hidden * (self.q_dim + 2 * self.kv_dim) + self.q_dim * self.hidden
                     + 3 * self.hidden * self.intermediate + 2 * self.hidden)
        if self.qkv_bias:
            per_layer += self.q_dim + 2 * self.kv_dim
        head = 0 if self.tie_embeddings else self.vocab * self.hidden
        return self.layers * per_layer + self.vocab * self.hidden + head + self.hidden

    def validate_tp(self, world: int) -> None:
        """Divisibility rules for Megatron-style TP (reference: ``hrm_flash/utils.py:100-118``).

        KV heads may be replicated when ``kv_heads % world != 0`` (``engine/llama_tp.py:129-141``), but only
        if every rank's query heads map onto the replicated set, which holds when ``heads % world == 0``.
        """
        problems = []
        if self.hidden % world:
            problems.append(f"hidden={self.hidden}")
        if self.heads % world:
            problems.append(f"heads={self.heads}")
        if self.intermediate % world:
            problems.append(f"intermediate={self.intermediate}")
        if self.vocab % world:
            problems.append(f"vocab={self.vocab}")
        if self.heads % self.kv_heads:
            problems.append(f"heads={self.heads} not a multiple of kv_heads={self.kv_heads}")
        if problems:
            raise ValueError(f"model {self.name!r} is not shardable over world={world}: " + ", ".join(problems))

    def with_layers(self, layers: int) -> "ModelConfig":
        return replace(self, layers=int(layers), name=f"{self.name}-L{layers}")

    def to_dict(self) -> dict:
        d = asdict(self)
        d["eos_token_ids"] = list(self.eos_token_ids)
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "ModelConfig":
        """Inverse of :meth:`to_dict`."""
        d = dict(d)
        rs = d.get("rope_scaling")
        if isinstance(rs, dict):
            d["rope_scaling"] = RopeScaling(**rs)
        d["eos_token_ids"] = tuple(d.get("eos_token_ids", (2,)))
        return cls(**d)

    # ---- HF config.json ------------------------------------------------------------------------
    @classmethod
    def from_hf_config(cls, cfg: dict, name: str = "hf") -> "ModelConfig":
        hidden = int(cfg["hidden_size"])
        heads = int(cfg["num_attention_heads"])
        kv = int(cfg.get("num_key_value_heads", heads))
        head_dim = int(cfg.get("head_dim") or hidden // heads)
        rs = cfg.get("rope_scaling") or None
        scaling = None
        if isinstance(rs, dict) and (rs.get("rope_type") or rs.get("type")) == "llama3":
            scaling = RopeScaling(
                factor=float(rs.get("factor", 8.0)),
                low_freq_factor=float(rs.get("low_freq_factor", 1.0)),
                high_freq_factor=float(rs.get("high_freq_factor", 4.0)),
                original_max_position_embeddings=int(rs.get("original_max_position_embeddings", 8192)),
            )
        eos = cfg.get("eos_token_id", 2)
        eos_ids = tuple(int(e) for e in eos) if isinstance(eos, (list, tuple)) else (int(eos),)
        arch = " ".join(cfg.get("architectures") or [])
        qkv_bias = bool(cfg.get("attention_bias", False)) or "Qwen2" in arch or cfg.get("model_type") == "qwen2"
        return cls(
            name=name,
            hidden=hidden,
            layers=int(cfg["num_hidden_layers"]),
            heads=heads,
            kv_heads=kv,
            head_dim=head_dim,
            intermediate=int(cfg["intermediate_size"]),
            vocab=int(cfg["vocab_size"]),
            rms_eps=float(cfg.get("rms_norm_eps", 1e-6)),
            rope_theta=float(cfg.get("rope_theta", 10000.0)),
            rope_scaling=scaling,
            qkv_bias=qkv_bias,
            tie_embeddings=bool(cfg.get("tie_word_embeddings", False)),
            max_position_embeddings=int(cfg.get("max_position_embeddings", 4096)),
            bos_token_id=int(cfg.get("bos_token_id", 1) or 1),
            eos_token_ids=eos_ids,
        )

    @classmethod
    def from_hf_dir(cls, path: str | Path) -> "ModelConfig":
        p = Path(path)
        return cls.from_hf_config(json.loads((p / "config.json").read_text()), name=p.name)


# ------------------------------------------------------------------------------------------------
# Presets (the architectures named by the benchmark configs)
# ------------------------------------------------------------------------------------------------
TINY = ModelConfig()

QWEN25_32B = ModelConfig(
    name="qwen2.5-32b", hidden=5120, layers=64, heads=40, kv_heads=8, head_dim=128,
    intermediate=27648, vocab=152064, rms_eps=1e-6, rope_theta=1e6, qkv_bias=True,
    max_position_embeddings=32768, bos_token_id=151643, eos_token_ids=(151643, 151645),
)

LLAMA31_70B = ModelConfig(
    name="llama3.1-70b", hidden=8192, layers=80, heads=64, kv_heads=8, head_dim=128,
    intermediate=28672, vocab=128256, rms_eps=1e-5, rope_theta=500000.0,
    rope_scaling=RopeScaling(8.0, 1.0, 4.0, 8192), max_position_embeddings=131072,
    bos_token_id=128000, eos_token_ids=(128001, 128008, 128009),
)

# A 1-2 layer GPU-testable slice with production widths (used by numerics tests / smoke).
LLAMA70B_SLICE = LLAMA31_70B.with_layers(2)

PRESETS = {
    "tiny": TINY,
    "qwen2.5-32b": QWEN25_32B,
    "qwen32b": QWEN25_32B,
    "llama3.1-70b": LLAMA31_70B,
    "llama70b": LLAMA31_70B,
}


def get_preset(name: str) -> ModelConfig:
    key = name.strip().lower()
    if key not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[key]


@dataclass
class EngineConfig:
    """Runtime knobs of the inference engine (KV cache, batching, chunked prefill, graph capture)."""

    tp: int = 1
    block_size: int = 16                 # paged-KV block (tokens)
    max_seq_len: int = 8192
    max_batch: int = 64
    prefill_chunk: int = 4096            # tokens per chunked-prefill step
    num_kv_blocks: Optional[int] = None  # default: sized from max_batch * max_seq_len
    use_cuda_graphs: bool = True
    graph_batch_buckets: Sequence[int] = field(default_factory=lambda: (1, 2, 4, 8, 16, 32, 64))
    fused_collectives: bool = True       # False -> NCCL all-reduce after the local GEMM (baseline path)
    sequence_parallel: bool = False      # prefill with a token-sharded residual stream (TP > 1)
    chain_layers: bool = False           # decode: o_proj..next QKV as one multi-phase GEMM launch
    prefill_overlap_chunks: int = 1      # TP prefill (NCCL path): row-parallel GEMM / all-reduce pipelined in chunks
    prefix_cache: bool = False           # share the KV blocks of a prompt prefix seen before (shared system prompts)
    seed: int = 0


def rope_inv_freq(cfg: ModelConfig) -> "list[float]":
    """Per-pair inverse frequencies, HF semantics, including llama3 scaling.

    Computed in float64 on the host; the result is cast by the caller.  llama3 scaling follows the published
    Llama-3.1 recipe: long wavelengths (> original_ctx/low_freq_factor) are divided by ``factor``, short ones
    (< original_ctx/high_freq_factor) are kept, and the band in between is linearly blended in
    ``original_ctx / wavelen``.
    """
    half = cfg.head_dim // 2
    inv = [1.0 / (cfg.rope_theta ** (2.0 * i / cfg.head_dim)) for i in range(half)]
    s = cfg.rope_scaling
    if s is None:
        return inv
    low_wl = s.original_max_position_embeddings / s.low_freq_factor
    high_wl = s.original_max_position_embeddings / s.high_freq_factor
    out = []
    for f in inv:
        wl = 2.0 * math.pi / f
        if wl < high_wl:
            out.append(f)
        elif wl > low_wl:
            out.append(f / s.factor)
        else:
            smooth = (s.original_max_position_embeddings / wl - s.low_freq_factor) / (
                s.high_freq_factor - s.low_freq_factor)
            out.append((1.0 - smooth) * f / s.factor + smooth * f)
    return out
