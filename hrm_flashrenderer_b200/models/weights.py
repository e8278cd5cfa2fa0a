"""Int8 per-output-channel weights: quantisation, random-init synthesis and tensor-parallel sharding.

Quantisation follows the DSI8 exporter (``hrm_flash/deepseek_export.py:45-50``): symmetric, one fp32 scale per
output row, ``scale = max(|w_row|, 1e-8) / 127`` and ``q = clip(round_half_even(w / scale), -128, 127)``.
The same rule is used for the embedding and the lm_head (both are 2-D records in DSI8).

Tensor names are the HF names (``model.layers.{l}.self_attn.q_proj.weight`` ...) because the DSI8 records are
keyed by them.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterator, Tuple, Union

import torch

from ..config import ModelConfig


@dataclass
class QTensor:
    """Row-quantised matrix: ``w ~= q.float() * scale[:, None]``; ``q`` is int8 ``[rows, cols]``."""

    q: torch.Tensor
    scale: torch.Tensor

    @property
    def shape(self) -> Tuple[int, int]:
        return tuple(self.q.shape)

    def dequant(self, dtype=torch.float32) -> torch.Tensor:
        return (self.q.to(torch.float32) * self.scale.to(torch.float32)[:, None]).to(dtype)

    def rows(self, r0: int, r1: int) -> "QTensor":
        return QTensor(self.q[r0:r1], self.scale[r0:r1])

    def cols(self, c0: int, c1: int) -> "QTensor":
        # Row scales are per output channel, so a column (input) shard keeps the full scale vector.
        return QTensor(self.q[:, c0:c1], self.scale)

    def to(self, device) -> "QTensor":
        return QTensor(self.q.to(device), self.scale.to(device))

    def contiguous(self) -> "QTensor":
        return QTensor(self.q.contiguous(), self.scale.contiguous())


Tensorish = Union[QTensor, torch.Tensor]


def quantize_rows(w: torch.Tensor) -> QTensor:
    """Symmetric per-row int8 quantisation of a 2-D float tensor (any device)."""
    w = w.to(torch.float32)
    absmax = w.abs().amax(dim=-1).clamp_min(1e-8)
    scale = absmax / 127.0
    q = torch.round(w / scale[:, None]).clamp_(-128, 127).to(torch.int8)
    return QTensor(q, scale)


def layer_names(l: int) -> Dict[str, str]:
    p = f"model.layers.{l}"
    return {
        "q": f"{p}.self_attn.q_proj.weight",
        "k": f"{p}.self_attn.k_proj.weight",
        "v": f"{p}.self_attn.v_proj.weight",
        "o": f"{p}.self_attn.o_proj.weight",
        "gate": f"{p}.mlp.gate_proj.weight",
        "up": f"{p}.mlp.up_proj.weight",
        "down": f"{p}.mlp.down_proj.weight",
        "ln1": f"{p}.input_layernorm.weight",
        "ln2": f"{p}.post_attention_layernorm.weight",
        "bq": f"{p}.self_attn.q_proj.bias",
        "bk": f"{p}.self_attn.k_proj.bias",
        "bv": f"{p}.self_attn.v_proj.bias",
    }


EMBED = "model.embed_tokens.weight"
FINAL_NORM = "model.norm.weight"
LM_HEAD = "lm_head.weight"


def matrix_shapes(cfg: ModelConfig) -> Iterator[Tuple[str, Tuple[int, int]]]:
    """(name, [out, in]) of every 2-D weight in DSI8 record order (``deepseek_export.py:153-170``)."""
    yield EMBED, (cfg.vocab, cfg.hidden)
    for l in range(cfg.layers):
        n = layer_names(l)
        yield n["q"], (cfg.q_dim, cfg.hidden)
        yield n["k"], (cfg.kv_dim, cfg.hidden)
        yield n["v"], (cfg.kv_dim, cfg.hidden)
        yield n["o"], (cfg.hidden, cfg.q_dim)
        yield n["gate"], (cfg.intermediate, cfg.hidden)
        yield n["up"], (cfg.intermediate, cfg.hidden)
        yield n["down"], (cfg.hidden, cfg.intermediate)
    if not cfg.tie_embeddings:
        yield LM_HEAD, (cfg.vocab, cfg.hidden)


def vector_shapes(cfg: ModelConfig) -> Iterator[Tuple[str, int]]:
    """(name, length) of every 1-D weight in DSI8 record order."""
    for l in range(cfg.layers):
        n = layer_names(l)
        yield n["ln1"], cfg.hidden
        yield n["ln2"], cfg.hidden
        if cfg.qkv_bias:
            yield n["bq"], cfg.q_dim
            yield n["bk"], cfg.kv_dim
            yield n["bv"], cfg.kv_dim
    yield FINAL_NORM, cfg.hidden


def synth_weights(cfg: ModelConfig, seed: int = 0, std: float = 0.02, device: str | torch.device = "cpu",
                  norm_jitter: float = 0.0, bias_std: float = 0.02,
                  chunk_elems: int = 1 << 26) -> Dict[str, Tensorish]:
    """Random-init weights of ``cfg``: fp32 ``N(0, std)`` from ``seed``, then per-row int8 quantisation.

    Large matrices are generated in row chunks of ``chunk_elems`` elements so that a 70B synthesis on the GPU
    never materialises more than one fp32 chunk.  Every matrix draws from its own generator seeded by
    ``(seed, index)`` so that any subset (e.g. one TP shard, or a reduced-depth slice) is reproducible.
    Norm weights are ``1 + N(0, norm_jitter)`` (HF initialises them to ones); biases are ``N(0, bias_std)``.
    """
    dev = torch.device(device)
    out: Dict[str, Tensorish] = {}
    for idx, (name, (rows, cols)) in enumerate(matrix_shapes(cfg)):
        out[name] = synth_matrix(rows, cols, seed=seed * 1_000_003 + idx, std=std, device=dev,
                                 chunk_elems=chunk_elems)
    base = 10_000_000
    for idx, (name, n) in enumerate(vector_shapes(cfg)):
        g = torch.Generator(device="cpu").manual_seed(seed * 1_000_003 + base + idx)
        if name.endswith("layernorm.weight") or name == FINAL_NORM:
            v = torch.ones(n) + (torch.randn(n, generator=g) * norm_jitter if norm_jitter else 0.0)
        else:
            v = torch.randn(n, generator=g) * bias_std
        out[name] = v.to(torch.float32).to(dev)
    return out


def synth_matrix(rows: int, cols: int, seed: int, std: float = 0.02, device: torch.device | str = "cpu",
                 chunk_elems: int = 1 << 26) -> QTensor:
    dev = torch.device(device)
    q = torch.empty(rows, cols, dtype=torch.int8, device=dev)
    scale = torch.empty(rows, dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev).manual_seed(int(seed))
    step = max(1, chunk_elems // max(1, cols))
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        w = torch.randn(r1 - r0, cols, generator=g, device=dev, dtype=torch.float32) * std
        qt = quantize_rows(w)
        q[r0:r1] = qt.q
        scale[r0:r1] = qt.scale
        del w
    return QTensor(q, scale)


def get_lm_head(cfg: ModelConfig, w: Dict[str, Tensorish]) -> QTensor:
    return w[EMBED] if cfg.tie_embeddings or LM_HEAD not in w else w[LM_HEAD]


# ------------------------------------------------------------------------------------------------
# Tensor-parallel sharding (Megatron 1-D), reference semantics: ``tp/parallel_linear.py:9-90``,
# ``tp/vocab_parallel.py:9-57``, ``engine/llama_tp.py:110-152``.
# ------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class ShardPlan:
    rank: int
    world: int
    local_heads: int
    local_kv_heads: int
    kv_replicated: bool
    kv_head_offset: int
    head_map: Tuple[int, ...]   # local q head -> local kv head
    local_inter: int
    vocab_start: int
    vocab_per_rank: int


def shard_plan(cfg: ModelConfig, rank: int, world: int) -> ShardPlan:
    cfg.validate_tp(world)
    local_heads = cfg.heads // world
    if cfg.kv_heads % world == 0:
        kv_rep, lkv, off = False, cfg.kv_heads // world, rank * (cfg.kv_heads // world)
    else:
        kv_rep, lkv, off = True, cfg.kv_heads, 0
    group = cfg.heads // cfg.kv_heads
    hm = []
    for hq in range(local_heads):
        gkh = (rank * local_heads + hq) // group          # HF GQA mapping: head // group
        hm.append(gkh if kv_rep else gkh - off)
    if any(h < 0 or h >= lkv for h in hm):
        raise ValueError(f"world={world} incompatible with kv layout of {cfg.name}")
    vpr = cfg.vocab // world
    return ShardPlan(rank, world, local_heads, lkv, kv_rep, off, tuple(hm), cfg.intermediate // world,
                     rank * vpr, vpr)


def shard_weights(cfg: ModelConfig, w: Dict[str, Tensorish], rank: int, world: int) -> Dict[str, Tensorish]:
    """Slice full weights into rank ``rank``'s TP shard.

    Column-parallel (q, k, v, gate, up, embed rows, lm_head rows): rows sliced together with their scales.
    Row-parallel (o, down): columns sliced, full per-row scales kept.  K/V are replicated when
    ``kv_heads % world != 0``.  Norms are replicated; q/k/v biases follow their rows.
    """
    p = shard_plan(cfg, rank, world)
    out: Dict[str, Tensorish] = {}
    D = cfg.head_dim
    for l in range(cfg.layers):
        n = layer_names(l)
        q0, q1 = rank * p.local_heads * D, (rank + 1) * p.local_heads * D
        out[n["q"]] = w[n["q"]].rows(q0, q1)
        if p.kv_replicated:
            k0, k1 = 0, cfg.kv_dim
        else:
            k0, k1 = p.kv_head_offset * D, (p.kv_head_offset + p.local_kv_heads) * D
        out[n["k"]] = w[n["k"]].rows(k0, k1)
        out[n["v"]] = w[n["v"]].rows(k0, k1)
        out[n["o"]] = w[n["o"]].cols(q0, q1)
        f0, f1 = rank * p.local_inter, (rank + 1) * p.local_inter
        out[n["gate"]] = w[n["gate"]].rows(f0, f1)
        out[n["up"]] = w[n["up"]].rows(f0, f1)
        out[n["down"]] = w[n["down"]].cols(f0, f1)
        out[n["ln1"]] = w[n["ln1"]]
        out[n["ln2"]] = w[n["ln2"]]
        if cfg.qkv_bias:
            out[n["bq"]] = w[n["bq"]][q0:q1]
            out[n["bk"]] = w[n["bk"]][k0:k1]
            out[n["bv"]] = w[n["bv"]][k0:k1]
    v0, v1 = p.vocab_start, p.vocab_start + p.vocab_per_rank
    out[EMBED] = w[EMBED].rows(v0, v1)
    out[LM_HEAD] = get_lm_head(cfg, w).rows(v0, v1)
    out[FINAL_NORM] = w[FINAL_NORM]
    return out
