"""CPU correctness oracle: fp32 math on int8-dequantised weights, HF Llama/Qwen2 semantics.

This is the numerics reference every kernel and every parallel layout is tested against.  It deliberately does
*not* reproduce the reference's native-engine quirks (interleaved RoPE, ``head % KVH`` GQA, dropped QKV bias,
fp16 norm math; see ``scripts/deepseek_native_engine.sh:545-549,568`` and ``engine/llama_tp.py:127-143``): it uses
rotate-half RoPE with optional llama3 scaling, ``kv_head = head // group``, the Qwen2 q/k/v bias and fp32 norms.
Greedy ties resolve to the lowest token id (``torch.argmax`` returns the first maximum).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ..config import ModelConfig, rope_inv_freq
from .weights import QTensor, Tensorish, layer_names, EMBED, FINAL_NORM, get_lm_head


def rope_tables(cfg: ModelConfig, max_pos: int, device="cpu") -> Tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables ``[max_pos, head_dim/2]`` (fp32), angles computed in fp64."""
    inv = torch.tensor(rope_inv_freq(cfg), dtype=torch.float64)
    t = torch.arange(max_pos, dtype=torch.float64)
    ang = torch.outer(t, inv)
    return torch.cos(ang).to(torch.float32).to(device), torch.sin(ang).to(torch.float32).to(device)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.to(torch.float32)
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.to(torch.float32)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE.  ``x [..., T, H, D]`` with ``pos [..., T]``."""
    half = x.shape[-1] // 2
    c = cos[pos].unsqueeze(-2)
    s = sin[pos].unsqueeze(-2)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor, group: int) -> torch.Tensor:
    """Causal GQA attention of one sequence.  ``q [T, Hq, D]``, ``k/v [S, Hk, D]``, ``q_pos [T]`` absolute.

    Key ``j`` is visible to query ``i`` iff ``j <= q_pos[i]``.
    """
    T, Hq, D = q.shape
    S = k.shape[0]
    kk = k.repeat_interleave(group, dim=1)       # head h uses kv head h // group
    vv = v.repeat_interleave(group, dim=1)
    scores = torch.einsum("thd,shd->hts", q.float(), kk.float()) / math.sqrt(D)
    mask = torch.arange(S).view(1, 1, S) > q_pos.view(1, T, 1)
    scores = scores.masked_fill(mask, float("-inf"))
    p = torch.softmax(scores, dim=-1)
    return torch.einsum("hts,shd->thd", p, vv.float())


class OracleLlama:
    """Unsharded fp32 model over dequantised int8 weights with a contiguous per-sequence KV cache."""

    def __init__(self, cfg: ModelConfig, weights: Dict[str, Tensorish], max_pos: Optional[int] = None):
        self.cfg = cfg
        self.max_pos = int(max_pos or min(cfg.max_position_embeddings, 8192))
        self.cos, self.sin = rope_tables(cfg, self.max_pos)
        deq = lambda t: t.dequant() if isinstance(t, QTensor) else t.to(torch.float32)
        self.w = {k: deq(v) for k, v in weights.items()}
        self.lm_head = get_lm_head(cfg, weights).dequant()

    def forward(self, ids: torch.Tensor, pos: torch.Tensor, cache: List[Tuple[torch.Tensor, torch.Tensor]]):
        """One sequence: ``ids [T]`` at absolute positions ``pos [T]``; appends to ``cache`` (per layer k, v)."""
        cfg = self.cfg
        x = self.w[EMBED][ids]
        for l in range(cfg.layers):
            n = layer_names(l)
            h = rmsnorm(x, self.w[n["ln1"]], cfg.rms_eps)
            q = h @ self.w[n["q"]].t()
            k = h @ self.w[n["k"]].t()
            v = h @ self.w[n["v"]].t()
            if cfg.qkv_bias:
                q, k, v = q + self.w[n["bq"]], k + self.w[n["bk"]], v + self.w[n["bv"]]
            T = ids.shape[0]
            q = apply_rope(q.view(T, cfg.heads, cfg.head_dim), self.cos, self.sin, pos)
            k = apply_rope(k.view(T, cfg.kv_heads, cfg.head_dim), self.cos, self.sin, pos)
            v = v.view(T, cfg.kv_heads, cfg.head_dim)
            if len(cache) <= l:
                cache.append((k, v))
            else:
                ck, cv = cache[l]
                cache[l] = (torch.cat([ck, k]), torch.cat([cv, v]))
            ck, cv = cache[l]
            a = attention(q, ck, cv, pos, cfg.group).reshape(T, cfg.q_dim)
            x = x + a @ self.w[n["o"]].t()
            h = rmsnorm(x, self.w[n["ln2"]], cfg.rms_eps)
            g = h @ self.w[n["gate"]].t()
            u = h @ self.w[n["up"]].t()
            x = x + (torch.nn.functional.silu(g) * u) @ self.w[n["down"]].t()
        return rmsnorm(x, self.w[FINAL_NORM], cfg.rms_eps)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return h @ self.lm_head.t()

    @torch.no_grad()
    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int, stop_on_eos: bool = False,
                 return_logits: bool = False):
        """Greedy decode of each prompt independently.  Returns new token ids per prompt (and logits)."""
        outs, all_logits = [], []
        for p in prompts:
            ids = torch.tensor(list(p), dtype=torch.long)
            cache: list = []
            h = self.forward(ids, torch.arange(len(p)), cache)
            toks, lg = [], []
            cur = len(p)
            for _ in range(max_new_tokens):
                logit = self.logits(h[-1])
                lg.append(logit)
                t = int(torch.argmax(logit))
                toks.append(t)
                if stop_on_eos and t in self.cfg.eos_token_ids:
                    break
                h = self.forward(torch.tensor([t]), torch.tensor([cur]), cache)
                cur += 1
            outs.append(toks)
            all_logits.append(torch.stack(lg) if lg else torch.empty(0, self.cfg.vocab))
        return (outs, all_logits) if return_logits else outs
