"""Megatron 1-D tensor-parallel layers over int8 per-output-channel weights.

API parity with the reference ``tp/`` package (``tp/parallel_linear.py:9-90``, ``tp/vocab_parallel.py:9-57``,
``tp/norm.py:7-20``): ``ColumnParallelLinear``, ``RowParallelLinear``, ``ReplicatedLinear``,
``VocabParallelEmbedding``, ``VocabParallelLMHead``, ``RMSNorm``.  Differences: weights are int8 + fp32 row scales
(the DSI8 layout) instead of fp16, biases are supported (Qwen2 q/k/v), and RMSNorm math is fp32.

Compute goes through :mod:`hrm_flashrenderer_b200.ops`: on CUDA tensors that is the sm_100a W8A16 GEMM, on CPU the
fp32 reference.  These layers use plain ``torch.distributed`` collectives (NCCL / gloo); the fused
compute+collective kernels are used by :mod:`hrm_flashrenderer_b200.models.llama` instead.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .. import ops
from ..models.weights import QTensor, quantize_rows
from .dist import all_reduce_sum, rank_world


def _as_q(w) -> QTensor:
    """The reference's layers load fp16 tensors; these take a QTensor or a float matrix (quantised per row here,
    over the full row, so a column shard keeps the full-model scales)."""
    return w if isinstance(w, QTensor) else quantize_rows(w.to(torch.float32))


class _QLinearBase(nn.Module):
    def __init__(self, out_features: int, in_features: int, bias: bool, device):
        super().__init__()
        self.register_buffer("qweight", torch.zeros(out_features, in_features, dtype=torch.int8, device=device))
        self.register_buffer("scale", torch.ones(out_features, dtype=torch.float32, device=device))
        self.register_buffer("bias", torch.zeros(out_features, dtype=torch.float32, device=device) if bias else None)

    def load(self, w: QTensor, bias: Optional[torch.Tensor] = None) -> None:
        self.qweight.copy_(w.q.to(self.qweight.device))
        self.scale.copy_(w.scale.to(self.scale.device))
        if self.bias is not None and bias is not None:
            self.bias.copy_(bias.to(self.bias.device, torch.float32))

    def _mm(self, x: torch.Tensor) -> torch.Tensor:
        y = ops.w8a16_linear(x, self.qweight, self.scale)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y


class ColumnParallelLinear(_QLinearBase):
    """Output features sharded: rank r owns rows ``[r*out/world, (r+1)*out/world)``; no communication."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, device="cpu", group=None):
        rank, world = rank_world()
        assert out_features % world == 0
        self.rank, self.world, self.local_out = rank, world, out_features // world
        super().__init__(self.local_out, in_features, bias, device)

    def load_from_full(self, w: QTensor, bias: Optional[torch.Tensor] = None) -> None:
        r0, r1 = self.rank * self.local_out, (self.rank + 1) * self.local_out
        self.load(_as_q(w).rows(r0, r1), None if bias is None else bias[r0:r1])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._mm(x)


class RowParallelLinear(_QLinearBase):
    """Input features sharded; the partial products are summed with an all-reduce (reference M1)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, device="cpu", group=None):
        rank, world = rank_world()
        assert in_features % world == 0
        self.rank, self.world, self.local_in, self.group = rank, world, in_features // world, group
        super().__init__(out_features, self.local_in, bias, device)

    def load_from_full(self, w: QTensor, bias: Optional[torch.Tensor] = None) -> None:
        c0, c1 = self.rank * self.local_in, (self.rank + 1) * self.local_in
        self.load(_as_q(w).cols(c0, c1), bias)

    def forward(self, x_shard: torch.Tensor) -> torch.Tensor:
        y = ops.w8a16_linear(x_shard, self.qweight, self.scale, out_dtype=torch.float32)
        all_reduce_sum(y, group=self.group)
        if self.bias is not None:
            y = y + self.bias
        return y


class ReplicatedLinear(_QLinearBase):
    """Full weight on every rank (K/V projections when ``kv_heads % world != 0``)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, device="cpu"):
        super().__init__(out_features, in_features, bias, device)

    def load_from_full(self, w: QTensor, bias: Optional[torch.Tensor] = None) -> None:
        self.load(_as_q(w), bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._mm(x)


class VocabParallelEmbedding(nn.Module):
    """Rank r holds vocab rows ``[r*V/world, (r+1)*V/world)``; out-of-range ids contribute zeros and the rows are
    summed across ranks (reference M2)."""

    def __init__(self, vocab_size: int, hidden: int, device="cpu", group=None):
        super().__init__()
        rank, world = rank_world()
        assert vocab_size % world == 0
        self.vocab_per_rank = vocab_size // world
        self.vocab_start = rank * self.vocab_per_rank
        self.group = group
        self.register_buffer("qweight", torch.zeros(self.vocab_per_rank, hidden, dtype=torch.int8, device=device))
        self.register_buffer("scale", torch.ones(self.vocab_per_rank, dtype=torch.float32, device=device))

    def load_from_full(self, w: QTensor) -> None:
        qt = _as_q(w).rows(self.vocab_start, self.vocab_start + self.vocab_per_rank)
        self.qweight.copy_(qt.q.to(self.qweight.device))
        self.scale.copy_(qt.scale.to(self.scale.device))

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        out = ops.embedding_q8(ids, self.qweight, self.scale, self.vocab_start)
        return all_reduce_sum(out, group=self.group)


class VocabParallelLMHead(_QLinearBase):
    """Local vocab-slice logits; no gather (the selection is distributed, see ``greedy_select_distributed``)."""

    def __init__(self, hidden: int, vocab_size: int, device="cpu"):
        rank, world = rank_world()
        assert vocab_size % world == 0
        self.vocab_per_rank = vocab_size // world
        self.vocab_start = rank * self.vocab_per_rank
        super().__init__(self.vocab_per_rank, hidden, False, device)

    def load_from_full(self, w: QTensor) -> None:
        self.load(_as_q(w).rows(self.vocab_start, self.vocab_start + self.vocab_per_rank))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.w8a16_linear(x, self.qweight, self.scale, out_dtype=torch.float32)


class RMSNorm(nn.Module):
    """``x * rsqrt(mean(x^2) + eps) * w`` with fp32 statistics and fp32 math (reference computed in fp16)."""

    def __init__(self, dim: int, eps: float = 1e-6, device="cpu"):
        super().__init__()
        self.eps = float(eps)
        self.register_buffer("weight", torch.ones(dim, dtype=torch.float32, device=device))

    def load_from_full(self, w: torch.Tensor) -> None:
        self.weight.copy_(w.to(self.weight.device, torch.float32))

    def forward(self, x: torch.Tensor, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        return ops.rmsnorm(x, self.weight, self.eps, out_dtype=out_dtype)
