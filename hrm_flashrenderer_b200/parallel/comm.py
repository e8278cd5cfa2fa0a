"""Tensor-parallel communicator used by the model: baseline NCCL/gloo collectives.

The fused compute+collective kernels (peer-memory GEMM+all-reduce, argmax exchange) live in
:mod:`hrm_flashrenderer_b200.parallel.symm` and are selected by the engine; this class is the plain
``torch.distributed`` path they are measured against (reference: ``tp/dist_utils.py:31-39``, the all-reduces of
``tp/parallel_linear.py:65`` and ``tp/vocab_parallel.py:35``, and ``greedy_select_token_distributed``).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class TPComm:
    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t

    def all_reduce_max_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return t

    def barrier(self) -> None:
        if self.world > 1:
            dist.barrier(group=self.group)
