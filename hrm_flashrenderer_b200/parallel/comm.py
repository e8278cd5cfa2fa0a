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

    def all_reduce_async_(self, t: torch.Tensor):
        """Start an in-place SUM all-reduce; returns the work handle (``wait()`` makes the current stream wait for
        it without blocking the host), or None when there is nothing to reduce."""
        if self.world > 1:
            return dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        return None

    def all_reduce_max_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return t

    # ---------------------------------------------------------------- sequence parallel (token-sharded rows)
    def reduce_scatter_rows(self, full: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
        """Sum ``full [world * R, ...]`` over ranks and keep rows ``[rank * R, (rank + 1) * R)``."""
        if self.world == 1:
            if out is None:
                return full
            return out.copy_(full)
        rows = full.shape[0] // self.world
        if out is None:
            out = torch.empty((rows,) + tuple(full.shape[1:]), dtype=full.dtype, device=full.device)
        dist.reduce_scatter_tensor(out, full.contiguous(), op=dist.ReduceOp.SUM, group=self.group)
        return out

    def all_gather_rows(self, shard: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """``out [world * R, ...]``: rank r's ``shard [R, ...]`` at rows ``[r * R, (r + 1) * R)``."""
        if self.world == 1:
            return out.copy_(shard)
        dist.all_gather_into_tensor(out, shard.contiguous(), group=self.group)
        return out

    def all_gather_cols(self, shard: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """``out [C, world * R]``: rank r's ``shard [C, R]`` at columns ``[r * R, (r + 1) * R)``."""
        if self.world == 1:
            return out.copy_(shard)
        C, R = shard.shape
        buf = torch.empty(self.world * C, R, dtype=shard.dtype, device=shard.device)
        dist.all_gather_into_tensor(buf, shard.contiguous(), group=self.group)
        out.copy_(buf.view(self.world, C, R).permute(1, 0, 2).reshape(out.shape))
        return out

    def barrier(self) -> None:
        if self.world > 1:
            dist.barrier(group=self.group)
