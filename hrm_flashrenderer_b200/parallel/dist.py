"""Process-group bootstrap and plain collectives (the control plane and the NCCL/gloo baseline data plane).

Reference: ``tp/dist_utils.py:8-39`` (``init_dist_env``, ``init_dist``, ``all_reduce_sum``, ``all_gather_cat``).
Differences: the backend is NCCL when CUDA is available and gloo otherwise, the process group always gets a short
timeout (so a rank that disappears turns into an error on its peers instead of a hang), and rendezvous defaults
to 127.0.0.1.
"""
from __future__ import annotations

import datetime
import os
from typing import Optional, Tuple

import torch
import torch.distributed as dist

DEFAULT_TIMEOUT_S = float(os.environ.get("HRM_B200_PG_TIMEOUT_S", "120"))


def _timeout(seconds: Optional[float]) -> datetime.timedelta:
    return datetime.timedelta(seconds=float(seconds if seconds is not None else DEFAULT_TIMEOUT_S))


def init_dist_env(backend: Optional[str] = None, timeout_s: Optional[float] = None) -> Tuple[int, int, int]:
    """Initialise from torchrun's environment (RANK, WORLD_SIZE, LOCAL_RANK, MASTER_ADDR/PORT)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local_rank)
    if not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local_rank)
        dist.init_process_group(backend=backend, rank=rank, world_size=world, timeout=_timeout(timeout_s), **kw)
    return rank, local_rank, world


def init_dist(rank: int, world: int, master_addr: str = "127.0.0.1", master_port: int = 29533,
              local_rank: Optional[int] = None, backend: Optional[str] = None,
              timeout_s: Optional[float] = None) -> Tuple[int, int, int]:
    """Explicit initialisation (used by ``mp.spawn`` style launchers and the CPU tests)."""
    os.environ["MASTER_ADDR"] = master_addr
    os.environ["MASTER_PORT"] = str(master_port)
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    os.environ["LOCAL_RANK"] = str(local_rank if local_rank is not None else rank)
    return init_dist_env(backend=backend, timeout_s=timeout_s)


def is_dist() -> bool:
    return dist.is_available() and dist.is_initialized()


def rank_world() -> Tuple[int, int]:
    if is_dist():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def all_reduce_sum(x: torch.Tensor, group=None) -> torch.Tensor:
    if is_dist() and dist.get_world_size(group) > 1:
        dist.all_reduce(x, op=dist.ReduceOp.SUM, group=group)
    return x


def all_gather_cat(x: torch.Tensor, dim: int, group=None) -> torch.Tensor:
    if not is_dist() or dist.get_world_size(group) == 1:
        return x
    xs = [torch.empty_like(x) for _ in range(dist.get_world_size(group))]
    dist.all_gather(xs, x.contiguous(), group=group)
    return torch.cat(xs, dim=dim)


def reduce_scatter_cat(x: torch.Tensor, dim: int = 0, group=None) -> torch.Tensor:
    """Sum over ranks, then keep this rank's ``1/world`` slice along ``dim`` (sequence-parallel output)."""
    if not is_dist() or dist.get_world_size(group) == 1:
        return x
    w = dist.get_world_size(group)
    chunks = [c.contiguous() for c in x.chunk(w, dim=dim)]
    out = torch.empty_like(chunks[0])
    dist.reduce_scatter(out, chunks, op=dist.ReduceOp.SUM, group=group)
    return out


def barrier(group=None) -> None:
    if is_dist():
        dist.barrier(group=group)


def destroy() -> None:
    if is_dist():
        dist.destroy_process_group()


# ------------------------------------------------------------------------------------------------
# Deterministic distributed greedy selection (replaces the reference's MAX + MIN + per-row broadcast,
# ``engine/llama_tp.py:317-335``) with ONE all-reduce(MAX) of a packed int64 key per row.
# ------------------------------------------------------------------------------------------------
def float_order_key(v: torch.Tensor) -> torch.Tensor:
    """Monotone map float32 -> int64 in ``[-2^31, 2^31)`` (total order, -0 < +0, NaN above +inf)."""
    bits = v.to(torch.float32).contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    neg = (bits & 0x80000000) != 0
    ordered = torch.where(neg, (~bits) & 0xFFFFFFFF, bits | 0x80000000)
    return ordered - (1 << 31)


def pack_argmax(val: torch.Tensor, gidx: torch.Tensor) -> torch.Tensor:
    """Key whose max is (largest value, then lowest global id)."""
    return float_order_key(val) * (1 << 32) + ((1 << 32) - 1 - gidx.to(torch.int64))


def unpack_argmax(key: torch.Tensor) -> torch.Tensor:
    return (1 << 32) - 1 - (key & 0xFFFFFFFF)


def greedy_select_distributed(local_logits: torch.Tensor, vocab_start: int, group=None) -> torch.Tensor:
    """Global greedy token per row from vocab-sharded logits; ties go to the lowest global id."""
    lf = local_logits.to(torch.float32)
    val, idx = torch.max(lf, dim=-1)                 # torch.max returns the first (lowest) index on ties
    key = pack_argmax(val, idx.to(torch.int64) + int(vocab_start))
    if is_dist() and dist.get_world_size(group) > 1:
        dist.all_reduce(key, op=dist.ReduceOp.MAX, group=group)
    return unpack_argmax(key)
