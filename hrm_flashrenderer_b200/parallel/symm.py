"""Symmetric peer memory over NVLink/NVSwitch for the fused compute+collective kernels.

Every rank ``cudaMalloc``s one equally sized buffer, exports a CUDA IPC handle, exchanges handles over the
``torch.distributed`` control group and maps every peer's buffer (``cudaIpcOpenMemHandle``).  Kernels then read and
write peers directly through a device table of base pointers ``peers[r]`` (``peers[rank]`` is the local buffer).

Layout of the buffer (all offsets 256-byte aligned):

* ``partials``  fp32 [2][world][max_tiles][128][max_bn] -- receive area: every rank pushes its row-parallel partial
  tiles into slot [launch parity][its rank] of every rank (double-buffered by launch parity: a slow peer may still be
  reading the previous launch's data when this rank starts the next one);
* ``final``     fp32 [max_tiles][max_bn][128]  -- spare reduction space;
* ``flags``     int32 [world]: the epoch up to which each source rank's partials are complete (multi-phase chain);
* ``tile flags`` int32 [world][max_tiles], one 128-byte line each: the epoch up to which source rank r's partial of
  tile t has arrived
  (single-launch fused GEMM: each tile waits only for the same tile of the other ranks);
* ``scalars``: the per-launch epoch counter and two CTA tickets, the argmax exchange's epoch and row ticket;
* ``epoch-tagged words`` u64 [2][world][max_tiles][max_bn][128] (after the extra area): the flag-free variant of
  the fused all-reduce, where every pushed element carries its launch epoch in the same 64-bit word;
* ``argmax keys`` int64 [2][world][argmax_rows] and ``argmax flags`` int32 [world][argmax_rows] (one line each; extra
  area): the distributed greedy pick, where every rank pushes each row's packed (value, token) key to every rank.

Flags carry an epoch number that every fused launch increments once, so a flag written by a previous launch is never
mistaken for a current one and no reset pass is needed between launches.
"""
from __future__ import annotations

import warnings
from typing import Dict

import torch
import torch.distributed as dist

from .. import ops

ALIGN = 256
FLAG_LINE = 128   # every epoch flag owns one cache line (kernels: kFlagStrideInts ints)


def _al(x: int) -> int:
    return (x + ALIGN - 1) // ALIGN * ALIGN


def symm_layout(world: int, max_tiles: int, max_bn: int, extra_bytes: int = 1 << 20) -> Dict[str, int]:
    """Byte offsets of every region of one rank's symmetric buffer (all 256-byte aligned, in this order) and the
    total size.  ``regions`` maps each region to its (offset, length); the regions never overlap."""
    tile_bytes = max_bn * 128 * 4
    L: Dict[str, int] = {}
    L["off_partials"] = 0
    L["off_final"] = _al(2 * world * max_tiles * tile_bytes)
    L["off_flags"] = _al(L["off_final"] + max_tiles * tile_bytes)
    L["off_tile_flags"] = _al(L["off_flags"] + 2 * max_tiles * 4)
    L["off_scalars"] = _al(L["off_tile_flags"] + world * max_tiles * FLAG_LINE)
    L["off_extra"] = _al(L["off_scalars"] + 4096)
    # epoch-tagged receive words of the flag-free fused all-reduce: u64 [2][world][max_tiles][max_bn * 128]
    L["off_ll"] = _al(L["off_extra"] + extra_bytes)
    ll_bytes = 2 * world * max_tiles * max_bn * 128 * 8
    L["bytes"] = _al(L["off_ll"] + ll_bytes)
    # distributed argmax exchange inside the extra area: two key slots and one flag line per source rank and row
    per_row = world * (16 + FLAG_LINE)
    L["argmax_rows"] = int(min(ops.ARGMAX_XCHG_MAX_ROWS, (extra_bytes - 2 * ALIGN) // per_row))
    L["off_ax_keys"] = L["off_extra"]
    L["off_ax_flags"] = _al(L["off_ax_keys"] + 2 * world * L["argmax_rows"] * 8)
    L["regions"] = {
        "partials": (L["off_partials"], 2 * world * max_tiles * tile_bytes),
        "final": (L["off_final"], max_tiles * tile_bytes),
        "flags": (L["off_flags"], 2 * max_tiles * 4),
        "tile_flags": (L["off_tile_flags"], world * max_tiles * FLAG_LINE),
        "scalars": (L["off_scalars"], 4096),
        "argmax_keys": (L["off_ax_keys"], 2 * world * L["argmax_rows"] * 8),
        "argmax_flags": (L["off_ax_flags"], world * L["argmax_rows"] * FLAG_LINE),
        "ll_words": (L["off_ll"], ll_bytes),
    }
    return L


class SymmetricWorkspace:
    def __init__(self, rank: int, world: int, device: torch.device, max_tiles: int = 1024, max_bn: int = 64,
                 group=None, extra_bytes: int = 1 << 20):
        self.rank, self.world, self.device = rank, world, torch.device(device)
        self.max_tiles, self.max_bn = max_tiles, max_bn
        L = symm_layout(world, max_tiles, max_bn, extra_bytes)
        for k in ("off_partials", "off_final", "off_flags", "off_tile_flags", "off_scalars", "off_extra", "off_ll",
                  "bytes", "argmax_rows", "off_ax_keys", "off_ax_flags"):
            setattr(self, k, L[k])
        C = ops.ext()
        with torch.cuda.device(self.device):
            self.local_ptr, handle = C.symm_alloc(self.bytes)
        handles = [None] * world
        if world > 1:
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles = [handle]
        self.ptrs = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                self.ptrs.append(self.local_ptr if r == rank else C.symm_open(h))
        self.peers = torch.tensor(self.ptrs, dtype=torch.int64, device=self.device)
        # epoch counter lives in this rank's scalars (local memory); the CTA-completion ticket next to it
        self.epoch = C.tensor_from_ptr(self.local_ptr + self.off_scalars, [1], torch.int32, self.device.index or 0)
        self.ticket = C.tensor_from_ptr(self.local_ptr + self.off_scalars + 128, [2], torch.int32,
                                        self.device.index or 0)
        self.group = group

    @property
    def epoch_ptr(self) -> int:
        return self.local_ptr + self.off_scalars

    @property
    def argmax_epoch_ptr(self) -> int:
        return self.local_ptr + self.off_scalars + 256

    @property
    def argmax_ticket_ptr(self) -> int:
        return self.local_ptr + self.off_scalars + 384

    def view(self, offset: int, shape, dtype=torch.float32) -> torch.Tensor:
        return ops.ext().tensor_from_ptr(self.local_ptr + offset, list(shape), dtype, self.device.index or 0)

    def close(self) -> None:
        C = ops.ext()
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                try:
                    C.symm_close(p)
                except Exception as e:   # keep tearing down: the barrier below must still be reached
                    warnings.warn(f"symmetric workspace: unmapping rank {r}'s buffer failed: {e!r}")
        if self.world > 1:
            dist.barrier(group=self.group)   # peers unmapped before the owner frees
        C.symm_free(self.local_ptr)
        self.ptrs = []
