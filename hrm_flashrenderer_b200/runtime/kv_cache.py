"""Block-table paged KV cache (block size 16 by default) and its block manager.

Replaces the reference's per-sequence contiguous pages ``[B,Hk,P,PS,D]`` that grow by power-of-two reallocation
and copy (``engine/llama_tp.py:21-108``, reference quirk Q10): here a fixed pool of blocks is allocated once, every
sequence owns a list of block ids (its block table), and growth is a table append.  Pool layout per layer:
``[num_blocks, kv_heads, block_size, head_dim]`` so one (block, head) is a contiguous ``block_size*head_dim``
run (4 KB at bf16/D=128), the unit the attention kernels fetch.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch


class OutOfBlocks(RuntimeError):
    pass


class BlockManager:
    """Free-list allocator of KV blocks.  Deterministic: the lowest free block id is always handed out first."""

    def __init__(self, num_blocks: int, block_size: int = 16):
        self.num_blocks = int(num_blocks)
        self.block_size = int(block_size)
        self._free: List[int] = list(range(self.num_blocks - 1, -1, -1))   # pop() yields the lowest id
        self.tables: Dict[int, List[int]] = {}
        self.lengths: Dict[int, int] = {}

    @property
    def free_blocks(self) -> int:
        return len(self._free)

    def blocks_needed(self, seq_id: int, new_len: int) -> int:
        have = len(self.tables.get(seq_id, ()))
        need = (int(new_len) + self.block_size - 1) // self.block_size
        return max(0, need - have)

    def can_grow(self, seq_id: int, new_len: int) -> bool:
        return self.blocks_needed(seq_id, new_len) <= len(self._free)

    def grow(self, seq_id: int, new_len: int) -> List[int]:
        """Ensure ``seq_id`` can hold ``new_len`` tokens; returns its block table."""
        n = self.blocks_needed(seq_id, new_len)
        if n > len(self._free):
            raise OutOfBlocks(f"need {n} blocks for seq {seq_id}, {len(self._free)} free")
        tab = self.tables.setdefault(seq_id, [])
        for _ in range(n):
            tab.append(self._free.pop())
        self.lengths[seq_id] = max(self.lengths.get(seq_id, 0), int(new_len))
        return tab

    def free(self, seq_id: int) -> None:
        for b in reversed(self.tables.pop(seq_id, [])):
            self._free.append(b)
        self._free.sort(reverse=True)
        self.lengths.pop(seq_id, None)

    def reset(self) -> None:
        self.__init__(self.num_blocks, self.block_size)

    def table_tensor(self, seq_ids: Sequence[int], width: Optional[int] = None, device="cpu") -> torch.Tensor:
        """``[len(seq_ids), width]`` int32 block tables padded with 0 (padding is never read: lengths bound it)."""
        width = width or max((len(self.tables.get(s, ())) for s in seq_ids), default=1) or 1
        t = torch.zeros(len(seq_ids), width, dtype=torch.int32)
        for i, s in enumerate(seq_ids):
            tab = self.tables.get(s, [])
            if tab:
                t[i, :len(tab)] = torch.tensor(tab, dtype=torch.int32)
        return t.to(device)


@dataclass
class PagedKVPool:
    """Per-layer K and V block pools."""

    layers: int
    num_blocks: int
    kv_heads: int
    head_dim: int
    block_size: int = 16
    dtype: torch.dtype = torch.bfloat16
    device: str | torch.device = "cpu"
    k: List[torch.Tensor] = field(default_factory=list)
    v: List[torch.Tensor] = field(default_factory=list)

    def __post_init__(self):
        shape = (self.num_blocks, self.kv_heads, self.block_size, self.head_dim)
        self.k = [torch.zeros(shape, dtype=self.dtype, device=self.device) for _ in range(self.layers)]
        self.v = [torch.zeros(shape, dtype=self.dtype, device=self.device) for _ in range(self.layers)]

    @property
    def bytes(self) -> int:
        return 2 * self.layers * self.num_blocks * self.kv_heads * self.block_size * self.head_dim * \
            torch.finfo(self.dtype).bits // 8

    @staticmethod
    def blocks_for_budget(budget_bytes: int, layers: int, kv_heads: int, head_dim: int, block_size: int = 16,
                          dtype=torch.bfloat16) -> int:
        per_block = 2 * layers * kv_heads * block_size * head_dim * torch.finfo(dtype).bits // 8
        return max(1, int(budget_bytes // per_block))


def write_kv_reference(pool_k: torch.Tensor, pool_v: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       block_table: Sequence[int], start_pos: int) -> None:
    """Host-side reference of the paged append: token ``t`` of ``k [T, Hk, D]`` goes to position
    ``start_pos + t`` -> block ``table[pos // bs]``, slot ``pos % bs``."""
    bs = pool_k.shape[2]
    for t in range(k.shape[0]):
        pos = start_pos + t
        b = block_table[pos // bs]
        pool_k[b, :, pos % bs] = k[t].to(pool_k.dtype)
        pool_v[b, :, pos % bs] = v[t].to(pool_v.dtype)


def gather_kv_reference(pool: torch.Tensor, block_table: Sequence[int], length: int) -> torch.Tensor:
    """``[length, Hk, D]`` view of a sequence's cached keys or values."""
    bs = pool.shape[2]
    nb = (length + bs - 1) // bs
    blocks = pool[torch.as_tensor(list(block_table[:nb]), dtype=torch.long)]     # [nb, Hk, bs, D]
    return blocks.permute(0, 2, 1, 3).reshape(nb * bs, pool.shape[1], pool.shape[3])[:length]
