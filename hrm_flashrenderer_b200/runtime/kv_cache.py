"""Block-table paged KV cache (block size 16 by default) and its block manager.

Replaces the reference's per-sequence contiguous pages ``[B,Hk,P,PS,D]`` that grow by power-of-two reallocation
and copy (``engine/llama_tp.py:21-108``, reference quirk Q10): here a fixed pool of blocks is allocated once, every
sequence owns a list of block ids (its block table), and growth is a table append.  Pool layout per layer:
``[num_blocks, kv_heads, block_size, head_dim]`` so one (block, head) is a contiguous ``block_size*head_dim``
run (4 KB at bf16/D=128), the unit the attention kernels fetch.
"""
from __future__ import annotations

import hashlib
import heapq
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch


class OutOfBlocks(RuntimeError):
    pass


class BlockManager:
    """Free-list allocator of KV blocks, deterministic and tile-aware.

    The attention kernels read keys in tiles of ``tile_blocks`` consecutive table entries (128 keys = 8 blocks of 16)
    and fetch a tile with ONE TMA box when its block ids are consecutive, else one box per block.  So:
      * a block that starts a tile (table position % tile_blocks == 0) is the first id of the lowest fully free
        aligned group of ``tile_blocks`` ids, when one exists;
      * any other block is the id right after the sequence's previous block, when that id is free;
      * otherwise the lowest free id.
    Nothing is reserved: another sequence may take an id of a started group, which only costs that tile its fast
    fetch.  The reference grows contiguous per-sequence pages by reallocation instead (``engine/llama_tp.py:21-108``).

    ``prefix_cache``: full prompt blocks are published under a hash chain of their tokens (each key covers the
    whole prefix up to that block), blocks are reference-counted, and a new sequence whose prompt starts with
    published blocks shares them instead of recomputing them (:meth:`match_prefix`).  A published block whose last
    user leaves stays cached and is evicted least-recently-freed first when a sequence needs a block.  Shared blocks
    are never written: a sequence only writes positions at or after its own length, which starts behind its last
    shared block.
    """

    def __init__(self, num_blocks: int, block_size: int = 16, tile_blocks: int = 8, prefix_cache: bool = False):
        self.num_blocks = int(num_blocks)
        self.block_size = int(block_size)
        self.tile_blocks = max(1, int(tile_blocks))
        self._is_free = bytearray(b"\x01") * self.num_blocks
        self._nfree = self.num_blocks
        self._heap: List[int] = list(range(self.num_blocks))                 # lowest-free heap (lazy deletion)
        ng = self.num_blocks // self.tile_blocks                              # only whole groups are candidates
        self._gfree = [self.tile_blocks] * ng
        self._gheap: List[int] = list(range(ng))                              # fully free groups (lazy deletion)
        self.tables: Dict[int, List[int]] = {}
        self.lengths: Dict[int, int] = {}
        self.prefix_cache = bool(prefix_cache)
        self._ref = [0] * self.num_blocks                      # users of each block
        self._key_of: Dict[int, bytes] = {}                     # published block -> prefix key
        self._block_of: Dict[bytes, int] = {}                   # prefix key -> published block
        self._idle: "OrderedDict[int, None]" = OrderedDict()    # published blocks without users (evictable)
        self.prefix_hits = 0                                    # blocks shared instead of recomputed

    @property
    def free_blocks(self) -> int:
        """Blocks a sequence can still take: free ones plus cached blocks nobody uses."""
        return self._nfree + len(self._idle)

    def _keys(self, tokens: Sequence[int], nblocks: int) -> List[bytes]:
        bs, out, prev = self.block_size, [], b""
        for i in range(nblocks):
            h = hashlib.sha256(prev)
            h.update(",".join(str(int(t)) for t in tokens[i * bs:(i + 1) * bs]).encode())
            prev = h.digest()
            out.append(prev)
        return out

    def match_prefix(self, seq_id: int, tokens: Sequence[int]) -> int:
        """Share the longest run of published blocks that starts ``tokens`` with the new sequence ``seq_id``; at least
        one token is left to compute (its logits give the first generated token).  Returns the tokens covered."""
        if not self.prefix_cache or self.tables.get(seq_id):
            return 0
        tab = self.tables.setdefault(seq_id, [])
        for key in self._keys(tokens, (len(tokens) - 1) // self.block_size):
            b = self._block_of.get(key)
            if b is None:
                break
            if self._ref[b] == 0:
                self._idle.pop(b, None)
            self._ref[b] += 1
            tab.append(b)
        self.prefix_hits += len(tab)
        self.lengths[seq_id] = len(tab) * self.block_size
        return self.lengths[seq_id]

    def publish(self, seq_id: int, tokens: Sequence[int]) -> int:
        """Publish the full blocks of ``seq_id`` that hold ``tokens`` (its prompt, already in the cache); returns the
        number of newly published blocks.  A prefix some other block already publishes is left as it is."""
        if not self.prefix_cache:
            return 0
        tab = self.tables.get(seq_id, [])
        n = min(len(tokens) // self.block_size, len(tab))
        added = 0
        for b, key in zip(tab[:n], self._keys(tokens, n)):
            if key in self._block_of or b in self._key_of:
                continue
            self._block_of[key] = b
            self._key_of[b] = key
            added += 1
        return added

    def _evict(self, n: int) -> None:
        """Return ``n`` idle cached blocks (least recently freed first) to the free pool."""
        for _ in range(n):
            b, _ = self._idle.popitem(last=False)
            del self._block_of[self._key_of.pop(b)]
            self._release_block(b)

    def _release_block(self, b: int) -> None:
        tb = self.tile_blocks
        self._is_free[b] = 1
        self._nfree += 1
        heapq.heappush(self._heap, b)
        g = b // tb
        if g < len(self._gfree):
            self._gfree[g] += 1
            if self._gfree[g] == tb:
                heapq.heappush(self._gheap, g)

    def blocks_needed(self, seq_id: int, new_len: int) -> int:
        have = len(self.tables.get(seq_id, ()))
        need = (int(new_len) + self.block_size - 1) // self.block_size
        return max(0, need - have)

    def can_grow(self, seq_id: int, new_len: int) -> bool:
        return self.blocks_needed(seq_id, new_len) <= self.free_blocks

    def _take(self, b: int) -> int:
        self._is_free[b] = 0
        self._nfree -= 1
        self._ref[b] = 1
        g = b // self.tile_blocks
        if g < len(self._gfree):
            self._gfree[g] -= 1
        return b

    def _pick(self, tab: List[int]) -> int:
        tb = self.tile_blocks
        if tab and len(tab) % tb:
            nxt = tab[-1] + 1
            if nxt < self.num_blocks and self._is_free[nxt]:
                return self._take(nxt)
        else:
            while self._gheap and self._gfree[self._gheap[0]] != tb:
                heapq.heappop(self._gheap)
            if self._gheap:
                return self._take(heapq.heappop(self._gheap) * tb)
        while not self._is_free[self._heap[0]]:
            heapq.heappop(self._heap)
        return self._take(heapq.heappop(self._heap))

    def grow(self, seq_id: int, new_len: int) -> List[int]:
        """Ensure ``seq_id`` can hold ``new_len`` tokens; returns its block table."""
        n = self.blocks_needed(seq_id, new_len)
        if n > self.free_blocks:
            raise OutOfBlocks(f"need {n} blocks for seq {seq_id}, {self.free_blocks} free")
        if n > self._nfree:
            self._evict(n - self._nfree)
        tab = self.tables.setdefault(seq_id, [])
        for _ in range(n):
            tab.append(self._pick(tab))
        self.lengths[seq_id] = max(self.lengths.get(seq_id, 0), int(new_len))
        return tab

    def free(self, seq_id: int) -> None:
        for b in self.tables.pop(seq_id, []):
            self._ref[b] -= 1
            if self._ref[b] > 0:
                continue                       # still shared by another sequence
            if b in self._key_of:
                self._idle[b] = None           # cached: reusable until evicted
            else:
                self._release_block(b)
        self.lengths.pop(seq_id, None)

    def reset(self) -> None:
        self.__init__(self.num_blocks, self.block_size, self.tile_blocks, self.prefix_cache)

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
