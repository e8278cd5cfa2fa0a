"""Block manager: accounting, determinism and tile contiguity (CPU only)."""
import random

import pytest

from hrm_flashrenderer_b200.runtime.kv_cache import BlockManager, OutOfBlocks


def _tiles_contiguous(tab, tb=8):
    full = len(tab) // tb
    return sum(all(tab[t * tb + j] == tab[t * tb] + j for j in range(tb)) for t in range(full)), full


def test_prefill_gets_consecutive_ids():
    bm = BlockManager(1024)
    tab = bm.grow(0, 4096)
    assert tab == list(range(256))
    assert bm.free_blocks == 1024 - 256


def test_interleaved_decode_growth_keeps_tiles_contiguous():
    """16 sequences that each grow one block at a time, round robin: every whole 128-key tile stays one id run."""
    bm = BlockManager(4096)
    for s in range(16):
        bm.grow(s, 100)
    for L in range(101, 2048, 16):
        for s in range(16):
            bm.grow(s, L)
    for s in range(16):
        ok, full = _tiles_contiguous(bm.tables[s])
        assert full > 0 and ok == full
    ids = [b for s in range(16) for b in bm.tables[s]]
    assert len(ids) == len(set(ids))
    assert bm.free_blocks == 4096 - len(ids)


def test_free_and_reuse_accounting():
    rng = random.Random(0)
    bm = BlockManager(600)
    live = {}
    for step in range(3000):
        s = rng.randrange(12)
        if s in live and rng.random() < 0.2:
            bm.free(s)
            del live[s]
            continue
        L = live.get(s, 0) + rng.randrange(1, 80)
        if bm.can_grow(s, L):
            bm.grow(s, L)
            live[s] = L
        else:
            with pytest.raises(OutOfBlocks):
                bm.grow(s, L)
        used = [b for t in bm.tables.values() for b in t]
        assert len(used) == len(set(used))
        assert bm.free_blocks == 600 - len(used)
        assert all(0 <= b < 600 for b in used)


def test_deterministic():
    def run():
        bm = BlockManager(300)
        for s in range(5):
            bm.grow(s, 37 * (s + 1))
        bm.free(2)
        for s in (0, 1, 3, 4, 7):
            bm.grow(s, 400)
        return dict(bm.tables)
    assert run() == run()


def test_exhaustion_and_reset():
    bm = BlockManager(10)
    bm.grow(0, 160)
    assert bm.free_blocks == 0 and not bm.can_grow(1, 1)
    with pytest.raises(OutOfBlocks):
        bm.grow(1, 1)
    bm.reset()
    assert bm.free_blocks == 10 and bm.grow(1, 16) == [0]


def test_table_tensor_padding():
    bm = BlockManager(64)
    bm.grow(0, 40)
    bm.grow(1, 16)
    t = bm.table_tensor([0, 1])
    assert t.shape == (2, 3)
    assert t[1, 1:].tolist() == [0, 0]
