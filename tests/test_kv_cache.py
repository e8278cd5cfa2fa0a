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


# ---------------------------------------------------------------------------------------------- prefix cache
def _prompt(n, seed):
    r = random.Random(seed)
    return [r.randrange(1000) for _ in range(n)]


def test_prefix_cache_shares_published_blocks():
    bm = BlockManager(64, prefix_cache=True)
    sysp = _prompt(40, 1)                       # 2 full blocks + 8 tokens
    a = sysp + _prompt(20, 2)
    assert bm.match_prefix(0, a) == 0           # nothing published yet
    bm.grow(0, len(a))
    assert bm.publish(0, a) == 3                # 60 tokens: 3 full blocks
    b = sysp + _prompt(30, 3)
    assert bm.match_prefix(1, b) == 32          # the two blocks of the shared prefix, not the third (differs)
    assert bm.tables[1] == bm.tables[0][:2] and bm.lengths[1] == 32
    bm.grow(1, len(b))
    assert bm.tables[1][:2] == bm.tables[0][:2] and bm.tables[1][2] not in bm.tables[0]
    assert bm.match_prefix(2, a) == 48          # an identical prompt: every full block but the one with its last token
    # the same prompt exactly one block long leaves its only block to recompute (one token must be computed)
    assert bm.match_prefix(3, a[:16]) == 0


def test_prefix_cache_refcounts_idle_blocks_and_eviction():
    bm = BlockManager(16, prefix_cache=True, tile_blocks=4)
    a = _prompt(64, 5)
    bm.grow(0, 64)
    bm.publish(0, a)
    assert bm.free_blocks == 12
    bm.match_prefix(1, a)                       # shares 3 blocks
    bm.free(0)
    assert bm.free_blocks == 12 + 1             # block 3 idle (published, unused); blocks 0-2 still used by seq 1
    bm.free(1)
    assert bm.free_blocks == 16 and bm._nfree == 12 and len(bm._idle) == 4
    assert bm.match_prefix(2, a + [1]) == 64    # idle blocks are revived
    bm.free(2)
    # a sequence that needs every block evicts the idle cached ones (least recently freed first)
    bm.grow(3, 16 * 16)
    assert bm.free_blocks == 0 and not bm._block_of and not bm._idle
    bm.free(3)
    assert bm.free_blocks == 16
    assert bm.match_prefix(4, a) == 0           # evicted prefixes are gone


def test_prefix_cache_off_is_the_plain_allocator():
    for pc in (False, True):
        bm = BlockManager(256, prefix_cache=pc)
        tabs = [list(bm.grow(s, 100 + 37 * s)) for s in range(5)]
        assert bm.match_prefix(9, list(range(200))) == 0
        if pc:
            continue
        ref = BlockManager(256)
        assert tabs == [ref.grow(s, 100 + 37 * s) for s in range(5)]


def test_prefix_cache_random_workload_keeps_invariants():
    """Random admissions (shared and private prefixes), growth, publication and release: every block is free,
    idle-cached or used, reference counts equal the number of tables holding the block, and no table holds a
    block twice."""
    rng = random.Random(7)
    bm = BlockManager(96, prefix_cache=True)
    heads = [_prompt(48, 100 + i) for i in range(3)]
    live = {}
    for step in range(600):
        if live and (rng.random() < 0.4 or bm.free_blocks < 12):
            sid = rng.choice(list(live))
            bm.free(sid)
            del live[sid]
        else:
            sid = step
            p = rng.choice(heads)[: rng.randrange(1, 48)] + _prompt(rng.randrange(1, 40), step)
            bm.match_prefix(sid, p)
            try:
                bm.grow(sid, len(p) + rng.randrange(0, 20))
            except OutOfBlocks:
                bm.free(sid)
                continue
            bm.publish(sid, p)
            live[sid] = p
        used = {}
        for s, tab in bm.tables.items():
            assert len(set(tab)) == len(tab)
            for b in tab:
                used[b] = used.get(b, 0) + 1
        for b in range(bm.num_blocks):
            assert bm._ref[b] == used.get(b, 0)
            state = (bool(bm._is_free[b]), b in bm._idle, b in used)
            assert sum(state) == 1, (b, state)
        assert bm.free_blocks == bm._nfree + len(bm._idle)
        assert all(bm._block_of[k] == b for b, k in bm._key_of.items())
