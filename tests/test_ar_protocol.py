"""Host-side models of the peer-memory protocols: the fused row-parallel all-reduce's per-tile protocol
(``ar_tile_finish`` in ``csrc/gemm_w8a16_impl.cuh``) and, further down, the in-kernel argmax exchange.

Per launch (epoch ``ep``) and tile ``t``, the rank that finishes the tile
  1. pushes its fp32 partial into slot ``[dst][src = me][parity = ep & 1][t]`` of every rank,
  2. after a fence, stores ``flag[dst][src = me][t] = ep`` on every rank,
  3. waits until ``flag[me][src][t] >= ep`` for every source rank (epochs only grow), then
  4. reduces the tile from its own slots ``[me][src][ep & 1][t]`` in rank order.
A rank starts launch ``L + 1`` only after all of its tiles of launch ``L`` are done (stream order; the kernel's
programmatic-launch wait covers the previous grid's memory operations).

The model runs every rank's steps in random interleavings and checks that each reduction reads exactly the partials
of its own launch (no slot is overwritten before its reader is done) and that nothing deadlocks.  It also shows why
the wait is ">=": with an exact-equality wait, a fast peer that already published the next epoch's flag strands a
slow rank.  This checks the protocol, not the hardware.
"""
import random

import pytest


def _run(ranks, tiles, launches, seed, exact_wait=False):
    rng = random.Random(seed)
    slot = {}                       # (dst, src, parity, tile) -> (launch, src, tile)
    flag = {}                       # (dst, src, tile) -> epoch
    # per rank: current launch and, per tile, its step (0 push, 1 flag, 2 wait, 3 reduce, 4 done)
    launch = [0] * ranks
    step = [[0] * tiles for _ in range(ranks)]
    reads = 0
    while True:
        enabled = []
        for r in range(ranks):
            if launch[r] >= launches:
                continue
            ep = launch[r] + 1
            for t in range(tiles):
                s = step[r][t]
                if s in (0, 1, 3):
                    enabled.append((r, t))
                elif s == 2:
                    ok = all((flag.get((r, src, t), 0) == ep) if exact_wait else (flag.get((r, src, t), 0) >= ep)
                             for src in range(ranks))
                    if ok:
                        enabled.append((r, t))
        if not enabled:
            done = all(l >= launches for l in launch)
            return done, reads
        r, t = rng.choice(enabled)
        L = launch[r]
        ep, par = L + 1, (L + 1) & 1
        s = step[r][t]
        if s == 0:
            for d in range(ranks):
                slot[(d, r, par, t)] = (L, r, t)
        elif s == 1:
            for d in range(ranks):
                flag[(d, r, t)] = ep
        elif s == 3:
            for src in range(ranks):
                assert slot[(r, src, par, t)] == (L, src, t), ("stale or overwritten partial", r, src, t, L)
            reads += 1
        step[r][t] = s + 1 if s != 2 else 3
        if all(x == 4 for x in step[r]):
            launch[r] += 1
            step[r] = [0] * tiles


@pytest.mark.parametrize("ranks,tiles", [(2, 1), (2, 3), (4, 2), (8, 2)])
def test_per_tile_protocol_reads_its_own_launch_and_never_deadlocks(ranks, tiles):
    for seed in range(150):
        done, reads = _run(ranks, tiles, launches=6, seed=seed)
        assert done, seed
        assert reads == ranks * tiles * 6


def test_exact_epoch_wait_can_strand_a_slow_rank():
    stranded = sum(not _run(2, 1, launches=6, seed=s, exact_wait=True)[0] for s in range(300))
    assert stranded > 0


def _run_argmax(ranks, rows, launches, seed):
    """The in-kernel argmax exchange (``argmax_exchange_row`` in ``csrc/attention.cu``): per launch, each row's
    final thread reads the rank's epoch counter (ep = counter + 1), writes its key into slot
    ``[ep & 1][me][row]`` of every rank, publishes ``flag[me][row] = ep`` on every rank, waits for
    ``flag[src][row] >= ep`` from every rank and takes the max of ``[ep & 1][src][row]``; then it takes a row ticket
    and the launch's last row advances the counter (every row read it before taking its ticket)."""
    rng = random.Random(seed)
    key, flag = {}, {}
    counter = [0] * ranks
    launch = [0] * ranks
    tickets = [0] * ranks
    # per (rank, row): step 0 read epoch, 1 write keys, 2 flags, 3 wait, 4 read + ticket, 5 done
    step = [[0] * rows for _ in range(ranks)]
    ep_of = [[0] * rows for _ in range(ranks)]
    while True:
        enabled = []
        for r in range(ranks):
            if launch[r] >= launches:
                continue
            for w in range(rows):
                s = step[r][w]
                if s in (0, 1, 2, 4):
                    enabled.append((r, w))
                elif s == 3 and all(flag.get((r, src, w), 0) >= ep_of[r][w] for src in range(ranks)):
                    enabled.append((r, w))
        if not enabled:
            return all(l >= launches for l in launch)
        r, w = rng.choice(enabled)
        L = launch[r]
        s = step[r][w]
        if s == 0:
            ep_of[r][w] = counter[r] + 1
        elif s == 1:
            for d in range(ranks):
                key[(d, ep_of[r][w] & 1, r, w)] = (L, r, w)
        elif s == 2:
            for d in range(ranks):
                flag[(d, r, w)] = max(flag.get((d, r, w), 0), ep_of[r][w])
        elif s == 4:
            for src in range(ranks):
                assert key[(r, ep_of[r][w] & 1, src, w)] == (L, src, w), ("wrong launch's key", r, src, w, L)
            tickets[r] += 1
            if tickets[r] == rows:
                tickets[r] = 0
                counter[r] = ep_of[r][w]
        step[r][w] = s + 1 if s != 3 else 4
        if all(x == 5 for x in step[r]):
            launch[r] += 1
            step[r] = [0] * rows


@pytest.mark.parametrize("ranks,rows", [(2, 1), (2, 4), (4, 3), (8, 2)])
def test_argmax_exchange_protocol(ranks, rows):
    for seed in range(150):
        assert _run_argmax(ranks, rows, launches=6, seed=seed), seed
