"""TP-group heartbeat watchdog: a fake store + clock (deterministic), and real processes on a TCPStore where one
rank dies without a word and another leaves cleanly (failures made on the host only)."""
import os
import socket
import time

import pytest
import torch.multiprocessing as mp

from hrm_flashrenderer_b200.parallel.watchdog import HeartbeatWatchdog, PeerFailure


class FakeStore:
    def __init__(self):
        self.kv = {}

    def set(self, k, v):
        self.kv[k] = v.encode() if isinstance(v, str) else v

    def get(self, k):
        return self.kv[k]

    def check(self, keys):
        return all(k in self.kv for k in keys)


def test_fake_clock_detects_silence_and_leave():
    st, now = FakeStore(), [0.0]
    clock = lambda: now[0]
    w = [HeartbeatWatchdog(st, r, 3, interval_s=1, timeout_s=3, clock=clock) for r in range(3)]
    for x in w:
        x.beat()
    w[0].check()                                   # everyone fresh
    for t in range(1, 5):                          # ranks 0 and 1 keep beating, rank 2 is silent
        now[0] = float(t)
        w[0].beat()
        w[1].beat()
        if t < 4:
            w[0].check()
    with pytest.raises(PeerFailure) as e:
        w[0].check()
    assert e.value.dead == [2] and e.value.left == []
    w[1].stop(clean=True)
    assert w[0].dead_peers() == [1, 2]


def test_peer_never_started_counts_from_watchdog_start():
    st, now = FakeStore(), [0.0]
    w0 = HeartbeatWatchdog(st, 0, 2, timeout_s=2, clock=lambda: now[0])
    w0.beat()
    now[0] = 1.0
    assert w0.dead_peers() == []
    now[0] = 3.0
    assert w0.dead_peers() == [1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _proc(rank, world, port, mode, q):
    import torch.distributed as dist
    st = dist.TCPStore("127.0.0.1", port, world, is_master=rank == 0, timeout=__import__("datetime").timedelta(30))
    w = HeartbeatWatchdog(st, rank, world, interval_s=0.1, timeout_s=1.0).start()
    if rank == 0:
        t0 = time.time()
        while time.time() - t0 < 15:
            try:
                w.check()
            except PeerFailure as e:
                q.put((e.dead, e.left, round(time.time() - t0, 1)))
                break
            time.sleep(0.05)
        else:
            q.put(None)
        time.sleep(0.5)
        w.stop()
        return
    if rank == 2 and mode == "crash":
        time.sleep(0.5)
        os._exit(0)                                # dies without stopping its watchdog
    if rank == 1 and mode == "leave":
        time.sleep(0.5)
        w.stop(clean=True)
        return
    time.sleep(6)
    w.stop()


@pytest.mark.parametrize("mode,expect", [("crash", ([2], [])), ("leave", ([], [1]))])
def test_tcpstore_ranks(mode, expect):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_proc, args=(r, 3, port, mode, q)) for r in range(3)]
    for p in ps:
        p.start()
    res = q.get(timeout=60)
    for p in ps:
        p.join(timeout=30)
    assert res is not None, "rank 0 never noticed the lost peer"
    dead, left, after = res
    assert (dead, left) == expect
    assert after < 5.0
