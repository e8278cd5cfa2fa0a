"""Continuous-batching scheduler on the CPU engine: concurrent requests with different lengths join and leave the
decode batch; each request's tokens equal an isolated greedy run."""
import pytest
import torch

from hrm_flashrenderer_b200.config import TINY, EngineConfig
from hrm_flashrenderer_b200.models.llama import LlamaW8
from hrm_flashrenderer_b200.models.weights import synth_weights
from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
from hrm_flashrenderer_b200.runtime.scheduler import Scheduler


def _engine():
    w = synth_weights(TINY, seed=4)
    m = LlamaW8.from_weights(TINY, w, device="cpu", max_pos=512)
    return InferenceEngine(m, EngineConfig(max_seq_len=256, max_batch=4, prefill_chunk=40, use_cuda_graphs=False,
                                           graph_batch_buckets=(1, 2, 4)), num_blocks=96)


def test_scheduler_matches_isolated_runs():
    g = torch.Generator().manual_seed(7)
    reqs = [(torch.randint(0, 1024, (int(torch.randint(5, 30, (1,), generator=g)),), generator=g).tolist(),
             int(torch.randint(3, 12, (1,), generator=g))) for _ in range(7)]
    ref_eng = _engine()
    ref = [ref_eng.generate([p], n, stop_on_eos=False)[0] for p, n in reqs]
    sched = Scheduler(_engine()).start()
    try:
        handles = [sched.submit(p, n, stop_on_eos=False) for p, n in reqs]
        got = [h.future.result(timeout=120) for h in handles]
    finally:
        sched.stop()
    assert got == ref
    m = sched.metrics()
    assert m["completed"] == 7 and m["generated_tokens"] == sum(n for _, n in reqs)
    assert m["ttft_p50_ms"] is not None


def test_scheduler_rejects_oversize():
    sched = Scheduler(_engine())
    import pytest
    with pytest.raises(ValueError):
        sched.submit(list(range(250)), 100)


def test_scheduler_tight_kv_pool_never_runs_out():
    """A pool that holds only a few requests at a time: admission waits for blocks instead of over-committing, so
    every request completes (decode staging reserves each sequence's own remaining length)."""
    w = synth_weights(TINY, seed=4)
    m = LlamaW8.from_weights(TINY, w, device="cpu", max_pos=512)
    eng = InferenceEngine(m, EngineConfig(max_seq_len=256, max_batch=4, prefill_chunk=64, use_cuda_graphs=False,
                                          graph_batch_buckets=(1, 2, 4)), num_blocks=14)
    g = torch.Generator().manual_seed(11)
    reqs = [(torch.randint(0, 1024, (int(torch.randint(5, 40, (1,), generator=g)),), generator=g).tolist(),
             int(torch.randint(2, 40, (1,), generator=g))) for _ in range(12)]
    sched = Scheduler(eng).start()
    try:
        handles = [sched.submit(p, n, stop_on_eos=False) for p, n in reqs]
        got = [h.future.result(timeout=300) for h in handles]
    finally:
        sched.stop()
    assert [len(t) for t in got] == [n for _, n in reqs]
    assert sched.metrics()["completed"] == 12
    assert eng.bm.free_blocks == 14


def test_scheduler_rejects_request_larger_than_pool():
    import pytest
    w = synth_weights(TINY, seed=4)
    m = LlamaW8.from_weights(TINY, w, device="cpu", max_pos=512)
    eng = InferenceEngine(m, EngineConfig(max_seq_len=256, max_batch=2, use_cuda_graphs=False), num_blocks=4)
    with pytest.raises(ValueError):
        Scheduler(eng).submit(list(range(60)), 10)     # 71 positions = 5 blocks > 4


def _fail_prefill(eng, exc, times=None):
    """Make the engine's prefill raise ``exc`` (``times`` calls, then work again)."""
    real = eng.prefill
    left = [times]

    def bad(*a, **k):
        if left[0] is None or left[0] > 0:
            if left[0] is not None:
                left[0] -= 1
            raise exc
        return real(*a, **k)
    eng.prefill = bad


def test_sticky_cuda_error_makes_the_scheduler_fatal():
    """A context-poisoning CUDA error: in-flight and queued requests fail, new ones are refused at once and the
    scheduler reports itself dead (lane health false -> failover and a supervisor restart)."""
    import pytest
    from hrm_flashrenderer_b200.runtime.scheduler import is_context_fatal
    eng = _engine()
    err = RuntimeError("CUDA error: an illegal memory access was encountered")
    assert is_context_fatal(err) and not is_context_fatal(RuntimeError("shape mismatch"))
    _fail_prefill(eng, err)
    sched = Scheduler(eng).start()
    try:
        r = sched.submit(list(range(5, 15)), 4)
        with pytest.raises(RuntimeError, match="illegal memory access"):
            r.future.result(timeout=60)
        sched._thread.join(timeout=30)
        assert not sched.alive() and "illegal memory access" in sched.metrics()["fatal"]
        assert eng.bm.free_blocks == eng.bm.num_blocks          # the failed request's blocks went back
        with pytest.raises(RuntimeError, match="fatal error"):
            sched.submit([5, 6, 7], 2)
    finally:
        sched.stop()


def test_transient_errors_keep_serving_until_the_limit():
    import pytest
    eng = _engine()
    _fail_prefill(eng, ValueError("transient"), times=1)
    sched = Scheduler(eng).start()
    try:
        with pytest.raises(ValueError):
            sched.submit([5, 6, 7, 8], 3).future.result(timeout=60)
        assert len(sched.submit([5, 6, 7, 8], 3).future.result(timeout=60)) == 3   # served after one failure
        assert sched.alive() and sched.metrics()["fatal"] is None
        _fail_prefill(eng, ValueError("broken"))
        for _ in range(sched.max_consecutive_failures):
            with pytest.raises((ValueError, RuntimeError)):
                sched.submit([5, 6, 7, 8], 3).future.result(timeout=60)
        sched._thread.join(timeout=30)
        assert not sched.alive() and "broken" in sched.metrics()["fatal"]
    finally:
        sched.stop()


class _Recorder:
    """Wraps an engine and records the order of prefill forwards (prompt tokens) and decode steps."""

    def __init__(self, eng):
        self.eng, self.log = eng, []

    def __getattr__(self, k):
        return getattr(self.eng, k)

    def prefill(self, seqs, *rest):
        self.log.append(("prefill", sum(len(t) for _, t in seqs)))
        return self.eng.prefill(seqs, *rest)

    def decode_step(self, g):
        self.log.append(("decode", 0))
        return self.eng.decode_step(g)


def test_long_prompt_prefill_interleaves_with_decode():
    """A long prompt that arrives while another request decodes is prefilled in interleave-sized chunks with decode
    steps in between, and both requests still produce exactly their isolated greedy tokens."""
    import time
    g = torch.Generator().manual_seed(3)
    short = torch.randint(0, 1024, (8,), generator=g).tolist()
    long_ = torch.randint(0, 1024, (100,), generator=g).tolist()
    ref_eng = _engine()
    ref = [ref_eng.generate([p], n, stop_on_eos=False)[0] for p, n in ((short, 40), (long_, 5))]
    rec = _Recorder(_engine())
    sched = Scheduler(rec, interleave_chunk=16).start()
    try:
        h1 = sched.submit(short, 40, stop_on_eos=False)
        t0 = time.time()
        while not h1.tokens and time.time() - t0 < 60:   # the short request is decoding
            time.sleep(0.001)
        h2 = sched.submit(long_, 5, stop_on_eos=False)
        got = [h1.future.result(timeout=120), h2.future.result(timeout=120)]
    finally:
        sched.stop()
    assert got == ref
    pre = [i for i, (k, _) in enumerate(rec.log) if k == "prefill"]
    long_chunks = [rec.log[i][1] for i in pre[1:]]
    assert sum(long_chunks) == 100 and max(long_chunks) <= 16, rec.log
    # a decode step between consecutive chunks of the long prompt
    assert all(any(k == "decode" for k, _ in rec.log[a + 1:b]) for a, b in zip(pre[1:], pre[2:])), rec.log


class _FlakyEngine:
    """Engine wrapper whose decode step raises once (a transient, non-fatal error)."""

    def __init__(self, eng):
        self.eng, self.failed = eng, False

    def __getattr__(self, k):
        return getattr(self.eng, k)

    def decode_step(self, g):
        if not self.failed:
            self.failed = True
            raise RuntimeError("transient decode failure")
        return self.eng.decode_step(g)


def test_transient_decode_error_fails_only_running_requests():
    """A non-fatal error fails (and frees) only the requests that were in the engine; requests still queued are
    served afterwards."""
    import pytest
    g = torch.Generator().manual_seed(5)
    reqs = [torch.randint(0, 1024, (12,), generator=g).tolist() for _ in range(6)]
    eng = _FlakyEngine(_engine())
    sched = Scheduler(eng, max_batch=2)
    handles = [sched.submit(p, 6, stop_on_eos=False) for p in reqs]   # queued before the loop starts
    sched.start()
    try:
        outcomes = []
        for h in handles:
            try:
                outcomes.append(len(h.future.result(timeout=120)))
            except RuntimeError as e:
                assert "transient decode failure" in str(e)
                outcomes.append("failed")
    finally:
        sched.stop()
    assert outcomes.count("failed") == 2 and outcomes[2:] == [6, 6, 6, 6]
    assert sched.fatal is None and eng.bm.free_blocks == eng.bm.num_blocks


def test_concurrent_submitters_get_their_isolated_tokens():
    """Eight threads submit 24 requests at once (greedy and sampled, different lengths); every request still gets
    exactly the tokens of its isolated run: batching, admission order and the submitting thread change nothing."""
    import threading
    from hrm_flashrenderer_b200.runtime.sampling import SamplingParams
    g = torch.Generator().manual_seed(11)
    reqs = []
    for i in range(24):
        prompt = torch.randint(0, 1024, (int(torch.randint(3, 40, (1,), generator=g)),), generator=g).tolist()
        sp = SamplingParams(temperature=0.7 + 0.1 * (i % 3), top_k=(0, 8, 50)[i % 3], seed=1000 + i) if i % 2 else None
        reqs.append((prompt, 4 + i % 7, sp))
    ref_eng = _engine()
    want = [ref_eng.generate([p], n, stop_on_eos=False, sampling=sp)[0] for p, n, sp in reqs]
    sched = Scheduler(_engine(), interleave_chunk=16).start()
    got = [None] * len(reqs)
    errors = []

    def worker(ids):
        try:
            hs = [(i, sched.submit(reqs[i][0], reqs[i][1], stop_on_eos=False, sampling=reqs[i][2])) for i in ids]
            for i, h in hs:
                got[i] = h.future.result(timeout=300)
        except BaseException as e:   # surfaced by the main thread
            errors.append(e)

    try:
        ts = [threading.Thread(target=worker, args=(list(range(t, 24, 8)),)) for t in range(8)]
        for t in ts:
            t.start()
        for t in ts:
            t.join(timeout=600)
    finally:
        sched.stop()
    assert not errors, errors
    assert got == want


def _engine_pc(prefix_cache, num_blocks=96):
    w = synth_weights(TINY, seed=4)
    m = LlamaW8.from_weights(TINY, w, device="cpu", max_pos=512)
    return InferenceEngine(m, EngineConfig(max_seq_len=256, max_batch=4, prefill_chunk=40, use_cuda_graphs=False,
                                           graph_batch_buckets=(1, 2, 4), prefix_cache=prefix_cache),
                           num_blocks=num_blocks)


def test_prefix_cache_gives_the_same_tokens_and_skips_shared_blocks():
    """Requests that share a 48-token system prefix: with the prefix cache the later ones reuse its KV blocks (fewer
    prompt tokens prefilled) and every request still produces its isolated tokens, greedy and sampled; a pool too
    small to keep everything cached evicts and stays correct."""
    from hrm_flashrenderer_b200.runtime.sampling import SamplingParams
    g = torch.Generator().manual_seed(21)
    system = torch.randint(0, 1024, (48,), generator=g).tolist()
    reqs = [(system + torch.randint(0, 1024, (int(n),), generator=g).tolist(), 6,
             SamplingParams(0.8, 20, 40 + i) if i % 3 == 2 else None)
            for i, n in enumerate(torch.randint(1, 30, (9,), generator=g))]
    ref = _engine_pc(False)
    want = [ref.generate([p], n, stop_on_eos=False, sampling=sp)[0] for p, n, sp in reqs]
    for blocks in (96, 24):
        eng = _engine_pc(True, blocks)
        rec = _Recorder(eng)
        sched = Scheduler(rec, interleave_chunk=16).start()
        try:
            got = []
            for p, n, sp in reqs:                  # one after another: each finds the published prefix
                got.append(sched.generate(p, n, timeout=120, stop_on_eos=False, sampling=sp))
            hits = sched.metrics()["prefix_cache_hit_blocks"]
        finally:
            sched.stop()
        assert got == want, blocks
        prefilled = sum(t for k, t in rec.log if k == "prefill")
        assert hits >= 3 * (len(reqs) - 1) and prefilled == sum(len(p) for p, _, _ in reqs) - 16 * hits


def test_cancel_running_waiting_and_timed_out_requests():
    """A cancelled request leaves the batch before its next step and gives its KV blocks back; a request cancelled
    while queued never reaches the engine; ``generate`` cancels a request whose wait timed out; requests that run
    alongside still produce their isolated tokens."""
    import time
    from concurrent.futures import CancelledError
    from concurrent.futures import TimeoutError as FutureTimeout
    g = torch.Generator().manual_seed(13)
    keep = torch.randint(0, 1024, (10,), generator=g).tolist()
    ref = _engine().generate([keep], 30, stop_on_eos=False)[0]
    eng = _engine()
    total = eng.bm.free_blocks
    sched = Scheduler(eng, max_batch=2).start()
    try:
        long_ = sched.submit(torch.randint(0, 1024, (12,), generator=g).tolist(), 200, stop_on_eos=False)
        other = sched.submit(keep, 30, stop_on_eos=False)
        queued = sched.submit([1, 2, 3], 5, stop_on_eos=False)      # batch full: waits
        sched.cancel(queued)
        t0 = time.time()
        while len(long_.tokens) < 5 and time.time() - t0 < 60:
            time.sleep(0.001)
        sched.cancel(long_)
        with pytest.raises(CancelledError):
            long_.future.result(timeout=60)
        with pytest.raises(CancelledError):
            queued.future.result(timeout=60)
        assert queued.seq_id == -1 and len(long_.tokens) < 200
        assert other.future.result(timeout=120) == ref
        with pytest.raises(FutureTimeout):
            sched.generate([4, 5, 6], 200, timeout=0.05, stop_on_eos=False)
        t0 = time.time()
        while (sched.metrics()["batch_size"] or sched.metrics()["prefilling"]) and time.time() - t0 < 60:
            time.sleep(0.01)
        assert sched.metrics()["cancelled"] == 3
        assert eng.bm.free_blocks == total
    finally:
        sched.stop()


def test_stop_fails_requests_in_flight_and_refuses_new_ones():
    import time
    eng = _engine()
    step = eng.decode_step

    def slow(g):
        time.sleep(0.01)
        return step(g)
    eng.decode_step = slow
    sched = Scheduler(eng, max_batch=1).start()
    running = sched.submit([1, 2, 3], 200, stop_on_eos=False)
    queued = sched.submit([4, 5, 6], 5, stop_on_eos=False)
    t0 = time.time()
    while not running.tokens and time.time() - t0 < 60:
        time.sleep(0.001)
    sched.stop()
    for r in (running, queued):
        with pytest.raises(RuntimeError, match="stopped"):
            r.future.result(timeout=10)
    with pytest.raises(RuntimeError, match="stopped"):
        sched.submit([7], 2)
    assert eng.bm.free_blocks == eng.bm.num_blocks
