"""Continuous-batching scheduler over :class:`~hrm_flashrenderer_b200.runtime.engine.InferenceEngine`.

One background thread owns the engine (and its CUDA graphs).  Each iteration it

1. admits waiting requests while the decode batch has room and the KV pool has blocks, and runs ONE prefill forward
   over the admitted prompts: up to ``prefill_chunk`` prompt tokens when nothing is decoding, up to
   ``interleave_chunk`` while other requests decode (a long prompt is prefilled over several iterations, so it
   delays each decode step by one bounded chunk instead of stalling the batch for its whole prefill).  A request
   whose prompt is complete yields its first token and joins the decode batch;
2. runs one graph-replayed decode step for every running request (the batch is re-staged on the device only when
   its membership changed; otherwise the sampled tokens are fed back on the device);
3. streams tokens to the requests, retires finished ones (EOS or ``max_new_tokens``) and frees their blocks.

The reference serves one request at a time per engine process (``hrm_flash/serve.py:147,235-301`` with the
``max_concurrent=1`` semaphore and file IPC into ``deepseek_native_engine``); this scheduler is what lets one lane
serve many concurrent requests with one weight stream per step.  Metrics (TTFT, inter-token latency, queue depth,
batch size, tok/s) are kept for ``/v1/health``.
"""
from __future__ import annotations

import collections
import queue
import threading
import time
from concurrent.futures import CancelledError, Future
from concurrent.futures import TimeoutError as FutureTimeout
from dataclasses import dataclass, field
from typing import Callable, Deque, Dict, List, Optional, Sequence

import torch

from .sampling import SamplingParams


# CUDA errors after which the context is unusable (every later CUDA call in the process fails as well)
_STICKY_CUDA = ("illegal memory access", "illegal instruction", "misaligned address", "unspecified launch failure",
                "device-side assert", "uncorrectable ecc", "launch timed out", "hardware stack error",
                "invalid program counter", "mmu fault", "context is destroyed", "cuda-capable device")


def is_context_fatal(e: BaseException) -> bool:
    """True for a CUDA error that leaves the process's CUDA context unusable."""
    msg = str(e).lower()
    return ("cuda" in msg or "cublas" in msg or "acceleratorerror" in type(e).__name__.lower()) and \
        any(k in msg for k in _STICKY_CUDA)


@dataclass
class GenRequest:
    prompt_ids: List[int]
    max_new_tokens: int
    stop_on_eos: bool = True
    on_token: Optional[Callable[[int], None]] = None
    rid: int = 0
    arrival: float = field(default_factory=time.perf_counter)
    first_token_at: Optional[float] = None
    finished_at: Optional[float] = None
    tokens: List[int] = field(default_factory=list)
    future: Future = field(default_factory=Future)
    seq_id: int = -1
    error: Optional[BaseException] = None
    sampling: Optional[SamplingParams] = None   # None: greedy
    cancelled: bool = False                     # set by Scheduler.cancel; the loop drops the request

    @property
    def ttft_s(self) -> Optional[float]:
        return None if self.first_token_at is None else self.first_token_at - self.arrival


class Scheduler:
    def __init__(self, engine, max_batch: Optional[int] = None, prefill_chunk: Optional[int] = None,
                 idle_sleep_s: float = 0.0005, interleave_chunk: Optional[int] = 512):
        """``interleave_chunk``: prompt tokens prefilled per iteration while requests are decoding (None or 0:
        admitted prompts are prefilled to completion before the next decode step)."""
        self.engine = engine
        self.max_batch = int(max_batch or engine.ecfg.max_batch)
        self.prefill_chunk = int(prefill_chunk or engine.ecfg.prefill_chunk)
        self.interleave_chunk = int(interleave_chunk or 0)
        self.prefix_cache = bool(getattr(engine.ecfg, "prefix_cache", False))
        self.idle_sleep_s = idle_sleep_s
        self._inbox: "queue.Queue[GenRequest]" = queue.Queue()
        self._waiting: Deque[GenRequest] = collections.deque()
        self._prefilling: List[GenRequest] = []   # admitted, prompt partly in the KV cache (r._done tokens)
        self._running: List[GenRequest] = []
        self.prefill_calls: List[int] = []        # prompt tokens of each prefill forward (bounded record)
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._next_rid = 0
        self._lock = threading.Lock()
        self.eos = set(engine.cfg.eos_token_ids)
        # metrics
        self.completed = 0
        self.cancelled_total = 0
        self.generated_tokens = 0
        self.ttfts: Deque[float] = collections.deque(maxlen=4096)
        self.itls: Deque[float] = collections.deque(maxlen=4096)
        self.started_at = time.perf_counter()
        self.last_error: Optional[str] = None
        # fatal: the engine cannot serve any more (a CUDA error that poisons the context, or
        # max_consecutive_failures failed iterations in a row).  The loop then stops, every queued request fails,
        # submit() refuses new ones and alive() is False, so the lane's health turns false: the router fails over
        # and the process supervisor restarts the lane (a lost CUDA context cannot be rebuilt in-process).
        self.fatal: Optional[str] = None
        self.max_consecutive_failures = 3
        self._fails = 0

    # ------------------------------------------------------------------ lifecycle
    def start(self) -> "Scheduler":
        if self._thread is None:
            self._thread = threading.Thread(target=self._loop, name="hrm-b200-scheduler", daemon=True)
            self._thread.start()
        return self

    def stop(self, timeout: float = 10.0) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout)
            self._thread = None

    def alive(self) -> bool:
        return self._thread is not None and self._thread.is_alive() and self.fatal is None

    # ------------------------------------------------------------------ API
    def submit(self, prompt_ids: Sequence[int], max_new_tokens: int, stop_on_eos: bool = True,
               on_token: Optional[Callable[[int], None]] = None,
               sampling: Optional[SamplingParams] = None) -> GenRequest:
        if self.fatal is not None:
            raise RuntimeError(f"engine stopped after a fatal error: {self.fatal}")
        if self._stop.is_set():
            raise RuntimeError("scheduler stopped")
        if not prompt_ids:
            raise ValueError("empty prompt")
        if int(max_new_tokens) < 1:
            raise ValueError(f"max_new_tokens must be >= 1, got {max_new_tokens}")
        limit = self.engine.max_blocks * self.engine.block_size
        if len(prompt_ids) + max_new_tokens > limit:
            raise ValueError(f"prompt ({len(prompt_ids)}) + max_new_tokens ({max_new_tokens}) exceeds the "
                             f"engine's max sequence length {limit}")
        need = min(self.engine.max_blocks, self.engine.bm.blocks_needed(-1, len(prompt_ids) + max_new_tokens + 1))
        if need > self.engine.bm.num_blocks:   # could never be admitted: fail now instead of waiting forever
            raise ValueError(f"request needs {need} KV blocks, the pool has {self.engine.bm.num_blocks}")
        with self._lock:
            rid = self._next_rid
            self._next_rid += 1
        r = GenRequest(list(map(int, prompt_ids)), int(max_new_tokens), stop_on_eos, on_token, rid,
                       sampling=sampling if sampling is not None and not sampling.greedy else None)
        self._inbox.put(r)
        if self.fatal is not None:   # the loop stopped between the check above and the put
            self._fail_queued()
        return r

    def generate(self, prompt_ids: Sequence[int], max_new_tokens: int, timeout: Optional[float] = None,
                 stop_on_eos: bool = True, sampling: Optional[SamplingParams] = None) -> List[int]:
        """Submit and wait; a request that outlives ``timeout`` is cancelled (its KV blocks and batch slot are
        given back) before the timeout propagates."""
        r = self.submit(prompt_ids, max_new_tokens, stop_on_eos, sampling=sampling)
        try:
            return r.future.result(timeout)
        except FutureTimeout:
            self.cancel(r)
            raise

    def cancel(self, r: GenRequest) -> None:
        """Stop ``r``: the loop drops it before its next prefill chunk or decode step, releases its KV blocks and
        fails its future with ``CancelledError``.  No effect on a finished request."""
        r.cancelled = True

    def metrics(self) -> Dict:
        el = max(1e-9, time.perf_counter() - self.started_at)
        tt = sorted(self.ttfts)
        it = sorted(self.itls)
        pct = lambda a, q: (a[min(len(a) - 1, int(q * len(a)))] * 1e3) if a else None
        return {"queue_depth": len(self._waiting) + self._inbox.qsize(), "batch_size": len(self._running),
                "prefilling": len(self._prefilling),
                "completed": self.completed, "generated_tokens": self.generated_tokens,
                "tok_per_s": self.generated_tokens / el, "ttft_p50_ms": pct(tt, 0.5), "ttft_p99_ms": pct(tt, 0.99),
                "itl_p50_ms": pct(it, 0.5), "last_error": self.last_error, "fatal": self.fatal,
                "prefix_cache_hit_blocks": getattr(getattr(self.engine, "bm", None), "prefix_hits", 0),
                "cancelled": self.cancelled_total}

    # ------------------------------------------------------------------ loop
    def _finish(self, r: GenRequest) -> None:
        r.finished_at = time.perf_counter()
        self.engine.release(r.seq_id)
        self.completed += 1
        if not r.future.done():
            r.future.set_result(list(r.tokens))

    def _emit(self, r: GenRequest, tok: int) -> bool:
        """Append a token; returns True when the request is finished."""
        r.tokens.append(tok)
        self.generated_tokens += 1
        if r.on_token is not None:
            try:
                r.on_token(tok)
            except Exception as e:   # a broken stream consumer must not stop generation for the batch
                self.last_error = f"on_token callback of request {r.rid}: {e!r}"
        return len(r.tokens) >= r.max_new_tokens or (r.stop_on_eos and tok in self.eos)

    def _full_need(self, r: GenRequest) -> int:
        """Blocks ``r`` still has to take to hold prompt + max_new_tokens + 1 positions (see _decode's staging)."""
        eng = self.engine
        total = min(eng.max_blocks * eng.block_size, len(r.prompt_ids) + r.max_new_tokens + 1)
        return eng.bm.blocks_needed(r.seq_id, total)

    def _admit(self) -> bool:
        """Admission plus one prefill forward; True when a prefill ran."""
        while True:
            try:
                self._waiting.append(self._inbox.get_nowait())
            except queue.Empty:
                break
        eng = self.engine
        # every admitted request's whole reservation is counted, so staging never runs out of blocks
        committed = self._pending_growth() + sum(self._full_need(r) for r in self._prefilling)
        while self._waiting and len(self._running) + len(self._prefilling) < self.max_batch:
            r = self._waiting[0]
            if r.cancelled:   # cancelled while it arrived: never touches the engine
                self._waiting.popleft()
                self._cancel_future(r)
                continue
            if self._full_need(r) > eng.bm.free_blocks - committed:
                break
            self._waiting.popleft()
            r.seq_id = eng.new_seq()
            # prefix cache: the prompt's leading blocks may already be in the KV cache (a shared system prompt)
            r._done = eng.match_prefix(r.seq_id, r.prompt_ids) if self.prefix_cache else 0
            committed += self._full_need(r)
            self._prefilling.append(r)
        if not self._prefilling:
            return False
        budget = self.prefill_chunk
        if self._running and self.interleave_chunk > 0:
            budget = min(budget, self.interleave_chunk)
        chunks, used = [], 0
        for r in self._prefilling:
            if used >= budget:
                break
            take = min(len(r.prompt_ids) - r._done, budget - used)
            chunks.append((r, take))
            used += take
        # a failure here propagates to the loop, which fails every request that holds engine state
        seqs = [(r.seq_id, r.prompt_ids[r._done:r._done + n]) for r, n in chunks]
        if any(r.sampling is not None for r, _ in chunks):
            firsts = eng.prefill(seqs, [r.sampling for r, _ in chunks])
        else:
            firsts = eng.prefill(seqs)
        if len(self.prefill_calls) < 4096:
            self.prefill_calls.append(used)
        now = time.perf_counter()
        done = []
        for (r, n), t in zip(chunks, firsts):
            r._done += n
            if r._done < len(r.prompt_ids):
                continue   # the token after a partial prompt is not a generated token
            done.append(r)
            if self.prefix_cache:
                eng.publish_prefix(r.seq_id, r.prompt_ids)
            r.first_token_at = now
            self.ttfts.append(now - r.arrival)
            r._last_tok_at = now
            r._pos = len(r.prompt_ids)
            if self._emit(r, int(t)):
                self._finish(r)
            else:
                self._running.append(r)
        if done:
            gone = {id(r) for r in done}
            self._prefilling = [r for r in self._prefilling if id(r) not in gone]
        return True

    def _pending_growth(self) -> int:
        """Blocks the running sequences will still take when the batch is next staged (admitted but not yet grown
        to their full reservation)."""
        bm = self.engine.bm
        return sum(bm.blocks_needed(r.seq_id, r._pos + r.max_new_tokens - len(r.tokens) + 1) for r in self._running)

    def _decode(self, staged: bool, g) -> tuple:
        eng = self.engine
        if not staged:
            # each sequence reserves only what it can still generate (admission counted exactly that)
            extra = {}
            if any(r.sampling is not None for r in self._running):
                extra["sampling"] = [r.sampling for r in self._running]
            g = eng.load_decode_batch([r.seq_id for r in self._running], [r.tokens[-1] for r in self._running],
                                      reserve=[r.max_new_tokens - len(r.tokens) + 1 for r in self._running],
                                      positions=[r._pos for r in self._running], **extra)
        tok = eng.decode_step(g)
        host = tok[:len(self._running)].tolist()
        now = time.perf_counter()
        still, changed = [], False
        for r, t in zip(self._running, host):
            r._pos += 1
            self.itls.append(now - r._last_tok_at)
            r._last_tok_at = now
            if self._emit(r, int(t)):
                self._finish(r)
                changed = True
            else:
                still.append(r)
        self._running = still
        return (not changed), g

    def _drop_cancelled(self) -> bool:
        """Remove cancelled requests from every stage; True when the decode batch changed."""
        changed = False
        for name in ("_prefilling", "_running"):
            keep = []
            for r in getattr(self, name):
                if r.cancelled:
                    self.engine.release(r.seq_id)
                    self._cancel_future(r)
                    changed |= name == "_running"
                else:
                    keep.append(r)
            setattr(self, name, keep)
        if any(r.cancelled for r in self._waiting):
            for r in [r for r in self._waiting if r.cancelled]:
                self._cancel_future(r)
            self._waiting = collections.deque(r for r in self._waiting if not r.cancelled)
        return changed

    def _cancel_future(self, r: GenRequest) -> None:
        self.cancelled_total += 1
        if not r.future.done():
            r.future.set_exception(CancelledError(f"request {r.rid} cancelled"))

    def _loop(self) -> None:
        staged, g = False, None
        dev = self.engine.device
        if dev.type == "cuda":
            torch.cuda.set_device(dev)
        while not self._stop.is_set():
            try:
                if self._drop_cancelled():
                    staged = False
                admitted = self._admit()
                if admitted:
                    staged = False
                if self._running:
                    staged, g = self._decode(staged, g)
                elif not admitted:
                    time.sleep(self.idle_sleep_s)
                if admitted or self._running:
                    self._fails = 0
            except BaseException as e:
                # fail the requests that hold engine state (decoding or partly prefilled); queued requests never
                # reached the engine and stay queued, unless the engine cannot serve any more
                self.last_error = repr(e)
                self._fails += 1
                fatal = is_context_fatal(e) or self._fails >= self.max_consecutive_failures
                victims = self._running + self._prefilling + (list(self._waiting) if fatal else [])
                for r in victims:
                    if not r.future.done():
                        r.future.set_exception(e)
                    if r.seq_id >= 0:
                        try:
                            self.engine.release(r.seq_id)
                        except Exception:
                            pass
                self._running, self._prefilling, staged = [], [], False
                if fatal:
                    self._waiting.clear()
                    self.fatal = repr(e)
                    break
        if self.fatal is not None:   # nothing queued waits for a loop that is gone
            self._fail_queued()
        else:                        # stopped: every request still in flight ends with an error
            self._fail_outstanding(RuntimeError("scheduler stopped"))

    def _fail_outstanding(self, err: BaseException) -> None:
        for r in self._running + self._prefilling + list(self._waiting):
            if r.seq_id >= 0 and r in self._running + self._prefilling:
                try:
                    self.engine.release(r.seq_id)
                except Exception:
                    pass
            if not r.future.done():
                r.future.set_exception(err)
        self._running, self._prefilling = [], []
        self._waiting.clear()
        while True:
            try:
                r = self._inbox.get_nowait()
            except queue.Empty:
                return
            if not r.future.done():
                r.future.set_exception(err)

    def _fail_queued(self) -> None:
        err = RuntimeError(f"engine stopped after a fatal error: {self.fatal}")
        while True:
            try:
                r = self._inbox.get_nowait()
            except queue.Empty:
                return
            try:
                r.future.set_exception(err)
            except Exception:   # already resolved
                pass
