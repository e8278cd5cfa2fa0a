"""Generation backends behind the HTTP service.

* :class:`EngineBackend` -- the in-process B200 engine + continuous-batching scheduler (replaces the reference's
  ``DeepSeekNativeEngine``: a child process driven through prompt/tokens/done files polled every 50-200 ms,
  ``hrm_flash/deepseek_native.py:182-369``).  Weights come from a DSI8 file or from random-init synthesis of a preset
  architecture; the tokenizer is a local HF tokenizer or the byte tokenizer.
* :class:`EchoBackend` -- deterministic stand-in used by tests and the mock lanes.

All backends expose ``tokenizer``, ``generate(prompt_text, max_new_tokens, timeout_s, sampling=None) -> str``,
``generate_stream(...)`` (an iterator of text deltas), ``is_running()``, ``stop()`` and ``metrics()``.
"""
from __future__ import annotations

import hashlib
import queue
import time
from typing import Dict, Iterator, List, Optional, Sequence


def cut_at_stop(pieces: Iterator[str], stops: Sequence[str]) -> Iterator[str]:
    """Pass text pieces through until the text contains one of ``stops``; the output ends just before the earliest
    stop string (which is not emitted) and the piece source is closed (for a backend stream that cancels the
    request).  Text that could still turn into a stop string is held back until it cannot."""
    stops = [s for s in stops if s]
    hold = max((len(s) for s in stops), default=1) - 1
    text, sent = "", 0
    try:
        for piece in pieces:
            text += piece
            hits = [i for i in (text.find(s, max(0, sent - len(s) + 1)) for s in stops) if i >= 0]
            if hits:
                cut = min(hits)
                if cut > sent:
                    yield text[sent:cut]
                return
            safe = len(text) - hold
            if safe > sent:
                yield text[sent:safe]
                sent = safe
        if len(text) > sent:
            yield text[sent:]
    finally:
        close = getattr(pieces, "close", None)
        if close is not None:
            close()


class ByteTokenizer:
    """UTF-8 byte tokenizer (ids 3..258 = bytes; 0 pad, 1 bos, 2 eos).  Used when no HF tokenizer is configured
    (synthetic random-init models); HF-compatible call signature for the prompt budget fitter."""

    pad_id, bos_id, eos_id, offset = 0, 1, 2, 3

    def __call__(self, text: str, add_special_tokens: bool = True, **_):
        ids = [b + self.offset for b in text.encode("utf-8")]
        if add_special_tokens:
            ids = [self.bos_id] + ids
        return {"input_ids": ids}

    def encode(self, text: str, add_special_tokens: bool = True) -> List[int]:
        return self(text, add_special_tokens)["input_ids"]

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        bs = bytes((int(i) - self.offset) % 256 for i in ids
                   if not (skip_special_tokens and int(i) < self.offset))
        return bs.decode("utf-8", errors="replace")


def load_tokenizer(source: Optional[str], local_files_only: bool = True):
    if not source or source == "bytes":
        return ByteTokenizer()
    from transformers import AutoTokenizer
    return AutoTokenizer.from_pretrained(str(source), local_files_only=bool(local_files_only))


class EchoBackend:
    """Deterministic fake LLM: a short text derived from a hash of the prompt (tests, mock lanes)."""

    def __init__(self, tokenizer=None, fail: bool = False):
        self.tokenizer = tokenizer or ByteTokenizer()
        self.fail = fail
        self.calls: List[Dict] = []

    def generate(self, prompt_text: str, max_new_tokens: int = 64, timeout_s: float = 180.0, sampling=None,
                 stop: Optional[Sequence[str]] = None) -> str:
        self.calls.append({"prompt": prompt_text, "max_new_tokens": max_new_tokens, "sampling": sampling,
                           "stop": stop})
        if self.fail:
            raise RuntimeError("echo backend configured to fail")
        h = hashlib.sha256(prompt_text.encode()).hexdigest()[:16]
        text = f"answer-{h}"[: max(1, max_new_tokens * 4)]
        return "".join(cut_at_stop(iter([text]), stop)) if stop else text

    def generate_stream(self, prompt_text: str, max_new_tokens: int = 64, timeout_s: float = 180.0,
                        sampling=None, cancel=None, stop: Optional[Sequence[str]] = None) -> Iterator[str]:
        """The same answer in 4-character pieces (stops early once ``cancel`` is set)."""
        text = self.generate(prompt_text, max_new_tokens, timeout_s, sampling)

        def pieces():
            for i in range(0, len(text), 4):
                if cancel is not None and cancel.is_set():
                    return
                yield text[i:i + 4]
        return cut_at_stop(pieces(), stop) if stop else pieces()

    def is_running(self) -> bool:
        return True

    def stop(self) -> None:
        pass

    def metrics(self) -> Dict:
        return {"calls": len(self.calls)}


class EngineBackend:
    """The B200 engine with a continuous-batching scheduler, on one GPU (TP=1) or as rank 0 of a TP group."""

    def __init__(self, model_source: str, tokenizer_source: Optional[str] = None, device: str = "cuda:0",
                 max_seq_len: int = 8192, max_batch: int = 64, prefill_chunk: int = 4096,
                 kv_fraction: float = 0.85, max_prompt_tokens: int = 2048, local_files_only: bool = True,
                 seed: int = 0, comm=None, rank: int = 0, world: int = 1, engine=None, prefix_cache: bool = False):
        import torch
        from ..config import EngineConfig, get_preset
        from ..models.llama import LlamaW8
        from ..runtime.engine import InferenceEngine
        from ..runtime.kv_cache import PagedKVPool
        from ..runtime.scheduler import Scheduler
        self.tokenizer = load_tokenizer(tokenizer_source, local_files_only)
        self.max_prompt_tokens = int(max_prompt_tokens)
        if engine is None:
            dev = torch.device(device)
            if str(model_source).startswith("synthetic:"):
                cfg = get_preset(model_source.split(":", 1)[1])
                model = LlamaW8.synthesize(cfg, rank=rank, world=world, device=dev, seed=seed, comm=comm,
                                           max_pos=max_seq_len + 16)
            else:
                import os
                model = LlamaW8.from_dsi8(model_source, rank=rank, world=world, device=dev, comm=comm,
                                          max_pos=max_seq_len + 16,
                                          cache_dir=os.environ.get("HRM_PACKED_CACHE") or None)
                cfg = model.cfg
            if dev.type == "cuda":
                free, _ = torch.cuda.mem_get_info(dev)
                nb = PagedKVPool.blocks_for_budget(int(free * kv_fraction), cfg.layers, model.plan.local_kv_heads,
                                                   cfg.head_dim)
            else:   # CPU (tests, oracle runs): room for max_batch full-length sequences
                nb = max_batch * ((max_seq_len + 15) // 16 + 1)
            ecfg = EngineConfig(tp=world, max_seq_len=max_seq_len, max_batch=max_batch, prefill_chunk=prefill_chunk,
                                prefix_cache=prefix_cache)
            engine = InferenceEngine(model, ecfg, num_blocks=nb)
        self.engine = engine
        self.scheduler = Scheduler(engine).start()

    def encode_prompt(self, text: str) -> List[int]:
        ids = self.tokenizer(text, add_special_tokens=True)["input_ids"]
        if len(ids) > self.max_prompt_tokens:          # left-truncate (reference: deepseek_native.py:345-346)
            ids = ids[-self.max_prompt_tokens:]
        return ids

    def generate_ids(self, ids: List[int], max_new_tokens: int, timeout_s: float = 180.0,
                     sampling=None) -> List[int]:
        """Token ids of the completion; ``sampling`` (a ``runtime.sampling.SamplingParams``) draws instead of the
        greedy pick."""
        # fit the context like the reference engine (prompt + output capped at its Tmax): keep the prompt's tail
        # and at least one new token, then cap the output
        limit = self.engine.max_blocks * self.engine.block_size
        ids = list(ids)[-max(1, limit - 1):]
        max_new_tokens = max(1, min(int(max_new_tokens), limit - len(ids)))
        return self.scheduler.generate(ids, max_new_tokens, timeout=timeout_s, sampling=sampling)

    def generate(self, prompt_text: str, max_new_tokens: int = 256, timeout_s: float = 180.0,
                 sampling=None, stop: Optional[Sequence[str]] = None) -> str:
        """The completion text; with ``stop`` strings it ends before the first one and generation stops there."""
        if stop:
            return "".join(self.generate_stream(prompt_text, max_new_tokens, timeout_s, sampling, stop=stop))
        out = self.generate_ids(self.encode_prompt(prompt_text), max_new_tokens, timeout_s, sampling)
        return self.tokenizer.decode(out, skip_special_tokens=True)

    def generate_stream(self, prompt_text: str, max_new_tokens: int = 256, timeout_s: float = 180.0,
                        sampling=None, cancel=None, stop: Optional[Sequence[str]] = None) -> Iterator[str]:
        """Text deltas of the completion as it is generated; with ``stop`` strings the stream ends before the first
        one and the request is cancelled there (see :meth:`_stream` for the rest)."""
        pieces = self._stream(prompt_text, max_new_tokens, timeout_s, sampling, cancel)
        return cut_at_stop(pieces, stop) if stop else pieces

    def _stream(self, prompt_text: str, max_new_tokens: int, timeout_s: float, sampling, cancel) -> Iterator[str]:
        """Text deltas as tokens are generated (the scheduler's per-token callback feeds a queue).  The deltas
        concatenate to :meth:`generate`'s text: each one is the growth of the decoded text, held back while it ends
        in an incomplete UTF-8 sequence.  A caller that stops early (closes the iterator, or sets the
        ``threading.Event`` ``cancel``, which is checked between tokens), or a wait longer than ``timeout_s``,
        cancels the request."""
        ids = self.encode_prompt(prompt_text)
        limit = self.engine.max_blocks * self.engine.block_size
        ids = list(ids)[-max(1, limit - 1):]
        n = max(1, min(int(max_new_tokens), limit - len(ids)))
        q: "queue.Queue" = queue.Queue()
        r = self.scheduler.submit(ids, n, on_token=q.put, sampling=sampling)
        r.future.add_done_callback(lambda f: q.put(None))
        toks: List[int] = []
        sent = ""
        deadline = time.monotonic() + float(timeout_s)
        try:
            while True:
                if cancel is not None and cancel.is_set():
                    return
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TimeoutError(f"generation exceeded {timeout_s} s")
                try:
                    t = q.get(timeout=min(left, 0.05))
                except queue.Empty:
                    continue                      # re-check the cancel flag and the deadline
                if t is None:
                    break
                toks.append(int(t))
                text = self.tokenizer.decode(toks, skip_special_tokens=True)
                if text.endswith("\ufffd"):
                    continue                      # an incomplete multi-byte character: wait for the rest
                if len(text) > len(sent) and text.startswith(sent):
                    yield text[len(sent):]
                    sent = text
            r.future.result()                     # raises the request's error, if any
            text = self.tokenizer.decode(r.future.result(), skip_special_tokens=True)
            if text != sent and text.startswith(sent):
                yield text[len(sent):]
        finally:
            if not r.future.done():
                self.scheduler.cancel(r)

    def is_running(self) -> bool:
        return self.scheduler.alive()

    def stop(self) -> None:
        self.scheduler.stop()

    def metrics(self) -> Dict:
        return self.scheduler.metrics()
