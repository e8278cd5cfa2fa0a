"""Inference engine: paged KV, chunked prefill, CUDA-graph decode steps with device-side bookkeeping.

Reference counterpart: ``generate_tp`` (``engine/llama_tp.py:338-382``: chunked prefill, then a decode loop that
syncs the host several times per token) and the native engine's token loop
(``scripts/deepseek_native_engine.sh:1012-1130``: prompt tokens one at a time through the decode path, ~6 device
syncs + 2 scale read-backs per layer, no EOS stop).  Here:

* prefill is batched GEMM work over chunks of up to ``prefill_chunk`` tokens (several sequences per chunk);
* a decode step is ONE CUDA-graph replay per batch bucket: slots / context lengths are derived on the device from
  the block tables, the sampled token is fed back on the device, so consecutive steps need no host input;
* generation stops per sequence on any EOS id of the config (reference quirk Q6 fixed).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

from .. import ops
from ..utils.nvtx import nvtx_range
from ..config import EngineConfig
from ..models.llama import BatchMeta, LlamaW8
from .kv_cache import BlockManager
from .sampling import SampleMeta, SamplingParams, any_sampled


@dataclass
class _DecodeGraph:
    bucket: int
    ids: torch.Tensor
    positions: torch.Tensor
    slots: torch.Tensor
    context_lens: torch.Tensor
    tables: torch.Tensor
    active: torch.Tensor
    last_rows: torch.Tensor
    tokens: torch.Tensor
    graph: Optional[torch.cuda.CUDAGraph] = None
    meta: Optional[BatchMeta] = None
    # sampled variant of the step (same buffers plus per-row sampling arrays); ``sampled`` selects it
    sample: Optional[SampleMeta] = None
    meta_sample: Optional[BatchMeta] = None
    graph_sample: Optional[torch.cuda.CUDAGraph] = None
    sampled: bool = False


class InferenceEngine:
    def __init__(self, model: LlamaW8, ecfg: Optional[EngineConfig] = None, num_blocks: Optional[int] = None):
        self.model = model
        self.cfg = model.cfg
        self.ecfg = ecfg or EngineConfig()
        self.device = model.device
        bs = self.ecfg.block_size
        self.block_size = bs
        self.max_blocks = (self.ecfg.max_seq_len + bs - 1) // bs
        nb = num_blocks or self.ecfg.num_kv_blocks or self.ecfg.max_batch * self.max_blocks
        model.alloc_kv(int(nb), bs)
        model.sequence_parallel = bool(self.ecfg.sequence_parallel)
        model.chain_layers = bool(self.ecfg.chain_layers)
        model.prefill_overlap_chunks = int(self.ecfg.prefill_overlap_chunks)
        self.bm = BlockManager(int(nb), bs, prefix_cache=bool(self.ecfg.prefix_cache))
        self._graphs: Dict[int, _DecodeGraph] = {}
        self._next_seq = 0
        self._pinned_tokens: Dict[int, torch.Tensor] = {}

    # ------------------------------------------------------------------ sequence bookkeeping
    def new_seq(self) -> int:
        s = self._next_seq
        self._next_seq += 1
        return s

    def release(self, seq_id: int) -> None:
        self.bm.free(seq_id)

    def match_prefix(self, seq_id: int, tokens: Sequence[int]) -> int:
        """Prefix cache: give the new sequence the published KV blocks its prompt starts with; returns the number of
        prompt tokens already in the cache (prefill continues from there).  0 when the cache is off."""
        return self.bm.match_prefix(seq_id, tokens)

    def publish_prefix(self, seq_id: int, tokens: Sequence[int]) -> int:
        """Prefix cache: publish the full blocks holding the (already prefilled) prompt ``tokens`` of ``seq_id``."""
        return self.bm.publish(seq_id, tokens)

    def reset(self) -> None:
        self.bm.reset()

    # ------------------------------------------------------------------ prefill
    def _prefill_meta(self, chunks: List[Tuple[int, List[int], int]],
                      sampling: Optional[Sequence[Optional[SamplingParams]]] = None) -> BatchMeta:
        """chunks: (seq_id, token ids of this chunk, absolute start position)."""
        dev = self.device
        bs = self.block_size
        ids, pos, slots, cu, qst, ctx = [], [], [], [0], [], []
        tabs = []
        for sid, toks, start in chunks:
            tab = self.bm.grow(sid, start + len(toks))
            for i, t in enumerate(toks):
                p = start + i
                ids.append(int(t))
                pos.append(p)
                slots.append(tab[p // bs] * bs + p % bs)
            cu.append(cu[-1] + len(toks))
            qst.append(start)
            ctx.append(start + len(toks))
            tabs.append(tab)
        width = max(len(t) for t in tabs)
        table = torch.zeros(len(tabs), width, dtype=torch.int32)
        for i, t in enumerate(tabs):
            table[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        last = [c - 1 for c in cu[1:]]
        host = dict(
            ids=torch.tensor(ids, dtype=torch.int64), positions=torch.tensor(pos, dtype=torch.int32),
            slots=torch.tensor(slots, dtype=torch.int32), block_tables=table,
            context_lens=torch.tensor(ctx, dtype=torch.int32), last_rows=torch.tensor(last, dtype=torch.int64),
            cu_q=torch.tensor(cu, dtype=torch.int32), q_start=torch.tensor(qst, dtype=torch.int32))
        dv = {k: v.pin_memory().to(dev, non_blocking=True) if dev.type == "cuda" else v for k, v in host.items()}
        meta = BatchMeta(is_decode=False, max_q=max(len(c[1]) for c in chunks), **dv)
        if any_sampled(sampling):
            # one row per chunk (its last token); the noise counter is that token's absolute position
            meta.sample = SampleMeta.alloc(len(chunks), dev)
            meta.sample.fill(sampling, positions=[start + len(toks) - 1 for _, toks, start in chunks])
        return meta

    @torch.no_grad()
    def prefill(self, seqs: Sequence[Tuple[int, Sequence[int]]],
                sampling: Optional[Sequence[Optional[SamplingParams]]] = None) -> List[int]:
        """Chunked prefill of whole prompts; returns the first generated token of each sequence (greedy, or drawn
        with ``sampling[i]`` for sequence ``i``)."""
        budget = int(self.ecfg.prefill_chunk)
        by_sid = {sid: (sampling[i] if sampling is not None else None) for i, (sid, _) in enumerate(seqs)}
        pending = [(sid, list(toks), self.bm.lengths.get(sid, 0)) for sid, toks in seqs]
        first: Dict[int, int] = {}
        while pending:
            chunks, used, nxt = [], 0, []
            for sid, toks, start in pending:
                if used >= budget:
                    nxt.append((sid, toks, start))
                    continue
                take = min(len(toks), budget - used)
                chunks.append((sid, toks[:take], start))
                used += take
                if take < len(toks):
                    nxt.append((sid, toks[take:], start + take))
            meta = self._prefill_meta(chunks, [by_sid[c[0]] for c in chunks] if sampling is not None else None)
            with nvtx_range(f"prefill chunk {used} tokens"):
                out = self.model.forward(meta).tolist()
            done_ids = {s for s, _, _ in nxt}
            for (sid, _, _), t in zip(chunks, out):
                if sid not in done_ids:
                    first[sid] = int(t)
            pending = nxt
        return [first[sid] for sid, _ in seqs]

    # ------------------------------------------------------------------ decode (graph per bucket)
    def _bucket(self, n: int) -> int:
        for b in sorted(self.ecfg.graph_batch_buckets):
            if n <= b:
                return b
        raise ValueError(f"decode batch {n} exceeds the largest graph bucket")

    def _decode_state(self, bucket: int) -> _DecodeGraph:
        g = self._graphs.get(bucket)
        if g is not None:
            return g
        dev = self.device
        z = lambda *s, dt=torch.int32: torch.zeros(*s, dtype=dt, device=dev)
        g = _DecodeGraph(bucket=bucket, ids=z(bucket, dt=torch.int64), positions=z(bucket), slots=z(bucket),
                         context_lens=z(bucket), tables=z(bucket, self.max_blocks), active=z(bucket),
                         last_rows=torch.arange(bucket, dtype=torch.int64, device=dev),
                         tokens=z(bucket, dt=torch.int64))
        splits, kps = ops.decode_splits(self.max_blocks * self.block_size, bucket * self.model.plan.local_kv_heads,
                                        self.block_size, ops.ext().sm_count() if ops.has_ext() else 148)
        g.meta = BatchMeta(ids=g.ids, positions=g.positions, slots=g.slots, block_tables=g.tables,
                           context_lens=g.context_lens, last_rows=g.last_rows, is_decode=True,
                           attn_splits=splits, attn_keys_per_split=kps)
        self._graphs[bucket] = g
        return g

    def _sample_state(self, g: _DecodeGraph) -> None:
        """The sampled variant's arrays; its noise counter is the step's device-side positions."""
        if g.sample is None:
            g.sample = SampleMeta.alloc(g.bucket, self.device)
            g.sample.pos = g.positions
            m = g.meta
            g.meta_sample = BatchMeta(ids=m.ids, positions=m.positions, slots=m.slots, block_tables=m.block_tables,
                                      context_lens=m.context_lens, last_rows=m.last_rows, is_decode=True,
                                      attn_splits=m.attn_splits, attn_keys_per_split=m.attn_keys_per_split,
                                      sample=g.sample)

    def _decode_body(self, g: _DecodeGraph, sampled: bool = False) -> None:
        ops.decode_prepare(g.positions, g.tables, self.block_size, g.active, g.slots, g.context_lens)
        tok = self.model.forward(g.meta_sample if sampled else g.meta)
        g.tokens.copy_(tok)
        ops.decode_advance(g.tokens, g.ids, g.positions, g.active)

    def release_graphs(self) -> None:
        """Drop every captured decode graph.  Graphs that captured NCCL calls must be released before the process
        group is destroyed, or the communicator teardown waits on them forever."""
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        for g in self._graphs.values():
            g.graph = None
            g.graph_sample = None
        self._graphs.clear()

    def capture(self, bucket: int, sampled: bool = False) -> None:
        """Warm up (sizes the workspace) and capture the decode step of ``bucket`` sequences (greedy, or the
        sampled variant)."""
        g = self._decode_state(bucket)
        if sampled:
            self._sample_state(g)
        if (g.graph_sample if sampled else g.graph) is not None or not self.ecfg.use_cuda_graphs:
            return
        saved = (g.ids.clone(), g.positions.clone(), g.active.clone())
        g.active.zero_()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self._decode_body(g, sampled)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        ws = ops.Workspace.get(self.device)
        ws.frozen = True
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._decode_body(g, sampled)
            if sampled:
                g.graph_sample = graph
            else:
                g.graph = graph
        finally:
            ws.frozen = False
        g.ids.copy_(saved[0]); g.positions.copy_(saved[1]); g.active.copy_(saved[2])

    def load_decode_batch(self, seq_ids: Sequence[int], last_tokens: Sequence[int], reserve,
                          positions: Optional[Sequence[int]] = None,
                          sampling: Optional[Sequence[Optional[SamplingParams]]] = None) -> _DecodeGraph:
        """Stage a decode batch: block tables grown for ``reserve`` more tokens (one count for every sequence, or a
        per-sequence list), current tokens and positions.

        ``positions[i]`` is the absolute position of ``last_tokens[i]`` (default: the prefilled length);
        ``sampling[i]`` the sampling parameters of sequence ``i`` (None or absent: greedy)."""
        n = len(seq_ids)
        bucket = self._bucket(n)
        g = self._decode_state(bucket)
        tabs = torch.zeros(bucket, self.max_blocks, dtype=torch.int32)
        pos = torch.zeros(bucket, dtype=torch.int32)
        ids = torch.zeros(bucket, dtype=torch.int64)
        act = torch.zeros(bucket, dtype=torch.int32)
        res = [int(reserve)] * n if isinstance(reserve, int) else [int(x) for x in reserve]
        for i, (sid, t) in enumerate(zip(seq_ids, last_tokens)):
            L = int(positions[i]) if positions is not None else self.bm.lengths.get(sid, 0)
            tab = self.bm.grow(sid, min(L + res[i], self.max_blocks * self.block_size))
            tabs[i, :len(tab)] = torch.tensor(tab, dtype=torch.int32)
            pos[i] = L
            ids[i] = int(t)
            act[i] = 1
        g.tables.copy_(tabs, non_blocking=False)
        g.positions.copy_(pos)
        g.ids.copy_(ids)
        g.active.copy_(act)
        g.sampled = any_sampled(sampling)
        if g.sampled:
            self._sample_state(g)
            g.sample.fill(sampling)
        return g

    def decode_step(self, g: _DecodeGraph) -> torch.Tensor:
        """One decode step for the staged batch; returns the device tensor of sampled tokens (bucket-sized)."""
        if self.ecfg.use_cuda_graphs and self.device.type == "cuda":
            graph = g.graph_sample if g.sampled else g.graph
            if graph is None:
                with nvtx_range(f"capture decode b{g.bucket}"):
                    self.capture(g.bucket, g.sampled)
                graph = g.graph_sample if g.sampled else g.graph
            with nvtx_range("decode step (graph)"):
                graph.replay()
        else:
            with nvtx_range("decode step"):
                self._decode_body(g, g.sampled)
        return g.tokens

    def step_host(self, g: _DecodeGraph, host_ids: torch.Tensor, host_out: torch.Tensor) -> torch.Tensor:
        """Serving step: H2D this step's input ids from pinned ``host_ids``, one decode step, D2H the sampled
        tokens into pinned ``host_out`` and wait for them."""
        cuda = self.device.type == "cuda"
        g.ids.copy_(host_ids, non_blocking=cuda)
        self.decode_step(g)
        host_out.copy_(g.tokens, non_blocking=cuda)
        if cuda:
            torch.cuda.current_stream(self.device).synchronize()
        return host_out

    # ------------------------------------------------------------------ public API
    @torch.no_grad()
    def generate(self, prompts: Sequence[Sequence[int]], max_new_tokens: int, stop_on_eos: bool = True,
                 eos_ids: Optional[Sequence[int]] = None,
                 on_token: Optional[Callable[[int, int], None]] = None,
                 sampling=None) -> List[List[int]]:
        """Generation for a batch of token-id prompts (prompt ids H2D, tokens D2H every step): greedy, or drawn with
        ``sampling`` (one :class:`SamplingParams` for every prompt, or one per prompt).  ``on_token(i, token)`` is
        called for every token kept for prompt ``i``, as soon as it is known."""
        if isinstance(sampling, SamplingParams):
            sampling = [sampling] * len(prompts)
        eos = set(self.cfg.eos_token_ids if eos_ids is None else eos_ids)
        sids = [self.new_seq() for _ in prompts]
        try:
            cached = [self.match_prefix(s, p) for s, p in zip(sids, prompts)]
            first = self.prefill([(s, list(p)[c:]) for s, p, c in zip(sids, prompts, cached)], sampling)
            for s, p in zip(sids, prompts):
                self.publish_prefix(s, p)
            outs = [[t] for t in first]
            if on_token is not None and max_new_tokens >= 1:
                for i, t in enumerate(first):
                    on_token(i, t)
            alive = [not (stop_on_eos and t in eos) for t in first]
            if max_new_tokens <= 1 or not any(alive):
                return [o[:max_new_tokens] for o in outs]
            g = self.load_decode_batch(sids, first, reserve=max_new_tokens, sampling=sampling)
            act_host = torch.zeros(g.bucket, dtype=torch.int32)
            act_host[:len(sids)] = torch.tensor([1 if a else 0 for a in alive], dtype=torch.int32)
            g.active.copy_(act_host)
            cuda = self.device.type == "cuda"
            pinned = torch.empty(g.bucket, dtype=torch.int64, pin_memory=cuda)
            for step in range(1, max_new_tokens):
                tok = self.decode_step(g)
                pinned.copy_(tok, non_blocking=cuda)
                if cuda:
                    torch.cuda.current_stream(self.device).synchronize()
                changed = False
                for i in range(len(sids)):
                    if not alive[i]:
                        continue
                    t = int(pinned[i])
                    outs[i].append(t)
                    if on_token is not None:
                        on_token(i, t)
                    if stop_on_eos and t in eos:
                        alive[i] = False
                        changed = True
                if not any(alive):
                    break
                if changed:
                    act_host[:len(sids)] = torch.tensor([1 if a else 0 for a in alive], dtype=torch.int32)
                    g.active.copy_(act_host)
            return outs
        finally:
            for sid in sids:
                self.release(sid)
