"""Per-request sampling parameters and their device-side batch form.

The reference engine decodes greedily only (``engine/llama_tp.py:317-335``; the renderer asks llama.cpp for
temperature 0 / top_k 1, ``renderer/hrm_render.py:162-164``), and greedy stays the default here.  A request may ask
for temperature / top-k sampling instead: the token is drawn on the device inside the argmax kernel (Gumbel-max over
the logits at or above the row's global k-th largest), from noise keyed by (seed, position, token id), so a draw is
reproducible from the request's seed and independent of batching and of the tensor-parallel layout.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from ..ops import SAMPLE_MAX_TOP_K


@dataclass(frozen=True)
class SamplingParams:
    temperature: float = 0.0      # 0: greedy (the reference's behaviour)
    top_k: int = 0                # 0: every token; else the top_k largest logits (ties at the cut are kept)
    seed: int = 0

    def __post_init__(self):
        if not (self.temperature >= 0.0) or self.temperature != self.temperature:
            raise ValueError(f"temperature must be >= 0, got {self.temperature!r}")
        if not 0 <= int(self.top_k) <= SAMPLE_MAX_TOP_K:
            raise ValueError(f"top_k must be in [0, {SAMPLE_MAX_TOP_K}], got {self.top_k!r}")

    @property
    def greedy(self) -> bool:
        return self.temperature == 0.0

    @property
    def inv_temp(self) -> float:
        return 0.0 if self.greedy else 1.0 / float(self.temperature)


GREEDY = SamplingParams()


def any_sampled(params: Optional[Sequence[Optional[SamplingParams]]]) -> bool:
    return params is not None and any(p is not None and not p.greedy for p in params)


@dataclass
class SampleMeta:
    """Device arrays of one batch's rows (``R`` rows feed the lm_head; arrays may be longer, e.g. a graph bucket)."""
    inv_temp: torch.Tensor        # f32 [R]
    top_k: torch.Tensor           # int32 [R]
    seed: torch.Tensor            # int64 [R]
    pos: torch.Tensor             # int32 [R]: position of the row's input token (noise counter)
    kmax: int = SAMPLE_MAX_TOP_K  # width of the per-rank candidate rows exchanged under tensor parallelism

    @staticmethod
    def alloc(rows: int, device) -> "SampleMeta":
        z = lambda dt: torch.zeros(rows, dtype=dt, device=device)
        return SampleMeta(z(torch.float32), z(torch.int32), z(torch.int64), z(torch.int32))

    def fill(self, params: Sequence[Optional[SamplingParams]], positions: Optional[Sequence[int]] = None) -> None:
        """Host values for the first ``len(params)`` rows (None = greedy); the remaining rows become greedy.
        ``positions`` sets ``pos`` (decode graphs instead share the step's device positions)."""
        n = self.inv_temp.numel()
        ps: List[SamplingParams] = [p if p is not None else GREEDY for p in params] + [GREEDY] * (n - len(params))
        cuda = self.inv_temp.is_cuda
        host = lambda vals, dt: torch.tensor(vals, dtype=dt).pin_memory() if cuda else torch.tensor(vals, dtype=dt)
        self.inv_temp.copy_(host([p.inv_temp for p in ps], torch.float32), non_blocking=cuda)
        self.top_k.copy_(host([int(p.top_k) for p in ps], torch.int32), non_blocking=cuda)
        self.seed.copy_(host([int(p.seed) for p in ps], torch.int64), non_blocking=cuda)
        if positions is not None:
            pos = [int(x) for x in positions] + [0] * (n - len(positions))
            self.pos.copy_(host(pos, torch.int32), non_blocking=cuda)


def sampling_from_request(temperature=None, top_k=None, seed=None) -> Optional[SamplingParams]:
    """Request fields -> parameters: no temperature (or 0) keeps the request greedy; a sampled request without a
    seed gets a random one, so two such requests do not share their noise."""
    if temperature is None or float(temperature) == 0.0:
        if top_k not in (None, 0) and int(top_k) < 0:
            raise ValueError(f"top_k must be >= 0, got {top_k!r}")
        return None
    if seed is None:
        import secrets
        seed = secrets.randbits(63)
    return SamplingParams(temperature=float(temperature), top_k=int(top_k or 0), seed=int(seed))
