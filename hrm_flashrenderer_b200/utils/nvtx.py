"""NVTX ranges for Nsight timelines: on when HRM_NVTX=1 and CUDA is available, otherwise a no-op.

Ranges mark the engine steps: each prefill chunk, each decode step (graph replay or eager) and each decode-graph
capture.  Inside a captured CUDA graph a range is host-side only (it brackets the capture, not the replays)."""
from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("HRM_NVTX", "0") == "1" and torch.cuda.is_available()


@contextlib.contextmanager
def _on(name: str):
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def nvtx_range(name: str):
    """``with nvtx_range("layer 3/attention"): ...``"""
    return _on(name) if ENABLED else contextlib.nullcontext()
