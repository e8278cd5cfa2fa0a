"""NVTX ranges: a no-op when off; when on, every push is popped, also when the body raises."""
import pytest
import torch

from hrm_flashrenderer_b200.utils import nvtx


def test_off_is_a_null_context(monkeypatch):
    monkeypatch.setattr(nvtx, "ENABLED", False)
    with nvtx.nvtx_range("x"):
        pass


def test_on_pushes_and_pops_even_on_error(monkeypatch):
    log = []
    monkeypatch.setattr(nvtx, "ENABLED", True)
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda n: log.append(("push", n)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: log.append(("pop",)))
    with nvtx.nvtx_range("decode step"):
        with nvtx.nvtx_range("inner"):
            pass
    with pytest.raises(ValueError):
        with nvtx.nvtx_range("prefill chunk"):
            raise ValueError("boom")
    assert log == [("push", "decode step"), ("push", "inner"), ("pop",), ("pop",), ("push", "prefill chunk"),
                   ("pop",)]
