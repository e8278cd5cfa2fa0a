"""DSI8 file-IPC shim: the reference engine's prompt / tokens / done-flag protocol on the CPU engine."""
import pytest
import torch

from hrm_flashrenderer_b200.config import TINY, EngineConfig
from hrm_flashrenderer_b200.models.llama import LlamaW8
from hrm_flashrenderer_b200.models.weights import synth_weights
from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
from hrm_flashrenderer_b200.serving import dsi8_ipc as ipc


@pytest.fixture(scope="module")
def engine():
    model = LlamaW8.from_weights(TINY, synth_weights(TINY, seed=0), device="cpu", max_pos=256)
    return InferenceEngine(model, EngineConfig(max_seq_len=128, max_batch=1, use_cuda_graphs=False), num_blocks=16)


def _paths(tmp_path):
    return ipc.IpcPaths(tmp_path / "p.txt", tmp_path / "pt.txt", tmp_path / "tok.txt", tmp_path / "done.flag")


def test_env_defaults_and_tgen_clamp():
    p = ipc.IpcPaths.from_env({})
    assert str(p.prompt) == "/tmp/deepseek_prompt.txt" and str(p.done) == "/tmp/deepseek_done.flag"
    assert ipc.tgen_from_env({}) == 64
    assert ipc.tgen_from_env({"DSI8_TGEN": "0"}) == 1 and ipc.tgen_from_env({"DSI8_TGEN": "99999"}) == 2048


def test_request_round_trip(engine, tmp_path):
    p = _paths(tmp_path)
    assert not ipc.poll_once(engine, p, 128, 1, 8, log=lambda s: None)       # nothing pending
    prompt = [5, 17, 300, 42, 7]
    p.tokens.write_text("999\n")                                               # stale result from before
    p.prompt.write_text("hello world\nsecond line ignored\n")
    p.prompt_tokens.write_text("".join(f"{t}\n" for t in prompt) + "junk\n")
    logs = []
    assert ipc.poll_once(engine, p, 128, 1, 8, log=logs.append)
    assert logs == ["> Received Prompt: hello world"]
    assert not p.prompt.exists() and not p.prompt_tokens.exists()
    got = [int(x) for x in p.tokens.read_text().split()]
    assert got == engine.generate([prompt], 8, stop_on_eos=False)[0]
    assert p.done.read_text() == "done\n"


def test_empty_tokens_use_bos_and_context_cap(engine, tmp_path):
    p = _paths(tmp_path)
    p.prompt.write_text("x\n")
    assert ipc.poll_once(engine, p, 6, 1, 64, log=lambda s: None)             # BOS + at most 5 new tokens
    assert len(p.tokens.read_text().split()) == 5
    assert p.done.exists()
