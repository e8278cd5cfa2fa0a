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


def test_telemetry_packets_carry_loss_and_projection(tmp_path):
    """With telemetry on, every generated token's packet carries the greedy token's cross-entropy (the reference
    engine's step loss; 0 for the first token) and a projection of the final hidden row; the loss equals
    logsumexp(logits) - max(logits) of that step computed independently."""
    import socket
    from hrm_flashrenderer_b200.serving.telemetry import Telemetry, unpack
    model = LlamaW8.from_weights(TINY, synth_weights(TINY, seed=0), device="cpu", max_pos=256)
    model.collect_stats = True
    eng = InferenceEngine(model, EngineConfig(max_seq_len=128, max_batch=1, use_cuda_graphs=False), num_blocks=16)
    rx = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
    rx.bind(("127.0.0.1", 0))
    rx.settimeout(5)
    tel = Telemetry("tiny", hidden=TINY.hidden, env={"TELEM_ENABLE": "1", "TELEM_PORT": str(rx.getsockname()[1])})
    p = _paths(tmp_path)
    prompt = [5, 17, 300, 42, 7]
    p.prompt.write_text("hi\n")
    p.prompt_tokens.write_text("".join(f"{t}\n" for t in prompt))
    seen = []
    orig = model.forward

    def spy(b):   # the loss each step should report, from the model's own logits path
        out = orig(b)
        seen.append(float(model.stat_nll[0]))
        return out
    model.forward = spy
    assert ipc.poll_once(eng, p, 128, 1, 6, log=lambda s: None, telemetry=tel)
    pk = [unpack(rx.recv(1024)) for _ in range(6)]
    toks = [int(x) for x in p.tokens.read_text().split()]
    assert [q["prompt"] for q in pk] == [f"TokenID: {t}" for t in toks]
    assert [q["step"] for q in pk] == list(range(len(prompt), len(prompt) + 6))
    assert pk[0]["loss"] == 0.0 and all(q["loss"] > 0.0 for q in pk[1:])
    assert [round(q["loss"], 4) for q in pk[1:]] == [round(v, 4) for v in seen[1:6]]
    assert any(abs(c) > 0 for c in pk[2]["proj"])


def test_record_stats_is_greedy_cross_entropy():
    """stat_nll = -log softmax(logits)[argmax] and stat_hidden = the RMS-normalised row, against direct math."""
    model = LlamaW8.from_weights(TINY, synth_weights(TINY, seed=0), device="cpu", max_pos=64)
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(3, 1024, generator=g) * 4
    xl = torch.randn(3, TINY.hidden, generator=g)
    ssq = xl.pow(2).view(3, -1, 128).sum(-1).t().contiguous()
    model._record_stats(logits, xl, (ssq, TINY.hidden, 1e-5))
    want = -torch.log_softmax(logits, -1).gather(1, logits.argmax(1, keepdim=True)).squeeze(1)
    torch.testing.assert_close(model.stat_nll[:3], want, rtol=1e-5, atol=1e-5)
    rms = torch.rsqrt(xl.pow(2).mean(-1) + 1e-5)
    torch.testing.assert_close(model.stat_hidden[:3], xl * rms[:, None], rtol=1e-5, atol=1e-5)
