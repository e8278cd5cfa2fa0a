"""Counterparts of the reference's static / fresh-install / native-lock / mocked-benchmark suites:
every module imports, every console entry point answers --help, unsupported models are rejected, the serving
benchmark grid writes comparable CSVs against the mock stack, and the config-5 trace replays on the CPU engine."""
import csv
import importlib
import pkgutil

import pytest

import hrm_flashrenderer_b200 as pkg

SKIP_IMPORT = set()


def test_every_module_imports():
    bad = []
    for m in pkgutil.walk_packages(pkg.__path__, pkg.__name__ + "."):
        if m.name in SKIP_IMPORT:
            continue
        try:
            importlib.import_module(m.name)
        except Exception as e:   # pragma: no cover - the assertion shows which
            bad.append(f"{m.name}: {type(e).__name__}: {e}")
    assert not bad, bad


@pytest.mark.parametrize("mod", [
    "hrm_flashrenderer_b200.serving.cli", "hrm_flashrenderer_b200.serving.serve", "hrm_flashrenderer_b200.serving.router",
    "hrm_flashrenderer_b200.serving.daemon", "hrm_flashrenderer_b200.serving.dsi8_ipc",
    "hrm_flashrenderer_b200.launcher.service", "hrm_flashrenderer_b200.launcher.topology",
    "hrm_flashrenderer_b200.launcher.preflight", "hrm_flashrenderer_b200.launcher.e2e",
    "hrm_flashrenderer_b200.launcher.diag",
    "hrm_flashrenderer_b200.benchmarks.serving", "hrm_flashrenderer_b200.benchmarks.ops_sweep",
    "hrm_flashrenderer_b200.experiments.llm", "hrm_flashrenderer_b200.experiments.bench_cli"])
def test_entry_point_help(mod, capsys):
    m = importlib.import_module(mod)
    with pytest.raises(SystemExit) as e:
        m.main(["--help"])
    assert e.value.code == 0
    assert "usage" in capsys.readouterr().out.lower()


def test_native_lock_rejects_unsupported_models():
    from hrm_flashrenderer_b200.serving.utils import validate_native_model_config, validate_tp_world
    ok = {"hidden_size": 8192, "num_attention_heads": 64, "intermediate_size": 28672, "vocab_size": 128256,
          "architectures": ["LlamaForCausalLM"]}
    validate_native_model_config(ok)
    validate_tp_world(ok, 8)
    for bad in ({**ok, "architectures": ["MixtralMoEForCausalLM"]}, {**ok, "architectures": ["DeepseekV3ForCausalLM"]},
                {**ok, "num_local_experts": 8}, {**ok, "num_attention_heads": 32},
                {**ok, "hidden_size": 8190}):
        with pytest.raises(ValueError):
            validate_native_model_config(bad)
    with pytest.raises(ValueError):
        validate_tp_world({**ok, "vocab_size": 128257}, 8)


def test_serving_benchmark_grid_against_mock_stack(tmp_path):
    from hrm_flashrenderer_b200.benchmarks.serving import run_grid
    from hrm_flashrenderer_b200.launcher.e2e import mock_stack
    url, servers = mock_stack()
    try:
        summary = run_grid(url, tmp_path, scenarios=("short",), repeats=2, warmup=1)
    finally:
        for s in servers:
            s.close()
    rows = list(csv.DictReader(open(tmp_path / "raw.csv")))
    assert len(rows) == 3 * 2 and {r["mode"] for r in rows} == {"mixed", "retrieval", "deepseek_only"}
    assert {s["mode"] for s in summary} == {"mixed", "retrieval", "deepseek_only"}
    assert (tmp_path / "summary.csv").is_file() and (tmp_path / "summary.txt").read_text().strip()


def test_trace_replay_on_cpu_engine():
    from hrm_flashrenderer_b200.benchmarks.serving import make_trace, run_trace
    from hrm_flashrenderer_b200.config import TINY, EngineConfig
    from hrm_flashrenderer_b200.models.llama import LlamaW8
    from hrm_flashrenderer_b200.models.weights import synth_weights
    from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
    from hrm_flashrenderer_b200.runtime.scheduler import Scheduler
    # the trace's shared system prompt (first 32 tokens) plus the start of each request's own context
    trace = [(t, ids[:32] + ids[256:264], 4) for t, ids, _ in make_trace(n=6, rate=50.0, vocab=TINY.vocab, seed=3)]
    model = LlamaW8.from_weights(TINY, synth_weights(TINY, seed=0), device="cpu", max_pos=128)
    results = {}
    for pc in (False, True):
        eng = InferenceEngine(model, EngineConfig(max_seq_len=96, max_batch=4, use_cuda_graphs=False,
                                                  prefix_cache=pc), num_blocks=64)
        sch = Scheduler(eng)
        sch.start()
        try:
            res = run_trace(sch, trace, time_scale=0.1)
        finally:
            sch.stop()
        assert res["requests"] == 6 and res["generated_tokens"] == 6 * 4 and res["ttft_p50_ms"] > 0
        assert res["prompt_tokens"] == 6 * 40
        results[pc] = res
    assert results[False]["prefilled_tokens"] == 6 * 40 and results[False]["prefix_cache_hit_blocks"] == 0
    # with the cache, requests that arrive after the first one finished its prompt skip the two shared blocks
    hits = results[True]["prefix_cache_hit_blocks"]
    assert hits >= 2 and results[True]["prefilled_tokens"] == 6 * 40 - 16 * hits


def test_diag_runs_without_gpu(capsys):
    from hrm_flashrenderer_b200.launcher import diag
    import torch
    rep = diag.run(log=lambda s: None)
    assert rep["cuda_available"] == torch.cuda.is_available()
    if not rep["cuda_available"]:
        assert rep["devices"] == [] and rep["failures"] == []
