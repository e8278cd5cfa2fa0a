"""Pinned defaults of the serving surfaces (the reference's static regressions, ``tests/test_regressions.py:96-273``,
checked here by parsing the real parsers and calling the real prompt path instead of grepping source text):
retrieval top_k = k = 16 with top_m = 400, at most 16 sources, the HRM query timeout of 1.8 s, q8 as the only
quantisation, and the int8 engine as the default and only model backend."""
from hrm_flashrenderer_b200.serving import cli, prompt_builder as pb
from hrm_flashrenderer_b200.serving import serve


def _choices(parser, dest):
    for act in parser._actions:
        if act.dest == dest:
            return act.choices, act.default
    raise KeyError(dest)


def _generate_parser():
    ap = cli.build_arg_parser()
    sub = next(a for a in ap._actions if a.dest == "cmd")
    return sub.choices["generate"]


def test_generate_cli_defaults():
    g = _generate_parser()
    a = g.parse_args(["--hrm_model", "m", "--llm_model", "synthetic:tiny", "--prompt", "q"])
    assert (a.top_k, a.top_m, a.k, a.max_sources, a.max_chars_per_source) == (16, 400, 16, 16, 1200)
    assert a.mode == "mixed" and a.model_quant == "q8" and a.backend == "b200_int8"
    assert _choices(g, "model_quant")[0] == ["q8"]
    assert set(_choices(g, "backend")[0]) == {"b200_int8", "deepseek_int8"}   # deepseek_int8: the reference's name


def test_serve_cli_defaults():
    ap = serve.build_arg_parser()
    a = ap.parse_args(["--hrm_model", "m", "--llm_model", "synthetic:tiny"])
    assert a.max_sources == 16 and a.max_chars_per_source == 1200 and a.reserve_prompt_tokens == 16
    assert a.model_quant == "q8" and _choices(ap, "model_quant")[0] == ["q8"]
    assert a.backend == "b200_int8"
    st = serve.ServiceState()
    assert st.hrm_timeout_s == 1.8 and st.max_sources == 16


def test_prompt_path_queries_hrm_with_pinned_parameters():
    seen = {}

    class R:
        raw = {"chosen": [{"sid": f"s{i}", "txt": f"snippet {i}"} for i in range(40)]}

    def q(**kw):
        seen.update(kw)
        return R()

    st = serve.ServiceState(query_fn=q, disable_token_budget=True)
    text, sources, mode, active = serve.build_prompt(st, "question?", "default")
    assert mode == "mixed" and active and text
    assert (seen["top_k"], seen["top_m"], seen["k"], seen["timeout_s"]) == (16, 400, 16, 1.8)
    assert len(sources) == 16


def test_prompt_builder_defaults():
    assert pb.build_sources.__defaults__ == (16, 1200)
    assert pb.SILENT_SYSTEM_PROMPT == pb.MIXED_SYSTEM_PROMPT
