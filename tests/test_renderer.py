"""Grounded renderer: source block, JSON extraction, citation/quote validation, extractive fallback (CPU)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

from hrm_flashrenderer_b200.serving import renderer as R
from hrm_flashrenderer_b200.serving.utils import find_hrm_binary

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "fixtures"))
from hrm_corpus import corpus  # noqa: E402

HRM = find_hrm_binary()
needs_hrm = pytest.mark.skipif(not Path(HRM).is_file(), reason="hrm core not built")

CHOSEN = [{"sid": "0001:0000", "txt": "The silver bridge is guarded at night by two soldiers.", "txt_c": "silver bridge"},
          {"sid": "0002:0003", "txt": "x" * 1500}]


def test_sources_block_truncates_and_maps():
    block, src = R.sources_block(CHOSEN)
    assert block.startswith("[SOURCES]\n0001:0000: The silver") and block.endswith("[/SOURCES]")
    assert src["0002:0003"] == "x" * 1200 + "…"


def test_first_json_object_handles_braces_in_strings_and_junk():
    txt = 'noise {bad json} then {"answer": "a } b {", "citations": [], "quotes": []} trailing {"x": 1}'
    assert R.first_json_object(txt)["answer"] == "a } b {"
    with pytest.raises(ValueError):
        R.first_json_object("no object here")


def test_validation_rules():
    _, src = R.sources_block(CHOSEN)
    ok = {"answer": "two soldiers", "citations": ["0001:0000"],
          "quotes": [{"id": "0001:0000", "quote": "guarded at night"}]}
    assert R.validate(ok, src) == (True, "ok")
    assert R.validate({**ok, "citations": ["9999:0000"]}, src)[1] == "citation '9999:0000': no such source"
    assert R.validate({**ok, "quotes": [{"id": "0001:0000", "quote": "guarded by day"}]}, src)[1] == \
        "quotes[0]: text is not verbatim in 0001:0000"
    assert R.validate({**ok, "quotes": [{"id": "0001:0000", "quote": "  "}]}, src)[1] == \
        "quotes[0]: blank quote for 0001:0000"
    assert R.validate({"citations": []}, src) == (False, "answer: missing or not a string")
    assert R.validate([1], src) == (False, "rendered value is a list, not an object")
    # every problem is reported, in reading order
    bad = {"answer": 3, "citations": ["nope"], "quotes": ["x", {"id": "gone", "quote": "q"}]}
    assert R.grounding_problems(bad, src) == [
        "answer: missing or not a string", "citation 'nope': no such source", "quotes[0]: not an object",
        "quotes[1]: source 'gone' was not shown"]


def test_hrm_query_errors(tmp_path):
    fake = tmp_path / "hrm"
    fake.write_text("#!/bin/sh\ncat > /dev/null\necho \"$HRM_FAKE_OUT\"\nexit $HRM_FAKE_RC\n")
    fake.chmod(0o755)
    env = os.environ
    try:
        os.environ["HRM_FAKE_OUT"], os.environ["HRM_FAKE_RC"] = '{"cids": [3], "chosen": []}', "0"
        assert R.hrm_query(str(fake), "m", "q")["cids"] == [3]
        os.environ["HRM_FAKE_OUT"] = "not json"
        with pytest.raises(R.RetrievalError, match="not JSON"):
            R.hrm_query(str(fake), "m", "q")
        os.environ["HRM_FAKE_OUT"], os.environ["HRM_FAKE_RC"] = "", "3"
        with pytest.raises(R.RetrievalError, match="exited with status 3"):
            R.hrm_query(str(fake), "m", "q")
    finally:
        env.pop("HRM_FAKE_OUT", None)
        env.pop("HRM_FAKE_RC", None)


def test_render_answer_paths():
    hrm = {"cids": [1, 2], "chosen": CHOSEN}
    good = lambda p, n: 'Sure! {"answer": "two soldiers", "citations": ["0001:0000"], ' \
                        '"quotes": [{"id": "0001:0000", "quote": "two soldiers"}]}'
    out = R.render_answer("who guards the bridge", hrm, good)
    assert out["answer"] == "two soldiers" and "error" not in out and out["hrm"]["cids"] == [1, 2]
    bad = lambda p, n: '{"answer": "x", "citations": ["0001:0000"], "quotes": [{"id": "0001:0000", "quote": "nope"}]}'
    out = R.render_answer("q", hrm, bad)
    assert out["mode"] == "fallback_extractive" and out["error"].startswith("validation_failed")
    assert out["quotes"][1]["quote"] == "x" * 240
    out = R.render_answer("q", hrm, None)
    assert out["error"].startswith("renderer_failed") and out["citations"] == ["0001:0000", "0002:0003"]


def test_render_prompt_reaches_renderer():
    seen = {}

    def rec(p, n):
        seen["p"], seen["n"] = p, n
        return "{}"
    R.render_answer("who?", {"chosen": CHOSEN}, rec, max_tokens=17)
    assert seen["n"] == 17 and seen["p"].startswith("<|system|>\nYou are a grounded renderer.")
    assert "QUESTION:\nwho?\n\nReturn JSON now.\n<|assistant|>\n" in seen["p"]


@needs_hrm
def test_cli_end_to_end_extractive(tmp_path):
    (tmp_path / "c.txt").write_text(corpus(300))
    subprocess.run([str(HRM), "prep", "--input", str(tmp_path / "c.txt"), "--out", str(tmp_path / "p.jsonl"),
                    "--cluster-size", "20"], check=True, capture_output=True)
    subprocess.run([str(HRM), "build", "--payloads", str(tmp_path / "p.jsonl"), "--outdir", str(tmp_path / "m")],
                   check=True, capture_output=True)
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    p = subprocess.run([sys.executable, "-m", "hrm_flashrenderer_b200.serving.renderer", "--model", str(tmp_path / "m"),
                        "--prompt", "who guards the silver bridge at night", "--json", "--llm",
                        str(tmp_path / "missing.gguf")], capture_output=True, text=True, env=env, timeout=120)
    assert p.returncode == 0, p.stderr
    obj = json.loads(p.stdout)
    assert obj["mode"] == "fallback_extractive" and obj["error"].startswith("renderer_failed")
    assert obj["citations"] and obj["hrm"]["k"] == 8
