"""HRM retrieval core (C++17): unit tests, and byte-for-byte parity with the reference `hrm` binary.

The golden hashes in fixtures/hrm_golden/golden.json were produced by the reference hrm_core build on the corpus of
fixtures/hrm_corpus.py; this test rebuilds the index with this project's `hrm` and compares index files and every
query output (json and text formats, three parameter sets, stdin prompt)."""
import hashlib
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CORE = os.path.join(ROOT, "hrm_core")
HRM = os.path.join(CORE, "build", "hrm")
sys.path.insert(0, os.path.join(ROOT, "tests", "fixtures"))


@pytest.fixture(scope="module")
def built():
    subprocess.run(["make", "-C", CORE, "-j4", "all"], check=True, capture_output=True)
    return HRM


def test_unit(built):
    r = subprocess.run([os.path.join(CORE, "build", "hrm_tests")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


@pytest.fixture(scope="module")
def model(built, tmp_path_factory):
    from hrm_corpus import corpus
    d = tmp_path_factory.mktemp("hrm")
    (d / "corpus.txt").write_text(corpus())
    subprocess.run([HRM, "prep", "--input", str(d / "corpus.txt"), "--out", str(d / "p.jsonl"), "--cluster-size", "40"],
                   check=True, capture_output=True)
    subprocess.run([HRM, "build", "--payloads", str(d / "p.jsonl"), "--outdir", str(d / "m")], check=True,
                   capture_output=True)
    return d


def _sha(p):
    return hashlib.sha256(open(p, "rb").read()).hexdigest()


def test_index_files_match_reference(model):
    g = json.load(open(os.path.join(ROOT, "tests", "fixtures", "hrm_golden", "golden.json")))
    assert _sha(model / "p.jsonl") == g["payloads_sha256"]
    assert _sha(model / "m" / "router_index.bin") == g["router_index_sha256"]
    assert (model / "m" / "meta.json").read_text() == g["meta"]


def test_queries_match_reference(model):
    from hrm_corpus import PROMPTS
    g = json.load(open(os.path.join(ROOT, "tests", "fixtures", "hrm_golden", "golden.json")))
    mismatches = []
    for pi, p in enumerate(PROMPTS):
        for qi, extra in enumerate(g["params"]):
            for fmt in ("json", "text"):
                r = subprocess.run([HRM, "query", "--model", str(model / "m"), "--format", fmt, "--prompt", p] + extra,
                                   capture_output=True)
                want = g["queries"][f"{pi}-{qi}-{fmt}"]
                if r.returncode != want["rc"] or hashlib.sha256(r.stdout).hexdigest() != want["sha256"]:
                    mismatches.append((pi, qi, fmt))
    r = subprocess.run([HRM, "query", "--model", str(model / "m"), "--format", "json", "--prompt-stdin"],
                       input=b"silver bridge\nat night\n", capture_output=True)
    if hashlib.sha256(r.stdout).hexdigest() != g["queries"]["stdin-json"]["sha256"]:
        mismatches.append("stdin")
    assert not mismatches, mismatches


def test_c_abi_json_equals_cli(model):
    from hrm_flashrenderer_b200.serving.hrm_api import HRMHandle
    h = HRMHandle(str(model / "m"))
    try:
        js = h.query_json("who guards the silver bridge at night", top_k=16, top_m=400, k=16)
    finally:
        h.close()
    r = subprocess.run([HRM, "query", "--model", str(model / "m"), "--format", "json", "--prompt",
                        "who guards the silver bridge at night", "--top-k", "16", "--top-m", "400", "--k", "16"],
                       capture_output=True, text=True)
    assert js == r.stdout
    d = json.loads(js)
    assert set(d) == {"prompt", "cids", "chosen"}
    assert set(d["chosen"][0]) == {"sid", "cid", "rel", "txt", "txt_c"}


def test_c_abi_errors(built):
    from hrm_flashrenderer_b200.serving.hrm_api import HRMHandle, HRMError
    with pytest.raises(HRMError):
        HRMHandle("/nonexistent/model")
