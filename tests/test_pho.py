"""PHO index prototype: encoder, index file, scores (CPU reference and the CUDA kernel), server/client CLI."""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from hrm_flashrenderer_b200.experiments import pho

ROOT = Path(__file__).resolve().parents[1]


def test_fnv_vectors_and_encoder():
    assert pho.fnv1a32(b"a") == 0xE40C292C and pho.fnv1a32(b"foobar") == 0xBF9CF968
    ids = pho.encode_pho("Hello, WORLD! ab")
    assert ids == [1 + pho.fnv1a32(b"hel") % 8191, 8192 + pho.fnv1a32(b"llo") % 8191,
                   1 + pho.fnv1a32(b"wor") % 8191, 8192 + pho.fnv1a32(b"rld") % 8191,
                   1 + pho.fnv1a32(b"ab") % 8191, 8192 + pho.fnv1a32(b"ab") % 8191]
    assert pho.encode_pho("   ") == [1 + pho.fnv1a32(b"empty") % 8191]
    assert len(pho.encode_pho("w " * 100)) == 32
    assert pho.encode_pho("Fähre") == pho.encode_pho("F hre")   # non-ASCII bytes separate words


def test_index_roundtrip_and_query(tmp_path):
    p = str(tmp_path / "d.index")
    pho.build_index(p, pho.DEMO_ITEMS)
    raw = open(p, "rb").read()
    assert raw[:4] == b"XOHP" and len(raw) == 16 + 44 * len(pho.DEMO_ITEMS)
    recs = pho.load_index(p)
    assert int(recs[0]["id"]) == 2001 and int(recs[0]["len"]) == 8
    idx = pho.PhoIndex(p, device="cpu")
    r = idx.query("who guards the silver bridge at night", topk=3)
    assert r["top"][0]["index_id"] == 2001
    assert [t["score"] for t in r["top"]] == sorted([t["score"] for t in r["top"]], reverse=True)
    assert pho.resolve(p, [2001, 9])[0] == "silver bridge night guard" and pho.resolve(p, [9])[0] == "<unknown>"


def test_score_definition():
    recs = np.array([[5, 6, 7, 0, 0, 0, 0, 0], [5, 5, 0, 0, 0, 0, 0, 0]])
    s = pho.score_reference(recs, np.array([3, 2]), [5, 7])
    assert np.allclose(s, [2 - 0.05, 2.0])


def test_cli_server_and_client_cpu(tmp_path):
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    idx = str(tmp_path / "x.index")
    cmd = [sys.executable, "-m", "hrm_flashrenderer_b200.experiments.pho", "--index", idx, "--device", "cpu"]
    out = subprocess.run(cmd + ["--server", "--topk", "2"], input="paged kv cache\n/quit\n", capture_output=True,
                         text=True, env=env, timeout=120)
    assert out.returncode == 0, out.stderr
    top = json.loads(out.stdout.strip().splitlines()[-1])["top"]
    assert top[0]["index_id"] == 2006 and len(top) == 2
    out = subprocess.run(cmd + ["--client"], input="2006\n/quit\n", capture_output=True, text=True, env=env,
                         timeout=60)
    assert "paged kv cache block table" in out.stdout


@pytest.mark.gpu
def test_pho_kernel_matches_reference(tmp_path):
    rng = np.random.default_rng(0)
    n = 1_000_003
    items_pho = rng.integers(1, 300, size=(n, 8)).astype(np.uint32)
    lens = rng.integers(0, 9, size=n).astype(np.uint32)
    recs = np.zeros(n, dtype=pho.RECORD_DTYPE)
    recs["id"], recs["len"], recs["pho"] = np.arange(n), lens, items_pho
    p = str(tmp_path / "big.index")
    with open(p, "wb") as f:
        f.write(pho.HEADER.pack(pho.MAGIC, pho.VERSION, n, 0))
        f.write(recs.tobytes())
    idx = pho.PhoIndex(p, device="cuda")
    for q in ([1, 2, 3, 17, 250], list(range(1, 33)), [299]):
        got = idx.score(q)
        want = pho.score_reference(items_pho.astype(np.int64), lens.astype(np.int64), q)
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)
