"""PairIndex tokenizer (native core): determinism, round trip, IDX7 files, tables, CLI, reference semantics."""
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "fixtures"))
from hrm_corpus import corpus  # noqa: E402

pi_mod = pytest.importorskip("hrm_flashrenderer_b200.experiments.pairindex")
try:
    pi_mod.lib()
except FileNotFoundError:
    pytest.skip("libhrm_pairindex.so not built", allow_module_level=True)
PairIndex = pi_mod.PairIndex
CLI = ROOT / "hrm_core" / "build" / "pairindex"


def _py_reference(data: bytes, k1: int, k2: int):
    """Straight Python statement of the two-stage rules, used to check the native build and encoder."""
    cnt = {}
    for i in range(len(data) - 1):
        p = data[i] | (data[i + 1] << 8)
        cnt[p] = cnt.get(p, 0) + 1
    items = sorted(cnt.items(), key=lambda kv: (-kv[1], kv[0]))
    id2pair = [p for p, _ in items[:k1]]
    used = set(cnt)
    p = 0
    while len(id2pair) < k1:
        if p not in used:
            id2pair.append(p)
        p += 1
    pair2id = {p: 256 + i for i, p in enumerate(id2pair)}

    def stage1(b):
        out, i = [], 0
        while i < len(b):
            if i + 1 < len(b) and (b[i] | (b[i + 1] << 8)) in pair2id:
                out.append(pair2id[b[i] | (b[i + 1] << 8)])
                i += 2
            else:
                out.append(b[i])
                i += 1
        return out
    s1 = stage1(data)
    c2 = {}
    for a, b in zip(s1, s1[1:]):
        c2[(a << 16) | b] = c2.get((a << 16) | b, 0) + 1
    items2 = sorted(c2.items(), key=lambda kv: (-kv[1], kv[0]))
    id2pair2 = [k for k, _ in items2[:k2]]
    id2pair2 += [(0xFFFF << 16) | (j & 0xFFFF) for j in range(len(id2pair2), k2)]
    macro = {k: 256 + k1 + i for i, k in enumerate(id2pair2)}

    def encode(b):
        s = stage1(b)
        out, i = [], 0
        while i < len(s):
            if i + 1 < len(s) and ((s[i] << 16) | s[i + 1]) in macro:
                out.append(macro[(s[i] << 16) | s[i + 1]])
                i += 2
            else:
                out.append(s[i])
                i += 1
        return out
    return id2pair, id2pair2, encode


def test_build_matches_python_statement_and_roundtrips():
    data = corpus(400).encode()
    k1, k2 = 300, 200
    pi = PairIndex.build_bytes(data, k1, k2)
    id2pair, id2pair2, hk, hv = pi.tables()
    ref1, ref2, ref_encode = _py_reference(data, k1, k2)
    assert id2pair.tolist() == ref1 and id2pair2.tolist() == ref2
    assert hk.size == 512 and int((hk != 0xFFFFFFFF).sum()) == k2
    text = "ROMEO: who guards the silver bridge at night?\nJULIET: the winter tower's guard."
    ids = pi.encode(text)
    assert ids.tolist() == ref_encode(text.encode())
    assert pi.decode(ids) == text
    assert len(ids) < len(text.encode())        # it compresses
    assert int(ids.max()) < pi.vocab


def test_idx7_file_tables_and_small_corpus_padding(tmp_path):
    pi = PairIndex.build_bytes(b"abababab", 8, 4)   # fewer distinct pairs than k1 / k2: padded deterministically
    a, b, _, _ = pi.tables()
    assert a[0] == (ord("a") | ord("b") << 8) and len(a) == 8
    assert b[-1] >> 16 == 0xFFFF
    p = tmp_path / "i.bin"
    pi.save(str(p))
    raw = p.read_bytes()
    assert raw[:4] == b"IDX7" and int.from_bytes(raw[4:8], "little") == 1
    q = PairIndex.load(str(p))
    assert [t.tolist() for t in q.tables()] == [t.tolist() for t in pi.tables()]
    r = PairIndex.from_tables(pi.k1, pi.k2, *pi.tables())
    assert r.encode("abababx").tolist() == pi.encode("abababx").tolist()


def test_files_are_order_independent_and_cli(tmp_path):
    f1, f2 = tmp_path / "b.txt", tmp_path / "a.txt"
    f1.write_text(corpus(120, seed=3))
    f2.write_text(corpus(120, seed=4))
    x = PairIndex.build_files([str(f1), str(f2)], 128, 64)
    y = PairIndex.build_files([str(f2), str(f1)], 128, 64)
    assert [t.tolist() for t in x.tables()] == [t.tolist() for t in y.tables()]
    if CLI.is_file():
        out = tmp_path / "cli.bin"
        subprocess.run([str(CLI), "build", "--inputs", f"{f1}:{f2}", "--k1", "128", "--k2", "64", "--out", str(out)],
                       check=True, capture_output=True)
        z = PairIndex.load(str(out))
        assert [t.tolist() for t in z.tables()] == [t.tolist() for t in x.tables()]
        (tmp_path / "t.txt").write_text("silver bridge")
        subprocess.run([str(CLI), "encode", "--index", str(out), "--in", str(tmp_path / "t.txt"), "--out",
                        str(tmp_path / "ids.u16")], check=True, capture_output=True)
        ids = np.fromfile(tmp_path / "ids.u16", dtype=np.uint16)
        assert ids.tolist() == z.encode("silver bridge").tolist()
