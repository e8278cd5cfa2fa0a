"""PHO index prototype: text -> compact integer "PHO" ids; the server scores index records in PHO space only and
returns record ids, which a client resolves to text locally.

Reference: ``experiments/pho_index_cuda.sh`` -- encoder ``:72-111`` (alnum words, lower-case; per word the FNV-1a-32
of its first three and last three characters mapped to ids ``1 + h % 8191`` and ``8192 + h % 8191``; at most 32 query
ids; records keep the first 8), index file ``:54-66,113-148`` (header ``PHOX`` magic, version 1, record count; fixed
records of id, length, 8 ids, flags), scoring ``:159-175`` and the server / client REPLs ``:177-306``.

Kept identical: the encoder, the scores and the binary index layout (so index files interoperate).  Different by
design: all records live on the GPU (no 256-candidate cap), ties in the top-k are broken by record order so results
are deterministic, the client resolves ids through a JSON side file written at build time instead of a compiled-in
table, and the CLI is Python over the library's CUDA kernel (``pho_score``) with a CPU fallback.
"""
from __future__ import annotations

import argparse
import json
import struct
import sys
from pathlib import Path
from typing import Dict, Iterable, List, Sequence, Tuple

import numpy as np
import torch

MAGIC = 0x50484F58   # "PHOX"
VERSION = 1
MAX_QUERY = 32
MAX_IDS = 8
HEADER = struct.Struct("<IIII")
RECORD_DTYPE = np.dtype([("id", "<u4"), ("len", "<u4"), ("pho", "<u4", (MAX_IDS,)), ("flags", "<u4")])

DEMO_ITEMS = [
    (2001, "silver bridge night guard"), (2002, "winter tower lantern"), (2003, "merchant promise to the king"),
    (2004, "river stone legend"), (2005, "tensor core matrix multiply"), (2006, "paged kv cache block table"),
    (2007, "nvlink peer memory all reduce"), (2008, "int8 weight dequantization"), (2009, "greedy decode argmax"),
    (2010, "prefill attention causal mask"), (2011, "router lane failover"), (2012, "hrm signature bins"),
    (2013, "sqlite snippet store"), (2014, "mmr diversity selection"), (2015, "power limit governor"),
    (2016, "deterministic retrieval ids"),
]


def fnv1a32(s: bytes) -> int:
    h = 2166136261
    for c in s:
        h ^= c
        h = (h * 16777619) & 0xFFFFFFFF
    return h


def _words(text: str) -> List[bytes]:
    out, cur = [], bytearray()
    for c in text.encode("utf-8"):
        if c < 128 and (chr(c).isalnum()):
            cur.append(ord(chr(c).lower()))
        elif cur:
            out.append(bytes(cur))
            cur = bytearray()
    if cur:
        out.append(bytes(cur))
    return out


def encode_pho(text: str) -> List[int]:
    ids: List[int] = []
    for w in _words(text):
        head = w[:3]
        tail = w if len(w) <= 3 else w[-3:]
        ids.append(1 + fnv1a32(head) % 8191)
        if len(ids) < MAX_QUERY:
            ids.append(8192 + fnv1a32(tail) % 8191)
        if len(ids) >= MAX_QUERY:
            break
    if not ids:
        ids.append(1 + fnv1a32(b"empty") % 8191)
    return ids


def build_index(path: str, items: Sequence[Tuple[int, str]]) -> None:
    recs = np.zeros(len(items), dtype=RECORD_DTYPE)
    for i, (rid, text) in enumerate(items):
        pho = encode_pho(text)[:MAX_IDS]
        recs[i]["id"] = rid
        recs[i]["len"] = len(pho)
        recs[i]["pho"][:len(pho)] = pho
    with open(path, "wb") as f:
        f.write(HEADER.pack(MAGIC, VERSION, len(items), 0))
        f.write(recs.tobytes())
    with open(path + ".resolve.json", "w", encoding="utf-8") as f:
        json.dump({str(rid): text for rid, text in items}, f, indent=1)


def load_index(path: str) -> np.ndarray:
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    magic, version, count, _ = HEADER.unpack(bytes(raw[:HEADER.size]))
    if magic != MAGIC:
        raise ValueError(f"{path}: bad index magic")
    if version != VERSION:
        raise ValueError(f"{path}: unsupported version {version}")
    return np.frombuffer(raw, dtype=RECORD_DTYPE, count=count, offset=HEADER.size)


def score_reference(pho: np.ndarray, lens: np.ndarray, q: Sequence[int]) -> np.ndarray:
    """CPU scores, same definition as the GPU kernel."""
    q = np.asarray(q[:MAX_QUERY], dtype=np.int64)
    lens = np.minimum(lens.astype(np.int64), MAX_IDS)
    valid = np.arange(MAX_IDS)[None, :] < lens[:, None]
    eq = (pho.astype(np.int64)[:, :, None] == q[None, None, :]) & valid[:, :, None]
    return (eq.sum(axis=(1, 2)) - 0.05 * np.abs(lens - len(q))).astype(np.float32)


class PhoIndex:
    def __init__(self, path: str, device: str = "cuda"):
        recs = load_index(path)
        self.ids = recs["id"].astype(np.int64)
        self.lens_np = recs["len"].astype(np.int64)
        self.pho_np = recs["pho"].astype(np.int64)
        self.device = torch.device(device if (device != "cuda" or torch.cuda.is_available()) else "cpu")
        if self.device.type == "cuda":
            from .. import ops
            self._C = ops.ext()
            self.pho = torch.from_numpy(recs["pho"].view(np.int32).reshape(-1, MAX_IDS).copy()).to(self.device)
            self.lens = torch.from_numpy(recs["len"].view(np.int32).copy()).to(self.device)
            self.scores = torch.empty(len(recs), dtype=torch.float32, device=self.device)

    def score(self, q: Sequence[int]) -> np.ndarray:
        if self.device.type != "cuda":
            return score_reference(self.pho_np, self.lens_np, q)
        qt = torch.tensor(list(q[:MAX_QUERY]), dtype=torch.int32, device=self.device)
        self._C.pho_score(self.pho, self.lens, qt, self.scores)
        return self.scores.cpu().numpy()

    def query(self, text: str, topk: int = 8, cand_limit: int = 0) -> Dict:
        q = encode_pho(text)[:MAX_QUERY]
        s = self.score(q)
        n = len(s) if cand_limit <= 0 else min(len(s), cand_limit)
        s = s[:n]
        order = np.lexsort((np.arange(n), -s))[:min(topk, n)]   # score desc, then record order
        return {"q_pho": q, "top": [{"index_id": int(self.ids[k]), "score": round(float(s[k]), 6),
                                     "pho": [int(x) for x in self.pho_np[k, :self.lens_np[k]]]} for k in order]}


def resolve(path: str, ids: Iterable[int]) -> List[str]:
    table = json.load(open(path + ".resolve.json", encoding="utf-8"))
    return [table.get(str(int(i)), "<unknown>") for i in ids]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-pho", description="PHO index prototype (build / server / client)")
    g = ap.add_mutually_exclusive_group()
    g.add_argument("--build", action="store_true")
    g.add_argument("--server", action="store_true")
    g.add_argument("--client", action="store_true")
    ap.add_argument("--index", default="pho_demo.index")
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--cand-limit", type=int, default=0, help="score only the first N records (0 = all)")
    ap.add_argument("--device", default="cuda")
    a = ap.parse_args(argv)
    if a.build or not Path(a.index).exists():
        build_index(a.index, DEMO_ITEMS)
        print(f"[*] built demo index: {a.index} ({len(DEMO_ITEMS)} records)", flush=True)
        if a.build:
            return 0
    if a.client:
        print("[client] enter index ids to resolve locally; /quit to exit", flush=True)
        for line in sys.stdin:
            line = line.strip()
            if line == "/quit":
                break
            try:
                print(resolve(a.index, [int(line)])[0], flush=True)
            except ValueError:
                print("<unknown>", flush=True)
        return 0
    idx = PhoIndex(a.index, a.device)
    print("[server] PHO-only mode: text in, PHO / index ids out; /quit to exit", flush=True)
    for line in sys.stdin:
        line = line.rstrip("\n")
        if line == "/quit":
            break
        print(json.dumps(idx.query(line, a.topk, a.cand_limit)), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
