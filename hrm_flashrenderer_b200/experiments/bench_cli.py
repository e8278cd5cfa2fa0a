"""Benchmark grid for the experiments trainer: presets x learning rates x runners x repeats -> CSV + ranking.

    python -m hrm_flashrenderer_b200.experiments.bench_cli [--preset matrix|decision|large] [--repeats 2]
        [--steps 80] [--log-every 10] [--save-every 1000] [--gpus 1] [--lr-list 0.0001,0.0003,0.001]
        [--out bench_cli] [--corpus-dir DIR] [--extra "--dmodel 128 ..."]

Counterpart of the reference's ``experiments/benchmark_cli.sh`` (presets and scenarios ``:91-115``, one run per
(scenario, lr, runner, repeat) ``:133-148``, CSV columns ``runner,scenario,lr,rep,tok_s,elapsed_sec`` ``:61``,
ranking ``:170-233``).  Runners here are this package's trainer (``experiments/llm.py``): ``revlm`` (CUDA-graph
train step) and ``revlm_eager`` (``--no_graph``); on several GPUs a runner goes through ``torch.distributed.run``.

Corpora: the reference downloads tinyshakespeare and wikitext-2.  Nothing is downloaded here: ``--corpus-dir``
may hold ``shakespeare.txt`` / ``wikitext2_train.txt``; otherwise built-in stand-ins of the same role are written
(a public-domain verse excerpt repeated, and a deterministic synthetic word-level corpus), next to the small
``code`` and ``german`` texts.  ``mixed_large`` is 6 x wikitext + 20 x shakespeare as in the reference.

Ranking (same rule as the reference so its tables compare): per runner@lr the mean tok/s and mean run time; a
runner@lr wins a scenario when its mean tok/s is the best there; score = norm(tok/s) - norm(run time) + 0.08 x wins
with min-max normalisation (0.5 when all equal); the top five are printed and the best is the winner.
"""
from __future__ import annotations

import argparse
import csv
import os
import random
import re
import subprocess
import sys
import time
from collections import defaultdict
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple

PRESETS: Dict[str, List[Tuple[str, str, int, int]]] = {
    # name, corpus, seq, batch
    "matrix": [("shakespeare", "shakespeare", 32, 8), ("code", "code", 32, 8), ("german", "german", 32, 8)],
    "decision": [("shakespeare", "shakespeare", 32, 8), ("code", "code", 32, 8), ("german", "german", 32, 8),
                 ("shakespeare_long", "shakespeare", 64, 4)],
    "large": [("tiny", "shakespeare", 32, 8), ("medium", "wikitext2_train", 64, 4),
              ("large", "mixed_large", 64, 4)],
}

RUNNERS: Dict[str, List[str]] = {"revlm": [], "revlm_eager": ["--no_graph"]}

_VERSE = """Shall I compare thee to a summer's day?
Thou art more lovely and more temperate:
Rough winds do shake the darling buds of May,
And summer's lease hath all too short a date;
Sometime too hot the eye of heaven shines,
And often is his gold complexion dimm'd;
And every fair from fair sometime declines,
By chance or nature's changing course untrimm'd;
But thy eternal summer shall not fade,
Nor lose possession of that fair thou ow'st;
Nor shall death brag thou wander'st in his shade,
When in eternal lines to time thou grow'st:
So long as men can breathe or eyes can see,
So long lives this, and this gives life to thee.
"""

_CODE = """#include <cstdio>
int main() { std::printf("hi\\n"); return 0; }
def gcd(a, b):
    while b:
        a, b = b, a % b
    return a
"""

_GERMAN = """Ein kleiner deutscher Text dient als dritter Korpus dieses Vergleichs.
Alle Laeufe sehen dieselben Daten, damit die Zahlen vergleichbar bleiben.
"""


def _synthetic_words(n_lines: int, seed: int = 0) -> str:
    rng = random.Random(seed)
    vocab = ["the", "of", "and", "in", "to", "a", "was", "is", "for", "on", "as", "with", "by", "that", "at",
             "from", "his", "it", "an", "were", "are", "which", "this", "be", "also", "has", "or", "had", "first",
             "one", "their", "its", "new", "after", "who", "they", "two", "her", "she", "been", "other", "when",
             "there", "all", "during", "into", "school", "time", "may", "years", "more", "most", "only", "over",
             "city", "some", "world", "would", "where", "later", "up", "such", "used", "many", "can", "state"]
    lines = []
    for _ in range(n_lines):
        k = rng.randint(6, 18)
        lines.append(" ".join(rng.choice(vocab) for _ in range(k)) + " .")
    return "\n".join(lines) + "\n"


def prepare_corpora(out_dir: Path, corpus_dir: Optional[Path] = None) -> Dict[str, Path]:
    cdir = out_dir / "corpora"
    cdir.mkdir(parents=True, exist_ok=True)
    paths: Dict[str, Path] = {}

    def put(name: str, text_fn):
        p = cdir / f"{name}.txt"
        src = corpus_dir / f"{name}.txt" if corpus_dir else None
        if src is not None and src.is_file() and src.stat().st_size > 0:
            p.write_bytes(src.read_bytes())
        elif not (p.is_file() and p.stat().st_size > 0):
            p.write_text(text_fn())
        paths[name] = p

    put("shakespeare", lambda: _VERSE * 40)
    put("wikitext2_train", lambda: _synthetic_words(4000))
    put("code", lambda: _CODE)
    put("german", lambda: _GERMAN)
    mixed = cdir / "mixed_large.txt"
    mixed.write_bytes(b"".join([paths["wikitext2_train"].read_bytes() + b"\n"] * 6 +
                               [paths["shakespeare"].read_bytes() + b"\n"] * 20))
    paths["mixed_large"] = mixed
    return paths


def normalize_lr(x: float) -> str:
    return f"{float(x):.10f}".rstrip("0").rstrip(".")


def runner_command(runner: str, gpus: int, corpus: Path, seq: int, batch: int, lr: float, steps: int,
                   log_every: int, save_every: int, ckpt: Path, index: Path, extra: Sequence[str]) -> List[str]:
    args = ["--train", "--measure", "--data", str(corpus), "--steps", str(steps), "--log_every", str(log_every),
            "--save_every", str(save_every), "--gpus", str(gpus), "--seq", str(seq), "--batch", str(batch),
            "--lr", str(lr), "--ckpt", str(ckpt), "--index", str(index)] + RUNNERS[runner] + list(extra)
    if gpus > 1:
        return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
                "--master-addr", "127.0.0.1", "--master-port", str(29500 + random.randint(0, 400)),
                "-m", "hrm_flashrenderer_b200.experiments.llm"] + args
    return [sys.executable, "-m", "hrm_flashrenderer_b200.experiments.llm"] + args


_TOK = re.compile(r"tok/s=([0-9]+(?:\.[0-9]+)?)")


def run_once(runner: str, scenario: str, corpus: Path, seq: int, batch: int, lr: float, rep: int, a,
             out_dir: Path, extra: Sequence[str]) -> Tuple[str, str]:
    """One training run (fresh checkpoint); returns (tok/s, elapsed seconds) as CSV strings ('NA' on failure)."""
    tag = f"{runner}__{scenario}__lr{normalize_lr(lr)}__r{rep}"
    log = out_dir / "logs" / f"{tag}.log"
    ckpt = out_dir / "logs" / f"ckpt_{tag}.bin"
    ckpt.unlink(missing_ok=True)                      # --force-new: never continue from an earlier run
    cmd = runner_command(runner, a.gpus, corpus, seq, batch, lr, a.steps, a.log_every, a.save_every, ckpt,
                         out_dir / "logs" / "no_index.bin", extra)
    t0 = time.perf_counter()
    env = dict(os.environ)
    env.setdefault("PYTHONPATH", str(Path(__file__).resolve().parents[2]))
    with open(log, "w") as f:
        r = subprocess.run(cmd, stdout=f, stderr=subprocess.STDOUT, env=env)
    sec = time.perf_counter() - t0
    text = log.read_text(errors="replace")
    toks = _TOK.findall(text)
    tok = toks[-1] if (toks and r.returncode == 0) else "NA"
    return tok, (f"{sec:.2f}" if r.returncode == 0 else "NA")


def _mmss(x: float) -> str:
    m = int(x // 60)
    return f"{m}:{x - m * 60:05.2f}"


def summarize(csv_path: Path) -> Tuple[List[tuple], str]:
    """Ranking table lines and the winner (runner@lr)."""
    rows = list(csv.DictReader(open(csv_path)))

    def ff(x):
        try:
            return float(x)
        except (TypeError, ValueError):
            return None

    per_key = defaultdict(list)
    triple = defaultdict(list)
    for r in rows:
        t, s = ff(r["tok_s"]), ff(r["elapsed_sec"])
        if t is None or s is None:
            continue
        per_key[f"{r['runner']}@{r['lr']}"].append((t, s))
        triple[(r["runner"], r["scenario"], r["lr"])].append((t, s))
    if not per_key:
        return [], ""
    per_scen = defaultdict(list)
    for (runner, scen, lr), vals in triple.items():
        per_scen[scen].append((sum(t for t, _ in vals) / len(vals), f"{runner}@{lr}"))
    wins = defaultdict(int)
    for cands in per_scen.values():
        cands.sort(reverse=True)
        wins[cands[0][1]] += 1
    rep = []
    for k, vals in per_key.items():
        rep.append((k, sum(t for t, _ in vals) / len(vals), sum(s for _, s in vals) / len(vals),
                    sum(s for _, s in vals), wins.get(k, 0)))
    mts, mss = [x[1] for x in rep], [x[2] for x in rep]

    def norm(x, lo, hi):
        return 0.5 if lo == hi else (x - lo) / (hi - lo)

    scored = sorted(((norm(mt, min(mts), max(mts)) - norm(ms, min(mss), max(mss)) + w * 0.08, k, mt, ms, tot, w)
                     for k, mt, ms, tot, w in rep), reverse=True)
    return scored, scored[0][1]


def print_summary(scored, winner: str, csv_path: Path, out=None) -> None:
    out = out or sys.stdout
    line = "+--------------------+------------+----------+----------+------+"
    print("\n" + line, file=out)
    print("| runner@lr          | tok/s      | run      | total    | wins |", file=out)
    print(line, file=out)
    for _, k, mt, ms, tot, w in scored[:5]:
        print(f"| {k:<18} | {mt:10.1f} | {_mmss(ms):>8} | {_mmss(tot):>8} | {w:4d} |", file=out)
    print(line, file=out)
    print(f"WINNER: {winner}", file=out)
    print(f"CSV: {csv_path}", file=out)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-bench-cli", description="experiments trainer benchmark grid")
    ap.add_argument("--preset", default="decision", choices=sorted(PRESETS))
    ap.add_argument("--repeats", type=int, default=2)
    ap.add_argument("--steps", type=int, default=80)
    ap.add_argument("--log-every", type=int, default=10)
    ap.add_argument("--save-every", type=int, default=1000)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--lr-list", default="0.0001,0.0003,0.001")
    ap.add_argument("--runners", default=",".join(RUNNERS), help="subset of: " + ",".join(RUNNERS))
    ap.add_argument("--out", default="bench_cli")
    ap.add_argument("--corpus-dir", default="", help="directory with shakespeare.txt / wikitext2_train.txt")
    ap.add_argument("--extra", default="", help="extra trainer flags, e.g. '--dmodel 128 --layers 2'")
    a = ap.parse_args(argv)
    out_dir = Path(a.out)
    (out_dir / "logs").mkdir(parents=True, exist_ok=True)
    corpora = prepare_corpora(out_dir, Path(a.corpus_dir) if a.corpus_dir else None)
    csv_path = out_dir / "raw.csv"
    runners = [r for r in a.runners.split(",") if r]
    for r in runners:
        if r not in RUNNERS:
            raise SystemExit(f"unknown runner {r!r}")
    lrs = [float(x) for x in a.lr_list.split(",") if x]
    extra = a.extra.split()
    with open(csv_path, "w", newline="") as f:
        f.write("runner,scenario,lr,rep,tok_s,elapsed_sec\n")
    print(f"Starting benchmark preset={a.preset} repeats={a.repeats} steps={a.steps} lr_list={a.lr_list}")
    for name, corpus, seq, batch in PRESETS[a.preset]:
        for lr in lrs:
            for runner in runners:
                for rep in range(1, a.repeats + 1):
                    tok, sec = run_once(runner, name, corpora[corpus], seq, batch, lr, rep, a, out_dir, extra)
                    with open(csv_path, "a", newline="") as f:
                        f.write(f"{runner},{name},{normalize_lr(lr)},{rep},{tok},{sec}\n")
                    print(f"[run] {runner:<12} {name:<16} lr={normalize_lr(lr):<8} r{rep} tok/s={tok:<8} sec={sec}",
                          flush=True)
    scored, winner = summarize(csv_path)
    if not scored:
        print("no successful runs", file=sys.stderr)
        return 1
    print_summary(scored, winner, csv_path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
