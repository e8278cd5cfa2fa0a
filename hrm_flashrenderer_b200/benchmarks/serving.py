"""Serving benchmarks.

1. ``grid`` -- the reference benchmark harness (``scripts/benchmark_deepseek.sh:54-370``): scenario {short, medium,
   long} x mode x route_hint x repeats (after warm-up) through a router's ``/v1/generate``; per row the client wall
   latency, output tokens (tokenizer or chars/4) and tok/s; summary per (scenario, mode, route_hint): mean / p50 /
   p95 / min / max latency, mean tok/s, majority selected lane, score = tok/s / p95.  Writes raw.csv, summary.csv,
   summary.txt.
2. ``trace`` -- the continuous-batching serving workload: a Poisson arrival trace (N requests at R req/s, seed 0) of mixed-mode prompts =
   random-token system prefix (256) + retrieved-context block (3 chunks x 256 random tokens) + user part (uniform
   64..1024), outputs uniform 64..512 tokens, greedy; run in-process against the continuous-batching scheduler
   (token ids, no tokenizer), reporting p50 / p99 TTFT and aggregate generated tok/s.
"""
import argparse
import csv
import dataclasses
import json
import math
import random
import statistics
import time
import urllib.request
from collections import Counter, defaultdict
from pathlib import Path
from typing import Dict, List

SCENARIOS = {
    "short": ("Give one sentence about the silver bridge.", 64),
    "medium": ("Summarise in a few sentences what the merchants promised the king and why the tower is dark "
               "in winter; mention the river stone.", 192),
    "long": ("Write a detailed multi-paragraph explanation covering the bridge, the guards, the merchants, the king, "
             "the winter tower and the river stone, with background for each. " * 3, 512),
}


def _post(url: str, payload: Dict, timeout: float = 600.0) -> Dict:
    req = urllib.request.Request(url, data=json.dumps(payload).encode(), method="POST",
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.loads(r.read().decode())


def _pct(xs: List[float], q: float) -> float:
    xs = sorted(xs)
    if not xs:
        return float("nan")
    k = (len(xs) - 1) * q
    lo, hi = math.floor(k), math.ceil(k)
    return xs[lo] + (xs[hi] - xs[lo]) * (k - lo)


def run_grid(router_url: str, out_dir: Path, modes=("mixed", "retrieval", "deepseek_only"), route_hints=("auto",),
             scenarios=("short", "medium", "long"), repeats: int = 3, warmup: int = 1, tokenizer=None) -> List[Dict]:
    out_dir.mkdir(parents=True, exist_ok=True)
    rows = []
    count = (lambda t: len(tokenizer(t, add_special_tokens=False)["input_ids"])) if tokenizer else \
        (lambda t: max(1, len(t) // 4))
    for sc in scenarios:
        prompt, max_new = SCENARIOS[sc]
        for mode in modes:
            for rh in route_hints:
                payload = {"prompt": prompt, "mode": mode, "max_new_tokens": max_new, "allow_failover": True}
                if rh != "auto":
                    payload["route_hint"] = rh
                for i in range(warmup + repeats):
                    t0 = time.perf_counter()
                    r = _post(router_url.rstrip("/") + "/v1/generate", payload)
                    dt = time.perf_counter() - t0
                    if i < warmup:
                        continue
                    ntok = count(str(r.get("text", "")))
                    rows.append({"scenario": sc, "mode": mode, "route_hint": rh, "run": i - warmup,
                                 "latency_s": round(dt, 4), "out_tokens": ntok, "tok_s": round(ntok / dt, 2),
                                 "selected": (r.get("route") or {}).get("selected", ""),
                                 "source_count": r.get("source_count", 0)})
    with open(out_dir / "raw.csv", "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=list(rows[0].keys()))
        w.writeheader()
        w.writerows(rows)
    groups = defaultdict(list)
    for r in rows:
        groups[(r["scenario"], r["mode"], r["route_hint"])].append(r)
    summary = []
    for (sc, mode, rh), rs in groups.items():
        lat = [r["latency_s"] for r in rs]
        p95 = _pct(lat, 0.95)
        tps = statistics.mean(r["tok_s"] for r in rs)
        summary.append({"scenario": sc, "mode": mode, "route_hint": rh, "n": len(rs),
                        "lat_mean_s": round(statistics.mean(lat), 4), "lat_p50_s": round(_pct(lat, 0.5), 4),
                        "lat_p95_s": round(p95, 4), "lat_min_s": round(min(lat), 4), "lat_max_s": round(max(lat), 4),
                        "tok_s_mean": round(tps, 2),
                        "route_majority": Counter(r["selected"] for r in rs).most_common(1)[0][0],
                        "score": round(tps / p95, 3) if p95 > 0 else 0.0})
    with open(out_dir / "summary.csv", "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=list(summary[0].keys()))
        w.writeheader()
        w.writerows(summary)
    (out_dir / "summary.txt").write_text("\n".join(
        f"{s['scenario']:>6} {s['mode']:>13} {s['route_hint']:>8}  p50={s['lat_p50_s']:.3f}s p95={s['lat_p95_s']:.3f}s "
        f"tok/s={s['tok_s_mean']:.1f} lane={s['route_majority']} score={s['score']}" for s in summary) + "\n")
    return summary


def make_trace(n: int = 512, rate: float = 4.0, vocab: int = 128256, seed: int = 0):
    """Config-5 trace: [(arrival_s, prompt_ids, max_new_tokens)] with exponential inter-arrival times."""
    rng = random.Random(seed)
    system = [rng.randrange(vocab) for _ in range(256)]
    t, out = 0.0, []
    for _ in range(n):
        t += rng.expovariate(rate)
        ctx = [rng.randrange(vocab) for _ in range(3 * 256)]
        user = [rng.randrange(vocab) for _ in range(rng.randint(64, 1024))]
        out.append((t, system + ctx + user, rng.randint(64, 512)))
    return out


def run_trace(scheduler, trace, time_scale: float = 1.0, sampling=None) -> Dict:
    """Replay ``trace`` against a started Scheduler; arrivals are honoured in wall time (scaled).  ``sampling``
    (``runtime.sampling.SamplingParams``) draws every request's tokens instead of the greedy pick; request ``i``
    gets seed ``sampling.seed + i``."""
    t0 = time.perf_counter()
    reqs = []
    for arr, ids, n in trace:
        wait = arr * time_scale - (time.perf_counter() - t0)
        if wait > 0:
            time.sleep(wait)
        sp = None if sampling is None else dataclasses.replace(sampling, seed=sampling.seed + len(reqs))
        reqs.append(scheduler.submit(ids, n, stop_on_eos=False, sampling=sp))
    for r in reqs:
        r.future.result()
    wall = time.perf_counter() - t0
    ttft = [r.ttft_s for r in reqs]
    gen = sum(len(r.tokens) for r in reqs)
    m = scheduler.metrics()
    return {"requests": len(reqs), "wall_s": round(wall, 3), "generated_tokens": gen,
            "tok_s": round(gen / wall, 2), "ttft_p50_ms": round(_pct(ttft, 0.5) * 1e3, 2),
            "ttft_p99_ms": round(_pct(ttft, 0.99) * 1e3, 2),
            "prompt_tokens": sum(len(ids) for _, ids, _ in trace),
            "prefilled_tokens": sum(scheduler.prefill_calls),
            "prefix_cache_hit_blocks": m.get("prefix_cache_hit_blocks", 0)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-bench-serving")
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("grid")
    g.add_argument("--router_url", default="http://127.0.0.1:8090")
    g.add_argument("--out_dir", default="bench_out")
    g.add_argument("--repeats", type=int, default=3)
    g.add_argument("--warmup", type=int, default=1)
    g.add_argument("--modes", default="mixed,retrieval,deepseek_only")
    g.add_argument("--route_hints", default="auto")
    t = sub.add_parser("trace")
    t.add_argument("--model", default="synthetic:llama3.1-70b")
    t.add_argument("--requests", type=int, default=512)
    t.add_argument("--rate", type=float, default=4.0)
    t.add_argument("--max_batch", type=int, default=64)
    t.add_argument("--max_seq_len", type=int, default=2560)
    t.add_argument("--device", default="cuda:0")
    t.add_argument("--prefix_cache", action="store_true", help="share the trace's common system-prompt blocks")
    t.add_argument("--temperature", type=float, default=0.0, help="sampled decoding (0: greedy)")
    t.add_argument("--top_k", type=int, default=0)
    a = ap.parse_args(argv)
    if a.cmd == "grid":
        s = run_grid(a.router_url, Path(a.out_dir), modes=a.modes.split(","), route_hints=a.route_hints.split(","),
                     repeats=a.repeats, warmup=a.warmup)
        print(json.dumps(s, indent=1))
        return 0
    from ..serving.backend import EngineBackend
    be = EngineBackend(a.model, device=a.device, max_seq_len=a.max_seq_len, max_batch=a.max_batch,
                       prefix_cache=a.prefix_cache)
    try:
        from ..runtime.sampling import SamplingParams
        sp = SamplingParams(a.temperature, a.top_k, 0) if a.temperature > 0 else None
        res = run_trace(be.scheduler, make_trace(a.requests, a.rate, be.engine.cfg.vocab), sampling=sp)
        print(json.dumps(res))
    finally:
        be.stop()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
