"""Kernel-by-kernel time of one decode step at a tensor-parallel size, max over ranks.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m hrm_flashrenderer_b200.benchmarks.decode_breakdown [--layers 2] [--batch 16] [--ctx 4096]

Builds the Llama-3.1-70B architecture (``--layers`` decoder layers at full width, random-init int8 weights) sharded
over the ranks, prefills ``--batch`` random prompts of ``--ctx`` tokens, then:

* ``graph``: the CUDA-graph-replayed decode step (what ``bench.py`` times), per step, max over ranks;
* ``eager``: the same step launched op by op with a CUDA event pair around every op of the operator layer; per op
  name the time summed over the step's calls, averaged over ``--steps`` steps, then the max over ranks.  Events
  between ops remove the programmatic-dependent-launch overlap of the graph, so the eager sum is an upper bound;
  the shares are what matter.

Per-layer figures are the step's figures divided by ``--layers``; the lm_head / argmax / bookkeeping rows are once
per step.  Rank 0 prints a Markdown table and, with ``--json``, writes the numbers.
"""
from __future__ import annotations

import argparse
import json
import os
import time
from collections import defaultdict

import torch
import torch.distributed as dist

from .. import ops

# operator-layer entry points timed individually (module attribute name -> label)
_TIMED = {
    "embedding_q8": "embed",
    "norm_prep": "norm_prep",
    "w8a16_qkv_rope_append": "qkv (+RoPE, KV append)",
    "paged_decode_attention": "decode attention (+combine)",
    "w8a16_residual_ar_": "row-parallel GEMM + peer all-reduce",
    "w8a16_residual_": "row-parallel GEMM + residual",
    "w8a16_swiglu": "gate/up + SwiGLU",
    "w8a16_linear": "lm_head",
    "w8a16_linear_out": "row-parallel GEMM (NCCL path)",
    "w8a16_chain": "chain (o_proj..next qkv)",
    "argmax_rows": "argmax",
    "argmax_exchange_": "argmax exchange (peer memory)",
    "decode_prepare": "decode_prepare",
    "decode_advance": "decode_advance",
}


class _OpTimer:
    def __init__(self):
        self.on = False
        self.events = []   # (label, start, end)

    def wrap(self, label, fn):
        def timed(*args, **kw):
            if not self.on:
                return fn(*args, **kw)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*args, **kw)
            e.record()
            self.events.append((label, s, e))
            return out
        return timed


def main(argv=None):
    ap = argparse.ArgumentParser(prog="hrm-flash-decode-breakdown")
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--model", default="llama3.1-70b")
    ap.add_argument("--baseline-comm", action="store_true", help="NCCL all-reduce instead of the fused kernels")
    ap.add_argument("--chain", action="store_true")
    ap.add_argument("--json", default="")
    a = ap.parse_args(argv)

    from ..config import get_preset, EngineConfig
    from ..models.llama import LlamaW8
    from ..runtime.engine import InferenceEngine
    from ..parallel.comm import TPComm
    from ..parallel.dist import init_dist_env

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        rank, local, world = init_dist_env("nccl")
    else:
        rank, local = 0, 0
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = get_preset(a.model).with_layers(a.layers)
    comm = TPComm() if world > 1 else None
    total = a.ctx + a.warmup + 2 * a.steps + 64
    model = LlamaW8.synthesize(cfg, rank=rank, world=world, device=dev, seed=0, comm=comm, max_pos=total + 64)
    if world > 1 and not a.baseline_comm:
        model.enable_fused_collectives()
    ecfg = EngineConfig(tp=world, max_seq_len=total + 16, max_batch=a.batch, prefill_chunk=4096,
                        graph_batch_buckets=(a.batch,), chain_layers=bool(a.chain))
    eng = InferenceEngine(model, ecfg, num_blocks=a.batch * ((total + 15) // 16 + 1))
    g0 = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab, (a.ctx,), generator=g0).tolist() for _ in range(a.batch)]
    sids = [eng.new_seq() for _ in prompts]
    first = []
    for sid, p in zip(sids, prompts):
        first += eng.prefill([(sid, p)])
    g = eng.load_decode_batch(sids, first, reserve=a.warmup + 2 * a.steps + 8)

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- graph-replayed step
    eng.capture(g.bucket)
    for _ in range(a.warmup):
        eng.decode_step(g)
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.steps):
        eng.decode_step(g)
    e.record()
    barrier()
    graph_us = max_over_ranks([s.elapsed_time(e) * 1e3 / a.steps])[0]
    ops.check_status(dev)

    # ---- eager step with an event pair around every operator-layer call
    timer = _OpTimer()
    saved = {}
    for name, label in _TIMED.items():
        fn = getattr(ops, name, None)
        if fn is not None:
            saved[name] = fn
            setattr(ops, name, timer.wrap(label, fn))
    comm_saved = {}
    if comm is not None:   # NCCL collectives issued by the model (argmax exchange, NCCL-path all-reduces)
        for name in ("all_reduce_", "all_reduce_max_"):
            comm_saved[name] = getattr(comm, name)
            setattr(comm, name, timer.wrap(f"NCCL {name.rstrip('_')}", comm_saved[name]))
    try:
        for _ in range(a.warmup):
            eng._decode_body(g)
        barrier()
        timer.on = True
        t0 = time.perf_counter()
        for _ in range(a.steps):
            eng._decode_body(g)
        barrier()
        timer.on = False
        host_s = time.perf_counter() - t0
    finally:
        for name, fn in saved.items():
            setattr(ops, name, fn)
        for name, fn in comm_saved.items():
            setattr(comm, name, fn)
    ops.check_status(dev)
    per = defaultdict(float)
    calls = defaultdict(int)
    for label, s_, e_ in timer.events:
        per[label] += s_.elapsed_time(e_) * 1e3 / a.steps
        calls[label] += 1
    labels = sorted(per)
    # every rank has the same labels (same code path); reduce in a fixed order
    mx = max_over_ranks([per[k] for k in labels])
    eager_sum = sum(mx)
    rows = [(k, calls[k] // a.steps, v) for k, v in zip(labels, mx)]
    rows.sort(key=lambda r: -r[2])
    if rank == 0:
        L = a.layers
        print(f"# decode step breakdown: {cfg.name} x{L} layers, TP={world}, batch {a.batch}, ctx {a.ctx}"
              f"{' (NCCL baseline)' if a.baseline_comm else ''}{' (chain)' if a.chain else ''}")
        print(f"graph-replayed step: {graph_us:.1f} us ({graph_us / L:.1f} us per layer incl. once-per-step ops); "
              f"eager sum of ops: {eager_sum:.1f} us; eager host time per step {host_s / a.steps * 1e6:.0f} us")
        print("| op | calls / step | us / step (max over ranks) | share |")
        print("|---|---|---|---|")
        for k, c, v in rows:
            print(f"| {k} | {c} | {v:.1f} | {v / eager_sum:.2f} |")
        if a.json:
            with open(a.json, "w") as f:
                json.dump({"model": cfg.name, "layers": a.layers, "tp": world, "batch": a.batch, "ctx": a.ctx,
                           "graph_us_per_step": graph_us, "eager_sum_us": eager_sum,
                           "ops": [{"op": k, "calls": c, "us": v} for k, c, v in rows]}, f, indent=1)
    eng.release_graphs()
    if world > 1:
        barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
