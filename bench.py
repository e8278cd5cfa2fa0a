"""Headline benchmark: decode tokens/s of the Llama-3.1-70B architecture with int8 weights at TP = --gpus,
plus p50 TTFT, on synthetic random-token prompts with random-init weights.

    python bench.py --gpus N --steps K --warmup W          # this framework (one process per GPU via torchrun)
    python bench.py --impl reference --gpus N ...          # the reference's torch.distributed NCCL TP build

Config (the headline benchmark workload): 80 layers, hidden 8192, 64 q / 8 kv heads (head_dim 128), FFN 28672,
vocab 128256, llama3 RoPE; batch 16 sequences, each prefilled with 4096 random tokens, then decode.  A "step" is one decode step
of the whole batch (16 new tokens).  W untimed warm-up steps, then exactly K steps timed with CUDA events between
barriers + synchronizes; the per-rank times are reduced with MAX.  Weights (70 GB int8 at TP=1) are far larger than
L2 (126 MB), so every step streams them from HBM ("inputs larger than L2").
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "decode tok/s (70B int8, TP=1/2/4/8, max over ranks); p50 TTFT"
BASELINE_PUBLISHED = None   # the reference publishes no number for this metric


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--ctx", type=int, default=4096, help="prompt tokens prefilled per sequence")
    ap.add_argument("--model", default="llama3.1-70b")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=0, help="debug only: override layer count (invalid as a bench)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--baseline-comm", action="store_true",
                    help="NCCL all-reduce after the row-parallel GEMMs instead of the fused in-kernel all-reduce")
    ap.add_argument("--chain", action="store_true",
                    help="decode: o_proj, gate/up, down and the next QKV as one multi-phase GEMM launch")
    ap.add_argument("--embed-vocab-parallel", action="store_true",
                    help="TP: vocab-sharded embedding + all-reduce (the reference's layout) instead of the table on "
                         "every rank")
    ap.add_argument("--prefill-overlap", type=int, default=1,
                    help="TP prefill: pipeline each row-parallel GEMM with its all-reduce over N row chunks")
    return ap.parse_args()


def _dist_setup(n):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}: launch N>1 with torchrun")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def _prompts(batch, ctx, vocab, seed=1):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (ctx,), generator=g).tolist() for _ in range(batch)]


def _log(rank, msg):
    if rank == 0:
        print(f"[bench {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def _emit(rank, rec):
    if rank == 0:
        print(json.dumps(rec), flush=True)


def _teardown(world, eng, state, model):
    """Release the decode graphs (they hold NCCL calls) before the process group goes away.  The result line is
    already printed, so a teardown that still stalls is cut short by a watchdog instead of holding the GPUs."""
    import gc
    import threading
    sys.stdout.flush()
    sys.stderr.flush()
    wd = threading.Timer(60.0, lambda: os._exit(0))
    wd.daemon = True
    wd.start()
    eng.release_graphs()
    del state, eng
    if getattr(model, "symm", None) is not None:
        model.symm = None          # IPC mappings are closed by process exit
    gc.collect()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    wd.cancel()


# ====================================================================================================== ours
def run_ours(a):
    from hrm_flashrenderer_b200.config import get_preset, EngineConfig
    from hrm_flashrenderer_b200.models.llama import LlamaW8
    from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
    from hrm_flashrenderer_b200.parallel.comm import TPComm
    from hrm_flashrenderer_b200.utils.clocks import ClockSampler, visible_gpu_indices
    from hrm_flashrenderer_b200 import ops

    rank, world, local = _dist_setup(a.gpus)
    cfg = get_preset(a.model)
    if a.layers:
        cfg = cfg.with_layers(a.layers)
    dev = torch.device("cuda", local)
    comm = TPComm() if world > 1 else None
    t0 = time.time()
    model = LlamaW8.synthesize(cfg, rank=rank, world=world, device=dev, seed=0, comm=comm,
                               max_pos=a.ctx + a.steps + a.warmup + 256,
                               replicate_embedding=not a.embed_vocab_parallel)
    fused = world > 1 and not a.baseline_comm
    if fused:
        model.enable_fused_collectives()   # row-parallel GEMMs reduce over NVLink peer memory inside the kernel
    torch.cuda.synchronize()
    t_synth = time.time() - t0
    _log(rank, f"synthesized {cfg.name} shard in {t_synth:.1f}s ({model.weight_bytes() / 1e9:.1f} GB int8)")
    total_len = a.ctx + a.steps + a.warmup + 2 * 16 + (a.steps + 8 if not a.no_e2e else 0)
    ecfg = EngineConfig(tp=world, max_seq_len=total_len + 16, max_batch=a.batch, prefill_chunk=4096,
                        graph_batch_buckets=(a.batch,), chain_layers=bool(a.chain),
                        prefill_overlap_chunks=int(a.prefill_overlap))
    eng = InferenceEngine(model, ecfg, num_blocks=a.batch * ((total_len + 15) // 16 + 1))
    prompts = _prompts(a.batch, a.ctx, cfg.vocab)
    sids = [eng.new_seq() for _ in prompts]

    # ---- prefill: every request arrives at t=0; TTFT of request i = device time until its first token
    _barrier(world)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    ttft_ms, first = [], []
    for sid, p in zip(sids, prompts):
        first += eng.prefill([(sid, p)])
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        e.synchronize()
        ttft_ms.append(ev0.elapsed_time(e))
        _log(rank, f"prefilled seq {sid}: first token at {ttft_ms[-1]:.0f} ms")
    ops.check_status(dev)
    ttft_p50 = _max_over_ranks(statistics.median(ttft_ms), world)
    # the same prefill seen two more ways: one prompt alone (the first request's TTFT) and the whole batch (the time
    # at which the reference's batched prefill, which emits every first token together, would finish)
    ttft_first = _max_over_ranks(ttft_ms[0], world)
    prefill_all = _max_over_ranks(ttft_ms[-1], world)

    # ---- decode (device-timed; one CUDA graph replay per step)
    g = eng.load_decode_batch(sids, first, reserve=a.warmup + a.steps + 8)
    eng.capture(g.bucket)
    _log(rank, "decode graph captured")
    for _ in range(a.warmup):
        eng.decode_step(g)
    torch.cuda.synchronize()
    ops.check_status(dev)
    _log(rank, "warm-up done")
    _barrier(world)
    sampler = ClockSampler(visible_gpu_indices(world)).start() if rank == 0 else None
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(a.steps):
        eng.decode_step(g)
    e_ev.record()
    _barrier(world)
    clocks = sampler.stop() if sampler else None
    ms = _max_over_ranks(s_ev.elapsed_time(e_ev), world)
    ms_per_step = ms / a.steps
    value = a.batch * a.steps / (ms / 1e3)

    # ---- end-to-end through the serving step API: H2D step inputs from pinned memory, D2H sampled tokens
    e2e = None
    if not a.no_e2e:
        host_ids = torch.empty(g.bucket, dtype=torch.int64, pin_memory=True)
        host_out = torch.empty(g.bucket, dtype=torch.int64, pin_memory=True)
        host_ids.copy_(g.tokens)
        for _ in range(2):
            eng.step_host(g, host_ids, host_out)
            host_ids.copy_(host_out)
        _barrier(world)
        t1 = time.perf_counter()
        for _ in range(a.steps):
            eng.step_host(g, host_ids, host_out)
            host_ids.copy_(host_out)
        _barrier(world)
        e2e_s = _max_over_ranks(time.perf_counter() - t1, world)
        e2e = {"value": a.batch * a.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": host_ids.numel() * 8,
               "d2h_bytes_per_step": host_out.numel() * 8,
               "api": "InferenceEngine.step_host (pinned ids H2D, graph step, tokens D2H + sync)"}

    # launches per decode step (our kernels only), counted by the op layer over one eager step
    ops.LAUNCH_COUNTER.reset()
    ops.LAUNCH_COUNTER.enabled = True
    eng._decode_body(g)
    ops.LAUNCH_COUNTER.enabled = False
    launches = ops.LAUNCH_COUNTER.count * a.steps
    torch.cuda.synchronize()

    rec = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None if BASELINE_PUBLISHED is None else value / BASELINE_PUBLISHED,
        "dtype": "int8 weights (per-channel), f16 GEMM operands, fp32 accumulate/residual, bf16 KV",
        "data": "synthetic random-token prompts, random-init N(0,0.02) int8 weights",
        "config": {"model": cfg.name, "global_batch": a.batch, "seq_len": a.ctx, "parallelism": f"tp{world}",
                   "decode_context": f"{a.ctx}..{a.ctx + a.warmup + a.steps}", "l2": "inputs larger than L2",
                   "comm": ("fused GEMM+all-reduce over peer memory" if fused else "nccl") if world > 1 else "none",
                   "embedding": ("replicated" if model.embed_replicated else "vocab-parallel") if world > 1
                   else "full"},
        "p50_ttft_ms": round(ttft_p50, 2), "ttft_first_ms": round(ttft_first, 2),
        "prefill_all_ms": round(prefill_all, 2), "impl": "ours", "gpu_launches": launches,
        "clocks": clocks, "e2e": e2e, "synth_s": round(t_synth, 1),
    }
    if a.layers:
        rec["invalid"] = f"layers overridden to {a.layers} (debug run)"
    _emit(rank, rec)
    _teardown(world, eng, g, model)


# ====================================================================================================== reference
def _block_reference_extension() -> None:
    """Make ``from . import _ext`` inside the reference's ``flashattention_custom`` raise ImportError (a ``None``
    entry in ``sys.modules``), whether or not a build of the extension is present, so its ops take their own
    PyTorch fallbacks."""
    sys.modules["flashattention_custom._ext"] = None


def run_reference(a):
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "engine")):
        _emit(int(os.environ.get("RANK", "0")), {"impl": "reference", "unavailable": "baseline/_ref not installed"})
        return
    sys.path.insert(0, ref_root)
    rank, world, local = _dist_setup(a.gpus)
    if world == 1 and not dist.is_initialized():
        import datetime
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29600 + local))
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    from types import SimpleNamespace
    # The reference's compiled attention extension is never loaded: its D=128 kernel stores WMMA accumulators into
    # a per-thread local array (csrc/flash_attn_sm75.cu:310-311, :390-391).  wmma.store is defined only for global
    # or shared addresses, and the sm_100 build raised "unspecified launch failure" on the driver's B200s at every
    # N.  A None entry in sys.modules makes `from . import _ext` raise ImportError, so flashattention_custom.ops
    # takes its own PyTorch fallbacks (ops.py:19-72): the reference as `pip install` builds it on a host without
    # the extension.
    _block_reference_extension()
    import flashattention_custom.ops as fops
    if getattr(fops, "_HAS_EXT", False):
        _emit(rank, {"impl": "reference", "unavailable": "refusing to run the reference's sm75 attention extension "
                     "(faulted on B200: unspecified launch failure)"})
        if world > 1:
            dist.destroy_process_group()
        return
    from engine.llama_tp import TPLlamaForCausalLM, greedy_select_token_distributed
    from hrm_flashrenderer_b200.utils.clocks import ClockSampler, visible_gpu_indices
    from hrm_flashrenderer_b200.config import get_preset

    c = get_preset(a.model)
    if a.layers:
        c = c.with_layers(a.layers)
    hf = SimpleNamespace(vocab_size=c.vocab, hidden_size=c.hidden, num_attention_heads=c.heads,
                         num_key_value_heads=c.kv_heads, num_hidden_layers=c.layers, intermediate_size=c.intermediate,
                         rms_norm_eps=c.rms_eps, rope_theta=c.rope_theta)
    max_seq = a.ctx + a.warmup + a.steps + 16
    try:
        torch.manual_seed(0)
        with torch.no_grad():
            model = TPLlamaForCausalLM(hf, max_seq_len=max_seq, device="cuda")
        model.eval()
        prompts = torch.tensor(_prompts(a.batch, a.ctx, c.vocab), dtype=torch.long, device="cuda")
        B, T0 = prompts.shape
        chunk = 1024
        init_pages = max(4, (T0 + a.warmup + a.steps + 127) // 128)
        with torch.no_grad():
            model.reset_all_caches()
            _barrier(world)
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            cur, last = 0, None
            while cur < T0:   # generate_tp's chunked prefill (engine/llama_tp.py:347-354)
                end = min(T0, cur + chunk)
                pos = torch.arange(cur, end, device="cuda", dtype=torch.long)
                h = model(prompts[:, cur:end], pos, prefill=True, init_pages=init_pages, page_size=128)
                last = h[:, -1, :]
                cur = end
            nxt = greedy_select_token_distributed(model.logits_last(last))
            ev1.record()
            ev1.synchronize()
            ttft = _max_over_ranks(ev0.elapsed_time(ev1), world)

            def step(nxt, cur):   # generate_tp's decode loop body (engine/llama_tp.py:366-380)
                pos = torch.tensor([cur], device="cuda", dtype=torch.long)
                h1 = model(nxt.view(B, 1), pos, prefill=False, init_pages=init_pages, page_size=128)
                return greedy_select_token_distributed(model.logits_last(h1[:, -1, :]))

            for _ in range(a.warmup):
                nxt = step(nxt, cur)
                cur += 1
            _barrier(world)
            sampler = ClockSampler(visible_gpu_indices(world)).start() if rank == 0 else None
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            t_wall = time.perf_counter()
            for _ in range(a.steps):
                nxt = step(nxt, cur)
                cur += 1
            e_ev.record()
            _barrier(world)
            wall = _max_over_ranks(time.perf_counter() - t_wall, world)
            clocks = sampler.stop() if sampler else None
            ms = _max_over_ranks(s_ev.elapsed_time(e_ev), world)
    except torch.OutOfMemoryError as e:
        _emit(rank, {"impl": "reference", "unavailable": f"out of memory: fp16 weights + KV exceed the GPU ({e})"[:300]})
        if world > 1:
            dist.destroy_process_group()
        return
    except Exception as e:   # the reference's own code failed: report it instead of a traceback-only exit
        _emit(rank, {"impl": "reference",
                     "unavailable": f"reference run failed: {type(e).__name__}: {e}".replace("\n", " ")[:300]})
        if world > 1:
            dist.destroy_process_group()
        return
    value = a.batch * a.steps / (ms / 1e3)
    rec = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp16 (reference TP path has fp16 weights)",
        "data": "synthetic random-token prompts, random-init weights (reference __init__ N(0,0.02))",
        "config": {"model": c.name, "global_batch": a.batch, "seq_len": a.ctx, "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2", "attention_ext": bool(getattr(fops, "_HAS_EXT", False)),
                   "attention": "reference PyTorch fallback (ops.py); its CUDA extension is not run on B200"},
        "p50_ttft_ms": round(ttft, 2), "impl": "reference", "clocks": clocks,
        "e2e": {"value": a.batch * a.steps / wall, "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 8 * a.batch, "api": "reference decode loop (host syncs inside)"},
    }
    if a.layers:
        rec["invalid"] = f"layers overridden to {a.layers} (debug run)"
    _emit(rank, rec)
    if world > 1:
        dist.destroy_process_group()


def main():
    a = _args()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
