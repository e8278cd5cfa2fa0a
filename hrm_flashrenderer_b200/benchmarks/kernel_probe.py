"""Run ONE hand-written kernel at one Llama-3.1-70B shape a few times (one GPU): the small, self-ending case that a
profiler capture wraps.

    python -m hrm_flashrenderer_b200.benchmarks.kernel_probe --op NAME [--reps 3] [--time]

Each op builds its inputs once, runs ``--reps`` launches of the kernel, synchronizes and checks the bounded-wait
status word; the printed line gives the op, its shape and the algorithmic bytes / FLOPs of one launch, so a
profiler's per-launch DRAM bytes and duration can be set against them.  Ops (kernel in parentheses):

* ``gemm_prefill``  gate/up + SwiGLU at M = 4096 tokens, TP = 1 (w8a16_gemm_kernel<256, 3>)
* ``gemm_decode_tp8`` o_proj shard at TP = 8, 16 tokens, fp32 out (w8a16_gemm_kernel<16, 1>)
* ``attn_prefill``  paged causal prefill attention, 4096 tokens, 64 q / 8 kv heads (attn_prefill_tc_kernel)
* ``attn_decode_tp8`` decode attention at TP = 8: 16 sequences x 4096 keys, 8 q / 1 kv head (attn_decode_tc_kernel,
  decode_combine_kernel)
* ``norm_prep``     RMSNorm inputs of 16 tokens (norm_prep_kernel)
* ``embed``         int8 embedding lookup of 16 tokens (embed_q8_kernel)
* ``argmax``        split greedy pick over 16 x 128256 logits (argmax_kernel)
* ``topk_threshold`` k-th largest of 16 x 128256 logits, k = 50 (kth_largest_kernel)
* ``sample``        sampled pick (temperature 0.8, top-50 threshold) over 16 x 128256 logits (argmax_kernel<0, 1>)
* ``flash_train_fwd`` / ``flash_train_bwd``  the trainer's causal attention at 128 sequences x 512 tokens, 8 heads of
  16 (flash_train_fwd_kernel; flash_train_dq_kernel + flash_train_dkv_kernel).  FLOPs are the executed multiply-adds
  x 2: 4 D per visible (query, key) pair forward, 14 D backward (S and dP are computed in both passes).
"""
from __future__ import annotations

import argparse
import json

import torch

from .. import ops
from ..config import LLAMA31_70B


def _gemm_prefill(dev):
    c = LLAMA31_70B
    M, F, K = 4096, c.intermediate, c.hidden
    g = torch.Generator(device=dev).manual_seed(0)
    gate = torch.randint(-127, 128, (F, K), generator=g, device=dev, dtype=torch.int8)
    up = torch.randint(-127, 128, (F, K), generator=g, device=dev, dtype=torch.int8)
    s = torch.rand(F, generator=g, device=dev) * 1e-4
    w, sc = ops.interleave_gate_up(gate, up, s, s)
    w = ops.tile_w8(w)
    del gate, up
    x = torch.randn(M, K, device=dev).half()
    run = lambda: ops.w8a16_swiglu(x, w, sc)
    return run, f"M{M}xN{2 * F}xK{K}", 2 * F * K + 2 * M * K + 2 * M * F, 2.0 * M * 2 * F * K


def _gemm_decode_tp8(dev):
    M, N, K = 16, LLAMA31_70B.hidden, LLAMA31_70B.q_dim // 8
    w = ops.tile_w8(torch.randint(-127, 128, (N, K), device=dev, dtype=torch.int8))
    s = torch.rand(N, device=dev) * 1e-4
    x = torch.randn(M, K, device=dev).half()
    out = torch.empty(M, N, device=dev)
    run = lambda: ops.w8a16_linear_out(x, w, s, out)
    return run, f"M{M}xN{N}xK{K}", N * K + 2 * M * K + 4 * M * N, 2.0 * M * N * K


def _attn_prefill(dev):
    c = LLAMA31_70B
    T, Hq, Hk, D = 4096, c.heads, c.kv_heads, c.head_dim
    nb = T // 16 + 8
    kc = torch.randn(nb, Hk, 16, D, device=dev, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    tab = torch.arange(T // 16, device=dev, dtype=torch.int32).view(1, -1)
    q = torch.randn(T, Hq, D, device=dev, dtype=torch.bfloat16)
    cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
    qs = torch.zeros(1, dtype=torch.int32, device=dev)
    cl = torch.tensor([T], dtype=torch.int32, device=dev)
    out = torch.empty(T, Hq, D, device=dev, dtype=torch.float16)
    run = lambda: ops.paged_prefill_attention(q, kc, vc, tab, cu, qs, cl, T, out=out)
    return run, f"T{T}xHq{Hq}xHk{Hk}", 2 * T * Hq * D * 2 + 2 * T * Hk * D * 2, 4.0 * Hq * D * T * T / 2


def _attn_decode_tp8(dev):
    c = LLAMA31_70B
    B, L, Hq, Hk, D = 16, 4096, c.heads // 8, c.kv_heads // 8, c.head_dim
    nb = B * (L // 16) + 8
    kc = torch.randn(nb, Hk, 16, D, device=dev, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    tab = torch.arange(B * (L // 16), device=dev, dtype=torch.int32).view(B, L // 16)
    cl = torch.full((B,), L, dtype=torch.int32, device=dev)
    q = torch.randn(B, Hq, D, device=dev, dtype=torch.bfloat16)
    out = torch.empty(B, Hq, D, device=dev, dtype=torch.float16)
    run = lambda: ops.paged_decode_attention(q, kc, vc, tab, cl, out=out, max_ctx=L)
    return run, f"B{B}xL{L}xHq{Hq}xHk{Hk}", 2 * B * L * Hk * D * 2, 4.0 * B * Hq * L * D


def _norm_prep(dev):
    M, H = 16, LLAMA31_70B.hidden
    x = torch.randn(M, H, device=dev)
    g = torch.ones(H, device=dev)
    xg = torch.empty(M, H, device=dev, dtype=torch.float16)
    ssq = torch.empty(H // 128, M, device=dev)
    run = lambda: ops.norm_prep(x, None, g, xg, ssq)
    return run, f"M{M}xH{H}", M * H * (4 + 4 + 2), 0.0


def _embed(dev):
    V, H = LLAMA31_70B.vocab, LLAMA31_70B.hidden
    q = torch.randint(-127, 128, (V, H), device=dev, dtype=torch.int8)
    s = torch.rand(V, device=dev) * 1e-3
    ids = torch.randint(0, V, (16,), device=dev)
    run = lambda: ops.embedding_q8(ids, q, s, 0)
    return run, f"M16xH{H}", 16 * H * (1 + 4), 0.0


def _argmax(dev):
    logits = torch.randn(16, LLAMA31_70B.vocab, device=dev)
    run = lambda: ops.argmax_rows(logits, 0)
    return run, f"M16xV{LLAMA31_70B.vocab}", logits.numel() * 4, 0.0


def _topk_threshold(dev):
    logits = torch.randn(16, LLAMA31_70B.vocab, device=dev)
    k = torch.full((16,), 50, dtype=torch.int32, device=dev)
    run = lambda: ops.kth_largest(logits, k)
    return run, f"M16xV{LLAMA31_70B.vocab}", logits.numel() * 4 * 4, 0.0   # four radix passes over the row


def _sample(dev):
    logits = torch.randn(16, LLAMA31_70B.vocab, device=dev)
    thr = ops.kth_largest(logits, torch.full((16,), 50, dtype=torch.int32, device=dev))
    it = torch.full((16,), 1 / 0.8, device=dev)
    seed = torch.arange(16, dtype=torch.int64, device=dev)
    pos = torch.full((16,), 100, dtype=torch.int32, device=dev)
    run = lambda: ops.sample_rows(logits, 0, it, seed, pos, thr)
    return run, f"M16xV{LLAMA31_70B.vocab}", logits.numel() * 4, 0.0


def _flash_train(dev, backward: bool):
    B, T, H, D = 128, 512, 8, 16
    g = torch.Generator(device=dev).manual_seed(0)
    q, k, v, do = (torch.randn(B, T, H, D, generator=g, device=dev) for _ in range(4))
    o, lse = ops.flash_train_fwd(q, k, v)
    pairs = B * H * T * (T + 1) // 2
    row = B * T * H * D * 4
    if backward:
        run = lambda: ops.flash_train_bwd(q, k, v, o, lse, do)
        return run, f"B{B}xT{T}xH{H}xD{D}", 8 * row + B * H * T * 4, 14.0 * D * pairs
    run = lambda: ops.flash_train_fwd(q, k, v)
    return run, f"B{B}xT{T}xH{H}xD{D}", 4 * row + B * H * T * 4, 4.0 * D * pairs


OPS = {"gemm_prefill": _gemm_prefill, "gemm_decode_tp8": _gemm_decode_tp8, "attn_prefill": _attn_prefill,
       "attn_decode_tp8": _attn_decode_tp8, "norm_prep": _norm_prep, "embed": _embed, "argmax": _argmax,
       "topk_threshold": _topk_threshold, "sample": _sample,
       "flash_train_fwd": lambda dev: _flash_train(dev, False), "flash_train_bwd": lambda dev: _flash_train(dev, True)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-kernel-probe")
    ap.add_argument("--op", required=True, choices=sorted(OPS))
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--time", action="store_true",
                    help="after 3 warm-up calls, time --reps calls with CUDA events and print us per call")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    run, shape, nbytes, flops = OPS[a.op](dev)
    torch.cuda.synchronize()
    rec = {"op": a.op, "shape": shape, "bytes_per_launch": nbytes, "flops_per_launch": flops, "reps": a.reps}
    if a.time:
        for _ in range(3):
            run()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record()
        for _ in range(a.reps):
            run()
        t1.record()
        torch.cuda.synchronize()
        us = t0.elapsed_time(t1) * 1e3 / a.reps
        rec.update(us_per_call=round(us, 2), gbs=round(nbytes / us / 1e3, 1), tflops=round(flops / us / 1e6, 2))
    else:
        for _ in range(a.reps):
            run()
        torch.cuda.synchronize()
    ops.check_status(dev)
    print(json.dumps(rec), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
