"""Per-op device timing of the hot kernels at Llama-3.1-70B shapes (one GPU), with roofline fractions.

    python -m hrm_flashrenderer_b200.benchmarks.ops_sweep [--tp 1] [--m 1,16,64,512,4096] [--json out.json]

Each op runs `--iters` times between CUDA events after `--warmup` runs; between timed iterations a 256 MB buffer is
rewritten to flush the L2 (126 MB), and the flush is excluded from the timing by timing each iteration separately.
Roofline denominators come from MEASURED_PEAKS.json at the repo root (hbm_gbs, bf16_tflops) when present, else the
pool's fallback (6650 GB/s, 1590 TFLOP/s).  GEMM roofline = max(bytes/HBM, flops/peak); bytes = int8 weights +
f16 activations in + outputs.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from .. import ops
from ..config import LLAMA31_70B
from ..models.weights import quantize_rows

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def time_op(fn, iters=10, warmup=3, flush=None):
    for _ in range(warmup):
        fn()
    ts = []
    for _ in range(iters):
        if flush is not None:
            flush.add_(1)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e) * 1e3)
    ts.sort()
    return ts[len(ts) // 2]


def gemm_shapes(tp: int):
    c = LLAMA31_70B
    return {
        "qkv": ((c.q_dim + 2 * c.kv_dim) // tp, c.hidden),
        "o_proj": (c.hidden, c.q_dim // tp),
        "gate_up": (2 * c.intermediate // tp, c.hidden),
        "down": (c.hidden, c.intermediate // tp),
        "lm_head": (c.vocab // tp, c.hidden),
    }


def main(argv=None):
    ap = argparse.ArgumentParser(prog="hrm-flash-ops-sweep")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--m", default="1,16,64,512,4096")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--json", default="")
    ap.add_argument("--ops", default="gemm,attn,norm")
    ap.add_argument("--attn-b", default="1,16,64", help="decode-attention batch sizes (context 4096)")
    ap.add_argument("--gemm-order", default="n",
                    help="output-tile numbering(s) to time: n (n-fastest, default), m (m-fastest), or n,m")
    a = ap.parse_args(argv)
    hbm, tfl, src = peaks()
    dev = torch.device("cuda")
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    rows = []

    def rec(name, shape, us, bytes_, flops):
        t_bw = bytes_ / (hbm * 1e9) * 1e6
        t_fl = flops / (tfl * 1e12) * 1e6
        roof = max(t_bw, t_fl)
        r = dict(op=name, shape=shape, us=round(us, 2), gbs=round(bytes_ / us / 1e3, 1),
                 tflops=round(flops / us / 1e6, 1), roofline_us=round(roof, 2),
                 frac_of_roofline=round(roof / us, 3), bound="hbm" if t_bw >= t_fl else "tensor", peaks=src)
        rows.append(r)
        print(json.dumps(r), flush=True)

    Ms = [int(x) for x in a.m.split(",")]
    if "gemm" in a.ops:
        for name, (N, K) in gemm_shapes(a.tp).items():
            g = torch.Generator(device=dev).manual_seed(0)
            qt = quantize_rows(torch.randn(N, K, generator=g, device=dev) * 0.02)
            wt = ops.tile_w8(qt.q)   # the engine's weight layout (bulk-copy path)
            for M in Ms:
                x = torch.randn(M, K, device=dev, dtype=torch.float16)
                out = torch.empty(M, N, device=dev, dtype=torch.float16)
                for order in a.gemm_order.split(","):
                    ops.ext().set_gemm_m_fastest(order == "m")
                    try:
                        us = time_op(lambda: ops.w8a16_linear_out(x, wt, qt.scale, out), a.iters, a.warmup, flush)
                    finally:
                        ops.ext().set_gemm_m_fastest(False)
                    tag = "" if order == "n" else "/m-fastest"
                    rec(f"w8a16_gemm/{name}{tag}", f"M{M}xN{N}xK{K}", us, N * K + 2 * M * K + 2 * M * N,
                        2.0 * M * N * K)
            del qt, wt
    if "attn" in a.ops:
        c = LLAMA31_70B
        Hq, Hk, D = c.heads // a.tp, max(1, c.kv_heads // a.tp), c.head_dim
        for B, L in ((int(x), 4096) for x in a.attn_b.split(",") if x):
            nb = B * (L // 16) + 8
            kc = torch.randn(nb, Hk, 16, D, device=dev, dtype=torch.bfloat16)
            vc = torch.randn_like(kc)
            cl = torch.full((B,), L, dtype=torch.int32, device=dev)
            q = torch.randn(B, Hq, D, device=dev, dtype=torch.bfloat16)
            out = torch.empty(B, Hq, D, device=dev, dtype=torch.float16)
            # scattered block ids: one 4 KB TMA box per block; in-order ids: one box per 8 blocks (128 keys)
            for layout, ids in (("scattered", torch.randperm(nb - 8, device=dev)),
                                ("contiguous", torch.arange(nb - 8, device=dev))):
                tab = ids[:B * (L // 16)].view(B, L // 16).to(torch.int32)
                us = time_op(lambda: ops.paged_decode_attention(q, kc, vc, tab, cl, out=out, max_ctx=L), a.iters,
                             a.warmup, flush)
                rec("attn_decode", f"B{B}xL{L}xHq{Hq}xHk{Hk}/{layout}", us, 2 * B * L * Hk * D * 2,
                    4.0 * B * Hq * L * D)
            del kc, vc
        for T in (512, 4096):
            nb = T // 16 + 8
            kc = torch.randn(nb, Hk, 16, D, device=dev, dtype=torch.bfloat16)
            vc = torch.randn_like(kc)
            tab = torch.arange(T // 16, device=dev, dtype=torch.int32).view(1, -1)
            q = torch.randn(T, Hq, D, device=dev, dtype=torch.bfloat16)
            cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
            qs = torch.zeros(1, dtype=torch.int32, device=dev)
            cl = torch.tensor([T], dtype=torch.int32, device=dev)
            out = torch.empty(T, Hq, D, device=dev, dtype=torch.float16)
            us = time_op(lambda: ops.paged_prefill_attention(q, kc, vc, tab, cu, qs, cl, T, out=out), a.iters,
                         a.warmup, flush)
            rec("attn_prefill", f"T{T}xHq{Hq}xHk{Hk}", us, 2 * T * Hq * D * 2 + 2 * T * Hk * D * 2,
                4.0 * Hq * D * T * T / 2)
    if "norm" in a.ops:
        H = LLAMA31_70B.hidden
        w = torch.ones(H, device=dev)
        for M in (16, 4096):
            x = torch.randn(M, H, device=dev)
            h = torch.empty(M, H, device=dev, dtype=torch.float16)
            us = time_op(lambda: ops.rmsnorm(x, w, 1e-5, out=h), a.iters, a.warmup, flush)
            rec("rmsnorm", f"M{M}xH{H}", us, M * H * 6, 0.0)
    if a.json:
        json.dump(rows, open(a.json, "w"), indent=1)


if __name__ == "__main__":
    main()
