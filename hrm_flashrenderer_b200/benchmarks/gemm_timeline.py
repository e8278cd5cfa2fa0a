"""Per-CTA timeline of the W8A16 decode GEMM (one GPU): where a launch spends its time outside the weight stream.

    python -m hrm_flashrenderer_b200.benchmarks.gemm_timeline [--tp 1] [--m 16]

For each Llama-3.1-70B projection (sharded for ``--tp``) the GEMM runs right behind another GEMM of the same shape
on different (cold) weights, with programmatic dependent launch off and on.  The traced launch records, per CTA,
%globaltimer stamps (``_C.set_gemm_trace``): CTA start, first weight unit landed, last MMA complete, CTA end.
Printed per shape: min / median / max over CTAs of each stamp relative to the earliest CTA start (microseconds),
plus the weight bytes streamed per CTA-microsecond of mainloop.
"""
from __future__ import annotations

import argparse
import json

import torch

from .. import ops
from .ops_sweep import gemm_shapes


def timeline(N: int, K: int, M: int, pdl: bool, dev) -> dict:
    C = ops.ext()
    w = ops.tile_w8(torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev))
    w2 = ops.tile_w8(torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev))
    s = torch.rand(N, device=dev) * 1e-3
    x = torch.randn(M, K, device=dev).half()
    out = torch.empty(M, N, dtype=torch.float16, device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    tr = torch.zeros(16 * 1024, dtype=torch.int64, device=dev)
    C.set_pdl(pdl)
    try:
        for _ in range(3):
            ops.w8a16_linear_out(x, w, s, out)
        flush.add_(1)
        ops.w8a16_linear_out(x, w2, s, out)      # predecessor (cold weights)
        tr.zero_()
        C.set_gemm_trace(tr)
        ops.w8a16_linear_out(x, w, s, out)       # traced launch right behind it
        C.set_gemm_trace(None)
        torch.cuda.synchronize()
    finally:
        C.set_pdl(True)
    t = tr.view(16, 1024)[8:12].cpu()
    n = int((t[0] > 0).sum())
    t = t[:, :n].double()
    rel = (t - t[0].min()) / 1e3

    def mmm(v):
        return [round(float(v.min()), 2), round(float(v.median()), 2), round(float(v.max()), 2)]

    main_us = float((rel[2] - rel[1]).median())
    return {"ctas": n, "start": mmm(rel[0]), "first_weight": mmm(rel[1]), "mainloop_done": mmm(rel[2]),
            "end": mmm(rel[3]), "weight_gbs_in_mainloop": round(N * K / max(main_us, 1e-3) / 1e3, 1)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-gemm-timeline")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--m", type=int, default=16)
    ap.add_argument("--ops", default="qkv,o_proj,gate_up,down")
    a = ap.parse_args(argv)
    dev = torch.device("cuda")
    shapes = gemm_shapes(a.tp)
    for name in a.ops.split(","):
        N, K = shapes[name]
        for pdl in (False, True):
            rec = {"op": name, "M": a.m, "N": N, "K": K, "pdl": pdl, **timeline(N, K, a.m, pdl, dev)}
            print(json.dumps(rec), flush=True)
    ops.check_status()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
