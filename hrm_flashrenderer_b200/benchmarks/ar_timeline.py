"""Per-stage timeline of the fused row-parallel GEMM + peer-memory all-reduce, one process per GPU.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m hrm_flashrenderer_b200.benchmarks.ar_timeline [--tokens 16]

For the Llama-3.1-70B row-parallel projections (o_proj K 8192, down K 28672, N 8192; K sharded over the ranks)
every rank runs the fused kernel back to back; one launch, right behind an untraced one, records per CTA the
%globaltimer stamps of the GEMM (start, first weight unit, mainloop done, end) and, for the CTAs that complete an
output tile, of the per-tile all-reduce (tile pushed, every rank's flag of the tile seen, reduction written).
Printed per rank: the median over CTAs of each stage's length, plus the event-timed average of 20 launches of the
fused kernel and of the GEMM alone (max over ranks), so the all-reduce's share of a launch is explicit.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from .. import ops
from ..parallel.dist import init_dist_env
from ..parallel.symm import SymmetricWorkspace

_STAGES = [("start->first weight", 8, 9), ("mainloop", 9, 10), ("epilogue+fixup+push", 10, 12),
           ("fence+flags+wait for peers", 12, 14), ("reduce+outputs", 14, 15), ("tail to CTA end", 15, 11)]


def _avg_us(fn, iters, dev):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters * 1e3], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main(argv=None):
    ap = argparse.ArgumentParser(prog="hrm-flash-ar-timeline")
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    rank, local, world = init_dist_env("nccl")
    dev = torch.device("cuda", local)
    C = ops.ext()
    symm = SymmetricWorkspace(rank, world, dev, max_tiles=64, max_bn=64)
    M, N = a.tokens, 8192
    for name, K in (("o_proj", 8192), ("down", 28672)):
        Kl = K // world
        g = torch.Generator().manual_seed(rank + 7)
        w = ops.tile_w8(torch.randint(-127, 128, (N, Kl), generator=g, dtype=torch.int8).to(dev))
        s = (torch.rand(N, generator=g) * 1e-4).to(dev)
        x = torch.randn(M, Kl, generator=g).half().to(dev)
        resid = torch.zeros(M, N, device=dev)
        gamma = torch.ones(N, device=dev)
        xg = torch.empty(M, N, dtype=torch.float16, device=dev)
        ssq = torch.empty(N // 128, M, device=dev)
        part = torch.empty(M, N, device=dev)
        fused = lambda: ops.w8a16_residual_ar_(x, w, s, resid, symm, gamma, xg, ssq)
        alone = lambda: ops.w8a16_linear_out(x, w, s, part)
        t_fused = _avg_us(fused, a.iters, dev)
        t_alone = _avg_us(alone, a.iters, dev)
        tr = torch.zeros(16 * 1024, dtype=torch.int64, device=dev)
        torch.cuda.synchronize()
        dist.barrier()
        fused()
        C.set_gemm_trace(tr)
        fused()
        C.set_gemm_trace(None)
        torch.cuda.synchronize()
        ops.check_status(dev)
        t = tr.view(16, 1024).cpu().double()
        n = int((t[8] > 0).sum())
        t = t[:, :n]
        stages = {}
        for label, r0, r1 in _STAGES:
            ok = (t[r0] > 0) & (t[r1] > 0)
            stages[label] = round(float(((t[r1] - t[r0])[ok]).median()) / 1e3, 2) if ok.any() else None
        span = round(float(t[11].max() - t[8].min()) / 1e3, 2)
        rec = {"rank": rank, "op": name, "M": M, "N": N, "K_per_rank": Kl, "ctas": n, "span_us": span,
               "stage_median_us": stages, "fused_us_max_over_ranks": round(t_fused, 2),
               "gemm_alone_us_max_over_ranks": round(t_alone, 2)}
        recs = [None] * world
        dist.all_gather_object(recs, rec)
        if rank == 0:
            for r in recs:
                print(json.dumps(r), flush=True)
    symm.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
