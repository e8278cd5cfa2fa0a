"""Tensor-parallel collective-GEMM op sweep (Llama-70B projection shapes): one process per GPU under torchrun.

    torchrun --nproc-per-node N -m hrm_flashrenderer_b200.benchmarks.tp_sweep [--m 1,8,64,512,4096]

RowParallel projections of Llama-3.1-70B (o_proj: K 8192, down: K 28672, both N 8192), K sharded over the ranks:
  * ``baseline``: W8A16 GEMM into an fp32 partial, NCCL all-reduce, residual add + next-RMSNorm inputs (norm_prep);
  * ``fused`` (M <= 64): one kernel - GEMM, partial tiles pushed into every rank's receive area over NVLink, one
    epoch-flag hop, local rank-ordered reduction + residual + xg / ssq outputs.
ColumnParallel projections (qkv: N 10240, gate_up: N 57344, K 8192) are timed as the GEMM on the local N shard
(no collective in the TP decode path).  Every time is the max over ranks of CUDA-event averages.  Roofline of the
fused op = max(weights / HBM, (world - 1) x M x N x 4 B / NVLink), with the measured HBM copy bandwidth and
770 GB/s per direction for NVLink.
"""
import argparse
import json

import torch
import torch.distributed as dist

from .. import ops
from ..parallel.dist import init_dist_env
from ..parallel.symm import SymmetricWorkspace
from .ops_sweep import peaks

NVLINK_GBS = 770.0


def timeit(fn, iters, warm, dev):
    for _ in range(warm):
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
    ap = argparse.ArgumentParser(prog="hrm-flash-tp-sweep")
    ap.add_argument("--m", default="1,8,64,512,4096")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args(argv)
    rank, local, world = init_dist_env("nccl")
    dev = torch.device("cuda", local)
    hbm_gbs, tflops, _ = peaks()
    symm = SymmetricWorkspace(rank, world, dev, max_tiles=64, max_bn=64)
    Ms = [int(x) for x in a.m.split(",")]
    g = torch.Generator(device="cpu").manual_seed(rank)
    for name, N, K in (("o_proj", 8192, 8192), ("down", 8192, 28672)):
        Kl = K // world
        w = ops.tile_w8(torch.randint(-127, 128, (N, Kl), generator=g, dtype=torch.int8).to(dev))
        s = (torch.rand(N, generator=g) * 1e-3).to(dev)
        gamma = torch.ones(N, device=dev)
        for M in Ms:
            x = torch.randn(M, Kl, generator=g).half().to(dev)
            resid = torch.randn(M, N, device=dev)
            xg = torch.empty(M, N, dtype=torch.float16, device=dev)
            ssq = torch.empty(N // 128, M, device=dev)
            part = torch.empty(M, N, device=dev)

            def base():
                ops.w8a16_linear_out(x, w, s, part)
                dist.all_reduce(part)
                ops.norm_prep(resid, part, gamma, xg, ssq)

            rec = {"op": f"row_parallel_{name}+allreduce+residual+norm", "M": M, "N": N, "K_per_rank": Kl,
                   "world": world, "baseline_us": round(timeit(base, a.iters, a.warmup, dev), 2)}
            wbytes = N * Kl
            roof_us = max(wbytes / (hbm_gbs * 1e3), (world - 1) * M * N * 4 / (NVLINK_GBS * 1e3))
            if M <= 64:
                rec["fused_us"] = round(timeit(lambda: ops.w8a16_residual_ar_(x, w, s, resid, symm, gamma, xg, ssq),
                                               a.iters, a.warmup, dev), 2)
                rec["fused_speedup"] = round(rec["baseline_us"] / rec["fused_us"], 2)
                rec["fused_frac_of_roofline"] = round(roof_us / rec["fused_us"], 3)
            rec["roofline_us"] = round(roof_us, 2)
            if rank == 0:
                print(json.dumps(rec), flush=True)
    for name, N, K in (("qkv", 10240, 8192), ("gate_up", 57344, 8192)):
        Nl = N // world
        w = ops.tile_w8(torch.randint(-127, 128, (Nl, K), generator=g, dtype=torch.int8).to(dev))
        s = (torch.rand(Nl, generator=g) * 1e-3).to(dev)
        for M in Ms:
            x = torch.randn(M, K, generator=g).half().to(dev)
            out = torch.empty(M, Nl, dtype=torch.float16, device=dev)
            us = timeit(lambda: ops.w8a16_linear_out(x, w, s, out), a.iters, a.warmup, dev)
            roof_us = max(Nl * K / (hbm_gbs * 1e3), 2.0 * M * Nl * K / (tflops * 1e6))
            if rank == 0:
                print(json.dumps({"op": f"column_parallel_{name}", "M": M, "N_per_rank": Nl, "K": K, "world": world,
                                  "us": round(us, 2), "roofline_us": round(roof_us, 2),
                                  "frac_of_roofline": round(roof_us / us, 3)}), flush=True)
    ops.check_status(dev)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
