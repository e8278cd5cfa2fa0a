"""Console checks ``flash-kernel-test`` and ``flash-append-test`` (the reference's ``flash_tests/test_kernel.py`` and
``flash_tests/test_append_fast.py`` entry points): run the compatibility API on the GPU against fp32 attention
math and print the max / mean error; exit status 1 on a tolerance miss."""
from __future__ import annotations

import math
import sys

import torch

from .flashattention import flash_attn, flash_attn_paged, paged_kv_append


def _ref(q, k, v, causal, q_offset=0, k_offset=0):
    M, N = q.shape[2], k.shape[2]
    s = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    if causal:
        qp = torch.arange(q_offset, q_offset + M, device=q.device)
        kp = torch.arange(k_offset, k_offset + N, device=q.device)
        s = s.masked_fill(kp.view(1, 1, 1, N) > qp.view(1, 1, M, 1), float("-inf"))
    return torch.matmul(torch.softmax(s, -1), v)


def kernel_checks(device: str = "cuda", log=print) -> bool:
    torch.manual_seed(0)
    ok = True
    PS = 128
    for D in (64, 128):
        B, Hq, Hk, M, N = 1, 8, 8, 128, 256
        tol = 0.12 if D == 128 else 0.10
        q = torch.randn(B, Hq, M, D, device=device, dtype=torch.float16)
        k = torch.randn(B, Hq, N, D, device=device, dtype=torch.float16)
        v = torch.randn(B, Hq, N, D, device=device, dtype=torch.float16)
        ref = _ref(q.float(), k.float(), v.float(), True).half()
        d = (flash_attn(q, k, v, causal=True) - ref).abs()
        log(f"contig D {D} max {d.max().item():.5f} mean {d.mean().item():.6f}")
        ok &= d.max().item() < tol
        P = (N + PS - 1) // PS
        kp = torch.zeros(B, Hk, P, PS, D, device=device, dtype=torch.float16)
        vp = torch.zeros_like(kp)
        kp.view(B, Hk, P * PS, D)[:, :, :N] = k[:, :Hk]
        vp.view(B, Hk, P * PS, D)[:, :, :N] = v[:, :Hk]
        seqlen = torch.tensor([N], device=device, dtype=torch.int32)
        hm = torch.arange(Hq, device=device, dtype=torch.int32)
        d = (flash_attn_paged(q, kp, vp, seqlen, PS, hm, causal=True) - ref).abs()
        log(f"paged D {D} max {d.max().item():.5f} mean {d.mean().item():.6f}")
        ok &= d.max().item() < tol
        q2 = torch.randn(B, Hq, 64, D, device=device, dtype=torch.float16)
        ref2 = _ref(q2.float(), k.float(), v.float(), True, q_offset=128).half()
        d = (flash_attn_paged(q2, kp, vp, seqlen, PS, hm, causal=True, q_offset=128) - ref2).abs()
        log(f"paged offset D {D} max {d.max().item():.5f} mean {d.mean().item():.6f}")
        ok &= d.max().item() < tol
    return bool(ok)


def append_checks(device: str = "cuda", log=print) -> bool:
    torch.manual_seed(0)
    B, Hk, P, PS, D, T = 2, 4, 8, 128, 128, 96
    start = 128 + 17
    kp = torch.zeros(B, Hk, P, PS, D, device=device, dtype=torch.float16)
    vp = torch.zeros_like(kp)
    kn = torch.randn(B, Hk, T, D, device=device, dtype=torch.float16)
    vn = torch.randn_like(kn)
    kr, vr = kp.clone(), vp.clone()
    for t in range(T):
        pos = start + t
        kr[:, :, pos // PS, pos % PS] = kn[:, :, t]
        vr[:, :, pos // PS, pos % PS] = vn[:, :, t]
    paged_kv_append(kp, vp, kn, vn, start_pos=start, page_size=PS)
    dk, dv = (kp - kr).abs().max().item(), (vp - vr).abs().max().item()
    log(f"append max|diff| K: {dk} V: {dv}")
    return dk == 0.0 and dv == 0.0


def kernel_test_main() -> int:
    ok = kernel_checks()
    print("OK" if ok else "FAILED")
    return 0 if ok else 1


def append_test_main() -> int:
    ok = append_checks()
    print("OK" if ok else "FAILED")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(kernel_test_main() if "append" not in sys.argv[1:] else append_test_main())
