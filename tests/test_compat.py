"""Compatibility API of the reference's flashattention_custom.ops: CPU math semantics, append, and (GPU) the kernel
path against the math path, including GQA head maps, offsets, non-causal and decode rows."""
import math

import pytest
import torch

from hrm_flashrenderer_b200.compat import flash_attn, flash_attn_paged, paged_kv_append
from hrm_flashrenderer_b200.compat import flashattention as fa


def _ref(q, k, v, causal, qo=0, ko=0):
    M, N = q.shape[-2], k.shape[-2]
    s = q.double() @ k.double().transpose(-1, -2) / math.sqrt(q.shape[-1])
    if causal:
        mask = torch.arange(ko, ko + N).view(1, N) > torch.arange(qo, qo + M).view(M, 1)
        s = s.masked_fill(mask, float("-inf"))
    return (torch.softmax(s, -1) @ v.double()).float()


def _pages(k, PS):
    B, H, N, D = k.shape
    P = (N + PS - 1) // PS
    kp = torch.zeros(B, H, P, PS, D, dtype=k.dtype, device=k.device)
    kp.view(B, H, P * PS, D)[:, :, :N] = k
    return kp


@pytest.mark.parametrize("causal,qo,ko", [(True, 0, 0), (True, 40, 8), (False, 0, 0)])
def test_cpu_flash_attn_semantics(causal, qo, ko):
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(2, 4, n, 32, generator=g) for n in (24, 64, 64))
    out = flash_attn(q, k, v, causal=causal, q_offset=qo, k_offset=ko)
    assert torch.allclose(out, _ref(q, k, v, causal, qo, ko), atol=1e-5)


def test_cpu_paged_gqa_head_map_and_seqlen():
    g = torch.Generator().manual_seed(1)
    B, Hq, Hk, M, N, D, PS = 2, 6, 2, 8, 70, 16, 32
    q = torch.randn(B, Hq, M, D, generator=g)
    k, v = torch.randn(B, Hk, N, D, generator=g), torch.randn(B, Hk, N, D, generator=g)
    hm = torch.tensor([1, 0, 1, 0, 0, 1], dtype=torch.int32)
    seqlen = torch.tensor([70, 50], dtype=torch.int32)
    out = flash_attn_paged(q, _pages(k, PS), _pages(v, PS), seqlen, PS, hm, causal=True, q_offset=42)
    for b in range(B):
        L = int(seqlen[b])
        ref = _ref(q[b], k[b, hm.long(), :L], v[b, hm.long(), :L], True, 42, 0)
        assert torch.allclose(out[b], ref, atol=1e-5)


def test_append_matches_loop():
    g = torch.Generator().manual_seed(2)
    B, Hk, P, PS, D, T, start = 2, 3, 4, 16, 8, 21, 13
    kp, vp = torch.zeros(B, Hk, P, PS, D), torch.zeros(B, Hk, P, PS, D)
    kn, vn = torch.randn(B, Hk, T, D, generator=g), torch.randn(B, Hk, T, D, generator=g)
    kr, vr = kp.clone(), vp.clone()
    for t in range(T):
        pos = start + t
        kr[:, :, pos // PS, pos % PS] = kn[:, :, t]
        vr[:, :, pos // PS, pos % PS] = vn[:, :, t]
    paged_kv_append(kp, vp, kn, vn, start, PS)
    assert torch.equal(kp, kr) and torch.equal(vp, vr)


def test_group_order():
    assert fa._group_order(torch.tensor([1, 0, 1, 0]), 4, 2).tolist() == [1, 3, 0, 2]
    assert fa._group_order(torch.tensor([1, 1, 1, 0]), 4, 2) is None


# ------------------------------------------------------------------------------------------------ GPU kernel path
DEV = "cuda"


@pytest.mark.gpu
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal,qo,M", [(True, 0, 128), (True, 128, 64), (False, 0, 48), (True, 255, 1)])
def test_gpu_paged_kernel_path_matches_math(D, causal, qo, M):
    torch.manual_seed(0)
    B, Hq, Hk, N, PS = 2, 8, (8 if D == 64 else 2), 256, 128
    q = torch.randn(B, Hq, M, D, device=DEV, dtype=torch.float16)
    k = torch.randn(B, Hk, N, D, device=DEV, dtype=torch.float16)
    v = torch.randn(B, Hk, N, D, device=DEV, dtype=torch.float16)
    hm = (torch.arange(Hq, device=DEV) * Hk // Hq).to(torch.int32).flip(0).contiguous()
    seqlen = torch.tensor([N, N - 37], device=DEV, dtype=torch.int32)
    kp, vp = _pages(k, PS), _pages(v, PS)
    out = flash_attn_paged(q, kp, vp, seqlen, PS, hm, causal=causal, q_offset=qo)
    ref = fa._math_paged(q.float(), kp.float(), vp.float(), seqlen, PS, hm, causal, qo, 0)
    from hrm_flashrenderer_b200 import ops
    ops.check_status()
    assert out.dtype == torch.float16
    assert (out.float() - ref).abs().max().item() < 3e-2


@pytest.mark.gpu
@pytest.mark.parametrize("D", [64, 128])
def test_gpu_contiguous_kernel_path_matches_math(D):
    torch.manual_seed(1)
    q = torch.randn(1, 8, 128, D, device=DEV, dtype=torch.float16)
    k = torch.randn(1, 8, 250, D, device=DEV, dtype=torch.float16)
    v = torch.randn(1, 8, 250, D, device=DEV, dtype=torch.float16)
    for causal, qo, ko in ((True, 0, 0), (True, 122, 0), (False, 0, 0)):
        out = flash_attn(q, k, v, causal=causal, q_offset=qo, k_offset=ko)
        ref = fa._math_attn(q.float(), k.float(), v.float(), causal, qo, ko)
        assert (out.float() - ref).abs().max().item() < 3e-2, (causal, qo, ko)


@pytest.mark.gpu
def test_console_checks():
    from hrm_flashrenderer_b200.compat.kernel_test import kernel_checks, append_checks
    assert kernel_checks(log=lambda s: None)
    assert append_checks(log=lambda s: None)


@pytest.mark.parametrize("causal,qo,M", [(True, 0, 32), (True, 40, 16), (False, 0, 12), (True, 63, 1), (False, 0, 1)])
def test_kernel_path_layout_logic_on_cpu(monkeypatch, causal, qo, M):
    """Force the kernel path on CPU tensors: the package ops then run their CPU reference implementations over the
    same block pool, tables, query starts and context lengths, which checks the re-layout, head regrouping and
    offset handling that the GPU path uses."""
    monkeypatch.setattr(fa, "_kernel_ok", lambda q, group=1: True)
    g = torch.Generator().manual_seed(3)
    B, Hq, Hk, N, D, PS = 2, 6, 3, 64, 32, 32
    q = torch.randn(B, Hq, M, D, generator=g)
    k, v = torch.randn(B, Hk, N, D, generator=g), torch.randn(B, Hk, N, D, generator=g)
    hm = torch.tensor([2, 0, 1, 2, 1, 0], dtype=torch.int32)
    seqlen = torch.tensor([64, 45], dtype=torch.int32)
    kp, vp = _pages(k, PS), _pages(v, PS)
    out = flash_attn_paged(q, kp, vp, seqlen, PS, hm, causal=causal, q_offset=qo)
    ref = fa._math_paged(q, kp, vp, seqlen, PS, hm, causal, qo, 0)
    assert (out.float() - ref).abs().max().item() < 2e-2     # bf16 operands on the kernel path
    qc = torch.randn(B, 3, M, D, generator=g)
    kc, vc = torch.randn(B, 3, 50, D, generator=g), torch.randn(B, 3, 50, D, generator=g)
    outc = flash_attn(qc, kc, vc, causal=causal, q_offset=qo)
    assert (outc.float() - fa._math_attn(qc, kc, vc, causal, qo, 0)).abs().max().item() < 2e-2
