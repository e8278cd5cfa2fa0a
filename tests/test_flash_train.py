"""CPU side of the trainer's causal attention: the PyTorch math behind ``ops.flash_train_fwd`` / ``_bwd`` on CPU
tensors (base-2 log-sum-exp, gradients) and the reversible LM's autograd wrapper around it."""
import math

import torch
import torch.nn.functional as Fn

from hrm_flashrenderer_b200 import ops


def _sdpa(q, k, v):
    return Fn.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=True).transpose(1, 2)


def test_cpu_forward_and_lse():
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(2, 33, 3, 16, generator=g) for _ in range(3))
    o, lse = ops.flash_train_fwd(q, k, v)
    torch.testing.assert_close(o, _sdpa(q, k, v), rtol=1e-5, atol=1e-5)
    s = torch.einsum("bihd,bjhd->bhij", q, k) / 4.0
    s = s.masked_fill(torch.ones(33, 33, dtype=torch.bool).triu(1), -float("inf"))
    torch.testing.assert_close(lse, torch.logsumexp(s, -1) * math.log2(math.e), rtol=1e-5, atol=1e-5)
    assert o.shape == q.shape and lse.shape == (2, 3, 33)


def test_cpu_backward_and_autograd_wrapper():
    from hrm_flashrenderer_b200.experiments.revlm import _FlashAttn
    g = torch.Generator().manual_seed(2)
    q, k, v, dout = (torch.randn(1, 20, 2, 32, generator=g) for _ in range(4))
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    want = torch.autograd.grad(_sdpa(qq, kk, vv), (qq, kk, vv), dout)
    o, lse = ops.flash_train_fwd(q, k, v)
    got = ops.flash_train_bwd(q, k, v, o, lse, dout)
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5)
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    y = _FlashAttn.apply(qq, kk, vv)
    y.backward(dout)
    for a, b in zip((qq.grad, kk.grad, vv.grad), want):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5)
