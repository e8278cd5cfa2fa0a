"""The trainer's causal flash attention (``ops.flash_train_fwd`` / ``ops.flash_train_bwd``, head dims 16 and 32) on
the GPU against fp64 PyTorch math of the same op, its determinism, and the reversible LM's loss / gradient with it
against PyTorch's scaled_dot_product_attention path."""
import math

import pytest
import torch

from hrm_flashrenderer_b200 import ops

pytestmark = pytest.mark.gpu


def _ref(q, k, v, dout):
    qq, kk, vv = (t.detach().double().requires_grad_(True) for t in (q, k, v))
    T, D = q.shape[1], q.shape[3]
    s = torch.einsum("bihd,bjhd->bhij", qq, kk) / math.sqrt(D)
    s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=q.device).triu(1), -float("inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.einsum("bhij,bjhd->bihd", torch.softmax(s, -1), vv)
    dq, dk, dv = torch.autograd.grad(o, (qq, kk, vv), dout.double())
    return o, lse * math.log2(math.e), dq, dk, dv


@pytest.mark.parametrize("rpt", [1, 2])
@pytest.mark.parametrize("B,T,H,D", [(2, 1, 3, 16), (1, 7, 2, 16), (2, 64, 8, 16), (1, 130, 4, 32), (3, 512, 8, 16),
                                     (1, 300, 2, 32), (1, 1000, 1, 16), (2, 129, 8, 16), (1, 257, 2, 16)])
def test_flash_train_matches_fp64_math(B, T, H, D, rpt, monkeypatch):
    monkeypatch.setattr(ops, "FLASH_RPT", rpt)
    monkeypatch.setattr(ops, "FLASH_FWD_RPT", rpt)
    g = torch.Generator(device="cpu").manual_seed(B * 1000 + T + H + D)
    q, k, v, dout = (torch.randn(B, T, H, D, generator=g).cuda() for _ in range(4))
    o, lse = ops.flash_train_fwd(q, k, v)
    dq, dk, dv = ops.flash_train_bwd(q, k, v, o, lse, dout)
    torch.cuda.synchronize()
    ro, rlse, rdq, rdk, rdv = _ref(q, k, v, dout)
    torch.testing.assert_close(o.double(), ro, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(lse.double(), rlse, rtol=1e-5, atol=1e-4)
    for got, want in ((dq, rdq), (dk, rdk), (dv, rdv)):
        torch.testing.assert_close(got.double(), want, rtol=1e-3, atol=2e-4 * max(1.0, T ** 0.5))


@pytest.mark.parametrize("rpt", [1, 2])
def test_flash_train_backward_is_deterministic(rpt, monkeypatch):
    monkeypatch.setattr(ops, "FLASH_RPT", rpt)
    monkeypatch.setattr(ops, "FLASH_FWD_RPT", rpt)
    g = torch.Generator(device="cpu").manual_seed(11)
    q, k, v, dout = (torch.randn(4, 384, 8, 16, generator=g).cuda() for _ in range(4))
    o, lse = ops.flash_train_fwd(q, k, v)
    a = ops.flash_train_bwd(q, k, v, o, lse, dout)
    b = ops.flash_train_bwd(q, k, v, o, lse, dout)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_revlm_loss_and_grads_on_flash_attention():
    """The reversible LM's loss and parameter gradient through the flash kernels agree with the SDPA path (fp32
    matmuls in both, so only the attention differs)."""
    from hrm_flashrenderer_b200.experiments import revlm as R
    cfg = R.RevConfig(k1=256, k2=128, d=128, heads=4, layers=2, ffn=256, tmax=128)
    flat = R.init_flat(cfg, 5)
    g = torch.Generator().manual_seed(4)
    tok = torch.randint(0, cfg.vocab, (4, 96), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab, (4, 96), generator=g).cuda()
    out = {}
    try:
        for fl in (True, False):
            R.FLASH_ATTN = fl
            m = R.RevLM(cfg, "cuda", flat.clone(), lowp=False)
            loss = m.loss(tok, tgt)
            loss.backward()
            out[fl] = (float(loss), m.flat.grad.detach().clone())
    finally:
        R.FLASH_ATTN = True
    assert abs(out[True][0] - out[False][0]) < 1e-4 * abs(out[False][0])
    ga, gb = out[True][1], out[False][1]
    assert float((ga - gb).norm() / gb.norm()) < 1e-3
