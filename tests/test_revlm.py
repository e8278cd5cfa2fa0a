"""Reversible LM of the experiments plane: reversible backward == plain autograd, loss/decode consistency,
checkpoint v11 round trip (CPU, fp32)."""

import numpy as np
import torch

from hrm_flashrenderer_b200.experiments.revlm import (ChatState, RevConfig, RevLM, init_flat, load_ckpt, save_ckpt,
                                                     views)

TINY = RevConfig(k1=40, k2=24, d=32, heads=2, layers=2, ffn=48, tmax=32)


def _batch(cfg, B=2, T=12, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(0, cfg.vocab, (B, T + 1), generator=g)
    return x[:, :-1], x[:, 1:]


def test_layout_and_init():
    assert TINY.vocab == 320 and TINY.vpad == 320 and TINY.dh == 8
    n = TINY.weights_floats()
    assert n == 320 * 32 + 32 * 32 + 2 * (16 + 4 * 16 * 16 + 16 + 16 * 48 + 48 * 16) + 32 + 32 * 320
    v = views(TINY, init_flat(TINY, 7))
    assert torch.all(v["gf.1"] == 1) and torch.all(v["gout"] == 1) and float(v["Wq.0"].abs().max()) <= 0.02


def test_reversible_backward_matches_autograd():
    tok, tgt = _batch(TINY)
    # the trainer's init scale: rebuilt activations are exact to fp32 rounding (with much larger weights the
    # reconstruction error of a reversible stack grows, as it does in the reference)
    flat = init_flat(TINY, 3)
    a = RevLM(TINY, "cpu", flat.clone(), lowp=False, reversible=True)
    b = RevLM(TINY, "cpu", flat.clone(), lowp=False, reversible=False)
    la, lb = a.loss(tok, tgt), b.loss(tok, tgt)
    la.backward()
    lb.backward()
    assert abs(la.item() - lb.item()) < 1e-6
    torch.testing.assert_close(a.flat.grad, b.flat.grad, rtol=1e-4, atol=1e-7)


def test_streaming_loss_equals_full_cross_entropy():
    tok, tgt = _batch(TINY)
    m = RevLM(TINY, "cpu", init_flat(TINY, 5) * 10, lowp=False)
    with torch.no_grad():
        full = torch.nn.functional.cross_entropy(m.logits(tok).reshape(-1, TINY.vocab), tgt.reshape(-1))
        assert abs(float(m.loss(tok, tgt, vchunk=7)) - float(full)) < 1e-5


def test_incremental_decode_matches_full_forward():
    m = RevLM(TINY, "cpu", init_flat(TINY, 9) * 10, lowp=False)
    ids = [3, 100, 7, 250, 18, 44]
    with torch.no_grad():
        full = m.logits(torch.tensor([ids])).argmax(-1)[0].tolist()
    st = ChatState(m)
    got = [st.step(t) for t in ids]
    assert got == full


def test_ckpt_v11_roundtrip(tmp_path):
    flat = init_flat(TINY, 11)
    tables = (np.arange(TINY.k1, dtype=np.uint16), np.arange(TINY.k2, dtype=np.uint32) + (300 << 16),
              np.full(64, 0xFFFFFFFF, np.uint32), np.full(64, 0xFFFF, np.uint16))
    p = tmp_path / "c.bin"
    save_ckpt(str(p), TINY, tables, flat)
    raw = p.read_bytes()
    assert int.from_bytes(raw[:4], "little") == 0x43484452 and int.from_bytes(raw[4:8], "little") == 11
    assert len(raw) == 36 + 2 * 40 + 4 * 24 + 4 + 64 * 6 + 4 * TINY.weights_floats()
    cfg, t2, f2 = load_ckpt(str(p), TINY)
    assert cfg == TINY and torch.equal(f2, flat)
    assert all(np.array_equal(x, y) for x, y in zip(tables, t2))


def test_tc_matmul_wiring_on_cpu():
    """The tensor-core product's autograd wiring (forward and both backward products expressed as C = A . B^T) on
    the op's CPU reference path, against PyTorch autograd on the same bf16-rounded operands."""
    import torch
    from hrm_flashrenderer_b200.experiments.revlm import _TcMatmul
    g = torch.Generator().manual_seed(2)
    x = torch.randn(3, 16, 32, generator=g).requires_grad_(True)
    w = torch.randn(64, 48, generator=g)[:32].requires_grad_(False)
    w = w.clone().requires_grad_(True)
    dy = torch.randn(3, 16, 48, generator=g)
    y = _TcMatmul.apply(x, w)
    y.backward(dy)
    xr = x.detach().bfloat16().float().requires_grad_(True)
    wr = w.detach().bfloat16().float().requires_grad_(True)
    (xr @ wr).backward(dy.bfloat16().float())
    torch.testing.assert_close(y, (xr @ wr).detach(), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(x.grad, xr.grad, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(w.grad, wr.grad, rtol=1e-5, atol=1e-5)
