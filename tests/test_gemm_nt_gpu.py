"""The experiments plane's tensor-core NT GEMM (``ops.gemm_nt``: C = A . B^T, bf16 / f16 operands, fp32 out) against
fp32 math of the same rounded operands, its autograd wrapper in the reversible LM against PyTorch's, and one
reversible-LM loss / gradient on it against PyTorch's bf16 matmul path."""
import pytest
import torch

from hrm_flashrenderer_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (300, 260, 200), (8192, 128, 128), (256, 4096, 256),
                                   (1000, 1024, 1024), (128, 48, 16), (7, 8, 8)])
def test_gemm_nt_matches_fp32_math(M, N, K, dt):
    g = torch.Generator(device="cpu").manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(dt).cuda()
    b = torch.randn(N, K, generator=g).to(dt).cuda()
    c = ops.gemm_nt(a, b)
    torch.cuda.synchronize()
    ops.check_status()
    ref = a.float() @ b.float().t()
    torch.testing.assert_close(c, ref, rtol=1e-4, atol=1e-3 * max(1.0, K ** 0.5))


def test_gemm_nt_strided_operands():
    """Column slices of wider row-major matrices (leading dimension > K) and a slice of C."""
    g = torch.Generator(device="cpu").manual_seed(5)
    A = torch.randn(384, 320, generator=g).bfloat16().cuda()
    B = torch.randn(256, 320, generator=g).bfloat16().cuda()
    C = torch.full((384, 512), float("nan"), device="cuda")
    ops.gemm_nt(A[:, 64:256], B[:, 64:256], out=C[:, 128:384])
    torch.cuda.synchronize()
    ref = A[:, 64:256].float() @ B[:, 64:256].float().t()
    torch.testing.assert_close(C[:, 128:384], ref, rtol=1e-4, atol=2e-2)
    assert torch.isnan(C[:, :128]).all() and torch.isnan(C[:, 384:]).all()   # nothing outside the slice


def test_tc_matmul_forward_backward_matches_torch():
    from hrm_flashrenderer_b200.experiments.revlm import _TcMatmul
    g = torch.Generator(device="cpu").manual_seed(9)
    x = torch.randn(4, 64, 128, generator=g).cuda().requires_grad_(True)
    w = torch.randn(128, 1024, generator=g).cuda().mul_(0.05).requires_grad_(True)
    dy = torch.randn(4, 64, 1024, generator=g).cuda()
    y = _TcMatmul.apply(x, w)
    y.backward(dy)
    xr = x.detach().bfloat16().float().requires_grad_(True)
    wr = w.detach().bfloat16().float().requires_grad_(True)
    yr = xr @ wr
    yr.backward(dy.bfloat16().float())
    torch.testing.assert_close(y, yr, rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(x.grad, xr.grad, rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(w.grad, wr.grad, rtol=2e-3, atol=5e-2)


def test_revlm_loss_and_grads_on_tensor_core_gemm():
    """The reversible LM's loss and parameter gradient through the NT GEMM agree with PyTorch's bf16 matmul path."""
    from hrm_flashrenderer_b200.experiments import revlm as R
    cfg = R.RevConfig(k1=256, k2=128, d=128, heads=4, layers=2, ffn=256, tmax=128)
    flat = R.init_flat(cfg, 7)
    g = torch.Generator().manual_seed(3)
    tok = torch.randint(0, cfg.vocab, (4, 64), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab, (4, 64), generator=g).cuda()
    out = {}
    try:
        for tc in (True, False):
            R.TC_GEMM = tc
            m = R.RevLM(cfg, "cuda", flat.clone(), lowp=True)
            loss = m.loss(tok, tgt)
            loss.backward()
            out[tc] = (float(loss), m.flat.grad.detach().clone())
    finally:
        R.TC_GEMM = True
    ops.check_status()
    assert abs(out[True][0] - out[False][0]) < 2e-3 * abs(out[False][0])
    ga, gb = out[True][1], out[False][1]
    cos = float((ga * gb).sum() / (ga.norm() * gb.norm()))
    assert cos > 0.999, cos
