"""sm_100a kernels vs plain PyTorch fp32 references of the same op (run on a B200 with -m gpu)."""
import os

import pytest
import torch

from hrm_flashrenderer_b200 import ops
from hrm_flashrenderer_b200.models.weights import quantize_rows

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _qw(N, K, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    qt = quantize_rows(torch.randn(N, K, generator=g) * 0.02)
    return qt.q.to(DEV), qt.scale.to(DEV)


def _x(M, K, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(M, K, generator=g).to(DEV, torch.float16)


def _ref(x, q, s):
    return x.float() @ (q.float() * s[:, None]).t()


def test_extension_loaded():
    assert ops.has_ext(), "the CUDA extension must be built and loaded on a GPU box"


@pytest.mark.parametrize("M", [1, 5, 16, 33, 64, 100, 257])
@pytest.mark.parametrize("N,K", [(128, 128), (384, 512), (1000, 1024), (256, 4096)])
def test_w8a16_gemm(M, N, K):
    q, s = _qw(N, K, 1)
    x = _x(M, K, 2)
    y = ops.w8a16_linear(x, q, s, out_dtype=torch.float32)
    ref = _ref(x, q, s)
    err = (y - ref).abs().max().item()
    assert err <= 1e-3 * max(1.0, ref.abs().max().item()), err


@pytest.mark.parametrize("M", [1, 16, 64, 130, 300])
@pytest.mark.parametrize("N,K", [(1000, 1024), (1536, 4096)])
def test_w8a16_tiled_weights_bitwise_equal_plain(M, N, K):
    """Pre-tiled weights (bulk-copy path) give bit-identical results to the plain row-major TMA path."""
    q, s = _qw(N, K, 11)
    x = _x(M, K, 12)
    t = ops.tile_w8(q)
    assert torch.equal(ops.untile_w8(t, N), q)
    a = ops.w8a16_linear(x, q, s, out_dtype=torch.float32)
    b = ops.w8a16_linear(x, t, s, out_dtype=torch.float32)
    assert torch.equal(a, b)


@pytest.mark.skipif(os.environ.get("HRM_TEST_MFAST") != "1", reason="m-fastest tile order: set HRM_TEST_MFAST=1")
@pytest.mark.parametrize("M,N,K", [(300, 1000, 1024), (4096, 1536, 4096), (257, 384, 512)])
def test_w8a16_m_fastest_tile_order(M, N, K):
    """m-fastest tile numbering computes the same product (stream-K split points move, so not bitwise)."""
    q, s = _qw(N, K, 13)
    x = _x(M, K, 14)
    t = ops.tile_w8(q)
    C = ops.ext()
    try:
        C.set_gemm_m_fastest(False)
        a = ops.w8a16_linear(x, t, s, out_dtype=torch.float32)
        C.set_gemm_m_fastest(True)
        b = ops.w8a16_linear(x, t, s, out_dtype=torch.float32)
        torch.cuda.synchronize()
    finally:
        C.set_gemm_m_fastest(False)
    ops.check_status()
    torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-3)
    ref = _ref(x, q, s)
    assert (b - ref).abs().max().item() <= 1e-3 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 37, 148])
def test_w8a16_stream_k_deterministic(splits):
    q, s = _qw(512, 2048, 3)
    x = _x(16, 2048, 4)
    a = ops.w8a16_linear(x, q, s, out_dtype=torch.float32, force_ctas=splits)
    b = ops.w8a16_linear(x, q, s, out_dtype=torch.float32, force_ctas=splits)
    assert torch.equal(a, b)
    ref = _ref(x, q, s)
    assert (a - ref).abs().max().item() < 1e-3


def test_w8a16_f16_out_and_bias():
    q, s = _qw(256, 512, 5)
    x = _x(9, 512, 6)
    bias = torch.randn(256, device=DEV)
    y = ops.w8a16_linear(x, q, s, bias=bias)
    assert y.dtype == torch.float16
    ref = _ref(x, q, s) + bias
    assert (y.float() - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("M", [1, 16, 130, 300])
def test_w8a16_residual(M):
    q, s = _qw(1024, 768, 7)
    x = _x(M, 768, 8)
    r0 = torch.randn(M, 1024, device=DEV)
    r = r0.clone()
    ops.w8a16_residual_(x, q, s, r)
    assert (r - (r0 + _ref(x, q, s))).abs().max().item() < 1e-3


@pytest.mark.parametrize("M", [1, 16, 130, 300])
def test_w8a16_residual_norm_outputs_and_folded_norm(M):
    """Residual epilogue writes xg = x*gamma and per-tile sums of squares; a consumer GEMM with in_norm equals
    rmsnorm(x)*gamma @ W^T."""
    H, N2 = 1024, 512
    q, s = _qw(H, 768, 17)
    x = _x(M, 768, 18)
    r = torch.randn(M, H, device=DEV)
    gamma = torch.rand(H, device=DEV) + 0.5
    xg = torch.empty(M, H, dtype=torch.float16, device=DEV)
    ssq = torch.empty(H // 128, M, device=DEV)
    r_ref = r + _ref(x, q, s)
    ops.w8a16_residual_(x, q, s, r, gamma_next=gamma, xg_out=xg, ssq_out=ssq)
    assert (r - r_ref).abs().max().item() < 1e-3
    assert (xg.float() - r_ref * gamma).abs().max().item() < 1e-2 * max(1.0, (r_ref * gamma).abs().max().item())
    assert torch.allclose(ssq.sum(0), r_ref.pow(2).sum(-1), rtol=1e-4)
    w2, s2 = _qw(N2, H, 19)
    y = ops.w8a16_linear(xg, w2, s2, out_dtype=torch.float32, in_norm=(ssq, H, 1e-5))
    h = r_ref * torch.rsqrt(r_ref.pow(2).mean(-1, keepdim=True) + 1e-5) * gamma
    ref = _ref(h.half(), w2, s2)
    assert (y - ref).abs().max().item() < 2e-2 * max(1.0, ref.abs().max().item())


def test_norm_prep_matches_reference():
    M, H = 7, 2048
    x = torch.randn(M, H, device=DEV)
    d = torch.randn(M, H, device=DEV)
    g = torch.rand(H, device=DEV)
    xg = torch.empty(M, H, dtype=torch.float16, device=DEV)
    ssq = torch.empty(H // 128, M, device=DEV)
    x2 = x.clone()
    ops.norm_prep(x2, d, g, xg, ssq)
    xr = x + d
    assert torch.allclose(x2, xr)
    assert (xg.float() - xr * g).abs().max().item() < 1e-2
    assert torch.allclose(ssq, xr.view(M, H // 128, 128).pow(2).sum(-1).t(), rtol=1e-4)


@pytest.mark.parametrize("M", [1, 16, 70, 165, 300])
def test_w8a16_swiglu(M):
    F, K = 384, 512
    gq, gs = _qw(F, K, 9)
    uq, us = _qw(F, K, 10)
    wq, ws = ops.interleave_gate_up(gq, uq, gs, us)
    x = _x(M, K, 11)
    y = ops.w8a16_swiglu(x, wq, ws)
    ref = torch.nn.functional.silu(_ref(x, gq, gs)) * _ref(x, uq, us)
    assert (y.float() - ref).abs().max().item() < 1e-2


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("M", [1, 7, 40, 165, 300])
def test_w8a16_qkv_rope_append(D, M):
    from hrm_flashrenderer_b200.models.oracle import apply_rope, rope_tables
    from hrm_flashrenderer_b200.config import TINY
    from dataclasses import replace
    Hq, Hk, K = 4, 2, 256
    cfg = replace(TINY, head_dim=D, rope_theta=10000.0)
    cos, sin = rope_tables(cfg, 512)
    q_rows, kv_rows = Hq * D, Hk * D
    wq, ws = _qw(q_rows + 2 * kv_rows, K, 12)
    bias = torch.randn(q_rows + 2 * kv_rows, device=DEV) * 0.1
    x = _x(M, K, 13)
    pos = torch.randint(0, 500, (M,), dtype=torch.int32)
    nb, bs = 64, 16
    perm = torch.randperm(nb * bs)[:M]
    slots = perm.to(torch.int32)
    slots[0] = -1 if M > 1 else slots[0]
    kc = torch.zeros(nb, Hk, bs, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q = ops.w8a16_qkv_rope_append(x, wq, ws, bias, q_rows, kv_rows, D, pos.to(DEV), slots.to(DEV), cos.to(DEV),
                                  sin.to(DEV), kc, vc)
    y = (_ref(x, wq, ws) + bias).cpu()
    qr = apply_rope(y[:, :q_rows].view(M, Hq, D), cos, sin, pos.long()).reshape(M, q_rows)
    kr = apply_rope(y[:, q_rows:q_rows + kv_rows].view(M, Hk, D), cos, sin, pos.long())
    vr = y[:, q_rows + kv_rows:].view(M, Hk, D)
    assert (q.float().cpu() - qr).abs().max().item() < 2e-2
    kcc, vcc = kc.float().cpu(), vc.float().cpu()
    for m in range(M):
        sl = int(slots[m])
        if sl < 0:
            continue
        assert (kcc[sl // bs, :, sl % bs] - kr[m]).abs().max().item() < 2e-2
        assert (vcc[sl // bs, :, sl % bs] - vr[m]).abs().max().item() < 2e-2


def _paged(B, lens, Hk, D, bs=16, seed=0, contiguous=False):
    g = torch.Generator().manual_seed(seed)
    nb = sum((L + bs - 1) // bs for L in lens) + 4
    perm = torch.arange(nb) if contiguous else torch.randperm(nb, generator=g)
    kc = torch.randn(nb, Hk, bs, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(nb, Hk, bs, D, generator=g).to(torch.bfloat16)
    maxb = max((L + bs - 1) // bs for L in lens)
    tab = torch.zeros(B, maxb, dtype=torch.int32)
    i = 0
    for b, L in enumerate(lens):
        n = (L + bs - 1) // bs
        tab[b, :n] = perm[i:i + n].to(torch.int32)
        i += n
    return kc, vc, tab


@pytest.mark.parametrize("D,Hq,Hk", [(128, 8, 1), (128, 40, 8), (128, 64, 8), (64, 8, 2)])
@pytest.mark.parametrize("lens", [[1, 17, 300], [4096], [33, 2000, 129, 128]])
@pytest.mark.parametrize("splits", [0, 1, 3])
@pytest.mark.parametrize("tc", [True, False])
def test_paged_decode_attention(D, Hq, Hk, lens, splits, tc):
    B = len(lens)
    kc, vc, tab = _paged(B, lens, Hk, D)
    q = torch.randn(B, Hq, D).to(torch.bfloat16)
    cl = torch.tensor(lens, dtype=torch.int32)
    ref = ops.paged_decode_attention(q, kc, vc, tab, cl)
    kw = {}
    if splits:
        tiles = (tab.shape[1] * 16 + 127) // 128
        per = (tiles + splits - 1) // splits
        kw = dict(splits=(tiles + per - 1) // per, keys_per_split=per * 128)
    out = ops.paged_decode_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), tab.to(DEV), cl.to(DEV), allow_tc=tc, **kw)
    ops.check_status()
    assert (out.float().cpu() - ref.float()).abs().max().item() < 2e-2


@pytest.mark.parametrize("lens", [[4096], [33, 2000, 129, 128], [1, 17, 300]])
@pytest.mark.parametrize("splits", [0, 3])
@pytest.mark.parametrize("kv_prefetch", [False, True])
def test_paged_decode_attention_contiguous_blocks(lens, splits, kv_prefetch):
    """Pool blocks handed out in order: whole 128-key tiles come in as 8-block TMA boxes (plus one-block boxes at
    sequence tails), same results as the reference."""
    B = len(lens)
    kc, vc, tab = _paged(B, lens, 8, 128, contiguous=True)
    q = torch.randn(B, 64, 128).to(torch.bfloat16)
    cl = torch.tensor(lens, dtype=torch.int32)
    ref = ops.paged_decode_attention(q, kc, vc, tab, cl)
    kw = {}
    if splits:
        tiles = (tab.shape[1] * 16 + 127) // 128
        per = (tiles + splits - 1) // splits
        kw = dict(splits=(tiles + per - 1) // per, keys_per_split=per * 128)
    out = ops.paged_decode_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), tab.to(DEV), cl.to(DEV),
                                     kv_prefetch=kv_prefetch, **kw)
    ops.check_status()
    assert (out.float().cpu() - ref.float()).abs().max().item() < 2e-2


@pytest.mark.parametrize("lens", [[4096] * 3, [33, 2000, 129, 128], [1, 17, 300]])
@pytest.mark.parametrize("splits", [0, 2, 5])
def test_paged_decode_attention_in_kernel_merge(lens, splits, monkeypatch):
    """Split merge done by the last split CTA of each (sequence, kv head) (tickets re-armed between calls)."""
    monkeypatch.setattr(ops, "_ATTN_MERGE", True)
    B = len(lens)
    kc, vc, tab = _paged(B, lens, 8, 128, contiguous=True)
    q = torch.randn(B, 64, 128).to(torch.bfloat16)
    cl = torch.tensor(lens, dtype=torch.int32)
    ref = ops.paged_decode_attention(q, kc, vc, tab, cl)
    kw = {}
    if splits:
        tiles = (tab.shape[1] * 16 + 127) // 128
        per = (tiles + splits - 1) // splits
        kw = dict(splits=(tiles + per - 1) // per, keys_per_split=per * 128)
    args = (q.to(DEV), kc.to(DEV), vc.to(DEV), tab.to(DEV), cl.to(DEV))
    outs = [ops.paged_decode_attention(*args, **kw) for _ in range(3)]
    ops.check_status()
    assert (outs[0].float().cpu() - ref.float()).abs().max().item() < 2e-2
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


@pytest.mark.parametrize("chunks", [[(0, 300)], [(200, 1029), (0, 17)], [(0, 2048)]])
def test_paged_prefill_attention_contiguous_blocks(chunks):
    lens = [a + b for a, b in chunks]
    kc, vc, tab = _paged(len(chunks), lens, 8, 128, seed=4, contiguous=True)
    Tq = sum(b for _, b in chunks)
    q = torch.randn(Tq, 64, 128).to(torch.bfloat16)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor([b for _, b in chunks]), 0)), dtype=torch.int32)
    qs = torch.tensor([a for a, _ in chunks], dtype=torch.int32)
    cl = torch.tensor(lens, dtype=torch.int32)
    mq = max(b for _, b in chunks)
    ref = ops.paged_prefill_attention(q, kc, vc, tab, cu, qs, cl, mq)
    out = ops.paged_prefill_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), tab.to(DEV), cu.to(DEV), qs.to(DEV),
                                      cl.to(DEV), mq)
    ops.check_status()
    assert (out.float().cpu() - ref.float()).abs().max().item() < 2e-2


def test_decode_attention_tc_deterministic():
    lens = [4000, 1500]
    kc, vc, tab = _paged(2, lens, 8, 128, seed=9)
    q = torch.randn(2, 64, 128).to(torch.bfloat16).to(DEV)
    args = (kc.to(DEV), vc.to(DEV), tab.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV))
    a = ops.paged_decode_attention(q, *args)
    b = ops.paged_decode_attention(q, *args)
    assert torch.equal(a, b)


@pytest.mark.parametrize("D,Hq,Hk", [(128, 8, 2), (64, 4, 4), (128, 16, 2), (128, 10, 2), (128, 4, 4)])
@pytest.mark.parametrize("chunks", [[(0, 100)], [(0, 37), (50, 64), (7, 1)], [(0, 300)], [(200, 129), (0, 17)]])
@pytest.mark.parametrize("tc", [True, False])
def test_paged_prefill_attention(D, Hq, Hk, chunks, tc):
    """chunks: (q_start, q_len) per sequence; context = q_start + q_len."""
    lens = [a + b for a, b in chunks]
    kc, vc, tab = _paged(len(chunks), lens, Hk, D, seed=3)
    Tq = sum(b for _, b in chunks)
    q = torch.randn(Tq, Hq, D).to(torch.bfloat16)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor([b for _, b in chunks]), 0)), dtype=torch.int32)
    qs = torch.tensor([a for a, _ in chunks], dtype=torch.int32)
    cl = torch.tensor(lens, dtype=torch.int32)
    mq = max(b for _, b in chunks)
    ref = ops.paged_prefill_attention(q, kc, vc, tab, cu, qs, cl, mq)
    out = ops.paged_prefill_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), tab.to(DEV), cu.to(DEV), qs.to(DEV),
                                      cl.to(DEV), mq, allow_tc=tc)
    ops.check_status()
    assert (out.float().cpu() - ref.float()).abs().max().item() < 2e-2


def test_rmsnorm_and_add():
    x = torch.randn(5, 1024, device=DEV)
    d = torch.randn(5, 1024, device=DEV)
    w = torch.randn(1024, device=DEV)
    ref_x = x + d
    ref = ref_x * torch.rsqrt(ref_x.pow(2).mean(-1, keepdim=True) + 1e-5) * w
    xx = x.clone()
    h = ops.add_rmsnorm_(xx, d, w, 1e-5)
    assert torch.allclose(xx, ref_x)
    assert (h.float() - ref).abs().max().item() < 1e-2


def test_embedding_vocab_parallel():
    q, s = _qw(100, 64, 14)
    ids = torch.tensor([0, 99, 150, 250, 120], device=DEV)
    out = ops.embedding_q8(ids, q, s, vocab_start=100)
    ref = ops.embedding_q8(ids.cpu(), q.cpu(), s.cpu(), vocab_start=100)
    assert torch.allclose(out.cpu(), ref)


@pytest.mark.parametrize("M,V", [(1, 128256), (16, 128256), (16, 16032), (4, 40001), (300, 4099), (5000, 999)])
def test_argmax_split_matches_torch(M, V):
    """Split over many CTAs per row (atomicMax of packed keys), ties across slice boundaries, repeated calls
    (accumulators / tickets re-armed), rows beyond the split limit (one CTA per row)."""
    from hrm_flashrenderer_b200.parallel.dist import pack_argmax
    g = torch.Generator(device="cpu").manual_seed(M + V)
    for rep in range(3):
        logits = torch.randn(M, V, generator=g).to(DEV)
        if V > 9000:
            logits[0, V - 1] = 50.0
            logits[0, 3] = 50.0              # tie in another slice: lowest id wins
        keys = torch.empty(M, dtype=torch.int64, device=DEV)
        t = ops.argmax_rows(logits, vocab_start=7, keys=keys)
        val, idx = torch.max(logits.cpu(), -1)
        assert torch.equal(t.cpu(), idx + 7)
        assert torch.equal(keys.cpu(), pack_argmax(val, idx + 7))
    if V > 9000:
        assert t[0].item() == 10


def test_argmax_ties_lowest_index():
    logits = torch.randn(4, 5000, device=DEV)
    logits[1, 17] = 100.0
    logits[1, 4000] = 100.0
    keys = torch.empty(4, dtype=torch.int64, device=DEV)
    t = ops.argmax_rows(logits, vocab_start=10, keys=keys)
    assert t[1].item() == 27
    ref = torch.argmax(logits, -1) + 10
    assert torch.equal(t, ref)
    from hrm_flashrenderer_b200.parallel.dist import pack_argmax
    val, idx = torch.max(logits, -1)
    assert torch.equal(keys.cpu(), pack_argmax(val.cpu(), idx.cpu() + 10))
