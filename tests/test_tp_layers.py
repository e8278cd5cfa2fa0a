"""The reference-API tensor-parallel layers (``parallel/layers.py``): each layer at world 1 against plain fp32 math
of the same int8 weights, and a Column -> Row MLP, the vocab-parallel embedding and the LM head + distributed greedy
select at world 2 over gloo against world 1."""
import socket

import torch
import torch.multiprocessing as mp

from hrm_flashrenderer_b200.models.weights import quantize_rows
from hrm_flashrenderer_b200.parallel import layers as L

H, F, V = 64, 96, 128


def _w(seed):
    g = torch.Generator().manual_seed(seed)
    return {"up": torch.randn(F, H, generator=g) * 0.1, "down": torch.randn(H, F, generator=g) * 0.1,
            "bias": torch.randn(F, generator=g), "emb": torch.randn(V, H, generator=g),
            "head": torch.randn(V, H, generator=g) * 0.1, "norm": torch.rand(H, generator=g) + 0.5,
            "x": torch.randn(5, H, generator=g), "ids": torch.randint(0, V, (7,), generator=g)}


def _run(w):
    up = L.ColumnParallelLinear(H, F, bias=True)
    up.load_from_full(w["up"], w["bias"])
    down = L.RowParallelLinear(F, H)
    down.load_from_full(w["down"])
    emb = L.VocabParallelEmbedding(V, H)
    emb.load_from_full(w["emb"])
    head = L.VocabParallelLMHead(H, V)
    head.load_from_full(w["head"])
    norm = L.RMSNorm(H, 1e-5)
    norm.load_from_full(w["norm"])
    from hrm_flashrenderer_b200.parallel.dist import greedy_select_distributed
    h = up(w["x"])
    y = down(torch.nn.functional.silu(h))
    e = emb(w["ids"])
    logits = head(norm(e))
    tok = greedy_select_distributed(logits, head.vocab_start)
    return y, e, tok


def test_world1_matches_fp32_math():
    w = _w(0)
    y, e, tok = _run(w)
    dq = lambda m: quantize_rows(m).dequant()
    h = w["x"] @ dq(w["up"]).t() + w["bias"]
    ref_y = torch.nn.functional.silu(h) @ dq(w["down"]).t()
    assert torch.allclose(y, ref_y, rtol=1e-4, atol=1e-4)
    ref_e = dq(w["emb"])[w["ids"]]
    assert torch.allclose(e, ref_e, rtol=1e-5, atol=1e-6)
    n = ref_e * torch.rsqrt(ref_e.pow(2).mean(-1, keepdim=True) + 1e-5) * w["norm"]
    assert tok.tolist() == (n @ dq(w["head"]).t()).argmax(-1).tolist()
    rep = L.ReplicatedLinear(H, F)
    rep.load_from_full(quantize_rows(w["up"]))
    assert torch.allclose(rep(w["x"]), w["x"] @ dq(w["up"]).t(), rtol=1e-4, atol=1e-4)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    from hrm_flashrenderer_b200.parallel.dist import init_dist, destroy
    torch.set_num_threads(1)
    init_dist(rank, world, "127.0.0.1", port, backend="gloo", timeout_s=60)
    try:
        y, e, tok = _run(_w(0))
        q.put((rank, y, e, tok))
    finally:
        destroy()


def test_world2_matches_world1():
    y1, e1, t1 = _run(_w(0))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(2):
        r, y, e, tok = q.get(timeout=300)
        res[r] = (y, e, tok)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in (0, 1):
        y, e, tok = res[r]
        assert torch.allclose(y, y1, rtol=1e-4, atol=1e-4)
        assert torch.equal(e, e1)
        assert tok.tolist() == t1.tolist()
