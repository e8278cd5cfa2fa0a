"""The reference-named torch TP API (``compat.llama_tp``) on the engine, CPU: per-sequence KV pages, the distributed
greedy select, loading through a reference-style loader from an HF-style config, the low-level forward /
logits_last loop against generate_tp and the oracle, and TP=2 over gloo against TP=1."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from hrm_flashrenderer_b200.compat import llama_tp as lt
from hrm_flashrenderer_b200.config import TINY
from hrm_flashrenderer_b200.models.weights import QTensor, synth_weights

HF_TINY = {"hidden_size": 256, "num_attention_heads": 8, "num_key_value_heads": 2, "num_hidden_layers": 4,
           "intermediate_size": 688, "vocab_size": 1024, "rms_norm_eps": 1e-5, "rope_theta": 10000.0,
           "eos_token_id": 2, "bos_token_id": 1, "max_position_embeddings": 4096, "tie_word_embeddings": False,
           "model_type": "llama"}


class FakeLoader:
    """The reference loader interface over in-memory float tensors."""

    def __init__(self, tensors):
        self.t = tensors
        self.reads = []

    def get(self, key):
        self.reads.append(key)
        return self.t[key]

    def rows(self, key, a, b):
        return self.get(key)[a:b]

    def cols(self, key, a, b):
        return self.get(key)[:, a:b]


def _float_weights(seed=0):
    """Float weights whose per-row int8 quantisation reproduces synth_weights exactly (q * s with max |q| = 127)."""
    w = synth_weights(TINY, seed=seed)
    return {k: (v.dequant() if isinstance(v, QTensor) else v) for k, v in w.items()}, w


def _prompts(B=2, T=12, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(3, 1024, (B, T), generator=g)


# ------------------------------------------------------------------------------------------------ KV pages
def test_paged_kv_append_across_a_page_boundary_and_growth():
    """The reference's append check (flash_tests/test_append_fast.py:13-38): start 145, page 128, exact equality."""
    B, Hk, D, PS = 2, 3, 16, 128
    c = lt.PagedKVCache(B, Hk, D, page_size=PS, init_pages=1, device="cpu", dtype=torch.float32)
    T, start = 40, 145
    k = torch.randn(B, Hk, T, D)
    v = torch.randn(B, Hk, T, D)
    c.append(k, v, torch.arange(start, start + T))
    kp, vp, sl = c.get()
    assert kp.shape[2] == 2 and sl.tolist() == [start + T] * B and c.cur_len == start + T
    flat_k = kp.reshape(B, Hk, -1, D)
    flat_v = vp.reshape(B, Hk, -1, D)
    assert torch.equal(flat_k[:, :, start:start + T], k) and torch.equal(flat_v[:, :, start:start + T], v)
    c.append(k[:, :, :1], v[:, :, :1], torch.tensor([600]))       # grows to the next power of two of pages
    assert c.k_pages.shape[2] == 8 and torch.equal(c.k_pages.reshape(B, Hk, -1, D)[:, :, start:start + T], k)
    c.reset()
    assert c.cur_len == 0 and int(c.seqlen.sum()) == 0 and c.k_pages.shape[2] == 8


def test_paged_kv_append_per_row_positions():
    B, Hk, D = 3, 2, 8
    c = lt.PagedKVCache(B, Hk, D, page_size=16, init_pages=1, device="cpu", dtype=torch.float32)
    pos = torch.tensor([[0, 1], [20, 21], [5, 40]])
    k = torch.randn(B, Hk, 2, D)
    c.append(k, -k, pos)
    for b in range(B):
        for t in range(2):
            p = int(pos[b, t])
            assert torch.equal(c.k_pages[b, :, p // 16, p % 16], k[b, :, t])
            assert torch.equal(c.v_pages[b, :, p // 16, p % 16], -k[b, :, t])
    assert c.seqlen.tolist() == [2, 22, 41] and c.cur_len == 41
    with pytest.raises(ValueError):
        c.append(k, k, torch.zeros(2, 2, 2))


# ------------------------------------------------------------------------------------------------ argmax
def test_greedy_select_single_rank_ties_to_lowest_id():
    x = torch.tensor([[0.0, 3.0, 3.0, 1.0], [5.0, -1.0, 5.0, 5.0], [-2.0, -1.0, -3.0, -1.0]])
    assert lt.greedy_select_token_distributed(x).tolist() == [1, 0, 1]


# ------------------------------------------------------------------------------------------------ model
def test_config_forms_agree():
    class Obj:
        pass
    o = Obj()
    o.__dict__.update(HF_TINY)
    a = lt.TPLlamaForCausalLM(HF_TINY, 64, device="cpu").cfg
    b = lt.TPLlamaForCausalLM(o, 64, device="cpu").cfg
    c = lt.TPLlamaForCausalLM(TINY, 64, device="cpu").cfg
    for f in ("hidden", "layers", "heads", "kv_heads", "head_dim", "intermediate", "vocab", "rms_eps", "rope_theta",
              "eos_token_ids"):
        assert getattr(a, f) == getattr(b, f) == getattr(c, f), f


def test_loader_path_matches_oracle_and_low_level_loop():
    from hrm_flashrenderer_b200.models.oracle import OracleLlama
    fw, qw = _float_weights()
    loader = FakeLoader(fw)
    m = lt.TPLlamaForCausalLM(HF_TINY, max_seq_len=64, device="cpu").load_from_loader(loader)
    assert "lm_head.weight" in loader.reads
    ids = _prompts()
    n = 10
    out = lt.generate_tp(m, ids, n, eos_token_id=None, prefill_chunk_size=5)
    assert out.shape == (2, 12 + n) and torch.equal(out[:, :12], ids)
    ref = OracleLlama(TINY, qw, max_pos=128).generate(ids.tolist(), n)
    assert out[:, 12:].tolist() == ref

    # the reference's low-level decode loop: forward -> last hidden -> logits_last -> greedy select
    m.reset_all_caches()
    h = m.forward(ids, torch.arange(12), prefill=True)
    assert h.shape == (2, 12, 256)
    toks, cur = [], 12
    last = h[:, -1]
    for _ in range(n):
        nxt = lt.greedy_select_token_distributed(m.logits_last(last))
        toks.append(nxt)
        h1 = m.forward(nxt.view(2, 1), torch.tensor([cur]), prefill=False)
        last = h1[:, -1]
        cur += 1
    assert torch.stack(toks, 1).tolist() == ref


def test_generate_tp_stops_each_row_at_its_eos():
    fw, qw = _float_weights()
    m = lt.TPLlamaForCausalLM(HF_TINY, max_seq_len=64, device="cpu").load_weights(fw)
    ids = _prompts(B=2, T=8, seed=3)
    free = lt.generate_tp(m, ids, 12, eos_token_id=None)[:, 8:]
    eos = int(free[0, 3])               # the 4th token of row 0 acts as EOS
    out = lt.generate_tp(m, ids, 12, eos_token_id=[eos, 99999])[:, 8:]
    for b in range(2):
        row = free[b].tolist()
        stop = row.index(eos) + 1 if eos in row else len(row)
        assert out[b, :stop].tolist() == row[:stop]
        assert all(t == eos for t in out[b, stop:].tolist())
    assert out.shape[1] == max((free[b].tolist().index(eos) + 1) if eos in free[b].tolist() else 12
                               for b in range(2))


def test_forward_needs_weights_and_consistent_batch():
    m = lt.TPLlamaForCausalLM(HF_TINY, max_seq_len=64, device="cpu")
    with pytest.raises(RuntimeError):
        m.forward(torch.zeros(1, 2, dtype=torch.long), torch.arange(2))
    fw, _ = _float_weights()
    m.load_weights(fw)
    m.forward(_prompts(B=2, T=4), torch.arange(4))
    with pytest.raises(ValueError):
        m.forward(_prompts(B=3, T=1), torch.tensor([4]))
    m.reset_all_caches()
    assert m.forward(_prompts(B=3, T=4), torch.arange(4)).shape == (3, 4, 256)


# ------------------------------------------------------------------------------------------------ TP=2 (gloo)
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    from hrm_flashrenderer_b200.parallel.dist import init_dist, destroy
    torch.set_num_threads(2)
    init_dist(rank, world, "127.0.0.1", port, backend="gloo", timeout_s=60)
    try:
        fw, _ = _float_weights()
        loader = FakeLoader(fw)
        m = lt.TPLlamaForCausalLM(HF_TINY, max_seq_len=64, device="cpu").load_from_loader(loader)
        assert m.model.plan.world == world
        out = lt.generate_tp(m, _prompts(), 8, eos_token_id=None)
        m.reset_all_caches()
        h = m.forward(_prompts(), torch.arange(12))
        sel = lt.greedy_select_token_distributed(m.logits_last(h[:, -1]))
        q.put((rank, out.tolist(), sel.tolist()))
    finally:
        destroy()


def test_tp2_over_gloo_matches_tp1():
    fw, _ = _float_weights()
    m1 = lt.TPLlamaForCausalLM(HF_TINY, max_seq_len=64, device="cpu").load_weights(fw)
    ref = lt.generate_tp(m1, _prompts(), 8, eos_token_id=None).tolist()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(2):
        r, out, sel = q.get(timeout=300)
        res[r] = (out, sel)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]
    assert res[0][0] == ref
    assert res[0][1] == [row[12] for row in ref]


@pytest.mark.gpu
@pytest.mark.skipif(os.environ.get("HRM_TEST_COMPAT_GPU") != "1", reason="set HRM_TEST_COMPAT_GPU=1")
def test_gpu_generate_tp_and_low_level_first_token():
    """On the B200 (head_dim 128, the GPU kernels' shape): generate_tp against the oracle (f16 operands: a late
    divergence is allowed, as in the engine's own GPU oracle test), and the low-level forward / logits_last logits
    rank generate_tp's first token at the top."""
    from hrm_flashrenderer_b200.config import ModelConfig, RopeScaling
    from hrm_flashrenderer_b200.models.oracle import OracleLlama
    cfg = ModelConfig(name="gpu-small", hidden=1024, layers=2, heads=8, kv_heads=2, head_dim=128,
                      intermediate=2816, vocab=4096, rms_eps=1e-5, rope_theta=500000.0,
                      rope_scaling=RopeScaling(8.0, 1.0, 4.0, 8192), max_position_embeddings=8192)
    w = synth_weights(cfg, seed=0, norm_jitter=0.1)
    m = lt.TPLlamaForCausalLM(cfg, max_seq_len=128, device="cuda", max_batch=4, num_blocks=64).load_weights(w)
    ids = torch.randint(0, cfg.vocab, (2, 40), generator=torch.Generator().manual_seed(1)).cuda()
    out = lt.generate_tp(m, ids, 12, eos_token_id=None)
    assert out.is_cuda and out.shape == (2, 52)
    ref = OracleLlama(cfg, w, max_pos=512).generate(ids.cpu().tolist(), 12)
    for a, b in zip(out[:, 40:].cpu().tolist(), ref):
        n = next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), len(a))
        assert n >= 8, (a, b)
    m.reset_all_caches()
    h = m.forward(ids, torch.arange(40, device="cuda"))
    logits = m.logits_last(h[:, -1]).float().cpu()
    first = out[:, 40].cpu()
    for b in range(2):
        top = logits[b].max()
        assert logits[b, first[b]] >= top - 1e-2 * logits[b].abs().max(), (b, int(first[b]), int(logits[b].argmax()))
