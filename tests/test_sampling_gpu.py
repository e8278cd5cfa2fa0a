"""Sampling kernels on the GPU: the radix-select top-k threshold and candidates against torch.topk, the sampled argmax
against the host computation of the same noise, the draw frequencies against softmax(v / T), and sampled decoding
through the engine (graph replay equals eager steps, reproducible, greedy rows unchanged)."""
import pytest
import torch

from hrm_flashrenderer_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("V", [1000, 128256])
def test_kth_largest_and_candidates_match_topk(V):
    g = torch.Generator(device="cpu").manual_seed(V)
    x = torch.randn(8, V, generator=g)
    x[6] = torch.randint(0, 7, (V,), generator=g).float()          # heavy ties
    x[7] = -x[7].abs()                                               # all negative
    ks = [1, 5, 50, 1024, 0, V, 20, 300]
    k = torch.tensor(ks, dtype=torch.int32)
    xd, kd = x.cuda(), k.cuda()
    thr = ops.kth_largest(xd, kd)
    cand = ops.topk_candidates(xd, thr, kd, 1024)
    torch.cuda.synchronize()
    thr, cand = thr.cpu(), cand.cpu()
    for r, kr in enumerate(ks):
        if kr <= 0 or kr >= V:
            assert thr[r] == -float("inf")
            continue
        top = torch.topk(x[r], kr).values
        assert float(thr[r]) == float(top[-1]), r
        kk = min(kr, 1024)
        assert torch.equal(torch.sort(cand[r], descending=True).values[:kk], top[:kk]), r
        assert (cand[r, kk:] == -float("inf")).all()


def test_sampled_argmax_matches_host_noise():
    """The kernel's pick equals the argmax of v * inv_temp + noise computed on the host with the same generator (fp32
    log on both sides: a mismatch would need two perturbed values within a few ulps)."""
    g = torch.Generator(device="cpu").manual_seed(3)
    R, V = 64, 32000
    L = torch.randn(R, V, generator=g) * 3
    inv_t = torch.rand(R, generator=g) * 2 + 0.25
    inv_t[::7] = 0.0                                                 # greedy rows
    seed = torch.randint(0, 2 ** 62, (R,), generator=g, dtype=torch.int64)
    pos = torch.randint(0, 8192, (R,), generator=g, dtype=torch.int32)
    thr = ops.kth_largest(L, torch.tensor([0 if r % 3 else 40 for r in range(R)], dtype=torch.int32))
    want = ops.sample_rows(L, 1000, inv_t, seed, pos, thr)
    keys = torch.empty(R, dtype=torch.int64, device="cuda")
    got = ops.sample_rows(L.cuda(), 1000, inv_t.cuda(), seed.cuda(), pos.cuda(), thr.cuda(), keys=keys)
    torch.cuda.synchronize()
    ops.check_status()
    assert (got.cpu() == want).float().mean() >= 0.98
    from hrm_flashrenderer_b200.parallel.dist import unpack_argmax
    assert torch.equal(unpack_argmax(keys).cpu(), got.cpu())


def test_sampled_frequencies_follow_softmax():
    logits = torch.tensor([2.0, 1.0, 0.0, -1.0, 0.5, -3.0, 1.5, 0.25])
    T, n = 0.8, 20000
    L = logits.expand(n, -1).contiguous().cuda()
    tok = ops.sample_rows(L, 0, torch.full((n,), 1 / T, device="cuda"),
                          torch.arange(n, dtype=torch.int64, device="cuda") * 104729 + 17,
                          torch.full((n,), 11, dtype=torch.int32, device="cuda"))
    freq = torch.bincount(tok.cpu(), minlength=8).float() / n
    p = torch.softmax(logits / T, 0)
    assert ((freq - p).abs() <= 4.5 * (p * (1 - p) / n).sqrt() + 1e-9).all(), (freq, p)
    # top-3 restriction: only the three largest logits, renormalised
    thr = ops.kth_largest(L, torch.full((n,), 3, dtype=torch.int32, device="cuda"))
    tok = ops.sample_rows(L, 0, torch.full((n,), 1 / T, device="cuda"),
                          torch.arange(n, dtype=torch.int64, device="cuda") * 104729 + 17,
                          torch.full((n,), 11, dtype=torch.int32, device="cuda"), thr)
    assert set(tok.unique().tolist()) <= {0, 1, 6}
    q = torch.softmax(logits[[0, 1, 6]] / T, 0)
    f = torch.stack([(tok == t).float().mean().cpu() for t in (0, 1, 6)])
    assert ((f - q).abs() <= 4.5 * (q * (1 - q) / n).sqrt()).all(), (f, q)


def test_engine_sampled_decode_graph_equals_eager():
    from hrm_flashrenderer_b200.config import EngineConfig, ModelConfig
    from hrm_flashrenderer_b200.models.llama import LlamaW8
    from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
    from hrm_flashrenderer_b200.runtime.sampling import SamplingParams
    cfg = ModelConfig(name="gpu-sample", hidden=1024, layers=2, heads=8, kv_heads=2, head_dim=128,
                      intermediate=2816, vocab=4096, rms_eps=1e-5, rope_theta=500000.0)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (12, 5, 30)]
    sampling = [SamplingParams(0.9, 20, 7), None, SamplingParams(1.5, 0, 8)]
    outs = {}
    for graphs in (True, False):
        m = LlamaW8.synthesize(cfg, device="cuda", max_pos=512 + 16)
        eng = InferenceEngine(m, EngineConfig(max_seq_len=512, max_batch=8, use_cuda_graphs=graphs), num_blocks=256)
        outs[graphs] = eng.generate(prompts, 24, stop_on_eos=False, sampling=sampling)
        again = eng.generate(prompts, 24, stop_on_eos=False, sampling=sampling)
        assert again == outs[graphs]
        greedy = eng.generate(prompts, 24, stop_on_eos=False)
        assert greedy[1] == outs[graphs][1] and greedy[0] != outs[graphs][0]
    ops.check_status()
    assert outs[True] == outs[False]
