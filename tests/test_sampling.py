"""Temperature / top-k sampling on CPU: the noise generator, the Gumbel-max draw against softmax(v / T), the top-k
threshold (local and sharded over ranks), engine / scheduler reproducibility and the request fields."""
import math

import pytest
import torch

from hrm_flashrenderer_b200 import ops
from hrm_flashrenderer_b200.runtime.sampling import SampleMeta, SamplingParams, sampling_from_request


def test_gumbel_noise_moments_and_determinism():
    g = ops.gumbel_noise_host(123, 7, range(200000))
    assert abs(float(g.mean()) - 0.5772156649) < 0.01
    assert abs(float(g.var()) - math.pi ** 2 / 6) < 0.03
    assert torch.equal(g[:100], ops.gumbel_noise_host(123, 7, range(100)))
    assert not torch.equal(g[:100], ops.gumbel_noise_host(123, 8, range(100)))
    assert not torch.equal(g[:100], ops.gumbel_noise_host(124, 7, range(100)))
    assert torch.isfinite(g).all()


def _draws(logits, inv_temp, n, thresh=None, pos=3):
    R = n
    L = logits.expand(R, -1).contiguous()
    seeds = torch.arange(R, dtype=torch.int64) * 7919 + 1
    t = None if thresh is None else torch.full((R,), float(thresh))
    return ops.sample_rows(L, 0, torch.full((R,), inv_temp), seeds, torch.full((R,), pos, dtype=torch.int32), t)


def test_gumbel_max_draws_follow_softmax():
    logits = torch.tensor([[2.0, 1.0, 0.0, -1.0, 0.5]])
    T = 0.7
    n = 8000
    tok = _draws(logits, 1 / T, n)
    freq = torch.bincount(tok, minlength=5).float() / n
    p = torch.softmax(logits[0] / T, 0)
    # each frequency within 4.5 standard deviations of its probability
    assert ((freq - p).abs() <= 4.5 * (p * (1 - p) / n).sqrt() + 1e-9).all(), (freq, p)


def test_top_k_threshold_restricts_and_renormalises():
    logits = torch.tensor([[2.0, 1.0, 0.0, -1.0, 0.5]])
    thr = ops.kth_largest(logits, torch.tensor([2], dtype=torch.int32))
    assert float(thr[0]) == 1.0
    n = 6000
    tok = _draws(logits, 1.0, n, thresh=float(thr[0]))
    assert set(tok.tolist()) <= {0, 1}
    p0 = math.exp(2.0) / (math.exp(2.0) + math.exp(1.0))
    f0 = float((tok == 0).float().mean())
    assert abs(f0 - p0) < 4.5 * math.sqrt(p0 * (1 - p0) / n)


def test_greedy_rows_are_argmax_and_vocab_offset():
    g = torch.Generator().manual_seed(0)
    L = torch.randn(6, 40, generator=g)
    z = torch.zeros(6)
    tok = ops.sample_rows(L, 100, z, torch.zeros(6, dtype=torch.int64), torch.zeros(6, dtype=torch.int32))
    assert torch.equal(tok, L.argmax(-1) + 100)


def test_kth_largest_and_candidates_match_topk():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(5, 300, generator=g)
    x[4] = torch.randint(0, 4, (300,), generator=g).float()          # heavy ties
    k = torch.tensor([1, 7, 64, 0, 100], dtype=torch.int32)
    thr = ops.kth_largest(x, k)
    for r in range(5):
        kr = int(k[r])
        want = -float("inf") if kr == 0 else float(torch.topk(x[r], kr).values[-1])
        assert float(thr[r]) == want
    cand = ops.topk_candidates(x, thr, k, 128)
    for r in range(5):
        kr = int(k[r])
        got = torch.sort(cand[r], descending=True).values[:kr]
        if kr:
            assert torch.equal(got, torch.topk(x[r], kr).values)
        assert (cand[r, kr:] == -float("inf")).all()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_threshold_equals_global(world):
    """Every rank's candidates (its local top-k, or its whole shard when the shard is smaller than k), joined, give
    the global k-th largest: the rule the tensor-parallel pick uses."""
    g = torch.Generator().manual_seed(world)
    V = 1000
    x = torch.randn(3, V, generator=g)
    x[2] = torch.randint(0, 5, (V,), generator=g).float()
    k = torch.tensor([5, 200, 33], dtype=torch.int32)
    kmax = 256
    shards = torch.chunk(x, world, dim=1)
    cands = [ops.topk_candidates(s.contiguous(), ops.kth_largest(s.contiguous(), k), k, kmax) for s in shards]
    joined = torch.cat(cands, dim=1)
    assert torch.equal(ops.kth_largest(joined, k), ops.kth_largest(x, k))


def test_sampling_params_validation_and_request_fields():
    assert sampling_from_request(None, None, None) is None
    assert sampling_from_request(0, 5, 1) is None
    sp = sampling_from_request(0.5, 3, 9)
    assert sp == SamplingParams(temperature=0.5, top_k=3, seed=9) and sp.inv_temp == 2.0
    a, b = sampling_from_request(1.0), sampling_from_request(1.0)
    assert a.seed != b.seed                                   # unseeded requests do not share noise
    for bad in ((-1.0, 0, 0), (1.0, -1, 0), (1.0, ops.SAMPLE_MAX_TOP_K + 1, 0), (float("nan"), 0, 0)):
        with pytest.raises(ValueError):
            sampling_from_request(*bad)


def test_sample_meta_fill_pads_greedy_rows():
    m = SampleMeta.alloc(4, "cpu")
    m.fill([SamplingParams(2.0, 5, 7), None], positions=[10, 11])
    assert m.inv_temp.tolist() == [0.5, 0.0, 0.0, 0.0]
    assert m.top_k.tolist() == [5, 0, 0, 0] and m.seed.tolist() == [7, 0, 0, 0] and m.pos.tolist() == [10, 11, 0, 0]


def _engine():
    from hrm_flashrenderer_b200.config import TINY, EngineConfig
    from hrm_flashrenderer_b200.models.llama import LlamaW8
    from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
    m = LlamaW8.synthesize(TINY, device="cpu", max_pos=256 + 16)
    return InferenceEngine(m, EngineConfig(max_seq_len=256, max_batch=8, use_cuda_graphs=False), num_blocks=128)


def test_engine_sampling_reproducible_and_batch_independent():
    eng = _engine()
    pr = [[1, 2, 3, 4, 5], [9, 8, 7]]
    sp = SamplingParams(temperature=1.0, top_k=50, seed=3)
    a = eng.generate(pr, 10, stop_on_eos=False, sampling=[sp, None])
    b = eng.generate(pr, 10, stop_on_eos=False, sampling=[sp, None])
    assert a == b
    assert a[1] == eng.generate(pr, 10, stop_on_eos=False)[1]                      # greedy row unchanged
    alone = eng.generate([pr[0]], 10, stop_on_eos=False, sampling=sp)[0]
    assert alone == a[0]                                                           # batch composition is irrelevant
    other = eng.generate([pr[0]], 10, stop_on_eos=False, sampling=SamplingParams(1.0, 50, 4))[0]
    assert other != alone


def test_scheduler_carries_sampling():
    from hrm_flashrenderer_b200.runtime.scheduler import Scheduler
    eng = _engine()
    sp = SamplingParams(temperature=0.9, top_k=10, seed=21)
    want = eng.generate([[4, 5, 6, 7]], 8, stop_on_eos=False, sampling=sp)[0]
    sched = Scheduler(eng).start()
    try:
        got = sched.generate([4, 5, 6, 7], 8, timeout=120, stop_on_eos=False, sampling=sp)
        greedy = sched.generate([4, 5, 6, 7], 8, timeout=120, stop_on_eos=False)
    finally:
        sched.stop()
    assert got == want
    assert greedy == eng.generate([[4, 5, 6, 7]], 8, stop_on_eos=False)[0]
