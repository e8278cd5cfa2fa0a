"""Config 1: tiny Llama on CPU/gloo, TP world_size=2 must match the unsharded TP=1 run token-for-token.

Architecture: 4 layers, hidden 256, 8 q heads / 2 kv heads (head_dim 32), SwiGLU 688, vocab 1024, eps 1e-5,
theta 1e4, no bias; weights N(0, 0.02) from seed 0 quantised per row; paged KV block 16; 2 prompts x 16 ids from
seed 1; 32 greedy tokens.
"""
import socket

import torch
import torch.multiprocessing as mp

from hrm_flashrenderer_b200.config import TINY, EngineConfig
from hrm_flashrenderer_b200.models.weights import synth_weights


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompts():
    g = torch.Generator().manual_seed(1)
    return [torch.randint(0, 1024, (16,), generator=g).tolist() for _ in range(2)]


def _run(rank, world, port, q, sp=False, prompts=None, overlap=1, replicate=True, sampling=None):
    from hrm_flashrenderer_b200.parallel.dist import init_dist, destroy
    from hrm_flashrenderer_b200.parallel.comm import TPComm
    from hrm_flashrenderer_b200.models.llama import LlamaW8
    from hrm_flashrenderer_b200.runtime.engine import InferenceEngine
    torch.set_num_threads(2)
    init_dist(rank, world, "127.0.0.1", port, backend="gloo", timeout_s=60)
    try:
        w = synth_weights(TINY, seed=0)
        comm = TPComm()
        model = LlamaW8.from_weights(TINY, w, rank=rank, world=world, device="cpu", comm=comm, max_pos=256,
                                     replicate_embedding=replicate)
        assert model.embed_replicated == (world > 1 and replicate)
        calls = {"all_reduce_": 0}
        inner = comm.all_reduce_

        def counted(t, *a, **k):
            calls["all_reduce_"] += 1
            return inner(t, *a, **k)
        comm.all_reduce_ = counted
        eng = InferenceEngine(model, EngineConfig(max_seq_len=160, max_batch=4, use_cuda_graphs=False,
                                                  sequence_parallel=sp, prefill_overlap_chunks=overlap),
                              num_blocks=48)
        out = eng.generate(prompts or _prompts(), 32, stop_on_eos=False, sampling=sampling)
        q.put((rank, out, calls["all_reduce_"]))
    finally:
        destroy()


def _spawn(world, sp=False, prompts=None, overlap=1, replicate=True, with_calls=False, sampling=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_run, args=(r, world, port, q, sp, prompts, overlap, replicate, sampling))
          for r in range(world)]
    for p in ps:
        p.start()
    res, calls = {}, {}
    for _ in range(world):
        r, out, n = q.get(timeout=300)
        res[r], calls[r] = out, n
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return (res, calls) if with_calls else res


def test_tp2_matches_tp1_token_for_token():
    tp1 = _spawn(1)[0]
    tp2 = _spawn(2)
    assert tp2[0] == tp2[1], "ranks disagree"
    assert tp2[0] == tp1
    assert all(len(o) == 32 for o in tp1)


def test_tp1_matches_oracle():
    from hrm_flashrenderer_b200.models.oracle import OracleLlama
    w = synth_weights(TINY, seed=0)
    ref = OracleLlama(TINY, w, max_pos=256).generate(_prompts(), 32)
    assert _spawn(1)[0] == ref


def test_tp2_sequence_parallel_prefill_matches_tp1():
    """Prefill with a token-sharded residual (reduce-scatter / all-gather) gives the TP=1 tokens; 2 prompts x 16
    tokens = 32 rows split 16 / 16 per rank."""
    tp1 = _spawn(1)[0]
    sp = _spawn(2, sp=True)
    assert sp[0] == sp[1] == tp1


def test_tp2_sequence_parallel_odd_rows():
    """23 prompt rows over 2 ranks: one pad row (zeros, slot -1) on the last rank."""
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (7, 11, 5)]
    assert _spawn(2, sp=True, prompts=prompts)[0] == _spawn(1, prompts=prompts)[0]


def test_tp2_prefill_overlap_chunks_match_tp1():
    """Row-parallel GEMM + asynchronous all-reduce pipelined over 2 row chunks (2 x 80 = 160 prompt rows)."""
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 1024, (80,), generator=g).tolist() for _ in range(2)]
    assert _spawn(2, prompts=prompts, overlap=2)[0] == _spawn(1, prompts=prompts)[0]


def test_tp2_embedding_layouts_match_tp1():
    """The whole embedding table on every rank (default) and the reference's vocab-parallel table give the TP=1
    tokens; the replicated table saves one all-reduce per forward (prefill and every decode step)."""
    tp1 = _spawn(1)[0]
    rep, n_rep = _spawn(2, with_calls=True)
    vp, n_vp = _spawn(2, replicate=False, with_calls=True)
    assert rep[0] == rep[1] == tp1
    assert vp[0] == vp[1] == tp1
    forwards = 1 + 31   # one prefill forward (both prompts in one batch) and 31 decode steps
    assert n_vp[0] - n_rep[0] == forwards, (n_vp, n_rep)


def test_tp2_sequence_parallel_vocab_parallel_embedding():
    """Sequence-parallel prefill with the vocab-parallel table (reduce-scatter of the lookup) and with the
    replicated table (each rank looks up its own token rows), odd row count."""
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (7, 11, 5)]
    tp1 = _spawn(1, prompts=prompts)[0]
    assert _spawn(2, sp=True, prompts=prompts, replicate=False)[0] == tp1
    assert _spawn(2, sp=True, prompts=prompts)[0] == tp1


def test_tp2_sampled_decode_matches_tp1():
    """Temperature / top-k sampling: the noise is keyed by (seed, position, global token id) and the top-k threshold
    is the global one (local candidates joined by one all-gather), so TP = 2 draws the TP = 1 tokens; a greedy row in
    the same batch keeps its greedy tokens."""
    from hrm_flashrenderer_b200.runtime.sampling import SamplingParams
    sampling = [SamplingParams(temperature=0.8, top_k=20, seed=11), None]
    tp1 = _spawn(1, sampling=sampling)[0]
    tp2 = _spawn(2, sampling=sampling)
    assert tp2[0] == tp2[1] == tp1
    assert tp1[1] == _spawn(1)[0][1]          # the greedy row is unchanged
    assert tp1[0] != _spawn(1)[0][0]          # the sampled row is not the greedy continuation
