"""Llama / Qwen2 decoder on the sm_100a kernels, tensor-parallel over one process per GPU.

Per layer and token batch (rows = tokens of all scheduled sequences, decode or chunked prefill):

    h   = rmsnorm(x)                         (fp32 residual x -> f16 GEMM operand)
    q   = QKV GEMM + bias + RoPE, K/V -> paged cache          (one kernel)
    o   = paged attention(q)                 (decode split-K or varlen causal prefill)
    x  += all_reduce(o @ Wo^T) ; h = rmsnorm(x)               (fused GEMM+AR+residual+norm when TP > 1)
    a   = silu(h @ Wg^T) * (h @ Wu^T)        (one kernel, gate/up interleaved per tile)
    x  += all_reduce(a @ Wd^T) ; h = rmsnorm(x)

Reference counterparts: ``TPLlamaAttention`` / ``TPLlamaMLP`` / ``TPLlamaBlock`` / ``TPLlamaForCausalLM``
(``engine/llama_tp.py:110-311``) and the native engine's per-layer loop (``scripts/deepseek_native_engine.sh:1041-1099``).
Semantics follow HF (rotate-half RoPE with llama3 scaling, ``kv_head = head // group``, Qwen2 QKV bias), not the
reference's quirks.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import TYPE_CHECKING, Dict, List, Optional, Tuple

import torch

from .. import ops
from ..config import ModelConfig
from ..models.oracle import rope_tables
from ..models.weights import (QTensor, Tensorish, ShardPlan, layer_names, shard_plan, synth_matrix, matrix_shapes,
                              vector_shapes, EMBED, FINAL_NORM, LM_HEAD, get_lm_head)
from ..runtime.kv_cache import PagedKVPool

if TYPE_CHECKING:
    from ..runtime.sampling import SampleMeta


@dataclass
class LayerWeights:
    w_qkv: torch.Tensor
    s_qkv: torch.Tensor
    b_qkv: Optional[torch.Tensor]
    w_o: torch.Tensor
    s_o: torch.Tensor
    w_gu: torch.Tensor
    s_gu: torch.Tensor
    w_d: torch.Tensor
    s_d: torch.Tensor
    ln1: torch.Tensor
    ln2: torch.Tensor


@dataclass
class BatchMeta:
    """Device-side description of one forward step (all int32 unless noted).

    ``ids`` int64 [T]; ``positions`` [T]; ``slots`` [T] (block*bs + offset, -1 = no KV write);
    decode: ``block_tables`` [B, maxb], ``context_lens`` [B]; prefill: additionally ``cu_q`` [S+1], ``q_start`` [S],
    ``max_q``; ``last_rows`` int64 [S] rows whose hidden state feeds the lm_head.
    """

    ids: torch.Tensor
    positions: torch.Tensor
    slots: torch.Tensor
    block_tables: torch.Tensor
    context_lens: torch.Tensor
    last_rows: torch.Tensor
    is_decode: bool
    cu_q: Optional[torch.Tensor] = None
    q_start: Optional[torch.Tensor] = None
    max_q: int = 1
    attn_splits: int = 0
    attn_keys_per_split: int = 0
    sample: Optional["SampleMeta"] = None   # per-row temperature / top-k / seed / position; None = greedy


def pack_layer(cfg: ModelConfig, w: Dict[str, Tensorish], l: int, device) -> LayerWeights:
    """Pack one (already sharded) layer into the kernel layouts: fused QKV rows, interleaved gate/up tiles."""
    n = layer_names(l)
    q, k, v = w[n["q"]], w[n["k"]], w[n["v"]]
    w_qkv = torch.cat([q.q, k.q, v.q], 0).to(device).contiguous()
    s_qkv = torch.cat([q.scale, k.scale, v.scale], 0).to(device, torch.float32).contiguous()
    b_qkv = None
    if cfg.qkv_bias:
        b_qkv = torch.cat([w[n["bq"]], w[n["bk"]], w[n["bv"]]], 0).to(device, torch.float32).contiguous()
    g, u = w[n["gate"]], w[n["up"]]
    w_gu, s_gu = ops.interleave_gate_up(g.q.to(device), u.q.to(device), g.scale.to(device), u.scale.to(device))
    o, d = w[n["o"]], w[n["down"]]
    w_o, w_d = o.q.to(device).contiguous(), d.q.to(device).contiguous()
    if torch.device(device).type == "cuda":   # GPU layout: pre-tiled blocks streamed by contiguous bulk copies
        w_qkv, w_o, w_gu, w_d = (ops.tile_w8(t) for t in (w_qkv, w_o, w_gu, w_d))
    return LayerWeights(
        w_qkv=w_qkv, s_qkv=s_qkv, b_qkv=b_qkv,
        w_o=w_o, s_o=o.scale.to(device, torch.float32).contiguous(),
        w_gu=w_gu, s_gu=s_gu.to(torch.float32),
        w_d=w_d, s_d=d.scale.to(device, torch.float32).contiguous(),
        ln1=w[n["ln1"]].to(device, torch.float32).contiguous(), ln2=w[n["ln2"]].to(device, torch.float32).contiguous())


class LlamaW8:
    """Int8-weight decoder shard for TP rank ``plan.rank`` of ``plan.world`` on one CUDA device."""

    def __init__(self, cfg: ModelConfig, plan: ShardPlan, layers: List[LayerWeights], embed: QTensor,
                 lm_head: QTensor, final_norm: torch.Tensor, device, comm=None, max_pos: int = 8192,
                 head_pretiled: bool = False):
        self.cfg, self.plan, self.layers, self.device = cfg, plan, layers, torch.device(device)
        self.embed_q, self.embed_s = embed.q.contiguous(), embed.scale.contiguous()
        # The embedding table is either this rank's vocab slice (vocab-parallel: lookup, then a sum over ranks) or
        # the whole table on every rank (~1 GB int8 for a 128k x 8192 vocab): then the lookup is local and the
        # collective disappears.  Same rows either way (the non-owners' contributions are exact zeros).
        self.embed_replicated = plan.world > 1 and self.embed_q.shape[0] == cfg.vocab
        self.embed_start = 0 if self.embed_q.shape[0] == cfg.vocab else plan.vocab_start
        self.head_q, self.head_s = lm_head.q.contiguous(), lm_head.scale.contiguous()
        if self.head_q.is_cuda and not head_pretiled:
            self.head_q = ops.tile_w8(self.head_q)
        self.final_norm = final_norm
        self.comm = comm
        self.q_rows = plan.local_heads * cfg.head_dim
        self.kv_rows = plan.local_kv_heads * cfg.head_dim
        cos, sin = rope_tables(cfg, max_pos)
        self.cos, self.sin = cos.to(self.device).contiguous(), sin.to(self.device).contiguous()
        self.max_pos = max_pos
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.kv: Optional[PagedKVPool] = None
        self.symm = None   # SymmetricWorkspace: enables the fused GEMM + all-reduce kernels when TP > 1
        self.sequence_parallel = False   # prefill: token-sharded residual between blocks (TP > 1)
        self.chain_layers = False        # decode: o_proj, gate/up, down, next QKV in one multi-phase GEMM launch
        self.prefill_overlap_chunks = 1  # TP prefill: row-parallel GEMM + all-reduce pipelined over this many chunks
        self.prefill_comm_sms = 8        # SMs the pipelined GEMM leaves free for the collective's kernels
        # Per-step statistics for telemetry (off unless set before the first decode graph is captured): the greedy
        # token's negative log-probability and the final hidden row of every sampled row, in fixed buffers that
        # graph replays rewrite in place.
        self.collect_stats = False
        self.stat_nll: Optional[torch.Tensor] = None
        self.stat_hidden: Optional[torch.Tensor] = None

    def enable_fused_collectives(self, group=None) -> None:
        """Allocate / exchange the NVLink symmetric buffers (collective over the TP group)."""
        if self.plan.world > 1 and self.device.type == "cuda" and self.symm is None:
            from ..parallel.symm import SymmetricWorkspace
            self.symm = SymmetricWorkspace(self.plan.rank, self.plan.world, self.device,
                                           max_tiles=max(64, self.cfg.hidden // 128), max_bn=64, group=group)

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_dsi8(cls, path: str, rank: int = 0, world: int = 1, device="cuda", comm=None, max_pos: int = 8192,
                  cache_dir: Optional[str] = None, replicate_embedding: bool = True) -> "LlamaW8":
        """Load a DSI8 export for TP rank ``rank`` of ``world``.  With ``cache_dir`` the packed shard (fused QKV,
        interleaved gate/up, GPU tile layout) is kept in a per-rank cache file keyed by the export's fingerprint,
        the TP layout and the packing version, so later starts skip reading, sharding and re-tiling the export."""
        from .packed_cache import load_packed, save_packed, cache_path
        from ..formats.dsi8 import read_dsi8
        cp = cache_path(cache_dir, path, rank, world, device) if cache_dir else None
        if cp is not None and cp.is_file():
            return load_packed(cls, cp, device, comm, max_pos)
        cfg, w = read_dsi8(path)
        model = cls.from_weights(cfg, w, rank=rank, world=world, device=device, comm=comm, max_pos=max_pos,
                                 replicate_embedding=replicate_embedding)
        if cp is not None:
            save_packed(model, cp)
        return model

    @classmethod
    def from_weights(cls, cfg: ModelConfig, weights: Dict[str, Tensorish], rank: int = 0, world: int = 1,
                     device="cuda", comm=None, max_pos: int = 8192, replicate_embedding: bool = True) -> "LlamaW8":
        """``replicate_embedding`` (TP > 1): every rank keeps the whole embedding table, so the lookup needs no
        collective; False keeps the reference's vocab-parallel embedding (``tp/vocab_parallel.py:9-57``)."""
        from .weights import shard_weights
        plan = shard_plan(cfg, rank, world)
        w = shard_weights(cfg, weights, rank, world) if world > 1 else dict(weights)
        if world == 1:
            w[LM_HEAD] = get_lm_head(cfg, weights)
        elif replicate_embedding:
            w[EMBED] = weights[EMBED]
        layers = [pack_layer(cfg, w, l, device) for l in range(cfg.layers)]
        return cls(cfg, plan, layers, w[EMBED].to(device), w[LM_HEAD].to(device),
                   w[FINAL_NORM].to(device, torch.float32), device, comm, max_pos)

    @classmethod
    def synthesize(cls, cfg: ModelConfig, rank: int = 0, world: int = 1, device="cuda", seed: int = 0,
                   comm=None, max_pos: int = 8192, norm_jitter: float = 0.0,
                   replicate_embedding: bool = True) -> "LlamaW8":
        """Random-init int8 weights generated directly on the device, layer by layer (70B never exists in fp32).

        Matrix ``i`` (DSI8 record order) draws from a generator seeded ``seed*1000003 + i`` exactly like
        :func:`~hrm_flashrenderer_b200.models.weights.synth_weights`, so a shard equals the slice of the full model.
        """
        from .weights import shard_weights
        dev = torch.device(device)
        plan = shard_plan(cfg, rank, world)
        shapes = list(matrix_shapes(cfg))
        idx_of = {name: i for i, (name, _) in enumerate(shapes)}
        vec = {}
        base = 10_000_000
        for i, (name, n) in enumerate(vector_shapes(cfg)):
            g = torch.Generator(device="cpu").manual_seed(seed * 1_000_003 + base + i)
            if name.endswith("layernorm.weight") or name == FINAL_NORM:
                v = torch.ones(n) + (torch.randn(n, generator=g) * norm_jitter if norm_jitter else 0.0)
            else:
                v = torch.randn(n, generator=g) * 0.02
            vec[name] = v.to(torch.float32)

        def mat(name):
            rows, cols = dict(shapes)[name]
            return synth_matrix(rows, cols, seed=seed * 1_000_003 + idx_of[name], device=dev)

        layers = []
        for l in range(cfg.layers):
            n = layer_names(l)
            full = {k: mat(n[k]) for k in ("q", "k", "v", "o", "gate", "up", "down")}
            lw = {n[k]: t for k, t in full.items()}
            for k in ("ln1", "ln2", "bq", "bk", "bv"):
                if n[k] in vec:
                    lw[n[k]] = vec[n[k]]
            sub_cfg = cfg.with_layers(1)
            # re-key layer l as layer 0 for sharding/packing helpers
            re = {name.replace(f"model.layers.{l}.", "model.layers.0."): t for name, t in lw.items()}
            if world > 1:
                re.update({EMBED: QTensor(torch.zeros(cfg.vocab, 1, dtype=torch.int8), torch.ones(cfg.vocab)),
                           LM_HEAD: QTensor(torch.zeros(cfg.vocab, 1, dtype=torch.int8), torch.ones(cfg.vocab)),
                           FINAL_NORM: vec[FINAL_NORM]})
                re = shard_weights(sub_cfg, re, rank, world)
            layers.append(pack_layer(sub_cfg, re, 0, dev))
            del full, lw, re
        emb = mat(EMBED)
        head = emb if cfg.tie_embeddings else mat(LM_HEAD)
        v0, v1 = plan.vocab_start, plan.vocab_start + plan.vocab_per_rank
        head = head.rows(v0, v1).contiguous()
        if not replicate_embedding:
            emb = emb.rows(v0, v1).contiguous()
        return cls(cfg, plan, layers, emb, head, vec[FINAL_NORM].to(dev), dev, comm, max_pos)

    def weight_bytes(self) -> int:
        tot = 0
        for L in self.layers:
            for t in (L.w_qkv, L.w_o, L.w_gu, L.w_d):
                tot += t.numel()
        return tot + self.embed_q.numel() + self.head_q.numel()

    # ------------------------------------------------------------------ KV cache
    def alloc_kv(self, num_blocks: int, block_size: int = 16) -> PagedKVPool:
        self.kv = PagedKVPool(self.cfg.layers, num_blocks, self.plan.local_kv_heads, self.cfg.head_dim, block_size,
                              torch.bfloat16, self.device)
        return self.kv

    # ------------------------------------------------------------------ forward
    def _all_reduce_add_norm(self, x: torch.Tensor, partial: torch.Tensor, gamma: torch.Tensor, h_out: torch.Tensor):
        """TP reduction of a row-parallel partial + residual add + RMSNorm (baseline: NCCL then one norm kernel)."""
        self.comm.all_reduce_(partial)
        return ops.add_rmsnorm_(x, partial, gamma, self.cfg.rms_eps, out=h_out)

    @torch.no_grad()
    def forward(self, b: BatchMeta) -> torch.Tensor:
        """Runs all layers for the batch and returns greedy next tokens ``[len(last_rows)]`` (int64, global ids).

        RMSNorm is folded into the GEMMs: the residual stream ``x`` (fp32) is accompanied by ``xg = x * gamma``
        (the next GEMM's operand) and per-128-column sums of squares ``ssq``; the consuming GEMM scales each
        token's outputs by ``rsqrt(sum(ssq) / H + eps)``.  With TP=1 the residual GEMMs produce ``xg``/``ssq`` in
        their epilogue; with TP > 1 the row-parallel partial is all-reduced first.
        """
        cfg, p = self.cfg, self.plan
        if p.world > 1 and self.sequence_parallel and not b.is_decode:
            return self._forward_sp(b)
        xg, ssq = self._layers(b)
        H = cfg.hidden
        norm = (ssq, H, cfg.rms_eps)
        if b.is_decode:
            xl, nl = xg, norm
        else:
            xl = xg.index_select(0, b.last_rows)
            nl = (ssq.index_select(1, b.last_rows).contiguous(), H, cfg.rms_eps)
        logits = ops.w8a16_linear(xl, self.head_q, self.head_s, out_dtype=torch.float32, in_norm=nl)
        if self.collect_stats:
            self._record_stats(logits, xl, nl)
        return self._pick(logits, b)

    def _pick(self, logits: torch.Tensor, b: BatchMeta) -> torch.Tensor:
        """Next token per logits row, global ids: greedy, or sampled when the batch carries sampling rows."""
        p = self.plan
        if b.sample is not None:
            return self._sample(logits, b.sample)
        xchg_rows = min(self.symm.argmax_rows, ops.ARGMAX_XCHG_MAX_ROWS) if self.symm is not None else 0
        if p.world > 1 and logits.shape[0] <= xchg_rows:
            # global greedy pick through peer memory inside the argmax kernel (no NCCL call)
            return ops.argmax_exchange_(logits, p.vocab_start, self.symm)
        if p.world > 1:
            keys = torch.empty(logits.shape[0], dtype=torch.int64, device=self.device)
            ops.argmax_rows(logits, p.vocab_start, keys=keys)
            self.comm.all_reduce_max_(keys)
            from ..parallel.dist import unpack_argmax
            return unpack_argmax(keys)
        return ops.argmax_rows(logits, 0)

    def _sample(self, logits: torch.Tensor, sm) -> torch.Tensor:
        """Temperature / top-k pick.  Top-k threshold: the row's k-th largest logit; under tensor parallelism each
        rank contributes its local top-k values (``topk_candidates``), one all-gather joins them and the same radix
        select runs over the joined rows, so every rank applies the same global threshold.  The draw itself is the
        argmax kernel's Gumbel-max pick, exchanged like the greedy one."""
        p = self.plan
        R = logits.shape[0]
        k = sm.top_k[:R]
        thr = ops.kth_largest(logits, k)
        if p.world > 1:
            cand = ops.topk_candidates(logits, thr, k, sm.kmax)
            joined = torch.empty(R, p.world * sm.kmax, dtype=torch.float32, device=logits.device)
            self.comm.all_gather_cols(cand, joined)
            thr = ops.kth_largest(joined, k)
        xchg_rows = min(self.symm.argmax_rows, ops.ARGMAX_XCHG_MAX_ROWS) if self.symm is not None else 0
        args = (sm.inv_temp[:R], sm.seed[:R], sm.pos[:R], thr)
        if p.world > 1 and R <= xchg_rows:
            return ops.sample_rows(logits, p.vocab_start, *args, symm=self.symm)
        if p.world > 1:
            keys = torch.empty(R, dtype=torch.int64, device=self.device)
            ops.sample_rows(logits, p.vocab_start, *args, keys=keys)
            self.comm.all_reduce_max_(keys)
            from ..parallel.dist import unpack_argmax
            return unpack_argmax(keys)
        return ops.sample_rows(logits, 0, *args)

    def _record_stats(self, logits: torch.Tensor, xl: torch.Tensor, nl) -> None:
        """``stat_nll[i] = logsumexp(logits_i) - max(logits_i)``: the cross-entropy of the greedy token (the
        reference engine's per-step loss, ``scripts/deepseek_native_engine.sh:633-663,1112-1116``), reduced over the
        vocabulary shards under tensor parallelism; ``stat_hidden[i]`` = the final RMS-normalised hidden row."""
        rows = logits.shape[0]
        if self.stat_nll is None or self.stat_nll.numel() < rows:
            self.stat_nll = torch.zeros(max(rows, 64), dtype=torch.float32, device=logits.device)
            self.stat_hidden = torch.zeros(max(rows, 64), self.cfg.hidden, dtype=torch.float32,
                                           device=logits.device)
        top = logits.max(dim=-1).values
        if self.plan.world > 1:
            self.comm.all_reduce_max_(top)
        sumexp = torch.exp(logits - top[:, None]).sum(-1)
        if self.plan.world > 1:
            self.comm.all_reduce_(sumexp)
        self.stat_nll[:rows].copy_(torch.log(sumexp))
        ssq, H, eps = nl
        inv = torch.rsqrt(ssq.sum(0) / H + eps)
        self.stat_hidden[:rows].copy_(xl.float() * inv[:, None])

    @torch.no_grad()
    def hidden_states(self, b: BatchMeta) -> torch.Tensor:
        """Final RMS-normalised hidden states of every row, ``[T, H]`` fp32 (the reference model's ``forward``
        output, ``engine/llama_tp.py:304-311``); the lm_head is left to the caller."""
        xg, ssq = self._layers(b)
        inv = torch.rsqrt(ssq.sum(0) / self.cfg.hidden + self.cfg.rms_eps)
        return xg.float() * inv[:, None]

    def _layers(self, b: BatchMeta) -> Tuple[torch.Tensor, torch.Tensor]:
        """Embedding and every decoder layer of the batch.  Returns ``xg = x * final_norm`` (the lm_head's operand)
        and ``ssq [H / 128, T]``, the per-128-column sums of ``x^2`` that give each row's RMS scale."""
        cfg, p = self.cfg, self.plan
        T = b.ids.shape[0]
        H = cfg.hidden
        tp = p.world > 1
        dev = self.device
        cuda = dev.type == "cuda"
        x = ops.embedding_q8(b.ids, self.embed_q, self.embed_s, self.embed_start)
        if tp and not self.embed_replicated:
            self.comm.all_reduce_(x)
        xg = torch.empty(T, H, dtype=torch.float16 if cuda else torch.float32, device=dev)
        ssq = torch.empty(H // 128, T, dtype=torch.float32, device=dev)
        ops.norm_prep(x, None, self.layers[0].ln1, xg, ssq)
        norm = (ssq, H, cfg.rms_eps)
        D = cfg.head_dim
        q_out = torch.empty(T, self.q_rows, dtype=torch.bfloat16, device=dev)
        attn = torch.empty(T, p.local_heads, D, dtype=torch.float16 if cuda else torch.float32, device=dev)
        partial = torch.empty(T, H, dtype=torch.float32, device=dev) if tp else None
        # multi-phase chain: TP = 1, or TP with the fused peer-memory all-reduce (symmetric workspace present)
        chain = self.chain_layers and b.is_decode and T <= 32 and (not tp or self.symm is not None)
        act_buf = torch.empty(T, self.layers[0].s_gu.numel() // 2, dtype=xg.dtype, device=dev) if chain else None
        qkv_done = False   # the previous layer's chain already ran this layer's QKV GEMM
        for l, L in enumerate(self.layers):
            kc, vc = self.kv.k[l], self.kv.v[l]
            if not qkv_done:
                ops.w8a16_qkv_rope_append(xg, L.w_qkv, L.s_qkv, L.b_qkv, self.q_rows, self.kv_rows, D, b.positions,
                                          b.slots, self.cos, self.sin, kc, vc, q_out=q_out, in_norm=norm)
            qkv_done = False
            q3 = q_out.view(T, p.local_heads, D)
            if b.is_decode:
                # the QKV GEMM just above appends exactly one key per sequence: older KV tiles may stream early
                ops.paged_decode_attention(q3, kc, vc, b.block_tables, b.context_lens, self.scale,
                                           b.attn_splits, b.attn_keys_per_split, out=attn, kv_prefetch=True)
            else:
                ops.paged_prefill_attention(q3, kc, vc, b.block_tables, b.cu_q, b.q_start, b.context_lens, b.max_q,
                                            self.scale, out=attn)
            a2 = attn.view(T, self.q_rows)
            if chain:
                # o_proj + residual -> gate/up + SwiGLU -> down + residual (-> next layer's QKV): one launch
                g_next = self.layers[l + 1].ln1 if l + 1 < len(self.layers) else self.final_norm
                inv_h = 1.0 / H
                if tp:
                    phases = [("resid_ar", a2, L.w_o, L.s_o, x, self.symm, L.ln2, xg, ssq),
                              ("swiglu", xg, L.w_gu, L.s_gu, act_buf, ssq, inv_h, cfg.rms_eps),
                              ("resid_ar", act_buf, L.w_d, L.s_d, x, self.symm, g_next, xg, ssq)]
                else:
                    phases = [("resid", a2, L.w_o, L.s_o, x, L.ln2, xg, ssq),
                              ("swiglu", xg, L.w_gu, L.s_gu, act_buf, ssq, inv_h, cfg.rms_eps),
                              ("resid", act_buf, L.w_d, L.s_d, x, g_next, xg, ssq)]
                if l + 1 < len(self.layers):
                    Ln = self.layers[l + 1]
                    phases.append(("qkv", xg, Ln.w_qkv, Ln.s_qkv, Ln.b_qkv, self.q_rows, self.kv_rows, D,
                                   b.positions, b.slots, self.cos, self.sin, q_out, self.kv.k[l + 1],
                                   self.kv.v[l + 1], ssq, inv_h, cfg.rms_eps))
                    qkv_done = True
                ops.w8a16_chain(phases)
                continue
            fused = tp and self.symm is not None and T <= 64
            if fused:
                ops.w8a16_residual_ar_(a2, L.w_o, L.s_o, x, self.symm, L.ln2, xg, ssq)
            elif tp:
                self._row_parallel(a2, L.w_o, L.s_o, partial)
                ops.norm_prep(x, partial, L.ln2, xg, ssq)
            else:
                ops.w8a16_residual_(a2, L.w_o, L.s_o, x, gamma_next=L.ln2, xg_out=xg, ssq_out=ssq)
            act = ops.w8a16_swiglu(xg, L.w_gu, L.s_gu, in_norm=norm)
            g_next = self.layers[l + 1].ln1 if l + 1 < len(self.layers) else self.final_norm
            if fused:
                ops.w8a16_residual_ar_(act, L.w_d, L.s_d, x, self.symm, g_next, xg, ssq)
            elif tp:
                self._row_parallel(act, L.w_d, L.s_d, partial)
                ops.norm_prep(x, partial, g_next, xg, ssq)
            else:
                ops.w8a16_residual_(act, L.w_d, L.s_d, x, gamma_next=g_next, xg_out=xg, ssq_out=ssq)
        return xg, ssq

    def _row_parallel(self, a: torch.Tensor, w: torch.Tensor, s: torch.Tensor, partial: torch.Tensor) -> None:
        """``partial = all_reduce(a @ W^T)`` for a row-parallel projection (NCCL path).  With
        ``prefill_overlap_chunks = n > 1`` and enough rows, the rows are cut into n chunks: chunk i's all-reduce runs
        on the collective's stream while chunk i + 1's GEMM runs, on all SMs but ``prefill_comm_sms`` so the
        collective's kernels are resident alongside it.  Row chunks do not change any row's result."""
        n = int(self.prefill_overlap_chunks)
        T = a.shape[0]
        if n <= 1 or T < 64 * n:
            ops.w8a16_linear_out(a, w, s, partial)
            self.comm.all_reduce_(partial)
            return
        ctas = 0
        if a.is_cuda:
            ctas = max(1, ops.ext().sm_count() - int(self.prefill_comm_sms))
        step = (T + n - 1) // n
        works = []
        for r0 in range(0, T, step):
            r1 = min(T, r0 + step)
            ops.w8a16_linear_out(a[r0:r1], w, s, partial[r0:r1], force_ctas=ctas)
            works.append(self.comm.all_reduce_async_(partial[r0:r1]))
        for wk in works:
            if wk is not None:
                wk.wait()

    @torch.no_grad()
    def _forward_sp(self, b: BatchMeta) -> torch.Tensor:
        """Prefill with sequence parallelism (Megatron-SP): between blocks every rank keeps only its 1/world of the
        token rows of the residual stream.  The vocab-parallel embedding and each row-parallel GEMM output are
        reduce-scattered (sum over ranks, keep this rank's rows) instead of all-reduced; residual add + RMSNorm
        inputs run on the shard; the GEMM operand ``xg`` and its ``ssq`` are all-gathered before each
        column-parallel GEMM (QKV, gate/up) and before the lm_head.  Rows are padded to a multiple of the world
        size; pad rows carry zeros, position 0 and slot -1 (no KV write), and attention skips them.  Same sums as
        the all-reduce path, so the same tokens.  (The reference has no sequence parallelism.)"""
        cfg, p = self.cfg, self.plan
        comm, w = self.comm, p.world
        T = b.ids.shape[0]
        H, D = cfg.hidden, cfg.head_dim
        dev = self.device
        cuda = dev.type == "cuda"
        Ts = (T + w - 1) // w
        Tp = Ts * w
        fdt = torch.float16 if cuda else torch.float32
        pos = torch.zeros(Tp, dtype=b.positions.dtype, device=dev)
        pos[:T] = b.positions
        slots = torch.full((Tp,), -1, dtype=b.slots.dtype, device=dev)
        slots[:T] = b.slots
        if self.embed_replicated:   # this rank's token rows straight from the local table
            x = torch.zeros(Ts, H, dtype=torch.float32, device=dev)
            r0, r1 = min(T, p.rank * Ts), min(T, (p.rank + 1) * Ts)
            if r1 > r0:
                x[:r1 - r0] = ops.embedding_q8(b.ids[r0:r1], self.embed_q, self.embed_s, 0)
        else:
            emb = torch.zeros(Tp, H, dtype=torch.float32, device=dev)
            emb[:T] = ops.embedding_q8(b.ids, self.embed_q, self.embed_s, self.embed_start)
            x = comm.reduce_scatter_rows(emb)                       # [Ts, H] fp32, this rank's rows
        xg_s = torch.empty(Ts, H, dtype=fdt, device=dev)
        ssq_s = torch.empty(H // 128, Ts, dtype=torch.float32, device=dev)
        xg = torch.empty(Tp, H, dtype=fdt, device=dev)
        ssq = torch.empty(H // 128, Tp, dtype=torch.float32, device=dev)
        q_out = torch.empty(Tp, self.q_rows, dtype=torch.bfloat16, device=dev)
        attn = torch.zeros(Tp, p.local_heads, D, dtype=fdt, device=dev)
        partial = torch.empty(Tp, H, dtype=torch.float32, device=dev)
        ps = torch.empty(Ts, H, dtype=torch.float32, device=dev)
        norm = (ssq, H, cfg.rms_eps)

        def gather():
            comm.all_gather_rows(xg_s, xg)
            comm.all_gather_cols(ssq_s, ssq)

        ops.norm_prep(x, None, self.layers[0].ln1, xg_s, ssq_s)
        gather()
        for l, L in enumerate(self.layers):
            kc, vc = self.kv.k[l], self.kv.v[l]
            ops.w8a16_qkv_rope_append(xg, L.w_qkv, L.s_qkv, L.b_qkv, self.q_rows, self.kv_rows, D, pos, slots,
                                      self.cos, self.sin, kc, vc, q_out=q_out, in_norm=norm)
            q3 = q_out.view(Tp, p.local_heads, D)
            ops.paged_prefill_attention(q3[:T], kc, vc, b.block_tables, b.cu_q, b.q_start, b.context_lens, b.max_q,
                                        self.scale, out=attn[:T])
            ops.w8a16_linear_out(attn.view(Tp, self.q_rows), L.w_o, L.s_o, partial)
            ops.norm_prep(x, comm.reduce_scatter_rows(partial, ps), L.ln2, xg_s, ssq_s)
            gather()
            act = ops.w8a16_swiglu(xg, L.w_gu, L.s_gu, in_norm=norm)
            g_next = self.layers[l + 1].ln1 if l + 1 < len(self.layers) else self.final_norm
            ops.w8a16_linear_out(act, L.w_d, L.s_d, partial)
            ops.norm_prep(x, comm.reduce_scatter_rows(partial, ps), g_next, xg_s, ssq_s)
            gather()
        xl = xg.index_select(0, b.last_rows)
        nl = (ssq.index_select(1, b.last_rows).contiguous(), H, cfg.rms_eps)
        logits = ops.w8a16_linear(xl, self.head_q, self.head_s, out_dtype=torch.float32, in_norm=nl)
        if self.collect_stats:
            self._record_stats(logits, xl, nl)
        return self._pick(logits, b)

    def _mm_f32(self, x, w, s, out):
        return ops.w8a16_linear_out(x, w, s, out)
