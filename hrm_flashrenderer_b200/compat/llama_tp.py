"""Drop-in names for the reference's torch TP engine module: ``TPLlamaForCausalLM``, ``generate_tp``,
``greedy_select_token_distributed`` and ``PagedKVCache`` (reference ``engine/llama_tp.py:21-382``), running on this
package's int8 engine.

* ``TPLlamaForCausalLM(config, max_seq_len, device)`` takes an HF-style config (a ``transformers`` config, a dict
  or any object with the HF attribute names) or a :class:`~hrm_flashrenderer_b200.config.ModelConfig`.
  ``load_from_loader(loader)`` reads full-precision tensors through the reference loader interface (``get(key)``,
  ``rows(key, a, b)``, ``cols(key, a, b)``; ``engine/weight_loader.py:64-89``) and quantises every matrix per output
  row to int8, the engine's format; with ``torch.distributed`` initialised each rank keeps its tensor-parallel
  shard.  ``forward(input_ids [B, T], positions, prefill)`` returns the final RMS-normalised hidden states
  ``[B, T, H]`` (fp32) and ``logits_last(h [B, H])`` this rank's vocab slice of the logits, as in the reference.
  Rows of a batch are separate sequences in the engine's block-table KV pool; ``reset_all_caches()`` frees them.
* ``generate_tp(model, input_ids, max_new_tokens, eos_token_id, prefill_chunk_size)`` returns
  ``[B, T0 + n]`` (prompt followed by the new tokens) and runs the engine's own generation (batched prefill,
  graph-captured decode).  Differences from the reference, on purpose: every row stops at its own EOS (an id or a
  list of ids; the reference looks at row 0 only) and rows that stopped earlier are padded with their EOS id.
* ``greedy_select_token_distributed(local_logits)``: global greedy ids from vocab-sharded logits with ONE
  all-reduce of packed (value, id) keys; ties go to the lowest global id (the reference needs two all-reduces and
  one broadcast per row, ties to the lowest rank, which is the same id).
* ``WeightLoader`` (from :mod:`~hrm_flashrenderer_b200.formats.safetensors`): the reference loader interface over
  sharded safetensors checkpoints; ``TPLlamaForCausalLM.from_pretrained(model_dir, ...)`` uses it.
* ``PagedKVCache``: the reference's per-sequence page layout ``[B, Hk, P, PS, D]`` with ``seqlen [B]``, grown to a
  power of two of pages, for code that drives ``compat.flash_attn_paged`` directly.  The engine itself does not
  use it.
"""
from __future__ import annotations

from typing import Any, Dict, Iterator, List, Optional, Sequence, Union

import torch

from ..config import EngineConfig, ModelConfig
from ..formats.safetensors import WeightLoader
from ..models.weights import EMBED, LM_HEAD, QTensor, matrix_shapes, quantize_rows, vector_shapes
from ..parallel.dist import greedy_select_distributed, is_dist, rank_world
from .flashattention import paged_kv_append

__all__ = ["PagedKVCache", "TPLlamaForCausalLM", "WeightLoader", "generate_tp", "greedy_select_token_distributed"]


# ------------------------------------------------------------------------------------------------ KV pages
def _next_pow2(n: int) -> int:
    p = 1
    while p < n:
        p *= 2
    return p


class PagedKVCache:
    def __init__(self, bsz: int, kv_heads: int, head_dim: int, page_size: int = 128, init_pages: int = 4,
                 device: Union[str, torch.device] = "cuda", dtype=torch.float16):
        self.bsz, self.kv_heads, self.head_dim = int(bsz), int(kv_heads), int(head_dim)
        self.page_size, self.device, self.dtype = int(page_size), device, dtype
        shape = (self.bsz, self.kv_heads, max(1, int(init_pages)), self.page_size, self.head_dim)
        self.k_pages = torch.zeros(shape, device=device, dtype=dtype)
        self.v_pages = torch.zeros(shape, device=device, dtype=dtype)
        self.seqlen = torch.zeros(self.bsz, device=device, dtype=torch.int32)
        self.cur_len = 0

    def _ensure_pages(self, needed: int) -> None:
        have = self.k_pages.shape[2]
        if needed <= have:
            return
        n = _next_pow2(needed)
        for name in ("k_pages", "v_pages"):
            old = getattr(self, name)
            new = torch.zeros(self.bsz, self.kv_heads, n, self.page_size, self.head_dim, device=old.device,
                              dtype=old.dtype)
            new[:, :, :have] = old
            setattr(self, name, new)

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, positions: torch.Tensor) -> None:
        """``k_new, v_new [B, Hk, T, D]`` at ``positions``: ``[T]`` (consecutive, shared by every row) or ``[B, T]``
        (any positions per row)."""
        B, Hk, T, D = k_new.shape
        if (B, Hk, D) != (self.bsz, self.kv_heads, self.head_dim):
            raise ValueError(f"k_new {tuple(k_new.shape)} does not match the cache ({self.bsz}, {self.kv_heads}, "
                             f"T, {self.head_dim})")
        if positions.dim() == 1:
            start = int(positions[0])
            end = start + T
            self._ensure_pages((end + self.page_size - 1) // self.page_size)
            paged_kv_append(self.k_pages, self.v_pages, k_new, v_new, start, self.page_size)
            self.cur_len = max(self.cur_len, end)
            self.seqlen.fill_(self.cur_len)
            return
        if positions.dim() != 2 or tuple(positions.shape) != (B, T):
            raise ValueError("positions must be [T] or [B, T]")
        pos = positions.to(device=self.k_pages.device, dtype=torch.long)
        self._ensure_pages(int(pos.max()) // self.page_size + 1)
        page, off = pos // self.page_size, pos % self.page_size
        rows = torch.arange(B, device=pos.device).view(B, 1).expand(B, T)
        # [B, Hk, P, PS, D] viewed as [B, P, PS, Hk, D]: one advanced-index write for all (row, position) pairs
        self.k_pages.permute(0, 2, 3, 1, 4)[rows, page, off] = k_new.permute(0, 2, 1, 3).to(self.dtype)
        self.v_pages.permute(0, 2, 3, 1, 4)[rows, page, off] = v_new.permute(0, 2, 1, 3).to(self.dtype)
        self.seqlen.copy_(torch.maximum(self.seqlen, (pos.max(dim=1).values + 1).to(torch.int32)))
        self.cur_len = max(self.cur_len, int(self.seqlen.max()))

    def get(self):
        return self.k_pages, self.v_pages, self.seqlen

    def reset(self) -> None:
        """Logical reset; the pages stay allocated for the next request."""
        self.seqlen.zero_()
        self.cur_len = 0


# ------------------------------------------------------------------------------------------------ argmax
def greedy_select_token_distributed(local_logits: torch.Tensor, group=None) -> torch.Tensor:
    """``local_logits [B, V / world]`` (this rank's contiguous vocab slice) -> global greedy ids ``[B]`` int64."""
    rank = torch.distributed.get_rank(group) if is_dist() else 0
    return greedy_select_distributed(local_logits, rank * local_logits.shape[-1], group)


# ------------------------------------------------------------------------------------------------ model
def _model_config(config: Any) -> ModelConfig:
    if isinstance(config, ModelConfig):
        return config
    if isinstance(config, dict):
        d = dict(config)
    elif hasattr(config, "to_dict"):
        d = config.to_dict()
    else:
        d = {k: v for k, v in vars(config).items() if not k.startswith("_")}
    return ModelConfig.from_hf_config(d, name=str(d.get("_name_or_path") or d.get("model_type") or "hf"))


class _LoaderWeights:
    """Read-on-access mapping from weight names to engine tensors over a reference-style loader: matrices are
    quantised per output row to int8 (+ fp32 scales), vectors stay fp32.  Only what the sharding asks for is read;
    the embedding / lm_head are kept once read (the loading path asks for them twice)."""

    def __init__(self, loader, cfg: ModelConfig):
        self.loader, self.cfg = loader, cfg
        self._mats = {name for name, _ in matrix_shapes(cfg)} | {LM_HEAD}
        self._names = [n for n, _ in matrix_shapes(cfg)] + [n for n, _ in vector_shapes(cfg)]
        self._keep: Dict[str, Any] = {}
        self._has_head: Optional[bool] = None

    def _read(self, name: str):
        t = self.loader.get(name)
        if name in self._mats:
            return quantize_rows(t.to(torch.float32))
        return t.to(torch.float32, copy=True)   # never a view into the loader's storage

    def __getitem__(self, name: str):
        if name in self._keep:
            return self._keep[name]
        if name == LM_HEAD and not self._head_present():
            raise KeyError(name)
        v = self._read(name)
        if name in (EMBED, LM_HEAD):
            self._keep[name] = v
        return v

    def _head_present(self) -> bool:
        if self._has_head is None:
            if self.cfg.tie_embeddings:
                self._has_head = False
            else:
                try:
                    self._keep[LM_HEAD] = self._read(LM_HEAD)
                    self._has_head = True
                except Exception:   # a missing lm_head falls back to the embedding, as in the reference loader
                    self._has_head = False
        return self._has_head

    def __contains__(self, name: str) -> bool:
        if name == LM_HEAD:
            return self._head_present()
        return name in self._names

    def keys(self) -> Iterator[str]:
        names = list(self._names)
        if self._head_present() and LM_HEAD not in names:
            names.append(LM_HEAD)
        return iter(names)

    def __iter__(self):
        return self.keys()

    def __len__(self) -> int:
        return len(list(self.keys()))


class TPLlamaForCausalLM:
    def __init__(self, config: Any, max_seq_len: int, device: Union[str, torch.device] = "cuda",
                 max_batch: int = 16, num_blocks: Optional[int] = None):
        self.config = config
        self.cfg = _model_config(config)
        self.device_str = str(device)
        self.device = torch.device(device)
        self.rank, self.world = rank_world()
        c = self.cfg
        self.vocab_size, self.hidden, self.layers = c.vocab, c.hidden, c.layers
        self.num_heads, self.num_kv_heads, self.head_dim = c.heads, c.kv_heads, c.head_dim
        self.intermediate, self.eps, self.rope_theta = c.intermediate, c.rms_eps, c.rope_theta
        self.max_seq_len = int(max_seq_len)
        self.max_batch = int(max_batch)
        self.num_blocks = num_blocks
        self.model = None      # LlamaW8 shard of this rank
        self.engine = None     # InferenceEngine over it
        self._seqs: Optional[List[int]] = None

    # ---------------------------------------------------------------- loading
    def load_from_loader(self, loader) -> "TPLlamaForCausalLM":
        return self.load_weights(_LoaderWeights(loader, self.cfg))

    def load_weights(self, weights) -> "TPLlamaForCausalLM":
        """Full (unsharded) weights: ``{name: QTensor | float tensor}`` (float matrices are quantised per row)."""
        from ..models.llama import LlamaW8
        from ..parallel.comm import TPComm
        if not isinstance(weights, _LoaderWeights):
            mats = {n for n, _ in matrix_shapes(self.cfg)} | {LM_HEAD}
            weights = {k: (quantize_rows(v.to(torch.float32)) if k in mats and not isinstance(v, QTensor) else v)
                       for k, v in weights.items()}
        comm = TPComm() if self.world > 1 else None
        self.model = LlamaW8.from_weights(self.cfg, weights, rank=self.rank, world=self.world, device=self.device,
                                          comm=comm, max_pos=self.max_seq_len + 16)
        self._make_engine()
        return self

    @classmethod
    def from_pretrained(cls, model_dir, max_seq_len: int, device: Union[str, torch.device] = "cuda",
                        max_batch: int = 16, num_blocks: Optional[int] = None) -> "TPLlamaForCausalLM":
        """A local HF checkpoint directory: ``config.json`` plus safetensors shards read through
        :class:`~hrm_flashrenderer_b200.formats.safetensors.WeightLoader` (zero-copy views, quantised at load)."""
        import json
        from pathlib import Path
        cfg = json.loads((Path(model_dir) / "config.json").read_text())
        self = cls(cfg, max_seq_len, device, max_batch=max_batch, num_blocks=num_blocks)
        with WeightLoader(model_dir) as loader:
            self.load_from_loader(loader)
        return self

    @classmethod
    def from_model(cls, model, max_seq_len: int, max_batch: int = 16,
                   num_blocks: Optional[int] = None) -> "TPLlamaForCausalLM":
        """Wrap an already built :class:`~hrm_flashrenderer_b200.models.llama.LlamaW8` shard."""
        self = cls(model.cfg, max_seq_len, model.device, max_batch=max_batch, num_blocks=num_blocks)
        self.rank, self.world = model.plan.rank, model.plan.world
        self.model = model
        self._make_engine()
        return self

    def _make_engine(self) -> None:
        from ..runtime.engine import InferenceEngine
        ecfg = EngineConfig(tp=self.world, max_seq_len=self.max_seq_len, max_batch=self.max_batch,
                            use_cuda_graphs=self.device.type == "cuda")
        self.engine = InferenceEngine(self.model, ecfg, num_blocks=self.num_blocks)
        self._seqs = None

    def _need(self) -> None:
        if self.engine is None:
            raise RuntimeError("no weights: call load_from_loader() or load_weights() first")

    # ---------------------------------------------------------------- caches
    def reset_all_caches(self) -> None:
        """Free the sequences of the previous ``forward`` calls (their KV blocks return to the pool)."""
        if self.engine is not None and self._seqs is not None:
            for s in self._seqs:
                self.engine.release(s)
        self._seqs = None

    # ---------------------------------------------------------------- forward
    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, prefill: bool = True, init_pages: int = 4,
                page_size: int = 128) -> torch.Tensor:
        """``input_ids [B, T]`` at ``positions`` (``[T]`` shared by all rows, or ``[B, T]``; consecutive per row)
        -> final normalised hidden states ``[B, T, H]`` fp32.  Row ``b`` continues sequence ``b`` of the previous
        calls.  ``prefill``, ``init_pages`` and ``page_size`` are accepted for compatibility; the engine's KV pool
        is block-table paged with blocks of 16."""
        self._need()
        B, T = input_ids.shape
        if self._seqs is None:
            self._seqs = [self.engine.new_seq() for _ in range(B)]
        elif len(self._seqs) != B:
            raise ValueError(f"batch of {B} rows after a batch of {len(self._seqs)}: call reset_all_caches()")
        pos = positions.to("cpu", torch.long)
        starts = [int(pos[0])] * B if pos.dim() == 1 else [int(pos[b, 0]) for b in range(B)]
        ids = input_ids.to("cpu", torch.long)
        meta = self.engine._prefill_meta([(s, ids[b].tolist(), st) for b, (s, st) in enumerate(zip(self._seqs,
                                                                                                   starts))])
        return self.model.hidden_states(meta).view(B, T, self.hidden)

    __call__ = forward

    @torch.no_grad()
    def logits_last(self, hidden_last: torch.Tensor) -> torch.Tensor:
        """``[B, H]`` normalised hidden states -> this rank's logits ``[B, V / world]`` fp32."""
        from .. import ops
        self._need()
        m = self.model
        x = hidden_last.to(torch.float16 if m.device.type == "cuda" else torch.float32).contiguous()
        return ops.w8a16_linear(x, m.head_q, m.head_s, out_dtype=torch.float32)


# ------------------------------------------------------------------------------------------------ generate
@torch.no_grad()
def generate_tp(model: TPLlamaForCausalLM, input_ids: torch.Tensor, max_new_tokens: int,
                eos_token_id: Union[int, Sequence[int], None], prefill_chunk_size: int = 1024) -> torch.Tensor:
    """Greedy generation for ``input_ids [B, T0]``; returns ``[B, T0 + n]`` on ``input_ids``' device."""
    model._need()
    model.reset_all_caches()
    B, T0 = input_ids.shape
    n = max(0, min(int(max_new_tokens), model.max_seq_len - T0))
    if n == 0:
        return input_ids.clone()
    eos = [] if eos_token_id is None else ([int(eos_token_id)] if isinstance(eos_token_id, int)
                                           else [int(e) for e in eos_token_id])
    eng = model.engine
    old_chunk = eng.ecfg.prefill_chunk
    eng.ecfg.prefill_chunk = max(1, int(prefill_chunk_size))
    try:
        outs = eng.generate([row.tolist() for row in input_ids.to("cpu", torch.long)], n, stop_on_eos=bool(eos),
                            eos_ids=eos or None)
    finally:
        eng.ecfg.prefill_chunk = old_chunk
    width = max(len(o) for o in outs)
    new = torch.empty(B, width, dtype=torch.long)
    for b, o in enumerate(outs):
        pad = o[-1] if o and o[-1] in eos else (eos[0] if eos else 0)
        new[b] = torch.tensor(o + [pad] * (width - len(o)), dtype=torch.long)
    return torch.cat([input_ids.to("cpu", torch.long), new], dim=1).to(input_ids.device)
