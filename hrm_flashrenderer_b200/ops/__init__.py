"""Operator layer: sm_100a kernels for CUDA tensors, fp32 reference math for CPU tensors.

The CPU branch is the numerics oracle used by the CPU/gloo tests; it is not a fallback for CUDA tensors.  A CUDA
tensor always goes to the compiled extension and raises if the extension is missing (there is no silent eager path
on the GPU).

Scratch memory (split-K partials and tickets, attention split partials) comes from :class:`Workspace`, which the
engine sizes once before CUDA-graph capture so captured kernels always see the same addresses.
"""
from __future__ import annotations

import math
import os
import threading
from typing import Sequence, Optional, Tuple

import torch

_C = None
_C_ERR: Optional[BaseException] = None
try:  # the in-tree build: python setup.py build_ext --inplace
    from .. import _C as _C  # type: ignore[attr-defined]
except Exception as e:  # pragma: no cover - depends on the build
    _C_ERR = e


def ext():
    """The compiled extension; raises with the import error if it is unavailable."""
    if _C is None:
        raise RuntimeError(
            "hrm_flashrenderer_b200._C is not built or failed to load "
            f"({_C_ERR!r}); run `python setup.py build_ext --inplace`")
    return _C


def has_ext() -> bool:
    return _C is not None


class _LaunchCounter:
    """Counts kernels launched through this module (used by the benchmark to report its own launches)."""

    def __init__(self):
        self.enabled = False
        self.count = 0

    def reset(self):
        self.count = 0

    def add(self, n: int = 1):
        if self.enabled:
            self.count += n


LAUNCH_COUNTER = _LaunchCounter()


# ------------------------------------------------------------------------------------------------ workspace
_ATTN_MERGE = os.environ.get("HRM_ATTN_MERGE", "0") == "1"
# fused all-reduce protocol: fp32 partials + per-tile flags (default), or epoch-tagged 64-bit words with no fence
# and no flag (HRM_AR_LL=1; measured slower at TP = 8: twice the NVLink bytes)
_AR_LL = os.environ.get("HRM_AR_LL", "0") == "1"
# split argmax over many CTAs per row (HRM_ARGMAX_SPLIT=0: one CTA per row)
_ARGMAX_SPLIT = os.environ.get("HRM_ARGMAX_SPLIT", "1") != "0"


class Workspace:
    """Per-device scratch: fp32 split-K partials + int32 tickets (zeroed once; kernels re-arm them)."""

    _lock = threading.Lock()
    _per_device: dict = {}

    def __init__(self, device: torch.device, floats: int = 1 << 20, counters: int = 1 << 14):
        self.device = device
        self.ws = torch.empty(floats, dtype=torch.float32, device=device)
        self.counters = torch.zeros(counters, dtype=torch.int32, device=device)
        self.status = torch.zeros(4, dtype=torch.int32, device=device)   # bounded-wait error word of the kernels
        self.argmax = torch.zeros(2 * 4096, dtype=torch.int64, device=device)   # split-argmax accumulators + tickets
        self.attn_tickets = torch.zeros(1 << 16, dtype=torch.int32, device=device)   # decode split merge, per (b, hk)
        self.chain_bar = torch.zeros(8, dtype=torch.int32, device=device)   # multi-phase GEMM grid barriers + ticket
        self.frozen = False

    def ensure(self, floats: int, counters: int = 0) -> None:
        if floats > self.ws.numel():
            if self.frozen:
                raise RuntimeError(f"workspace frozen (graph capture) but {floats} floats requested")
            self.ws = torch.empty(int(floats * 1.25) + 1024, dtype=torch.float32, device=self.device)
        if counters > self.counters.numel():
            if self.frozen:
                raise RuntimeError("workspace frozen (graph capture) but more split-K counters requested")
            self.counters = torch.zeros(int(counters * 1.25) + 64, dtype=torch.int32, device=self.device)

    @classmethod
    def get(cls, device) -> "Workspace":
        device = torch.device(device)
        key = (device.type, device.index if device.index is not None else torch.cuda.current_device())
        with cls._lock:
            w = cls._per_device.get(key)
            if w is None:
                w = cls._per_device[key] = Workspace(torch.device("cuda", key[1]))
                if _C is not None:
                    _C.set_status_word(w.status)
            return w


def gemm_plan(M: int, N: int, K: int, force_ctas: int = 0) -> dict:
    bn, nt, mt, kt, splits, wsf, cnt, ku = ext().gemm_plan(int(M), int(N), int(K), int(force_ctas))
    return dict(bn=bn, n_tiles=nt, m_tiles=mt, k_units=kt, splits=splits, ws_floats=wsf, counters=cnt, ku=ku)


def _ws_for(M, N, K, device, force_ctas=0):
    p = gemm_plan(M, N, K, force_ctas)
    w = Workspace.get(device)
    w.ensure(p["ws_floats"], p["counters"])
    return w


def _as_f16_2d(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.float16:
        x2 = x2.to(torch.float16)
    if x2.stride(-1) != 1 or (x2.data_ptr() % 16) or (x2.stride(0) * 2) % 16:
        x2 = x2.contiguous()
    return x2


# ------------------------------------------------------------------------------------------------ GEMMs
# ``in_norm = (ssq, H, eps)`` folds an RMSNorm into a GEMM: X is the un-normalised input times gamma (see
# :func:`norm_prep`) and token m's outputs are scaled by rsqrt(sum_t ssq[t, m] / H + eps).
def _inv_rms(in_norm):
    ssq, H, eps = in_norm
    return torch.rsqrt(ssq.reshape(-1, ssq.shape[-1]).sum(0) / float(H) + float(eps))


def tile_w8(q: torch.Tensor) -> torch.Tensor:
    """Pre-tile an int8 weight ``[N, K]`` for the GEMM's streaming paths: ``[ceil(N/128), K/64, 8192]``; block
    ``(n, k)`` covers rows ``128n..128n+127`` x columns ``64k..64k+63`` stored chunk-major: byte
    ``c*2048 + r*16 + b`` = ``W[128n + r, 64k + 16c + b]``.  A warp reading 16-byte chunk c of 32 consecutive rows
    then touches 512 contiguous bytes (global loads fully coalesced, shared-memory reads conflict-free).  Rows past N
    are zero."""
    N, K = q.shape
    if K % 64:
        raise ValueError(f"K={K} must be a multiple of 64")
    NT = (N + 127) // 128
    if NT * 128 != N:
        q = torch.nn.functional.pad(q, (0, 0, 0, NT * 128 - N))
    return q.reshape(NT, 128, K // 64, 4, 16).permute(0, 2, 3, 1, 4).reshape(NT, K // 64, 8192).contiguous()


def untile_w8(t: torch.Tensor, N: int) -> torch.Tensor:
    """Inverse of :func:`tile_w8` (for checks and CPU math)."""
    NT, KT, _ = t.shape
    return t.view(NT, KT, 4, 128, 16).permute(0, 3, 1, 2, 4).reshape(NT * 128, KT * 64)[:N].contiguous()


def weight_nk(qweight: torch.Tensor, scale: torch.Tensor) -> Tuple[int, int]:
    """(N, K) of a plain ``[N, K]`` or pre-tiled int8 weight."""
    if qweight.dim() == 3:
        return int(scale.numel()), int(qweight.shape[1]) * 64
    return int(qweight.shape[0]), int(qweight.shape[1])


def _norm_kw(in_norm):
    if in_norm is None:
        return {}
    ssq, H, eps = in_norm
    return dict(in_ssq=ssq, inv_h=1.0 / float(H), eps=float(eps))


def w8a16_linear(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, bias: Optional[torch.Tensor] = None,
                 out_dtype: Optional[torch.dtype] = None, force_ctas: int = 0, in_norm=None) -> torch.Tensor:
    """``y = x @ (qweight * scale[:, None])^T (+ bias)``; int8 weights ``[N, K]`` (or pre-tiled by :func:`tile_w8`)
    with per-row fp32 scales."""
    N, K = weight_nk(qweight, scale)
    if not x.is_cuda:
        y = x.to(torch.float32) @ (qweight.to(torch.float32) * scale.to(torch.float32)[:, None]).t()
        if in_norm is not None:
            y = y * _inv_rms(in_norm).view(*([1] * (y.dim() - 2)), -1, 1)
        if bias is not None:
            y = y + bias.to(torch.float32)
        return y.to(out_dtype) if out_dtype is not None else y
    C = ext()
    lead = x.shape[:-1]
    x2 = _as_f16_2d(x)
    M = x2.shape[0]
    od = out_dtype or torch.float16
    out = torch.empty(M, N, dtype=torch.float32 if od == torch.float32 else torch.float16, device=x.device)
    w = _ws_for(M, N, K, x.device, force_ctas)
    C.w8a16_gemm(x2, qweight, scale, bias, out, w.ws, w.counters, force_ctas, **_norm_kw(in_norm))
    LAUNCH_COUNTER.add()
    out = out if out.dtype == od else out.to(od)
    return out.reshape(*lead, N)


def w8a16_linear_out(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, out: torch.Tensor,
                     force_ctas: int = 0, in_norm=None) -> torch.Tensor:
    """``out[:] = x @ W^T`` into a preallocated f16/f32 ``[M, N]`` buffer."""
    if not x.is_cuda:
        y = x.to(torch.float32) @ (qweight.to(torch.float32) * scale[:, None]).t()
        if in_norm is not None:
            y = y * _inv_rms(in_norm)[:, None]
        out.copy_(y)
        return out
    x2 = _as_f16_2d(x)
    w = _ws_for(x2.shape[0], *weight_nk(qweight, scale), x.device, force_ctas)
    ext().w8a16_gemm(x2, qweight, scale, None, out, w.ws, w.counters, force_ctas, **_norm_kw(in_norm))
    LAUNCH_COUNTER.add()
    return out


def w8a16_residual_(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, resid: torch.Tensor,
                    force_ctas: int = 0, gamma_next: Optional[torch.Tensor] = None,
                    xg_out: Optional[torch.Tensor] = None, ssq_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``resid += x @ W^T`` in place (fp32 residual stream); optionally also ``xg_out = resid * gamma_next`` and the
    per-128-column sums of squares ``ssq_out [N/128, M]`` for the next (folded) RMSNorm."""
    if not x.is_cuda:
        resid += x.to(torch.float32) @ (qweight.to(torch.float32) * scale[:, None]).t()
        if xg_out is not None:
            norm_prep(resid, None, gamma_next, xg_out, ssq_out)
        return resid
    x2 = _as_f16_2d(x)
    w = _ws_for(x2.shape[0], *weight_nk(qweight, scale), x.device, force_ctas)
    ext().w8a16_gemm_residual(x2, qweight, scale, resid, w.ws, w.counters, force_ctas, gamma_next, xg_out, ssq_out)
    LAUNCH_COUNTER.add()
    return resid


def w8a16_residual_ar_(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, resid: torch.Tensor, symm,
                       gamma_next: torch.Tensor, xg_out: torch.Tensor, ssq_out: torch.Tensor) -> torch.Tensor:
    """Tensor-parallel row-parallel GEMM fused with its all-reduce over NVLink peer memory (decode, M <= 64):
    ``resid += sum over ranks of x_r @ W_r^T``; also writes ``xg_out = resid * gamma_next`` and ``ssq_out``.
    Every rank ends with bitwise-identical outputs (rank-ordered reduction by the tile's owner rank)."""
    x2 = _as_f16_2d(x)
    w = _ws_for(x2.shape[0], *weight_nk(qweight, scale), x.device)
    ext().w8a16_gemm_residual_ar(x2, qweight, scale, resid, w.ws, w.counters, gamma_next, xg_out, ssq_out, symm.peers,
                                 symm.rank, symm.world, symm.off_partials, symm.off_final, symm.off_flags,
                                 symm.max_bn * 128, symm.max_tiles, symm.epoch_ptr, symm.ticket, symm.off_tile_flags,
                                 symm.off_ll, 1 if (_AR_LL and symm.off_ll) else 0)
    LAUNCH_COUNTER.add()
    return resid


def swiglu_half(F: int) -> int:
    """Gate (= up) rows per packed tile: 64 (the kernel's 128-row tile) when possible, else the whole F (CPU only)."""
    return 64 if F % 64 == 0 else F


def interleave_gate_up(gate_q: torch.Tensor, up_q: torch.Tensor, gate_s: torch.Tensor, up_s: torch.Tensor,
                       half: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Pack gate/up rows as [64 gate rows, the matching 64 up rows] per 128-row tile (the SwiGLU epilogue layout)."""
    F, K = gate_q.shape
    h = half or swiglu_half(F)
    assert F % h == 0
    q = torch.stack([gate_q.view(F // h, h, K), up_q.view(F // h, h, K)], dim=1).reshape(2 * F, K)
    s = torch.stack([gate_s.view(F // h, h), up_s.view(F // h, h)], dim=1).reshape(2 * F)
    return q.contiguous(), s.contiguous()


def w8a16_swiglu(x: torch.Tensor, w_gu: torch.Tensor, s_gu: torch.Tensor, force_ctas: int = 0,
                 in_norm=None) -> torch.Tensor:
    """``silu(x @ Wg^T) * (x @ Wu^T)`` with ``w_gu`` packed by :func:`interleave_gate_up`; f16 output."""
    N2, K = weight_nk(w_gu, s_gu)
    F = N2 // 2
    if not x.is_cuda:
        h = swiglu_half(F)
        y = x.to(torch.float32) @ (w_gu.to(torch.float32) * s_gu[:, None]).t()
        if in_norm is not None:
            y = y * _inv_rms(in_norm)[:, None]
        y = y.view(*y.shape[:-1], F // h, 2, h)
        return (torch.nn.functional.silu(y[..., 0, :]) * y[..., 1, :]).reshape(*x.shape[:-1], F)
    x2 = _as_f16_2d(x)
    out = torch.empty(x2.shape[0], F, dtype=torch.float16, device=x.device)
    w = _ws_for(x2.shape[0], N2, K, x.device, force_ctas)
    ext().w8a16_gemm_swiglu(x2, w_gu, s_gu, out, w.ws, w.counters, force_ctas, **_norm_kw(in_norm))
    LAUNCH_COUNTER.add()
    return out.reshape(*x.shape[:-1], F)


def w8a16_chain(phases: Sequence[tuple]) -> None:
    """Run decode GEMMs back to back in ONE persistent cooperative launch, phase p + 1 reading phase p's outputs.

    Phases (pre-tiled weights on the GPU; M <= 64), as tuples:
      ``("f16", x, w, scale, out, in_ssq | None, inv_h, eps)``
      ``("resid", x, w, scale, resid, gamma_next | None, xg_out | None, ssq_out | None)``
      ``("resid_ar", x, w, scale, resid, symm, gamma_next, xg_out, ssq_out)`` (tensor parallel: the partial tiles
      are all-reduced over NVLink peer memory inside the phase, as :func:`w8a16_residual_ar_`)
      ``("swiglu", x, w_gu, s_gu, out, in_ssq | None, inv_h, eps)``
      ``("qkv", x, w, scale, bias | None, q_rows, kv_rows, head_dim, positions, slots, cos, sin, q_out, k_cache,
      v_cache, in_ssq | None, inv_h, eps)``
    Supported sequences: resid, swiglu, resid[, qkv] (the decode layer transition), the same with resid_ar (tensor
    parallel) and f16, f16.  Between phases the
    kernel waits on a grid barrier; the next phase's weights stream before it.  On CPU tensors the phases run one
    after the other with the single-GEMM reference math."""
    x0 = phases[0][1]
    if not x0.is_cuda:
        for ph in phases:
            _chain_phase_reference(ph)
        return
    w = Workspace.get(x0.device)
    need_f = need_c = 0
    native = []
    for ph in phases:
        M, K = ph[1].shape
        _, wsf, cnt = ext().chain_phase_plan(int(M), int(ph[3].numel()), int(K))
        need_f, need_c = max(need_f, wsf), max(need_c, cnt)
        if ph[0] == "resid_ar":
            _, x, wt, sc, resid, symm, gamma_next, xg_out, ssq_out = ph
            ph = ("resid_ar", x, wt, sc, resid, gamma_next, xg_out, ssq_out, symm.peers, symm.rank, symm.world,
                  symm.off_partials, symm.off_final, symm.off_flags, symm.max_bn * 128, symm.max_tiles,
                  symm.epoch_ptr, symm.ticket)
        native.append(ph)
    w.ensure(need_f, need_c)
    ext().w8a16_chain(native, w.ws, w.counters, w.chain_bar)
    LAUNCH_COUNTER.add()


def _chain_phase_reference(ph: tuple) -> None:
    kind = ph[0]

    def norm(ssq, inv_h, eps):
        return None if ssq is None else (ssq, int(round(1.0 / inv_h)), eps)

    if kind == "f16":
        _, x, wt, sc, out, ssq, inv_h, eps = ph
        w8a16_linear_out(x, wt, sc, out, in_norm=norm(ssq, inv_h, eps))
    elif kind == "resid":
        _, x, wt, sc, resid, gamma_next, xg_out, ssq_out = ph
        w8a16_residual_(x, wt, sc, resid, gamma_next=gamma_next, xg_out=xg_out, ssq_out=ssq_out)
    elif kind == "swiglu":
        _, x, wt, sc, out, ssq, inv_h, eps = ph
        out.copy_(w8a16_swiglu(x, wt, sc, in_norm=norm(ssq, inv_h, eps)))
    elif kind == "qkv":
        (_, x, wt, sc, bias, q_rows, kv_rows, hd, pos, slots, cos_t, sin_t, q_out, kc, vc, ssq, inv_h, eps) = ph
        w8a16_qkv_rope_append(x, wt, sc, bias, q_rows, kv_rows, hd, pos, slots, cos_t, sin_t, kc, vc, q_out=q_out,
                              in_norm=norm(ssq, inv_h, eps))
    elif kind == "resid_ar":
        raise RuntimeError("resid_ar chain phases need CUDA tensors (peer-memory all-reduce)")
    else:
        raise ValueError(f"unknown chain phase {kind!r}")


def w8a16_qkv_rope_append(x: torch.Tensor, w_qkv: torch.Tensor, s_qkv: torch.Tensor, bias: Optional[torch.Tensor],
                          q_rows: int, kv_rows: int, head_dim: int, positions: torch.Tensor, slots: torch.Tensor,
                          cos_t: torch.Tensor, sin_t: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                          q_out: Optional[torch.Tensor] = None, force_ctas: int = 0, in_norm=None) -> torch.Tensor:
    """Fused QKV projection + bias + rotate-half RoPE + paged KV append.  Returns q ``[M, q_rows]`` bf16."""
    M = x.reshape(-1, x.shape[-1]).shape[0]
    if not x.is_cuda:
        y = w8a16_linear(x.reshape(M, -1), w_qkv, s_qkv, bias, in_norm=in_norm)
        D = head_dim
        q = y[:, :q_rows].view(M, -1, D)
        k = y[:, q_rows:q_rows + kv_rows].view(M, -1, D)
        v = y[:, q_rows + kv_rows:].view(M, -1, D)
        from ..models.oracle import apply_rope
        q = apply_rope(q, cos_t, sin_t, positions.long())
        k = apply_rope(k, cos_t, sin_t, positions.long())
        bs = k_cache.shape[2]
        for m in range(M):
            s = int(slots[m])
            if s >= 0:
                k_cache[s // bs, :, s % bs] = k[m].to(k_cache.dtype)
                v_cache[s // bs, :, s % bs] = v[m].to(v_cache.dtype)
        qb = q.reshape(M, q_rows).to(torch.bfloat16)
        if q_out is not None:
            q_out.copy_(qb)
            return q_out
        return qb
    x2 = _as_f16_2d(x)
    if q_out is None:
        q_out = torch.empty(M, q_rows, dtype=torch.bfloat16, device=x.device)
    w = _ws_for(M, *weight_nk(w_qkv, s_qkv), x.device, force_ctas)
    ext().w8a16_gemm_qkv(x2, w_qkv, s_qkv, bias, q_rows, kv_rows, head_dim, positions, slots, cos_t, sin_t, q_out,
                         k_cache, v_cache, w.ws, w.counters, force_ctas, **_norm_kw(in_norm))
    LAUNCH_COUNTER.add()
    return q_out


# ------------------------------------------------------------------------------------------------ norms / embed
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out_dtype: Optional[torch.dtype] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not x.is_cuda:
        xf = x.to(torch.float32)
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.to(torch.float32)
        if out is not None:
            out.copy_(y)
            return out
        return y.to(out_dtype) if out_dtype is not None else y
    xf = x if x.dtype == torch.float32 and x.is_contiguous() else x.to(torch.float32).contiguous()
    if out is None:
        out = torch.empty(xf.shape, dtype=torch.float16, device=x.device)
    ext().rmsnorm(xf, None, w, float(eps), out)
    LAUNCH_COUNTER.add()
    return out if out_dtype in (None, torch.float16) else out.to(out_dtype)


def add_rmsnorm_(x: torch.Tensor, delta: torch.Tensor, w: torch.Tensor, eps: float,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x += delta`` (in place, fp32) then return ``rmsnorm(x)`` (f16 on CUDA, fp32 on CPU)."""
    if not x.is_cuda:
        x += delta.to(x.dtype)
        return rmsnorm(x, w, eps, out=out)
    if out is None:
        out = torch.empty(x.shape, dtype=torch.float16, device=x.device)
    ext().rmsnorm(x, delta.contiguous(), w, float(eps), out)
    LAUNCH_COUNTER.add()
    return out


def norm_prep(x: torch.Tensor, delta: Optional[torch.Tensor], gamma: torch.Tensor, xg: torch.Tensor,
              ssq: torch.Tensor) -> None:
    """``x += delta`` (optional), ``xg = x * gamma`` (f16 on CUDA), ``ssq[t, m] = sum of x[m, 128t:128t+128]^2``."""
    if not x.is_cuda:
        if delta is not None:
            x += delta.to(x.dtype)
        xg.copy_(x * gamma)
        M, H = x.reshape(-1, x.shape[-1]).shape
        ssq.view(-1)[: (H // 128) * M].copy_(x.reshape(M, H // 128, 128).pow(2).sum(-1).t().reshape(-1))
        return
    ext().norm_prep(x, delta, gamma, xg, ssq)
    LAUNCH_COUNTER.add()


def embedding_q8(ids: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, vocab_start: int = 0,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Masked int8 row lookup: rows outside ``[vocab_start, vocab_start + V_local)`` are zero (vocab parallel)."""
    V, H = qweight.shape
    if not ids.is_cuda:
        local = ids.long() - vocab_start
        mask = (local >= 0) & (local < V)
        lc = local.clamp(0, V - 1)
        emb = qweight[lc].to(torch.float32) * scale[lc].unsqueeze(-1)
        return emb * mask.unsqueeze(-1).to(emb.dtype)
    ids64 = ids.to(torch.int64).contiguous()
    if out is None:
        out = torch.empty(*ids.shape, H, dtype=torch.float32, device=ids.device)
    ext().embed_q8(ids64, qweight, scale, int(vocab_start), out)
    LAUNCH_COUNTER.add()
    return out


# ------------------------------------------------------------------------------------------------ attention
KEYS_PER_TILE = 128   # the tensor-core decode kernel consumes 128-key tiles


def decode_splits(max_ctx: int, batch_heads: int, block_size: int = 16, sms: int = 148) -> Tuple[int, int]:
    """Split-K plan for decode attention: about two resident CTAs per SM, whole 128-key tiles per split."""
    tiles = max(1, (max_ctx + KEYS_PER_TILE - 1) // KEYS_PER_TILE)
    want = max(1, (2 * sms) // max(1, batch_heads))
    splits = max(1, min(want, tiles))
    per = (tiles + splits - 1) // splits
    splits = (tiles + per - 1) // per
    return splits, per * KEYS_PER_TILE


# Status-word codes written by the kernels' bounded waits (csrc/common.cuh).
STATUS_NAMES = {1: "full", 2: "empty", 3: "dequant", 4: "accumulator", 5: "peer flag", 6: "bad shape",
                7: "grid barrier", 8: "chain weight-empty", 9: "chain activation-empty", 10: "chain A-stage-empty",
                11: "chain weight-full", 12: "chain activation-full", 13: "chain A-stage-full",
                14: "chain accumulator-empty", 15: "chain accumulator-full"}


def check_status(device=None) -> None:
    """Raise if any kernel on ``device`` hit a bounded-wait timeout (reads the status word; synchronizes)."""
    w = Workspace.get(device if device is not None else torch.device("cuda"))
    v = int(w.status[0].item())
    if v:
        w.status.zero_()
        w.counters.zero_()   # stream-K tickets may be left mid-count by an aborted launch
        w.chain_bar.zero_()
        raise RuntimeError(f"a kernel reported a bounded-wait timeout (code {v}: {STATUS_NAMES.get(v, '?')})")


def paged_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                           context_lens: torch.Tensor, scale: Optional[float] = None, splits: int = 0,
                           keys_per_split: int = 0, out: Optional[torch.Tensor] = None,
                           max_ctx: Optional[int] = None, allow_tc: bool = True,
                           kv_prefetch: bool = False) -> torch.Tensor:
    """One query token per sequence.  ``q [B, Hq, D]`` bf16 -> ``[B, Hq, D]`` f16.

    ``kv_prefetch=True`` is a promise that the kernel launched right before this call writes no block table, no
    context length and no KV entry except each sequence's last key (the decode step's QKV + append GEMM); the
    tensor-core kernel then starts streaming the older KV tiles while that kernel finishes (programmatic dependent
    launch)."""
    B, Hq, D = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if not q.is_cuda:
        from ..runtime.kv_cache import gather_kv_reference
        Hk = k_cache.shape[1]
        outs = []
        for b in range(B):
            L = int(context_lens[b])
            tab = block_tables[b].tolist()
            k = gather_kv_reference(k_cache, tab, L).float()
            v = gather_kv_reference(v_cache, tab, L).float()
            kk = k.repeat_interleave(Hq // Hk, dim=1)
            vv = v.repeat_interleave(Hq // Hk, dim=1)
            s = torch.einsum("hd,shd->hs", q[b].float(), kk) * scale
            outs.append(torch.einsum("hs,shd->hd", torch.softmax(s, -1), vv))
        res = torch.stack(outs).to(torch.float16)
        if out is not None:
            out.copy_(res)
            return out
        return res
    bs = k_cache.shape[2]
    if splits <= 0:
        mc = int(max_ctx) if max_ctx is not None else int(block_tables.shape[1] * bs)
        splits, keys_per_split = decode_splits(mc, B * k_cache.shape[1], bs, ext().sm_count())
    if out is None:
        out = torch.empty(B, Hq, D, dtype=torch.float16, device=q.device)
    ws = Workspace.get(q.device)
    need = ext().decode_attn_ws_floats(B, Hq, D, splits) if splits > 1 else 0
    ws.ensure(need)
    # in-kernel split merge (last split CTA of each (sequence, kv head) combines) instead of a combine launch;
    # opt-in with HRM_ATTN_MERGE=1 until it is measured faster than the separate combine kernel
    merge = _ATTN_MERGE and B * k_cache.shape[1] <= ws.attn_tickets.numel()
    tickets = ws.attn_tickets if merge else None
    n = ext().decode_attention(q.contiguous(), k_cache, v_cache, block_tables, context_lens, out, ws.ws, splits,
                               keys_per_split, float(scale), ws.status, bool(allow_tc), bool(kv_prefetch), tickets)
    LAUNCH_COUNTER.add(int(n))
    return out


def paged_prefill_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            block_tables: torch.Tensor, cu_q: torch.Tensor, q_start: torch.Tensor,
                            context_lens: torch.Tensor, max_q: int, scale: Optional[float] = None,
                            out: Optional[torch.Tensor] = None, allow_tc: bool = True) -> torch.Tensor:
    """Causal attention of varlen query chunks ``q [Tq, Hq, D]`` against the paged cache (chunk already appended)."""
    Tq, Hq, D = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if not q.is_cuda:
        from ..runtime.kv_cache import gather_kv_reference
        from ..models.oracle import attention
        Hk = k_cache.shape[1]
        res = torch.zeros(Tq, Hq, D)
        for s in range(q_start.numel()):
            a, b = int(cu_q[s]), int(cu_q[s + 1])
            L = int(context_lens[s])
            tab = block_tables[s].tolist()
            k = gather_kv_reference(k_cache, tab, L).float()
            v = gather_kv_reference(v_cache, tab, L).float()
            pos = torch.arange(int(q_start[s]), int(q_start[s]) + (b - a))
            res[a:b] = attention(q[a:b].float() * (scale * math.sqrt(D)), k, v, pos, Hq // Hk)
        if out is not None:
            out.copy_(res)
            return out
        return res.to(torch.float16)
    if out is None:
        out = torch.empty(Tq, Hq, D, dtype=torch.float16, device=q.device)
    Workspace.get(q.device)   # registers the kernels' status word
    ext().prefill_attention(q.contiguous(), k_cache, v_cache, block_tables, cu_q, q_start, context_lens, out,
                            int(max_q), float(scale), bool(allow_tc))
    LAUNCH_COUNTER.add()
    return out


# ------------------------------------------------------------------------------------------------ sampling
def argmax_rows(logits: torch.Tensor, vocab_start: int = 0, keys: Optional[torch.Tensor] = None,
                tokens: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Greedy token per row (global id = local + vocab_start); ties -> lowest id.  Optionally packed keys."""
    if not logits.is_cuda:
        from ..parallel.dist import pack_argmax
        val, idx = torch.max(logits.float(), dim=-1)
        if keys is not None:
            keys.copy_(pack_argmax(val, idx + vocab_start))
        return idx.to(torch.int64) + vocab_start
    if tokens is None:
        tokens = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    scratch = Workspace.get(logits.device).argmax if _ARGMAX_SPLIT else None
    ext().argmax_rows(logits, int(vocab_start), keys, tokens, scratch)
    LAUNCH_COUNTER.add()
    return tokens


def gemm_nt(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``a [M, K] @ b [N, K]^T`` -> fp32 ``[M, N]`` (bf16 or f16 operands, fp32 accumulate) on the tensor cores; the
    experiments plane's dense product (the reference trainer's WMMA GEMM, llm_engine.cu:471-524).  CPU tensors
    use fp32 math of the same rounded operands."""
    if out is None:
        out = torch.empty(a.shape[0], b.shape[0], dtype=torch.float32, device=a.device)
    if not a.is_cuda:
        return torch.matmul(a.float(), b.float().t(), out=out)
    ext().gemm_nt(a, b, out)
    LAUNCH_COUNTER.add()
    return out


def _causal_attention_math(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 causal attention of ``[B, T, H, D]`` rows: (output, base-2 log-sum-exp ``[B, H, T]``)."""
    B, T, H, D = q.shape
    s = torch.einsum("bihd,bjhd->bhij", q.float(), k.float()) * (math.log2(math.e) / math.sqrt(D))
    s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=q.device).triu(1), -float("inf"))
    m = s.amax(-1, keepdim=True)
    p = torch.exp2(s - m)
    l = p.sum(-1, keepdim=True)
    o = torch.einsum("bhij,bjhd->bihd", p / l, v.float())
    return o.contiguous(), (m + torch.log2(l))[..., 0].contiguous()


# Rows per thread of the trainer's flash kernels at head dim 16.  Measured at B128 x T512 x H8: the two-row backward
# is 4 % faster than the one-row one, the two-row forward 2.1x slower, so the forward keeps one row per thread
# (HRM_FLASH_FWD_RPT=2 / HRM_FLASH_RPT=1 select the other variants).
FLASH_FWD_RPT = 2 if os.environ.get("HRM_FLASH_FWD_RPT", "1") == "2" else 1
FLASH_RPT = 1 if os.environ.get("HRM_FLASH_RPT", "2") == "1" else 2


def flash_train_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Causal attention for the trainer: ``q, k, v`` contiguous fp32 ``[B, T, H, D]`` (D 16 or 32) -> ``(o, lse)``
    with ``o`` like ``q`` and ``lse`` the base-2 log-sum-exp of each row's scaled scores, ``[B, H, T]`` (the
    reference trainer's ``flash_fwd_hf``, llm_engine.cu:856-948).  CPU tensors use the same math in PyTorch."""
    if not q.is_cuda:
        return _causal_attention_math(q, k, v)
    B, T, H, _ = q.shape
    o = torch.empty_like(q)
    lse = torch.empty(B, H, T, dtype=torch.float32, device=q.device)
    ext().flash_train_fwd(q, k, v, o, lse, FLASH_FWD_RPT)
    LAUNCH_COUNTER.add()
    return o, lse


def flash_train_bwd(q, k, v, o, lse, dout) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients of :func:`flash_train_fwd` (``dq, dk, dv``), from the saved output and log-sum-exp: a dQ pass and a
    dK/dV pass, deterministic (llm_engine.cu:950-1146).  CPU tensors go through autograd of the same math."""
    if not q.is_cuda:
        with torch.enable_grad():
            qq, kk, vv = (t.detach().float().requires_grad_(True) for t in (q, k, v))
            oo, _ = _causal_attention_math(qq, kk, vv)
            return torch.autograd.grad(oo, (qq, kk, vv), dout.float())
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ext().flash_train_bwd(q, k, v, o, lse, dout.contiguous(), dq, dk, dv, FLASH_RPT)
    LAUNCH_COUNTER.add(2)
    return dq, dk, dv


ARGMAX_XCHG_MAX_ROWS = 256


def argmax_exchange_(logits: torch.Tensor, vocab_start: int, symm, tokens: Optional[torch.Tensor] = None
                     ) -> torch.Tensor:
    """Tensor-parallel greedy token per row: this rank's logits cover vocab ids ``[vocab_start, vocab_start + V)``;
    every rank returns the global argmax (ties -> lowest id) after one exchange of packed keys over NVLink peer
    memory inside the argmax kernel (no collective library call).

    Each row's final CTA waits for the other ranks' key of its row, so every CTA of the launch must be resident at
    once: rows are limited to ``ARGMAX_XCHG_MAX_ROWS`` (about two CTAs per SM); larger batches take the collective
    path."""
    if logits.shape[0] > ARGMAX_XCHG_MAX_ROWS:
        raise ValueError(f"argmax exchange: {logits.shape[0]} rows > {ARGMAX_XCHG_MAX_ROWS}")
    if tokens is None:
        tokens = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    scratch = Workspace.get(logits.device).argmax if _ARGMAX_SPLIT else None
    ext().argmax_rows_xchg(logits, int(vocab_start), tokens, scratch, symm.peers, symm.rank, symm.world,
                           symm.argmax_rows, symm.off_ax_keys, symm.off_ax_flags, symm.argmax_epoch_ptr,
                           symm.argmax_ticket_ptr)
    LAUNCH_COUNTER.add()
    return tokens


# ------------------------------------------------------------------------------------------------ sampling
# Temperature / top-k sampling on the argmax path (Gumbel-max): a row's token is the argmax over the kept logits of
# v / T + Gumbel(seed, position, global token id); "kept" = v >= the row's global k-th largest logit.  The noise is a
# counter-based hash of (seed, position, id), so a request's draw does not depend on its batch or on the vocabulary
# sharding, and tensor-parallel ranks agree without exchanging noise.
SAMPLE_MAX_TOP_K = 1024
_GAMMA = 0x9E3779B97F4A7C15
_MIX1, _MIX2 = 0xBF58476D1CE4E5B9, 0x94D049BB133111EB


def _mix64(z):
    import numpy as np
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(_MIX1)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(_MIX2)
        return z ^ (z >> np.uint64(31))


def gumbel_noise_host(seed: int, pos: int, ids) -> torch.Tensor:
    """The kernels' sampling noise for global token ids ``ids`` of one row (fp32), computed on the host: the SplitMix64
    output mix (Steele, Lea, Flood, OOPSLA 2014) of ``mix64(seed + gamma * (pos + 1)) + gamma * (id + 1)``, top 23
    bits -> u in (0, 1), ``-log(-log(u))``."""
    import numpy as np
    with np.errstate(over="ignore"):
        s = np.array([seed], dtype=np.int64).view(np.uint64)
        p = np.array([pos + 1], dtype=np.int64).view(np.uint64)
        rk = _mix64(s + np.uint64(_GAMMA) * p)
        i = np.asarray(ids, dtype=np.int64).view(np.uint64) + np.uint64(1)
        h = _mix64(rk + np.uint64(_GAMMA) * i)
    u = ((h >> np.uint64(41)).astype(np.float32) + np.float32(0.5)) * np.float32(1.0 / 8388608.0)
    return torch.from_numpy(-np.log(-np.log(u)))


def kth_largest(x: torch.Tensor, k: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out[r]`` = the ``k[r]``-th largest value of row ``r`` of ``x [R, n]`` (fp32); ``-inf`` when ``k[r] <= 0`` or
    ``k[r] >= n`` (no restriction).  Radix select in three passes, each spread over many CTAs per row."""
    R, n = x.shape
    if out is None:
        out = torch.empty(R, dtype=torch.float32, device=x.device)
    if not x.is_cuda:
        for r in range(R):
            kr = int(k[r])
            out[r] = -float("inf") if kr <= 0 or kr >= n else torch.topk(x[r].float(), kr).values[-1]
        return out
    state = torch.empty(int(ext().kth_largest_state_words(R)), dtype=torch.int32, device=x.device)
    ext().kth_largest_rows(x, k, out, state)
    LAUNCH_COUNTER.add(7)
    return out


def topk_candidates(x: torch.Tensor, thresh: torch.Tensor, k: torch.Tensor, kmax: int) -> torch.Tensor:
    """Each row's top-``k`` values as ``[R, kmax]``: the values above ``thresh[r]``, then ``thresh[r]`` up to ``k[r]``
    slots, then ``-inf`` (in no particular order; ``k[r] <= kmax``).  Rows with ``k[r] <= 0`` are all ``-inf``."""
    R, n = x.shape
    cand = torch.empty(R, kmax, dtype=torch.float32, device=x.device)
    if not x.is_cuda:
        cand.fill_(-float("inf"))
        for r in range(R):
            kr = min(int(k[r]), kmax)
            if kr <= 0:
                continue
            t = float(thresh[r])
            above = x[r][x[r].float() > t].float()[:kmax]
            cand[r, :above.numel()] = above
            if t != -float("inf") and above.numel() < kr:
                cand[r, above.numel():kr] = t
        return cand
    ext().topk_candidates_rows(x, thresh, k, cand)
    LAUNCH_COUNTER.add()
    return cand


def sample_rows(logits: torch.Tensor, vocab_start: int, inv_temp: torch.Tensor, seed: torch.Tensor,
                pos: torch.Tensor, thresh: Optional[torch.Tensor] = None, keys: Optional[torch.Tensor] = None,
                symm=None, tokens: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Sampled token per row of this rank's logits ``[R, V]`` (global ids from ``vocab_start``): rows with
    ``inv_temp == 0`` stay greedy, the others take the argmax of ``v * inv_temp + Gumbel(seed, pos, id)`` over the
    logits ``>= thresh`` (all when ``thresh`` is None).  ``keys`` receives the packed (value, lowest id) keys for a
    collective max; with ``symm`` the keys are exchanged over peer memory inside the kernel and the returned tokens
    are already global.  ``inv_temp`` f32, ``seed`` int64, ``pos`` int32, all ``[>= R]``."""
    R, V = logits.shape
    if not logits.is_cuda:
        from ..parallel.dist import pack_argmax
        lf = logits.float()
        vals = torch.empty(R, dtype=torch.float32)
        idx = torch.empty(R, dtype=torch.int64)
        ids = torch.arange(V, dtype=torch.int64) + int(vocab_start)
        for r in range(R):
            it = float(inv_temp[r])
            if it == 0.0:
                v, i = torch.max(lf[r], dim=0)
            else:
                z = lf[r] * it + gumbel_noise_host(int(seed[r]), int(pos[r]), ids.numpy())
                if thresh is not None:
                    z = torch.where(lf[r] >= float(thresh[r]), z, torch.full_like(z, -float("inf")))
                v, i = torch.max(z, dim=0)
            vals[r], idx[r] = v, i
        if keys is not None:
            keys.copy_(pack_argmax(vals, idx + int(vocab_start)))
        return idx + int(vocab_start)
    if tokens is None:
        tokens = torch.empty(R, dtype=torch.int64, device=logits.device)
    scratch = Workspace.get(logits.device).argmax if _ARGMAX_SPLIT else None
    if symm is not None:
        if R > min(symm.argmax_rows, ARGMAX_XCHG_MAX_ROWS):
            raise ValueError(f"sampled exchange: {R} rows > {min(symm.argmax_rows, ARGMAX_XCHG_MAX_ROWS)}")
        ext().argmax_rows_sample(logits, int(vocab_start), keys, tokens, scratch, inv_temp, thresh, seed, pos,
                                 symm.peers, symm.rank, symm.world, symm.argmax_rows, symm.off_ax_keys,
                                 symm.off_ax_flags, symm.argmax_epoch_ptr, symm.argmax_ticket_ptr)
    else:
        ext().argmax_rows_sample(logits, int(vocab_start), keys, tokens, scratch, inv_temp, thresh, seed, pos,
                                 None, 0, 1, 0, 0, 0, 0, 0)
    LAUNCH_COUNTER.add()
    return tokens


# ------------------------------------------------------------------------------------------------ decode bookkeeping
def decode_prepare(positions: torch.Tensor, tables: torch.Tensor, block_size: int, active: Optional[torch.Tensor],
                   slots: torch.Tensor, context_lens: torch.Tensor) -> None:
    """``slots[b] = table[b][pos // bs] * bs + pos % bs`` (``-1`` when inactive); ``context_lens = pos + 1``."""
    if positions.is_cuda:
        ext().decode_prepare(positions, tables, int(block_size), active, slots, context_lens)
        LAUNCH_COUNTER.add()
        return
    pos = positions.long()
    blk = (pos // block_size).clamp(max=tables.shape[1] - 1)
    s = tables.gather(1, blk.view(-1, 1)).view(-1).long() * block_size + pos % block_size
    if active is not None:
        s = torch.where(active != 0, s, torch.full_like(s, -1))
    slots.copy_(s.to(slots.dtype))
    context_lens.copy_((pos + 1).to(context_lens.dtype))


def decode_advance(tokens: torch.Tensor, ids: torch.Tensor, positions: torch.Tensor,
                   active: Optional[torch.Tensor]) -> None:
    """``ids = tokens``, ``positions += 1`` for active rows."""
    if tokens.is_cuda:
        ext().decode_advance(tokens, ids, positions, active)
        LAUNCH_COUNTER.add()
        return
    on = torch.ones_like(positions, dtype=torch.bool) if active is None else active != 0
    ids.copy_(torch.where(on, tokens, ids))
    positions.copy_(torch.where(on, positions + 1, positions))
