"""Drop-in for the reference's ``flashattention_custom.ops`` API: ``flash_attn``, ``flash_attn_paged``,
``paged_kv_append`` with the same arguments and semantics (reference ``flashattention_custom/ops.py:79-99``,
kernels ``csrc/flash_attn_sm75.cu``).

Layouts kept from the reference: contiguous ``q [B, Hq, M, D]``, ``k, v [B, H, N, D]``; per-sequence pages
``k_pages, v_pages [B, Hk, P, PS, D]`` with ``seqlen [B]`` valid keys and ``head_map [Hq]`` (query head -> kv head).
Causal masking hides key position ``k_offset + j`` from query position ``q_offset + i`` when it is larger.

On a GPU the calls run this package's paged attention kernels (tcgen05 for head_dim 128, CUDA cores for 64): the
keys are re-laid once per call into the kernels' block pool ``[blocks, Hk, 16, D]`` (bf16; one copy of the cache),
query heads are regrouped by ``head_map``, and one query row per sequence takes the decode kernel.  Cases the
kernels do not express (a query before the first key, uneven ``head_map`` groups, page sizes not a multiple of 16,
other head dims) and CPU tensors use the same math in PyTorch.  The result has ``q``'s dtype.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from .. import ops

__all__ = ["flash_attn", "flash_attn_paged", "paged_kv_append"]


# ------------------------------------------------------------------------------------------------ reference math
def _math_attn(q, k, v, causal, q_offset, k_offset):
    M, N, D = q.shape[-2], k.shape[-2], q.shape[-1]
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) / math.sqrt(D)
    if causal:
        qp = torch.arange(q_offset, q_offset + M, device=q.device)
        kp = torch.arange(k_offset, k_offset + N, device=q.device)
        s = s.masked_fill(kp.view(1, N) > qp.view(M, 1), float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), v.float()).to(q.dtype)


def _math_paged(q, k_pages, v_pages, seqlen, page_size, head_map, causal, q_offset, k_offset):
    B, Hq, M, D = q.shape
    Hk, P, PS = k_pages.shape[1:4]
    out = torch.zeros_like(q)
    hm = head_map.long().tolist()
    for b in range(B):
        L = int(seqlen[b])
        kf = k_pages[b].reshape(Hk, P * PS, D)[:, :L]
        vf = v_pages[b].reshape(Hk, P * PS, D)[:, :L]
        out[b] = _math_attn(q[b], kf[hm], vf[hm], causal, q_offset, k_offset)
    return out


# ------------------------------------------------------------------------------------------------ kernel path
def _group_order(head_map: torch.Tensor, Hq: int, Hk: int) -> Optional[torch.Tensor]:
    """Permutation of query heads that puts heads of kv head h at [h*G, (h+1)*G), or None if groups are uneven."""
    if Hq % Hk:
        return None
    G = Hq // Hk
    hm = head_map.long().cpu()
    if hm.numel() != Hq or int(hm.min()) < 0 or int(hm.max()) >= Hk:
        return None
    if not torch.equal(torch.bincount(hm, minlength=Hk), torch.full((Hk,), G, dtype=torch.long)):
        return None
    return torch.sort(hm, stable=True).indices


def _run_kernels(q: torch.Tensor, pool_k: torch.Tensor, pool_v: torch.Tensor, tables: torch.Tensor,
                 q_start: torch.Tensor, ctx: torch.Tensor) -> torch.Tensor:
    """q [B, Hq, M, D] (heads already grouped) against the block pool; returns [B, Hq, M, D] in q's dtype."""
    B, Hq, M, D = q.shape
    dev = q.device
    if M == 1:
        # a single query at position q_start sees keys < min(ctx, q_start + 1)
        cl = torch.minimum(ctx, q_start + 1).to(torch.int32)
        o = ops.paged_decode_attention(q[:, :, 0].to(torch.bfloat16).contiguous(), pool_k, pool_v, tables, cl,
                                       max_ctx=int(cl.max()))
        return o.view(B, Hq, 1, D).to(q.dtype)
    qt = q.permute(0, 2, 1, 3).reshape(B * M, Hq, D).to(torch.bfloat16).contiguous()
    cu = torch.arange(0, (B + 1) * M, M, dtype=torch.int32, device=dev)
    o = ops.paged_prefill_attention(qt, pool_k, pool_v, tables, cu, q_start.to(torch.int32), ctx.to(torch.int32), M)
    return o.view(B, M, Hq, D).permute(0, 2, 1, 3).to(q.dtype)


def _pool_from_pages(pages: torch.Tensor) -> Tuple[torch.Tensor, int]:
    """[B, Hk, P, PS, D] -> ([B * P * PS/16, Hk, 16, D] bf16, blocks per sequence)."""
    B, Hk, P, PS, D = pages.shape
    nbs = P * PS // 16
    pool = pages.reshape(B, Hk, P, PS // 16, 16, D).permute(0, 2, 3, 1, 4, 5).reshape(B * nbs, Hk, 16, D)
    return pool.to(torch.bfloat16).contiguous(), nbs


def _kernel_ok(q: torch.Tensor, group: int = 1) -> bool:
    """head_dim 128: tcgen05 kernels (group <= 16); head_dim 64: CUDA-core kernels (group <= 8)."""
    D = q.shape[-1]
    return (q.is_cuda and q.dtype in (torch.float16, torch.bfloat16, torch.float32)
            and ((D == 128 and group <= 16) or (D == 64 and group <= 8)))


# ------------------------------------------------------------------------------------------------ public API
def flash_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True, q_offset: int = 0,
               k_offset: int = 0) -> torch.Tensor:
    """Attention of ``q [B, H, M, D]`` over contiguous ``k, v [B, H, N, D]``."""
    B, H, M, D = q.shape
    N = k.shape[2]
    rel = int(q_offset) - int(k_offset) if causal else N - 1
    if not _kernel_ok(q) or rel < 0 or k.shape[1] != H:
        return _math_attn(q, k, v, causal, q_offset, k_offset)
    Np = (N + 15) // 16 * 16
    pad = (0, 0, 0, Np - N)
    kp = torch.nn.functional.pad(k, pad).view(B, H, 1, Np, D)
    vp = torch.nn.functional.pad(v, pad).view(B, H, 1, Np, D)
    pool_k, nbs = _pool_from_pages(kp)
    pool_v, _ = _pool_from_pages(vp)
    tables = torch.arange(B * nbs, dtype=torch.int32, device=q.device).view(B, nbs)
    qs = torch.full((B,), rel, dtype=torch.int32, device=q.device)
    ctx = torch.full((B,), N, dtype=torch.int32, device=q.device)
    return _run_kernels(q, pool_k, pool_v, tables, qs, ctx)


def flash_attn_paged(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor, seqlen: torch.Tensor,
                     page_size: int, head_map: torch.Tensor, causal: bool = True, q_offset: int = 0,
                     k_offset: int = 0) -> torch.Tensor:
    """Attention of ``q [B, Hq, M, D]`` over per-sequence pages ``[B, Hk, P, PS, D]`` (``seqlen`` valid keys)."""
    B, Hq, M, D = q.shape
    Hk, P, PS = k_pages.shape[1:4]
    if int(page_size) != PS:
        raise ValueError(f"page_size {page_size} does not match the pages' dimension {PS}")
    rel = int(q_offset) - int(k_offset)
    order = _group_order(head_map, Hq, Hk) if (Hq % Hk == 0 and _kernel_ok(q, Hq // Hk)) else None
    if order is None or PS % 16 or (causal and rel < 0):
        return _math_paged(q, k_pages, v_pages, seqlen, page_size, head_map, causal, q_offset, k_offset)
    pool_k, nbs = _pool_from_pages(k_pages)
    pool_v, _ = _pool_from_pages(v_pages)
    tables = torch.arange(B * nbs, dtype=torch.int32, device=q.device).view(B, nbs)
    ctx = seqlen.to(device=q.device, dtype=torch.int32)
    # non-causal: put every query at the last key so all keys are visible
    qs = torch.full((B,), rel, dtype=torch.int32, device=q.device) if causal else (ctx - 1).clamp(min=0)
    order = order.to(q.device)
    o = _run_kernels(q[:, order], pool_k, pool_v, tables, qs, ctx)
    out = torch.empty_like(o)
    out[:, order] = o
    return out


def paged_kv_append(k_pages: torch.Tensor, v_pages: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                    start_pos: int, page_size: int) -> None:
    """Write ``k_new, v_new [B, Hk, T, D]`` at positions ``start_pos .. start_pos + T - 1`` of every sequence."""
    T = k_new.shape[2]
    pos = torch.arange(int(start_pos), int(start_pos) + T, device=k_pages.device)
    p, off = pos // int(page_size), pos % int(page_size)
    k_pages[:, :, p, off] = k_new.to(k_pages.dtype)
    v_pages[:, :, p, off] = v_new.to(v_pages.dtype)
