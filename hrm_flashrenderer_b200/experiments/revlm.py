"""Reversible decoder LM of the experiments plane (the reference's ``llm_engine.cu`` model), in PyTorch.

Architecture (``llm_engine.cu:63-118,1636-1795``): width D = 256 split into two halves of 128; per layer
    y1 = x1 + F(x2),  F = RMSNorm(g_f) -> Q, K, V (128 x 128 each) -> interleaved RoPE (theta 1e4, head dim 16,
         8 heads) -> causal attention -> W_o
    y2 = x2 + G(y1),  G = RMSNorm(g_g) -> W1 (128 x F) -> tanh-GELU -> W2 (F x 128)
with learned token + position embeddings, a final RMSNorm over the concatenated halves and an untied output matrix;
all matrices are ``[in, out]`` (``y = x @ W``), RMSNorm eps 1e-6, loss = mean next-token cross entropy over the real
vocabulary (256 + K1 + K2; the padded columns are excluded).

Design: every weight is a view of ONE flat fp32 parameter laid out exactly as checkpoint version 11
(``weights_floats`` / ``pack_W``, :344-385), so checkpoints are a single copy, data-parallel gradient exchange is one
all-reduce of one buffer, and the optimizer is one fused kernel over it (``csrc/train_ops.cu``).  The backward of the
layer stack is reversible: activations are not stored; each layer's inputs are rebuilt from its outputs
(x2 = y2 - G(y1), x1 = y1 - F(x2)) while walking the layers backwards, as the reference does.  On the GPU the
matmuls run on the tensor-core NT GEMM with bf16 operands and fp32 accumulation, and causal attention on the fp32
flash kernels (``csrc/flash_train.cu``); residual halves and master weights are fp32.
"""
from __future__ import annotations

import math
import os
import struct
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn.functional as Fn

CKPT_MAGIC = 0x43484452
CKPT_VERSION = 11


@dataclass(frozen=True)
class RevConfig:
    k1: int = 8192
    k2: int = 8192
    d: int = 256
    heads: int = 8
    layers: int = 6
    ffn: int = 1024
    tmax: int = 512
    eps: float = 1e-6
    rope_theta: float = 10000.0

    @property
    def vocab(self) -> int:
        return 256 + self.k1 + self.k2

    @property
    def vpad(self) -> int:
        return (self.vocab + 15) // 16 * 16

    @property
    def dhf(self) -> int:
        return self.d // 2

    @property
    def dh(self) -> int:
        return self.dhf // self.heads

    def layout(self) -> List[Tuple[str, Tuple[int, ...]]]:
        """(name, shape) in checkpoint order."""
        h, f = self.dhf, self.ffn
        out = [("wte", (self.vpad, self.d)), ("wpe", (self.tmax, self.d))]
        for l in range(self.layers):
            out += [(f"gf.{l}", (h,)), (f"Wq.{l}", (h, h)), (f"Wk.{l}", (h, h)), (f"Wv.{l}", (h, h)),
                    (f"Wo.{l}", (h, h)), (f"gg.{l}", (h,)), (f"W1.{l}", (h, f)), (f"W2.{l}", (f, h))]
        out += [("gout", (self.d,)), ("Wout", (self.d, self.vpad))]
        return out

    def weights_floats(self) -> int:
        return sum(int(np.prod(s)) for _, s in self.layout())


def views(cfg: RevConfig, flat: torch.Tensor) -> Dict[str, torch.Tensor]:
    out, off = {}, 0
    for name, shape in cfg.layout():
        n = int(np.prod(shape))
        out[name] = flat[off:off + n].view(*shape)
        off += n
    assert off == flat.numel()
    return out


def init_flat(cfg: RevConfig, seed: int = 123) -> torch.Tensor:
    """Uniform(-0.02, 0.02) everywhere, norm gains 1 (the reference's init distribution; its RNG stream differs)."""
    g = torch.Generator().manual_seed(seed)
    flat = (torch.rand(cfg.weights_floats(), generator=g) * 2 - 1) * 0.02
    v = views(cfg, flat)
    for l in range(cfg.layers):
        v[f"gf.{l}"].fill_(1.0)
        v[f"gg.{l}"].fill_(1.0)
    v["gout"].fill_(1.0)
    return flat


# ------------------------------------------------------------------------------------------------ math
def rms(x: torch.Tensor, g: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)) * g


def rope_tables(cfg: RevConfig, device) -> Tuple[torch.Tensor, torch.Tensor]:
    i = torch.arange(cfg.dh // 2, dtype=torch.float32)
    inv = cfg.rope_theta ** (-(2.0 * i) / cfg.dh)
    ang = torch.arange(cfg.tmax, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cos(ang).to(device), torch.sin(ang).to(device)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved pairs (2i, 2i+1) of each head; x [..., T, H, Dh], cos/sin [T, Dh/2]."""
    xs = x.float().unflatten(-1, (-1, 2))
    a, b = xs[..., 0], xs[..., 1]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return Fn.gelu(x, approximate="tanh")


# Dense products on CUDA run on this library's tensor-core NT GEMM (HRM_REVLM_TC=0: PyTorch's bf16 matmul instead).
TC_GEMM = os.environ.get("HRM_REVLM_TC", "1") != "0"


class _TcMatmul(torch.autograd.Function):
    """``y = x @ W`` (``x [..., K]`` fp32, ``W [K, N]`` fp32, possibly a column slice) with bf16 operands and fp32
    accumulation on the tensor-core NT GEMM (``ops.gemm_nt``, C = A . B^T with both operands K-major).  Backward goes
    through the same kernel after transposing into that form, as the reference trainer does around its WMMA GEMM
    (llm_engine.cu:500-524): ``dx = dy . W^T`` is ``gemm_nt(dy, W)`` and ``dW = x^T . dy`` is
    ``gemm_nt(x^T, dy^T)``."""

    @staticmethod
    def forward(ctx, x, w):
        from .. import ops
        K, N = w.shape
        xb = x.reshape(-1, K).to(torch.bfloat16).contiguous()
        y = ops.gemm_nt(xb, _bf16_copy(w.t()))
        ctx.save_for_backward(xb, w)
        ctx.xshape = x.shape
        return y.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        from .. import ops
        xb, w = ctx.saved_tensors
        K, N = w.shape
        dyb = dy.reshape(-1, N).to(torch.bfloat16).contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = ops.gemm_nt(dyb, _bf16_copy(w)).view(ctx.xshape)
        if ctx.needs_input_grad[1]:
            dw = ops.gemm_nt(_bf16_copy(xb.t()), _bf16_copy(dyb.t()))
        return dx, dw


def _bf16_copy(t: torch.Tensor) -> torch.Tensor:
    """A contiguous bf16 copy of a (possibly transposed or sliced) 2-D view in one copy kernel (conversion and
    layout change together, where ``.to(bf16).contiguous()`` of a transposed view takes two)."""
    out = torch.empty(t.shape, dtype=torch.bfloat16, device=t.device)
    out.copy_(t)
    return out


def _tc_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    """Shapes the NT GEMM takes in both directions: every leading dimension a multiple of 8 elements."""
    K, N = w.shape
    M = x.numel() // max(1, K)
    return TC_GEMM and x.is_cuda and K % 8 == 0 and N % 8 == 0 and M % 8 == 0 and M > 0


def _mm(x: torch.Tensor, w: torch.Tensor, lowp: bool) -> torch.Tensor:
    if lowp:
        if _tc_ok(x, w):
            return _TcMatmul.apply(x, w)
        return (x.to(torch.bfloat16) @ w.to(torch.bfloat16)).float()
    return x.float() @ w


# Causal attention on CUDA runs on this library's trainer flash kernels for head dims 16 and 32 (HRM_REVLM_FLASH=0:
# PyTorch's scaled_dot_product_attention instead).
FLASH_ATTN = os.environ.get("HRM_REVLM_FLASH", "1") != "0"


class _FlashAttn(torch.autograd.Function):
    """Causal attention of ``[B, T, H, Dh]`` fp32 rows on ``ops.flash_train_fwd`` / ``ops.flash_train_bwd``: the
    forward keeps only the output and the per-row log-sum-exp, and the backward recomputes the probabilities tile by
    tile, as the reference trainer's flash kernels do (llm_engine.cu:856-1146)."""

    @staticmethod
    def forward(ctx, q, k, v):
        from .. import ops
        q, k, v = (t.float().contiguous() for t in (q, k, v))
        o, lse = ops.flash_train_fwd(q, k, v)
        ctx.save_for_backward(q, k, v, o, lse)
        return o

    @staticmethod
    def backward(ctx, dout):
        from .. import ops
        return ops.flash_train_bwd(*ctx.saved_tensors, dout.float().contiguous())


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lowp: bool) -> torch.Tensor:
    """``q, k, v [B, T, H, Dh]`` -> fp32 ``[B, T, H, Dh]``."""
    if FLASH_ATTN and q.is_cuda and q.shape[-1] in (16, 32):
        return _FlashAttn.apply(q, k, v)
    dt = torch.bfloat16 if lowp else torch.float32
    o = Fn.scaled_dot_product_attention(q.transpose(1, 2).to(dt), k.transpose(1, 2).to(dt),
                                        v.transpose(1, 2).to(dt), is_causal=True)
    return o.transpose(1, 2).float()


def f_block(cfg: RevConfig, x2, gf, Wq, Wk, Wv, Wo, cos, sin, lowp):
    B, T, _ = x2.shape
    n = rms(x2, gf, cfg.eps)
    q = _mm(n, Wq, lowp).view(B, T, cfg.heads, cfg.dh)
    k = _mm(n, Wk, lowp).view(B, T, cfg.heads, cfg.dh)
    v = _mm(n, Wv, lowp).view(B, T, cfg.heads, cfg.dh)
    q, k = apply_rope(q, cos[:T], sin[:T]), apply_rope(k, cos[:T], sin[:T])
    o = causal_attention(q, k, v, lowp).reshape(B, T, cfg.dhf)
    return _mm(o, Wo, lowp)


def g_block(cfg: RevConfig, y1, gg, W1, W2, lowp):
    n = rms(y1, gg, cfg.eps)
    return _mm(gelu_tanh(_mm(n, W1, lowp)), W2, lowp)


def _layer_params(p: Dict[str, torch.Tensor], l: int):
    return [p[f"gf.{l}"], p[f"Wq.{l}"], p[f"Wk.{l}"], p[f"Wv.{l}"], p[f"Wo.{l}"]], [p[f"gg.{l}"], p[f"W1.{l}"], p[f"W2.{l}"]]


class _ReversibleStack(torch.autograd.Function):
    """All layers; saves only the outputs and rebuilds each layer's inputs in backward."""

    @staticmethod
    def forward(ctx, cfg, cos, sin, lowp, x1, x2, *params):
        L = cfg.layers
        fp = [params[8 * l:8 * l + 5] for l in range(L)]
        gp = [params[8 * l + 5:8 * l + 8] for l in range(L)]
        with torch.no_grad():
            y1, y2 = x1, x2
            for l in range(L):
                y1 = y1 + f_block(cfg, y2, *fp[l], cos, sin, lowp)
                y2 = y2 + g_block(cfg, y1, *gp[l], lowp)
        ctx.cfg, ctx.cos, ctx.sin, ctx.lowp = cfg, cos, sin, lowp
        ctx.save_for_backward(y1, y2, *params)
        return y1, y2

    @staticmethod
    def backward(ctx, dy1, dy2):
        cfg, cos, sin, lowp = ctx.cfg, ctx.cos, ctx.sin, ctx.lowp
        y1, y2, *params = ctx.saved_tensors
        L = cfg.layers
        grads = [None] * len(params)
        dy1, dy2 = dy1.float(), dy2.float()
        for l in range(L - 1, -1, -1):
            fp = [p.detach().requires_grad_(True) for p in params[8 * l:8 * l + 5]]
            gp = [p.detach().requires_grad_(True) for p in params[8 * l + 5:8 * l + 8]]
            with torch.enable_grad():
                z1 = y1.detach().requires_grad_(True)
                gout = g_block(cfg, z1, *gp, lowp)
            dz1, *dgp = torch.autograd.grad(gout, [z1] + gp, dy2)
            with torch.no_grad():
                x2 = y2 - gout
            dy1 = dy1 + dz1
            with torch.enable_grad():
                w2 = x2.detach().requires_grad_(True)
                fout = f_block(cfg, w2, *fp, cos, sin, lowp)
            dw2, *dfp = torch.autograd.grad(fout, [w2] + fp, dy1)
            with torch.no_grad():
                x1 = y1 - fout
            dy2 = dy2 + dw2
            grads[8 * l:8 * l + 5] = dfp
            grads[8 * l + 5:8 * l + 8] = dgp
            y1, y2 = x1, x2
        return (None, None, None, None, dy1, dy2, *grads)


class RevLM(torch.nn.Module):
    def __init__(self, cfg: RevConfig, device="cpu", flat: Optional[torch.Tensor] = None, seed: int = 123,
                 lowp: Optional[bool] = None, reversible: bool = True):
        super().__init__()
        self.cfg = cfg
        self.device = torch.device(device)
        f = flat if flat is not None else init_flat(cfg, seed)
        self.flat = torch.nn.Parameter(f.to(self.device, torch.float32).contiguous())
        self.lowp = (self.device.type == "cuda") if lowp is None else lowp
        self.reversible = reversible
        self.cos, self.sin = rope_tables(cfg, self.device)

    def p(self) -> Dict[str, torch.Tensor]:
        return views(self.cfg, self.flat)

    def stack_params(self, p) -> List[torch.Tensor]:
        out = []
        for l in range(self.cfg.layers):
            a, b = _layer_params(p, l)
            out += a + b
        return out

    def hidden(self, tok: torch.Tensor) -> torch.Tensor:
        cfg, p = self.cfg, self.p()
        T = tok.shape[1]
        x = p["wte"][tok.long()] + p["wpe"][:T][None]
        x1, x2 = x[..., :cfg.dhf].contiguous(), x[..., cfg.dhf:].contiguous()
        if self.reversible and torch.is_grad_enabled():
            y1, y2 = _ReversibleStack.apply(cfg, self.cos, self.sin, self.lowp, x1, x2, *self.stack_params(p))
        else:
            y1, y2 = x1, x2
            for l in range(cfg.layers):
                fp, gp = _layer_params(p, l)
                y1 = y1 + f_block(cfg, y2, *fp, self.cos, self.sin, self.lowp)
                y2 = y2 + g_block(cfg, y1, *gp, self.lowp)
        return rms(torch.cat([y1, y2], -1), p["gout"], cfg.eps)

    def logits(self, tok: torch.Tensor) -> torch.Tensor:
        h = self.hidden(tok)
        return _mm(h, self.p()["Wout"][:, :self.cfg.vocab], self.lowp)

    def loss(self, tok: torch.Tensor, tgt: torch.Tensor, vchunk: int = 4096) -> torch.Tensor:
        """Mean next-token cross entropy; the logits are produced vocabulary chunk by chunk with an online
        log-sum-exp (no [N, V] matrix), as the reference's streaming head does."""
        cfg = self.cfg
        h = self.hidden(tok).reshape(-1, cfg.d)
        t = tgt.reshape(-1).long()
        W = self.p()["Wout"]
        m = torch.full((h.shape[0],), -float("inf"), device=h.device)
        s = torch.zeros(h.shape[0], device=h.device)
        tl = torch.zeros(h.shape[0], device=h.device)
        for v0 in range(0, cfg.vocab, vchunk):
            v1 = min(cfg.vocab, v0 + vchunk)
            z = _mm(h, W[:, v0:v1], self.lowp)
            zm = z.max(-1).values
            mn = torch.maximum(m, zm)
            s = s * torch.exp(m - mn) + torch.exp(z - mn[:, None]).sum(-1)
            m = mn
            inside = (t >= v0) & (t < v1)
            tl = tl + torch.where(inside, z.gather(1, (t - v0).clamp(0, v1 - v0 - 1)[:, None])[:, 0],
                                  torch.zeros_like(tl))
        return (m + torch.log(s) - tl).mean()


# ------------------------------------------------------------------------------------------------ incremental decode
class ChatState:
    """Incremental greedy decoding with a per-layer KV cache (batch 1), the reference's chat path (:1856-2165).

    Every step has static shapes (attention runs over the whole Tmax cache under a position mask, the cache row is
    written at a device-side index), so on a GPU the step is captured once as a CUDA graph and each token costs one
    graph replay plus one 8-byte device-to-host read of the next token."""

    def __init__(self, model: RevLM, use_graph: Optional[bool] = None):
        self.m = model
        cfg = model.cfg
        dev = model.device
        self.k = torch.zeros(cfg.layers, cfg.tmax, cfg.heads, cfg.dh, device=dev)
        self.v = torch.zeros_like(self.k)
        self.t = 0
        self.tok_in = torch.zeros((), dtype=torch.long, device=dev)
        self.pos_in = torch.zeros((), dtype=torch.long, device=dev)
        self.tok_out = torch.zeros((), dtype=torch.long, device=dev)
        self.ar = torch.arange(cfg.tmax, device=dev)
        self.graph = None
        self.use_graph = (dev.type == "cuda") if use_graph is None else use_graph

    def reset(self) -> None:
        self.k.zero_()
        self.v.zero_()
        self.t = 0

    @torch.no_grad()
    def _step_static(self) -> None:
        m, cfg = self.m, self.m.cfg
        p = m.p()
        t = self.pos_in
        x = p["wte"][self.tok_in] + p["wpe"][t]
        y1, y2 = x[:cfg.dhf], x[cfg.dhf:]
        cos, sin = m.cos[t].unsqueeze(0), m.sin[t].unsqueeze(0)
        visible = self.ar <= t
        for l in range(cfg.layers):
            n = rms(y2, p[f"gf.{l}"], cfg.eps)
            q = apply_rope((n @ p[f"Wq.{l}"]).view(1, cfg.heads, cfg.dh), cos, sin)[0]
            k = apply_rope((n @ p[f"Wk.{l}"]).view(1, cfg.heads, cfg.dh), cos, sin)[0]
            self.k[l].index_copy_(0, t.view(1), k.unsqueeze(0))
            self.v[l].index_copy_(0, t.view(1), (n @ p[f"Wv.{l}"]).view(1, cfg.heads, cfg.dh))
            sc = torch.einsum("hd,thd->ht", q, self.k[l]) / math.sqrt(cfg.dh)
            sc = sc.masked_fill(~visible[None, :], -float("inf"))
            o = torch.einsum("ht,thd->hd", torch.softmax(sc, -1), self.v[l]).reshape(cfg.dhf)
            y1 = y1 + o @ p[f"Wo.{l}"]
            n = rms(y1, p[f"gg.{l}"], cfg.eps)
            y2 = y2 + gelu_tanh(n @ p[f"W1.{l}"]) @ p[f"W2.{l}"]
        h = rms(torch.cat([y1, y2]), p["gout"], cfg.eps)
        self.tok_out.copy_(torch.argmax(h @ p["Wout"][:, :cfg.vocab]))

    def _capture(self) -> None:
        s = torch.cuda.Stream(device=self.m.device)
        s.wait_stream(torch.cuda.current_stream(self.m.device))
        with torch.cuda.stream(s):
            self._step_static()
        torch.cuda.current_stream(self.m.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._step_static()
        self.graph = g

    @torch.no_grad()
    def step(self, token: int) -> int:
        if self.t >= self.m.cfg.tmax:
            raise RuntimeError("context full")
        self.tok_in.fill_(int(token))
        self.pos_in.fill_(self.t)
        if self.use_graph:
            if self.graph is None:
                k0, v0 = self.k.clone(), self.v.clone()
                self._capture()                  # the warm-up and capture ran the step twice: restore the cache
                self.k.copy_(k0)
                self.v.copy_(v0)
            self.graph.replay()
        else:
            self._step_static()
        self.t += 1
        return int(self.tok_out)


# ------------------------------------------------------------------------------------------------ checkpoint v11
def save_ckpt(path: str, cfg: RevConfig, tables, flat: torch.Tensor) -> None:
    """Checkpoint version 11 (layout of ``save_ckpt``, llm_engine.cu:387-407): header, tokenizer tables, weights."""
    id2pair, id2pair2, hkeys, hvals = tables
    pow2 = int(hkeys.size).bit_length() - 1
    assert (1 << pow2) == hkeys.size
    with open(path, "wb") as f:
        f.write(struct.pack("<9I", CKPT_MAGIC, CKPT_VERSION, cfg.k1, cfg.k2, cfg.d, cfg.heads, cfg.layers, cfg.ffn,
                            cfg.tmax))
        f.write(np.ascontiguousarray(id2pair, np.uint16).tobytes())
        if cfg.k2 > 0:
            f.write(np.ascontiguousarray(id2pair2, np.uint32).tobytes())
        f.write(struct.pack("<I", pow2))
        f.write(np.ascontiguousarray(hkeys, np.uint32).tobytes())
        f.write(np.ascontiguousarray(hvals, np.uint16).tobytes())
        f.write(flat.detach().to("cpu", torch.float32).contiguous().numpy().tobytes())


def load_ckpt(path: str, cfg: Optional[RevConfig] = None):
    """Returns (cfg, tables, flat fp32 tensor).  With ``cfg`` given, its dimensions must match the file."""
    raw = open(path, "rb").read()
    magic, ver, k1, k2, d, h, nl, ff, tm = struct.unpack_from("<9I", raw, 0)
    if magic != CKPT_MAGIC:
        raise ValueError(f"{path}: bad checkpoint magic")
    if ver != CKPT_VERSION:
        raise ValueError(f"{path}: unsupported checkpoint version {ver}")
    file_cfg = RevConfig(k1=k1, k2=k2, d=d, heads=h, layers=nl, ffn=ff, tmax=tm)
    if cfg is not None and (cfg.k1, cfg.k2, cfg.d, cfg.heads, cfg.layers, cfg.ffn, cfg.tmax) != \
            (k1, k2, d, h, nl, ff, tm):
        raise ValueError(f"{path}: checkpoint dimensions do not match the configured model")
    off = 36
    id2pair = np.frombuffer(raw, np.uint16, k1, off)
    off += 2 * k1
    id2pair2 = np.frombuffer(raw, np.uint32, k2, off) if k2 else np.zeros(0, np.uint32)
    off += 4 * k2
    (pow2,) = struct.unpack_from("<I", raw, off)
    off += 4
    hs = 1 << pow2
    hkeys = np.frombuffer(raw, np.uint32, hs, off)
    off += 4 * hs
    hvals = np.frombuffer(raw, np.uint16, hs, off)
    off += 2 * hs
    n = file_cfg.weights_floats()
    if len(raw) < off + 4 * n:
        raise ValueError(f"{path}: truncated checkpoint")
    flat = torch.from_numpy(np.frombuffer(raw, np.float32, n, off).copy())
    return file_cfg, (id2pair.copy(), id2pair2.copy(), hkeys.copy(), hvals.copy()), flat
