"""Experiments-plane trainer and chat REPL for the reversible LM (the reference's ``llm_engine.cu`` main,
:2253-2415, and its launcher ``experiments/run_llm_orig.sh:2936-3030``).

    python -m hrm_flashrenderer_b200.experiments.llm --train --data corpus.txt --ckpt ckpt.bin [--steps N ...]
    torchrun --nproc-per-node 8 -m hrm_flashrenderer_b200.experiments.llm --train ...      (data parallel)
    python -m hrm_flashrenderer_b200.experiments.llm --chat --ckpt ckpt.bin [--measure] [--chat_prompt TEXT]

Same flags and semantics as the reference: the checkpoint (version 11: tokenizer tables + weights) is loaded when it
exists and training continues from it; otherwise the tokenizer comes from ``--index`` (an IDX7 file) or is built from
the corpus, and weights are initialised from ``--seed``.  Each step trains on random windows of ``--seq`` tokens;
``--batch`` is the global batch, split across ranks in proportion to device memory.  Logging every ``--log_every``
steps prints loss / ppl (and tok/s with ``--measure``); a non-finite loss aborts; the checkpoint is saved every
``--save_every`` steps and at the end.  ``--auto_ckpt DIR`` names the checkpoint after an md5 of the
hyper-parameters and resumes it automatically, like the reference launcher.

B200 design: one process per GPU (torchrun); gradients are exchanged with one NCCL all-reduce of the flat gradient
buffer; the optimizer is replicated on every rank (fused device-side clip + AdamW kernels, no host round trip); on a
single GPU the whole step (H2D of the step's tokens excluded) is captured in a CUDA graph.
"""
from __future__ import annotations

import argparse
import hashlib
import math
import os
import sys
import time
from pathlib import Path
from typing import List, Sequence

import numpy as np
import torch
import torch.distributed as dist

from .pairindex import PairIndex
from .revlm import ChatState, RevConfig, RevLM, init_flat, load_ckpt, save_ckpt


def split_batch(batch: int, mems: Sequence[int]) -> List[int]:
    """Per-device batch in proportion to device memory, each >= 1, summing to ``batch`` (reference :2318-2329;
    when ``batch`` is smaller than the device count every device still gets one sample, where the reference's
    loop never terminates)."""
    tot = float(sum(mems))
    b = [max(1, int(math.floor(m / tot * batch))) for m in mems]
    while sum(b) > batch and any(x > 1 for x in b):   # with batch < devices every device still keeps 1
        for i in range(len(b)):
            if sum(b) > batch and b[i] > 1:
                b[i] -= 1
    while sum(b) < batch:
        for i in range(len(b)):
            if sum(b) < batch:
                b[i] += 1
    return b


def auto_ckpt_path(directory: str, args) -> str:
    keys = ("data", "k1", "k2", "dmodel", "heads", "layers", "ffn", "tmax", "seq", "batch", "lr", "wd", "clip", "seed")
    sig = "|".join(f"{k}={getattr(args, k)}" for k in keys)
    return str(Path(directory) / f"ckpt_{hashlib.md5(sig.encode()).hexdigest()[:12]}.bin")


class Optimizer:
    """Decoupled AdamW with global-norm clipping over the flat parameter buffer (b1 0.9, b2 0.999, eps 1e-8)."""

    def __init__(self, flat: torch.nn.Parameter, lr: float, wd: float, clip: float):
        self.flat, self.lr, self.wd, self.clip = flat, lr, wd, clip
        self.m = torch.zeros_like(flat.data)
        self.v = torch.zeros_like(flat.data)
        dev = flat.device
        self.step_t = torch.ones(1, dtype=torch.int32, device=dev)    # 1-based step of the next update
        self.partial = torch.zeros(1024, dtype=torch.float32, device=dev)
        self.scalars = torch.zeros(2, dtype=torch.float32, device=dev)   # grad norm, clip factor
        self.native = dev.type == "cuda"
        if self.native:
            from .. import ops
            self._C = ops.ext()

    def step(self, grad: torch.Tensor) -> None:
        b1, b2, eps = 0.9, 0.999, 1e-8
        if self.native:
            self._C.grad_clip_factor(grad, self.clip, self.partial, self.scalars)
            self._C.adamw_flat(self.flat.data, self.m, self.v, grad, self.lr, self.wd, b1, b2, eps, self.step_t,
                               self.scalars)
            return
        g = torch.nan_to_num(grad, nan=0.0, posinf=0.0, neginf=0.0)
        norm = float(torch.sqrt((g * g).sum()))
        cs = self.clip / norm if (math.isfinite(norm) and norm > self.clip > 0) else 1.0
        g = grad * cs
        g = torch.where(torch.isfinite(g), g, torch.zeros_like(g))
        t = int(self.step_t.item())
        self.m.mul_(b1).add_(g, alpha=1 - b1)
        self.v.mul_(b2).addcmul_(g, g, value=1 - b2)
        mh, vh = self.m / (1 - b1 ** t), self.v / (1 - b2 ** t)
        w = self.flat.data
        w.sub_(self.lr * (mh / (vh.sqrt() + eps) + self.wd * w))
        self.step_t += 1


class Trainer:
    def __init__(self, cfg: RevConfig, flat: torch.Tensor, ids: np.ndarray, batch: int, seq: int, lr: float,
                 wd: float, clip: float, seed: int, device, rank: int = 0, world: int = 1, use_graph: bool = True):
        self.cfg, self.ids, self.B, self.T = cfg, ids, batch, seq
        self.rank, self.world, self.seed = rank, world, seed
        self.device = torch.device(device)
        self.model = RevLM(cfg, self.device, flat)
        self.opt = Optimizer(self.model.flat, lr, wd, clip)
        self.model.flat.grad = torch.zeros_like(self.model.flat.data)
        pin = self.device.type == "cuda"
        self.h_tok = torch.zeros(batch, seq, dtype=torch.int32).pin_memory() if pin else torch.zeros(batch, seq, dtype=torch.int32)
        self.h_tgt = torch.zeros_like(self.h_tok).pin_memory() if pin else torch.zeros_like(self.h_tok)
        self.tok = torch.zeros(batch, seq, dtype=torch.int32, device=self.device)
        self.tgt = torch.zeros_like(self.tok)
        self.loss_t = torch.zeros((), device=self.device)
        self.graph = None
        self.use_graph = use_graph and self.device.type == "cuda"

    def _fill(self, step: int) -> None:
        max_start = len(self.ids) - (self.T + 1)
        if max_start <= 0:
            raise RuntimeError("encoded corpus shorter than --seq + 1 tokens")
        rng = np.random.default_rng([self.seed, step, self.rank])
        starts = rng.integers(0, max_start, size=self.B)
        idx = starts[:, None] + np.arange(self.T + 1)[None, :]
        win = self.ids[idx].astype(np.int32)
        self.h_tok.numpy()[:] = win[:, :-1]
        self.h_tgt.numpy()[:] = win[:, 1:]
        self.tok.copy_(self.h_tok, non_blocking=True)
        self.tgt.copy_(self.h_tgt, non_blocking=True)

    def _fwd_bwd(self) -> None:
        g = self.model.flat.grad
        g.zero_()
        loss = self.model.loss(self.tok, self.tgt)
        loss.backward()
        self.loss_t.copy_(loss.detach())

    def _device_step(self) -> None:
        self._fwd_bwd()
        if self.world > 1:
            dist.all_reduce(self.model.flat.grad)
            self.model.flat.grad.div_(self.world)
        self.opt.step(self.model.flat.grad)

    def _capture(self) -> None:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):   # warm-up (allocator, autotuning) on a side stream, as graph capture requires
                self._fwd_bwd()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._fwd_bwd()
            if self.world == 1:
                self.opt.step(self.model.flat.grad)
        self.graph = g

    def train_step(self, step: int) -> torch.Tensor:
        self._fill(step)
        if self.use_graph and self.graph is None:
            try:
                self._capture()
            except Exception as e:   # capture is an optimisation: fall back to eager launches
                print(f"[train] CUDA graph capture unavailable ({type(e).__name__}: {e}); running eagerly",
                      file=sys.stderr)
                self.use_graph = False
                self.graph = None
        if self.graph is not None:
            self.graph.replay()
            if self.world > 1:
                dist.all_reduce(self.model.flat.grad)
                self.model.flat.grad.div_(self.world)
                self.opt.step(self.model.flat.grad)
        else:
            self._device_step()
        return self.loss_t


def resolve_tokenizer(args, data: bytes):
    """(PairIndex, weights or None, RevConfig): checkpoint > IDX7 index > build from the corpus."""
    base = dict(d=args.dmodel, heads=args.heads, layers=args.layers, ffn=args.ffn, tmax=args.tmax)
    if args.ckpt and Path(args.ckpt).is_file():
        cfg, tables, flat = load_ckpt(args.ckpt)
        return PairIndex.from_tables(cfg.k1, cfg.k2, *tables), flat, cfg
    if args.index and Path(args.index).is_file():
        pi = PairIndex.load(args.index)
    else:
        pi = PairIndex.build_bytes(data, args.k1, args.k2)
    return pi, None, RevConfig(k1=pi.k1, k2=pi.k2, **base)


def chat_repl(model: RevLM, pi: PairIndex, prompt: str, measure: bool, gen_max: int = 200, inp=None, out=None) -> None:
    inp = inp or sys.stdin
    out = out or sys.stdout
    st = ChatState(model)
    tmax = model.cfg.tmax
    nxt = None
    for t in (pi.encode(prompt).tolist() if prompt else []):
        if st.t >= tmax:
            break
        nxt = st.step(t)
    print("[chat] commands: /reset /quit  (greedy decode, incremental KV, up to %d tokens)" % gen_max, file=sys.stderr)
    for line in inp:
        line = line.rstrip("\n")
        if line == "/quit":
            break
        if line == "/reset":
            st.reset()
            nxt = None
            continue
        for t in pi.encode(line + "\n").tolist():
            if st.t >= tmax:
                break
            nxt = st.step(t)
        if st.t >= tmax or nxt is None:
            out.write("\n[ctx full]\n")
            out.flush()
            continue
        t0 = time.perf_counter()
        n = 0
        for _ in range(gen_max):
            if st.t >= tmax:
                break
            piece = pi.decode_bytes([nxt])
            out.write(piece.decode("utf-8", errors="replace"))
            out.flush()
            n += 1
            nxt = st.step(nxt)
            if b"\n" in piece:
                break
        if measure:
            print(f"\n[tok/s: {n / max(time.perf_counter() - t0, 1e-9):.1f}]", file=sys.stderr)
        if st.t >= tmax:
            out.write("\n[ctx full]\n")
            out.flush()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-llm", description="reversible LM trainer / chat (experiments)")
    ap.add_argument("--train", action="store_true")
    ap.add_argument("--chat", action="store_true")
    ap.add_argument("--measure", action="store_true")
    ap.add_argument("--chat_prompt", default="")
    ap.add_argument("--data", default="tinyshakespeare.txt")
    ap.add_argument("--ckpt", default="ckpt.bin")
    ap.add_argument("--auto_ckpt", default="", help="directory: checkpoint named by a hash of the hyper-parameters")
    ap.add_argument("--index", default="index_v7.bin")
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--seq", type=int, default=128)
    ap.add_argument("--gpus", type=int, default=2, help="ignored under torchrun (one process per GPU)")
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--wd", type=float, default=0.01)
    ap.add_argument("--clip", type=float, default=1.0)
    ap.add_argument("--log_every", type=int, default=50)
    ap.add_argument("--save_every", type=int, default=500)
    ap.add_argument("--seed", type=int, default=123)
    ap.add_argument("--graph", type=int, default=1)
    ap.add_argument("--no_graph", action="store_true")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--k1", type=int, default=8192)
    ap.add_argument("--k2", type=int, default=8192)
    ap.add_argument("--dmodel", type=int, default=256)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--layers", type=int, default=6)
    ap.add_argument("--ffn", type=int, default=1024)
    ap.add_argument("--tmax", type=int, default=512)
    a = ap.parse_args(argv)
    if not a.train and not a.chat:
        a.train = True
    if a.seq % 16 or not 16 <= a.seq <= a.tmax:
        raise SystemExit("--seq must be a multiple of 16 in [16, tmax]")
    if a.auto_ckpt:
        Path(a.auto_ckpt).mkdir(parents=True, exist_ok=True)
        a.ckpt = auto_ckpt_path(a.auto_ckpt, a)
    data = Path(a.data).read_bytes() if Path(a.data).is_file() else b""
    if not data and not (a.chat and Path(a.ckpt).is_file()):
        raise SystemExit(f"corpus not found or empty: {a.data}")
    pi, flat, cfg = resolve_tokenizer(a, data)
    if flat is None:
        flat = init_flat(cfg, a.seed)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device(a.device)
    if dev.type == "cuda":
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)

    if a.chat:
        model = RevLM(cfg, dev, flat, reversible=False)
        chat_repl(model, pi, a.chat_prompt, a.measure)
        return 0

    if world > 1:
        from ..parallel.dist import init_dist_env
        init_dist_env("nccl" if dev.type == "cuda" else "gloo")
        mems = [torch.cuda.get_device_properties(i).total_memory for i in range(world)] if dev.type == "cuda" \
            else [1] * world
    else:
        mems = [1]
    per = split_batch(a.batch, mems)
    ids = pi.encode(data)
    if len(ids) < a.seq + 2:
        raise SystemExit("encoded corpus too small for --seq")
    tr = Trainer(cfg, flat, ids, per[rank], a.seq, a.lr, a.wd, a.clip, a.seed, dev, rank, world,
                 use_graph=bool(a.graph) and not a.no_graph)
    if rank == 0:
        print(f"llm: V={cfg.vocab}(Vpad={cfg.vpad}) K={cfg.k1 + cfg.k2} D={cfg.d} Dh={cfg.dh} L={cfg.layers} "
              f"H={cfg.heads} F={cfg.ffn} T={a.seq} gpus={world} batch={a.batch} {per}", flush=True)
    t0 = time.perf_counter()
    for step in range(1, a.steps + 1):
        loss_t = tr.train_step(step)
        if step == 1 and a.measure:
            if dev.type == "cuda":
                torch.cuda.synchronize()
            t0 = time.perf_counter()
        if a.log_every > 0 and step % a.log_every == 0:
            lt = loss_t.detach().clone()
            if world > 1:
                dist.all_reduce(lt)
                lt /= world
            lm = float(lt)
            if rank == 0:
                msg = f"step {step}/{a.steps} loss={lm:.6f} ppl={math.exp(min(lm, 80)):.3f}"
                if a.measure:
                    el = time.perf_counter() - t0
                    msg += f" tok/s={a.log_every * a.batch * a.seq / max(el, 1e-9):.1f}"
                    t0 = time.perf_counter()
                print(msg, flush=True)
            if not math.isfinite(lm):
                raise SystemExit("loss NaN/Inf")
        if a.save_every > 0 and step % a.save_every == 0 and rank == 0:
            save_ckpt(a.ckpt, cfg, pi.tables(), tr.model.flat.data)
            print(f"[*] saved: {a.ckpt}", flush=True)
    if rank == 0:
        save_ckpt(a.ckpt, cfg, pi.tables(), tr.model.flat.data)
        print(f"[*] saved final: {a.ckpt}", flush=True)
    if world > 1:
        tr.graph = None
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
