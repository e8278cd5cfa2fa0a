"""Tensor-parallel lane: one process per GPU, rank 0 serves, the other ranks mirror its engine calls.

Reference: ``hrm_flash/flash_daemon.py:70-236`` (``mp.spawn`` TP workers; rank 0 owns a
``multiprocessing.connection`` RPC listener with ``ping`` / ``generate`` / ``shutdown`` and broadcasts command,
shape and token ids to the other ranks with NCCL before each request) and ``flash_daemon_client.py``
(``HRM_FLASH_DAEMON=host:port``, ``HRM_FLASH_AUTHKEY``).

Here the control plane is separate from the data plane: rank 0 runs the continuous-batching scheduler and mirrors
each engine call (prefill chunk, decode staging, decode step, release) to the other ranks over a gloo process group,
so the GPU collectives inside the model (NCCL / fused peer-memory kernels) always line up and device ranks never
block on host control traffic during a step.  The same worker runs either the RPC daemon (``hrm-flashd``) or the
HTTP lane (``hrm-flash serve --world N``).
"""
from __future__ import annotations

import argparse
import datetime
import os
import threading
from dataclasses import dataclass
from multiprocessing.connection import Client, Listener
from typing import Any, Callable, Dict, Optional

import torch
import torch.distributed as dist

from ..runtime.sampling import sampling_from_request


class MirroredEngine:
    """Rank-0 proxy of an :class:`InferenceEngine`: every state-changing call is first broadcast to the followers."""

    _MIRRORED = ("prefill", "load_decode_batch", "decode_step", "release", "new_seq", "capture", "reset",
                 "match_prefix", "publish_prefix")

    def __init__(self, engine, group, watchdog=None):
        self._engine = engine
        self._group = group
        self._lock = threading.Lock()
        self._watchdog = watchdog

    def _bcast(self, name: str, payload) -> None:
        # a lost follower is found on the host before the next broadcast / collective is issued
        if self._watchdog is not None and name != "__shutdown__":
            self._watchdog.check()
        dist.broadcast_object_list([(name, payload)], src=0, group=self._group)

    def __getattr__(self, item):
        eng = object.__getattribute__(self, "_engine")
        if item in MirroredEngine._MIRRORED:
            fn = getattr(eng, item)

            def call(*args, **kwargs):
                # decode graphs are addressed by bucket on the followers
                wire = tuple(a.bucket if hasattr(a, "bucket") and hasattr(a, "graph") else a for a in args)
                with self._lock:
                    self._bcast(item, (wire, kwargs))
                    return fn(*args, **kwargs)
            return call
        return getattr(eng, item)

    def shutdown(self) -> None:
        with self._lock:
            self._bcast("__shutdown__", ((), {}))


def follower_loop(engine, group, on_shutdown: Optional[Callable[[], None]] = None) -> None:
    """Replay rank 0's engine calls until shutdown."""
    while True:
        box = [None]
        dist.broadcast_object_list(box, src=0, group=group)
        name, (args, kwargs) = box[0]
        if name == "__shutdown__":
            if on_shutdown is not None:
                on_shutdown()
            return
        if name == "decode_step":
            engine.decode_step(engine._decode_state(args[0]))
        else:
            getattr(engine, name)(*args, **kwargs)


@dataclass
class LaneArgs:
    model: str
    world: int
    max_seq_len: int = 8192
    prefill_chunk_size: int = 4096
    max_batch: int = 64
    device: str = "cuda"
    seed: int = 0
    master_port: int = 29555
    kv_fraction: float = 0.85
    num_kv_blocks: int = 0
    heartbeat_timeout_s: float = 30.0   # a TP peer silent this long is treated as lost
    packed_cache_dir: str = ""           # per-rank packed-shard cache for DSI8 exports (default: HRM_PACKED_CACHE)
    fused_collectives: bool = True       # TP > 1 on CUDA: in-kernel NVLink all-reduce / argmax (False: NCCL calls)
    prefix_cache: bool = True            # share the KV blocks of prompt prefixes seen before (shared system prompts)


def build_engine(a: LaneArgs, rank: int, world: int, comm):
    from ..config import EngineConfig, get_preset
    from ..models.llama import LlamaW8
    from ..runtime.engine import InferenceEngine
    from ..runtime.kv_cache import PagedKVPool
    dev = torch.device("cuda", rank) if a.device == "cuda" else torch.device("cpu")
    if a.model.startswith("synthetic:"):
        cfg = get_preset(a.model.split(":", 1)[1])
        model = LlamaW8.synthesize(cfg, rank=rank, world=world, device=dev, seed=a.seed, comm=comm,
                                   max_pos=a.max_seq_len + 16)
    else:
        model = LlamaW8.from_dsi8(a.model, rank=rank, world=world, device=dev, comm=comm, max_pos=a.max_seq_len + 16,
                                  cache_dir=a.packed_cache_dir or os.environ.get("HRM_PACKED_CACHE") or None)
        cfg = model.cfg
    if a.fused_collectives:
        # the row-parallel GEMMs reduce over peer memory inside the kernel and the greedy pick exchanges its argmax
        # keys inside the argmax kernel; collective over the TP group, and a no-op at TP = 1 or on the CPU
        model.enable_fused_collectives()
    if a.num_kv_blocks:
        nb = a.num_kv_blocks
    elif dev.type == "cuda":
        free, _ = torch.cuda.mem_get_info(dev)
        nb = PagedKVPool.blocks_for_budget(int(free * a.kv_fraction), cfg.layers, model.plan.local_kv_heads,
                                           cfg.head_dim)
    else:
        nb = a.max_batch * ((a.max_seq_len + 15) // 16)
    # every rank must size the pool identically (block ids are mirrored): take the minimum over ranks
    if world > 1:
        t = torch.tensor([nb], dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=comm.control if hasattr(comm, "control") else None)
        nb = int(t.item())
    ecfg = EngineConfig(tp=world, max_seq_len=a.max_seq_len, max_batch=a.max_batch, prefill_chunk=a.prefill_chunk_size,
                        use_cuda_graphs=dev.type == "cuda", prefix_cache=a.prefix_cache)
    return InferenceEngine(model, ecfg, num_blocks=nb)


def run_worker(rank: int, a: LaneArgs, on_rank0: Callable[[Any], None]) -> None:
    """Body of one TP process: init process groups, build the shard, then serve (rank 0) or follow."""
    from ..parallel.dist import init_dist
    from ..parallel.comm import TPComm
    backend = "nccl" if a.device == "cuda" else "gloo"
    init_dist(rank, a.world, "127.0.0.1", a.master_port, backend=backend, timeout_s=600)
    control = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=3600)) if a.world > 1 else None
    comm = TPComm()
    comm.control = control
    engine = build_engine(a, rank, a.world, comm)
    watchdog = None
    closing = threading.Event()   # set once rank 0 has announced the shutdown: its exit is then expected
    if a.world > 1:
        from ..parallel.watchdog import HeartbeatWatchdog

        def lost(e):   # followers block inside the broadcast: a silent peer ends the process
            if closing.is_set():
                return
            print(f"[daemon rank {rank}] {e}; exiting", flush=True)
            os._exit(3)
        watchdog = HeartbeatWatchdog(dist.distributed_c10d._get_default_store(), rank, a.world,
                                     timeout_s=a.heartbeat_timeout_s, on_failure=None if rank == 0 else lost).start()
    try:
        if a.world == 1:
            on_rank0(engine)
        elif rank == 0:
            mirror = MirroredEngine(engine, control, watchdog)
            try:
                on_rank0(mirror)
            finally:
                mirror.shutdown()
        else:
            follower_loop(engine, control, on_shutdown=closing.set)
    finally:
        if watchdog is not None:
            watchdog.stop(clean=True)
        if a.device == "cuda":
            torch.cuda.synchronize()
            # captured decode graphs may hold NCCL calls (the NCCL collectives, a sampled step's all-gather): they
            # must go before the process group, or its teardown waits on them
            engine.release_graphs()
        del engine
        dist.destroy_process_group()


def spawn_lane(a: LaneArgs, on_rank0: Callable[[Any], None]) -> None:
    if a.world == 1:
        run_worker(0, a, on_rank0)
        return
    import torch.multiprocessing as mp
    mp.spawn(run_worker, args=(a, on_rank0), nprocs=a.world, join=True)


# ------------------------------------------------------------------------------------------------ RPC daemon
def rpc_serve(engine, host: str, port: int, authkey: bytes, tokenizer_source: Optional[str] = None,
              ready_file: Optional[str] = None) -> None:
    """Rank-0 RPC loop: {cmd: ping | generate | shutdown} over multiprocessing.connection (one client at a time
    per connection; requests from concurrent connections are batched by the scheduler)."""
    from .backend import load_tokenizer
    from ..runtime.scheduler import Scheduler
    tok = load_tokenizer(tokenizer_source)
    sched = Scheduler(engine).start()
    listener = Listener((host, port), authkey=authkey)
    addr = listener.address
    print(f"[hrm-flashd] listening on {addr[0]}:{addr[1]}", flush=True)
    if ready_file:
        with open(ready_file, "w") as f:
            f.write(f"{addr[0]}:{addr[1]}\n")
    stop = threading.Event()

    def handle(conn):
        try:
            while not stop.is_set():
                try:
                    msg = conn.recv()
                except EOFError:
                    return
                cmd = msg.get("cmd")
                if cmd == "ping":
                    conn.send({"ok": True, "metrics": sched.metrics()})
                elif cmd == "generate":
                    try:
                        ids = msg.get("input_ids") or tok(str(msg.get("prompt", "")), add_special_tokens=True)["input_ids"]
                        sp = sampling_from_request(msg.get("temperature"), msg.get("top_k"), msg.get("seed"))
                        out = sched.generate(ids, int(msg.get("max_new_tokens", 64)),
                                             stop_on_eos=bool(msg.get("stop_on_eos", True)), sampling=sp)
                        conn.send({"ok": True, "tokens": out, "text": tok.decode(out, skip_special_tokens=True)})
                    except Exception as e:
                        conn.send({"ok": False, "error": repr(e)})
                elif cmd == "shutdown":
                    conn.send({"ok": True})
                    stop.set()
                    try:   # wake the accept() of the main thread
                        Client(addr, authkey=authkey).close()
                    except Exception:
                        pass
                    return
                else:
                    conn.send({"ok": False, "error": f"unknown cmd {cmd!r}"})
        finally:
            conn.close()

    while not stop.is_set():
        try:
            conn = listener.accept()
        except Exception:
            if stop.is_set():
                break
            continue
        if stop.is_set():
            conn.close()
            break
        threading.Thread(target=handle, args=(conn,), daemon=True).start()
    listener.close()
    sched.stop()


@dataclass(frozen=True)
class DaemonAddr:
    host: str
    port: int
    authkey: bytes


def parse_daemon_addr() -> Optional[DaemonAddr]:
    s = os.environ.get("HRM_FLASH_DAEMON")
    if not s or ":" not in s:
        return None
    host, port = s.rsplit(":", 1)
    try:
        return DaemonAddr(host, int(port), os.environ.get("HRM_FLASH_AUTHKEY", "hrmflash").encode())
    except ValueError:
        return None


def client_ping(addr: DaemonAddr) -> bool:
    try:
        c = Client((addr.host, addr.port), authkey=addr.authkey)
        c.send({"cmd": "ping"})
        r = c.recv()
        c.close()
        return bool(r.get("ok"))
    except Exception:
        return False


def client_metrics(addr: DaemonAddr) -> Dict:
    """The lane scheduler's metrics (queue, batch, throughput, latency percentiles, prefix-cache hits)."""
    c = Client((addr.host, addr.port), authkey=addr.authkey)
    c.send({"cmd": "ping"})
    r = c.recv()
    c.close()
    return dict(r.get("metrics") or {})


def client_generate(addr: DaemonAddr, prompt: str = "", max_new_tokens: int = 64, input_ids=None,
                    stop_on_eos: bool = True, temperature: Optional[float] = None, top_k: Optional[int] = None,
                    seed: Optional[int] = None) -> Dict:
    """Generate through the lane daemon; ``temperature`` / ``top_k`` / ``seed`` request a sampled draw (absent:
    greedy)."""
    c = Client((addr.host, addr.port), authkey=addr.authkey)
    c.send({"cmd": "generate", "prompt": prompt, "max_new_tokens": int(max_new_tokens), "input_ids": input_ids,
            "stop_on_eos": stop_on_eos, "temperature": temperature, "top_k": top_k, "seed": seed})
    r = c.recv()
    c.close()
    if not r.get("ok"):
        raise RuntimeError(str(r.get("error", "unknown daemon error")))
    return r


def client_shutdown(addr: DaemonAddr) -> None:
    c = Client((addr.host, addr.port), authkey=addr.authkey)
    c.send({"cmd": "shutdown"})
    c.recv()
    c.close()


class _RpcEntry:
    """Picklable rank-0 entry for mp.spawn."""

    def __init__(self, host, port, authkey, tok, ready_file):
        self.host, self.port, self.authkey, self.tok, self.ready_file = host, port, authkey, tok, ready_file

    def __call__(self, engine):
        rpc_serve(engine, self.host, self.port, self.authkey, self.tok, self.ready_file)


def main(argv=None):
    ap = argparse.ArgumentParser(prog="hrm-flashd", description="Tensor-parallel engine daemon (RPC)")
    ap.add_argument("--model", required=True, help="DSI8 model_q8.bin or synthetic:<preset>")
    ap.add_argument("--world", type=int, choices=[1, 2, 4, 8], required=True)
    ap.add_argument("--max_seq_len", type=int, default=8192)
    ap.add_argument("--prefill_chunk_size", type=int, default=4096)
    ap.add_argument("--max_batch", type=int, default=64)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=0)
    ap.add_argument("--authkey", default=os.environ.get("HRM_FLASH_AUTHKEY", "hrmflash"))
    ap.add_argument("--device", choices=["cuda", "cpu"], default="cuda")
    ap.add_argument("--tokenizer_model", default=None)
    ap.add_argument("--ready_file", default=None, help="write host:port here once listening")
    ap.add_argument("--master_port", type=int, default=29555)
    ap.add_argument("--num_kv_blocks", type=int, default=0)
    ap.add_argument("--nccl_collectives", action="store_true",
                    help="TP all-reduce and argmax through NCCL calls instead of the fused peer-memory kernels")
    ap.add_argument("--no_prefix_cache", dest="prefix_cache", action="store_false",
                    help="recompute every prompt (default: share KV blocks of prompt prefixes seen before)")
    args = ap.parse_args(argv)
    lane = LaneArgs(args.model, args.world, args.max_seq_len, args.prefill_chunk_size, args.max_batch, args.device,
                    master_port=args.master_port, num_kv_blocks=args.num_kv_blocks,
                    fused_collectives=not args.nccl_collectives, prefix_cache=args.prefix_cache)
    spawn_lane(lane, _RpcEntry(args.host, args.port, args.authkey.encode(), args.tokenizer_model, args.ready_file))


if __name__ == "__main__":
    main()
