"""File-IPC shim with the reference native engine's protocol, on this package's engine.

    python -m hrm_flashrenderer_b200.serving.dsi8_ipc --dsi8 model_q8.bin [--device cuda] [--max_seq_len 4096]
    python -m hrm_flashrenderer_b200.serving.dsi8_ipc --preset tiny --device cpu      (random-init weights)

The reference's Python driver starts its engine binary and talks to it through files
(``scripts/deepseek_native_engine.sh:779-851,1010-1131``; driver ``hrm_flash/deepseek_native.py``).  This process
speaks the same protocol, so that driver can run unchanged against the B200 engine:

* once the model is loaded it prints ``[*] Ready. Entering interactive loop...``;
* it polls ``DSI8_PROMPT_FILE`` (default ``/tmp/deepseek_prompt.txt``) every 200 ms; a request is that file's
  first line (the file is removed) plus ``DSI8_PROMPT_TOKENS_FILE`` (default ``/tmp/deepseek_prompt_tokens.txt``,
  one id per line, removed; empty -> the BOS id);
* ``DSI8_TGEN`` (1..2048, default 64) tokens are generated greedily, capped so prompt + output fit the context;
  no EOS stop, as in the reference;
* ``DSI8_TOKENS_FILE`` (default ``/tmp/deepseek_tokens.txt``) and ``DSI8_DONE_FILE`` (default
  ``/tmp/deepseek_done.flag``) are removed before generation; every new id is appended to the tokens file as
  ``"<id>\\n"`` as soon as it is known, and the done file gets ``"done\\n"`` at the end;
* with ``TELEM_ENABLE=1`` the reference's UDP telemetry packets are sent (:mod:`.telemetry`).
"""
from __future__ import annotations

import argparse
import os
import sys
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, List, Optional

READY = "[*] Ready. Entering interactive loop..."


@dataclass
class IpcPaths:
    prompt: Path
    prompt_tokens: Path
    tokens: Path
    done: Path

    @classmethod
    def from_env(cls, env=None) -> "IpcPaths":
        env = os.environ if env is None else env

        def get(name, default):
            v = env.get(name, "")
            return Path(v if v else default)

        return cls(get("DSI8_PROMPT_FILE", "/tmp/deepseek_prompt.txt"),
                   get("DSI8_PROMPT_TOKENS_FILE", "/tmp/deepseek_prompt_tokens.txt"),
                   get("DSI8_TOKENS_FILE", "/tmp/deepseek_tokens.txt"),
                   get("DSI8_DONE_FILE", "/tmp/deepseek_done.flag"))


def tgen_from_env(env=None) -> int:
    env = os.environ if env is None else env
    s = env.get("DSI8_TGEN", "")
    if not s:
        return 64
    try:
        v = int(s)
    except ValueError:
        v = 0
    return max(1, min(2048, v))


def _read_ids(path: Path) -> List[int]:
    ids = []
    for line in path.read_text(errors="replace").splitlines():
        line = line.strip()
        try:
            t = int(line)
        except ValueError:
            continue
        if t >= 0:
            ids.append(t)
    return ids


def poll_once(engine, paths: IpcPaths, max_ctx: int, bos_id: int, tgen: int,
              log: Callable[[str], None] = print, telemetry=None) -> bool:
    """Serve one request if a prompt file is present; returns whether one was served.  With ``telemetry`` (a
    :class:`~hrm_flashrenderer_b200.serving.telemetry.Telemetry`) an idle poll sends an ``AWAITING_PROMPT`` packet
    and every generated token one packet with its step, the greedy token's cross-entropy, a projection of the final
    hidden row and ``TokenID: <id>``, as the reference engine does (the model must have ``collect_stats`` on)."""
    if not paths.prompt.is_file():
        if telemetry is not None:
            telemetry.send(0, 0.0, None, "AWAITING_PROMPT")
        return False
    model = getattr(engine, "model", None)
    lines = paths.prompt.read_text(errors="replace").splitlines()
    paths.prompt.unlink(missing_ok=True)
    log(f"> Received Prompt: {lines[0] if lines else ''}")
    ids = _read_ids(paths.prompt_tokens) if paths.prompt_tokens.is_file() else []
    paths.prompt_tokens.unlink(missing_ok=True)
    if not ids:
        ids = [bos_id]
    ids = ids[-max(1, max_ctx - 1):]
    n_new = max(0, min(tgen, max_ctx - len(ids)))
    paths.tokens.unlink(missing_ok=True)
    paths.done.unlink(missing_ok=True)
    if n_new > 0:
        step = [len(ids)]
        with open(paths.tokens, "a") as f:
            def on_token(_i, t):
                f.write(f"{int(t)}\n")
                f.flush()
                if telemetry is not None:
                    # the step's greedy-token cross-entropy (0 for the first token, as in the reference) and the
                    # final hidden row, recorded by the model in this step's forward
                    loss, hid = 0.0, None
                    if model is not None and getattr(model, "stat_nll", None) is not None:
                        if step[0] > len(ids):
                            loss = float(model.stat_nll[0])
                        hid = model.stat_hidden[0]
                    telemetry.send(step[0], loss, hid, f"TokenID: {int(t)}")
                step[0] += 1
            engine.generate([ids], n_new, stop_on_eos=False, on_token=on_token)
    paths.done.write_text("done\n")
    return True


def serve_forever(engine, paths: IpcPaths, max_ctx: int, bos_id: int, poll_s: float = 0.2,
                  max_requests: Optional[int] = None, log: Callable[[str], None] = print, telemetry=None) -> int:
    served = 0
    while max_requests is None or served < max_requests:
        if poll_once(engine, paths, max_ctx, bos_id, tgen_from_env(), log, telemetry):
            served += 1
        else:
            time.sleep(poll_s)
    return served


def build_engine(a):
    import torch
    from ..config import EngineConfig, get_preset
    from ..models.llama import LlamaW8
    from ..runtime.engine import InferenceEngine
    dev = torch.device(a.device)
    if a.dsi8:
        model = LlamaW8.from_dsi8(a.dsi8, device=dev, max_pos=a.max_seq_len + 16,
                                  cache_dir=os.environ.get("HRM_PACKED_CACHE") or None)
        cfg = model.cfg
    else:
        from ..models.weights import synth_weights
        cfg = get_preset(a.preset)
        model = LlamaW8.from_weights(cfg, synth_weights(cfg, seed=a.seed), device=dev, max_pos=a.max_seq_len + 16)
    ecfg = EngineConfig(max_seq_len=a.max_seq_len, max_batch=1, use_cuda_graphs=dev.type == "cuda")
    return InferenceEngine(model, ecfg), cfg


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-dsi8-ipc")
    ap.add_argument("--dsi8", default="", help="DSI8 model file (else --preset with random-init weights)")
    ap.add_argument("--preset", default="tiny")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--max_seq_len", type=int, default=4096, help="the reference engine's Tmax")
    ap.add_argument("--max_requests", type=int, default=0, help="exit after this many requests (0 = never)")
    a = ap.parse_args(argv)
    eng, cfg = build_engine(a)
    print(READY, flush=True)
    bos = int(getattr(cfg, "bos_token_id", 1) or 1)
    from .telemetry import Telemetry
    tel = Telemetry(model_id=cfg.name, hidden=cfg.hidden)   # TELEM_ENABLE=1 / TELEM_PORT / TELEM_TARGET
    eng.model.collect_stats = tel.enabled   # before the first decode graph is captured
    serve_forever(eng, IpcPaths.from_env(), a.max_seq_len, bos, max_requests=a.max_requests or None,
                  log=lambda s: print(s, flush=True), telemetry=tel if tel.enabled else None)
    return 0


if __name__ == "__main__":
    sys.exit(main())
