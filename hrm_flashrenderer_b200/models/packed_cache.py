"""Per-rank cache of a packed model shard (the layouts the kernels read), keyed by the source export.

Loading a DSI8 export means reading every tensor, sharding it for the TP rank, fusing q/k/v rows, interleaving
gate/up tiles and re-tiling the int8 weights for the GPU's bulk copies - minutes for a 70B export.  The cache file
holds the finished shard of one rank: every ``LayerWeights`` tensor, the embedding / lm_head shards (lm_head already
tiled on the GPU), the final norm, the model config and the shard plan.  Its name is a SHA-256 of the export's
fingerprint (path, size, mtime and a hash of its first MiB), TP rank and world, the device type (GPU and CPU layouts
differ) and ``LAYOUT_VERSION``, bumped whenever the packing changes.  Reference counterpart: the export-on-demand
cache of ``hrm_flash/deepseek_native.py:62-78`` (one quantised file per model, no packed/TP form).
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import asdict, fields
from pathlib import Path

import torch

LAYOUT_VERSION = 1


def _fingerprint(path: str) -> str:
    p = Path(path)
    st = p.stat()
    h = hashlib.sha256()
    with open(p, "rb") as f:
        h.update(f.read(1 << 20))
    return json.dumps({"path": str(p.resolve()), "size": st.st_size, "mtime_ns": st.st_mtime_ns,
                       "head": h.hexdigest()}, sort_keys=True)


def cache_path(cache_dir: str, source: str, rank: int, world: int, device) -> Path:
    dev = torch.device(device).type
    key = json.dumps({"src": _fingerprint(source), "rank": int(rank), "world": int(world), "device": dev,
                      "layout": LAYOUT_VERSION}, sort_keys=True)
    name = hashlib.sha256(key.encode()).hexdigest()[:32]
    d = Path(cache_dir)
    d.mkdir(parents=True, exist_ok=True)
    return d / f"packed_{name}_r{int(rank)}of{int(world)}.pt"


def save_packed(model, path: Path) -> Path:
    from .llama import LayerWeights
    layers = [{f.name: getattr(L, f.name) for f in fields(LayerWeights)} for L in model.layers]
    blob = {
        "layout": LAYOUT_VERSION,
        "cfg": model.cfg.to_dict(),
        "plan": asdict(model.plan),
        "layers": [{k: (v.cpu() if torch.is_tensor(v) else v) for k, v in L.items()} for L in layers],
        "embed_q": model.embed_q.cpu(), "embed_s": model.embed_s.cpu(),
        "head_q": model.head_q.cpu(), "head_s": model.head_s.cpu(),
        "head_tiled": bool(model.head_q.dim() == 3),
        "final_norm": model.final_norm.cpu(),
    }
    tmp = path.with_suffix(".tmp")
    torch.save(blob, tmp)
    os.replace(tmp, path)   # readers never see a half-written cache file
    return path


def load_packed(cls, path: Path, device, comm=None, max_pos: int = 8192):
    from ..config import ModelConfig
    from .llama import LayerWeights
    from .weights import QTensor, ShardPlan
    blob = torch.load(path, map_location="cpu", weights_only=False)
    if blob.get("layout") != LAYOUT_VERSION:
        raise ValueError(f"packed cache {path} has layout {blob.get('layout')}, expected {LAYOUT_VERSION}")
    dev = torch.device(device)
    cfg = ModelConfig.from_dict(blob["cfg"])
    plan_d = dict(blob["plan"])
    plan_d["head_map"] = tuple(plan_d["head_map"])
    plan = ShardPlan(**plan_d)
    layers = [LayerWeights(**{k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in L.items()})
              for L in blob["layers"]]
    return cls(cfg, plan, layers, QTensor(blob["embed_q"].to(dev), blob["embed_s"].to(dev)),
               QTensor(blob["head_q"].to(dev), blob["head_s"].to(dev)), blob["final_norm"].to(dev), dev, comm,
               max_pos, head_pretiled=blob["head_tiled"])
