"""DSI8 model file: reader, writer and HF-safetensors exporter.

The byte layout is kept bit-compatible with the reference exporter (``hrm_flash/deepseek_export.py:179-220``)
and the engine loader (``scripts/deepseek_native_engine.sh:315-357``) so files move between the two:

* header: ``b"DSI8"``, u32 version (4), 8 x u32 ``D, H, KVH, Dh, F, V, L, Tmax``, f64 rope_theta, f32 rms_eps,
  u32 bos, u32 eos;
* records until EOF: u32 name_len, name, u32 ttype (0 = Q8, 1 = F32), u32 ndim, ndim x u32 dims, payload;
* Q8 payload: ``rows`` f32 scales followed by ``rows*cols`` int8 row-major;  F32 payload: ``prod(dims)`` f32.

Differences from the reference (documented, forward compatible): ``Tmax`` is the config's
``max_position_embeddings`` (the reference hard-codes 4096), and the header ``eos`` is the first id of an EOS list.
Llama-3 rope-scaling parameters and the full EOS list are carried in an optional trailing F32 record named
``__hrm_b200_meta__`` (a JSON blob stored as bytes padded to 4), which the reference loader stores as an unused
F32 tensor and ignores.
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from dataclasses import replace
from pathlib import Path
from typing import Dict, Iterable, Tuple

import numpy as np
import torch

from ..config import ModelConfig, RopeScaling
from ..models.weights import (QTensor, Tensorish, matrix_shapes, vector_shapes, quantize_rows, EMBED, LM_HEAD)

MAGIC = b"DSI8"
VERSION = 4
TTYPE_Q8 = 0
TTYPE_F32 = 1
TTYPE_Q4 = 2
META_NAME = "__hrm_b200_meta__"


def _write_record(f, name: str, ttype: int, dims: Tuple[int, ...], payloads: Iterable[bytes]) -> None:
    nb = name.encode()
    f.write(struct.pack("<I", len(nb)))
    f.write(nb)
    f.write(struct.pack("<II", ttype, len(dims)))
    for d in dims:
        f.write(struct.pack("<I", int(d)))
    for p in payloads:
        f.write(p)


def write_dsi8(path: str | Path, cfg: ModelConfig, weights: Dict[str, Tensorish]) -> Path:
    """Write ``weights`` (QTensor matrices + fp32 vectors) in DSI8 record order."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    with tmp.open("wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<I", VERSION))
        f.write(struct.pack("<IIIIIIII", cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate,
                            cfg.vocab, cfg.layers, cfg.max_position_embeddings))
        f.write(struct.pack("<d", float(cfg.rope_theta)))
        f.write(struct.pack("<f", float(cfg.rms_eps)))
        f.write(struct.pack("<II", int(cfg.bos_token_id), int(cfg.eos_token_ids[0])))
        for name, (rows, cols) in matrix_shapes(cfg):
            if name not in weights:
                continue
            t = weights[name]
            if not isinstance(t, QTensor) or t.shape != (rows, cols):
                raise ValueError(f"{name}: expected an int8 QTensor {(rows, cols)}, got "
                                 f"{type(t).__name__} {tuple(getattr(t, 'shape', ()))}")
            _write_record(f, name, TTYPE_Q8, (rows, cols), [
                t.scale.detach().cpu().to(torch.float32).contiguous().numpy().tobytes(),
                t.q.detach().cpu().contiguous().numpy().tobytes()])
        for name, n in vector_shapes(cfg):
            if name not in weights:
                continue
            v = weights[name].detach().cpu().to(torch.float32).contiguous()
            if v.numel() != n:
                raise ValueError(f"{name}: expected {n} values, got {v.numel()}")
            _write_record(f, name, TTYPE_F32, (n,), [v.numpy().tobytes()])
        meta = {
            "name": cfg.name,
            "eos_token_ids": list(cfg.eos_token_ids),
            "qkv_bias": cfg.qkv_bias,
            "tie_embeddings": cfg.tie_embeddings,
            "rope_scaling": None if cfg.rope_scaling is None else cfg.rope_scaling.__dict__,
        }
        blob = json.dumps(meta, sort_keys=True).encode()
        blob += b" " * ((-len(blob)) % 4)
        _write_record(f, META_NAME, TTYPE_F32, (len(blob) // 4,), [blob])
    os.replace(tmp, path)
    return path


class DSI8File:
    """Memory-mapped DSI8 reader.  ``get`` returns zero-copy views into a private copy-on-write mapping (the file is
    never written): a 70B export is not copied into host memory, and the tensor-parallel ranks of one host share the
    page cache and touch only the pages their shard reads.  A view keeps the mapping alive after ``close()``."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        self._f = self.path.open("rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_COPY)
        buf = self._mm
        if len(buf) < 60:
            raise ValueError(f"{path}: truncated header ({len(buf)} bytes)")
        if buf[:4] != MAGIC:
            raise ValueError(f"{path}: bad magic {bytes(buf[:4])!r}")
        (self.version,) = struct.unpack_from("<I", buf, 4)
        if self.version < 3:
            raise ValueError(f"{path}: need version >= 3, got {self.version}")
        D, H, KVH, Dh, F, V, L, Tmax = struct.unpack_from("<IIIIIIII", buf, 8)
        (theta,) = struct.unpack_from("<d", buf, 40)
        (eps,) = struct.unpack_from("<f", buf, 48)
        bos, eos = struct.unpack_from("<II", buf, 52)
        o = 60
        self.records: Dict[str, Tuple[int, Tuple[int, ...], int]] = {}
        n = len(buf)

        def need(end: int, what: str) -> None:
            if end > n:
                raise ValueError(f"{path}: truncated in {what} (needs byte {end}, file has {n})")

        while o < n:   # records back to back up to the end of the file; a partial record is an error
            need(o + 4, f"record {len(self.records)} header")
            (nl,) = struct.unpack_from("<I", buf, o)
            o += 4
            need(o + nl + 8, f"record {len(self.records)} header")
            name = bytes(buf[o:o + nl]).decode(errors="replace")
            o += nl
            ttype, ndim = struct.unpack_from("<II", buf, o)
            o += 8
            if ndim < 1 or ndim > 4:
                raise ValueError(f"{path}: record {name!r} has {ndim} dimensions")
            need(o + 4 * ndim, f"record {name!r} header")
            dims = struct.unpack_from("<" + "I" * ndim, buf, o)
            o += 4 * ndim
            self.records[name] = (ttype, tuple(dims), o)
            if ttype == TTYPE_Q8:
                rows = dims[0]
                cols = dims[1] if ndim > 1 else 1
                o += rows * 4 + rows * cols
            elif ttype == TTYPE_Q4:
                rows = dims[0]
                cols = dims[1] if ndim > 1 else 1
                o += rows * 4 + rows * ((cols + 1) // 2)
            else:
                o += int(np.prod(dims)) * 4
            need(o, f"record {name!r} payload")
        meta = {}
        if META_NAME in self.records:
            _, dims, off = self.records[META_NAME]
            meta = json.loads(bytes(buf[off:off + dims[0] * 4]).decode().strip())
        rs = meta.get("rope_scaling")
        qkv_bias = bool(meta.get("qkv_bias", any(k.endswith("q_proj.bias") for k in self.records)))
        tie = bool(meta.get("tie_embeddings", LM_HEAD not in self.records))
        self.config = ModelConfig(
            name=str(meta.get("name", self.path.stem)), hidden=D, layers=L, heads=H, kv_heads=KVH, head_dim=Dh,
            intermediate=F, vocab=V, rms_eps=float(eps), rope_theta=float(theta),
            rope_scaling=RopeScaling(**rs) if rs else None, qkv_bias=qkv_bias, tie_embeddings=tie,
            max_position_embeddings=Tmax, bos_token_id=bos,
            eos_token_ids=tuple(meta.get("eos_token_ids", [eos])),
        )

    def close(self) -> None:
        try:
            self._mm.close()
        except BufferError:   # views are alive: they hold the mapping, which goes with the last of them
            pass
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def names(self):
        return [k for k in self.records if k != META_NAME]

    def get(self, name: str, copy: bool = False) -> Tensorish:
        """Tensor ``name``: a view into the mapping, or an independent copy with ``copy=True``.

        Record payloads follow names of any length, so an fp32 array (a row-scale vector or an F32 tensor) can start
        at an offset that is not a multiple of 4; such an array is always returned as an aligned copy (vectorised
        CPU kernels and pinned-memory copies assume element alignment).  The int8 matrices need no alignment and
        stay views."""
        ttype, dims, off = self.records[name]
        cp = (lambda a: a.copy()) if copy else (lambda a: a)

        def f32(count: int, at: int) -> np.ndarray:
            a = np.frombuffer(self._mm, dtype=np.float32, count=count, offset=at)
            return a.copy() if (copy or at % 4 != 0) else a
        if ttype == TTYPE_Q8:
            rows = dims[0]
            cols = dims[1] if len(dims) > 1 else 1
            scale = f32(rows, off)
            q = np.frombuffer(self._mm, dtype=np.int8, count=rows * cols, offset=off + rows * 4).reshape(rows, cols)
            return QTensor(torch.from_numpy(cp(q)), torch.from_numpy(scale))
        if ttype == TTYPE_F32:
            return torch.from_numpy(f32(int(np.prod(dims)), off))
        raise ValueError(f"{name}: unsupported tensor type {ttype} (only q8 is supported; q4 is rejected)")

    def load_all(self) -> Dict[str, Tensorish]:
        return {k: self.get(k) for k in self.names()}

    def check(self) -> None:
        """Every tensor the header's architecture needs is present with its shape and type (int8 matrices, fp32
        vectors); raises ValueError naming what is missing or wrong.  Extra records are allowed."""
        from ..models.weights import matrix_shapes, vector_shapes
        missing, wrong = [], []
        for name, (rows, cols) in matrix_shapes(self.config):
            r = self.records.get(name)
            if r is None:
                missing.append(name)
            elif r[0] != TTYPE_Q8 or r[1][:2] != (rows, cols):
                wrong.append(f"{name}: type {r[0]} dims {r[1]}, expected q8 {(rows, cols)}")
        for name, length in vector_shapes(self.config):
            r = self.records.get(name)
            if r is None:
                missing.append(name)
            elif r[0] != TTYPE_F32 or int(np.prod(r[1])) != length:
                wrong.append(f"{name}: type {r[0]} dims {r[1]}, expected f32 [{length}]")
        if missing or wrong:
            parts = []
            if missing:
                parts.append(f"{len(missing)} missing tensor(s): " + ", ".join(missing[:5])
                             + (" ..." if len(missing) > 5 else ""))
            if wrong:
                parts.append("; ".join(wrong[:5]) + (" ..." if len(wrong) > 5 else ""))
            raise ValueError(f"{self.path}: not a complete {self.config.name} export: " + " | ".join(parts))


def read_dsi8(path: str | Path) -> Tuple[ModelConfig, Dict[str, Tensorish]]:
    with DSI8File(path) as f:
        f.check()
        return f.config, f.load_all()


# ------------------------------------------------------------------------------------------------
# safetensors -> DSI8 exporter (reference: ``export_dsi_v4``, ``hrm_flash/deepseek_export.py:110-222``)
# ------------------------------------------------------------------------------------------------
class _ShardedExportWeights:
    """What :func:`write_dsi8` reads, streamed from the checkpoint's safetensors shards: each tensor is read from its
    shard's mapping and quantised only when the writer reaches its record, so one tensor is in memory at a time."""

    def __init__(self, files: Dict[str, "SafetensorsFile"], cfg: ModelConfig):
        self.files = files
        self.want_2d = dict(matrix_shapes(cfg))
        self.want_1d = dict(vector_shapes(cfg))

    def __contains__(self, name: str) -> bool:
        return name in self.files and (name in self.want_2d or name in self.want_1d)

    def __getitem__(self, name: str) -> Tensorish:
        t = self.files[name].tensor(name).to(torch.float32)
        if name in self.want_2d:
            return quantize_rows(t)
        return t.reshape(-1).clone()


def export_dsi8(model_dir: str | Path, out_path: str | Path, quant: str = "q8") -> Path:
    """Export a local HF checkpoint directory (config.json + *.safetensors) to DSI8 (q8 only), streaming one tensor
    at a time.  Matrices get one symmetric int8 scale per output row (``max|w| / 127``), vectors stay fp32.

    q4 is rejected: the reference engine parses tensor type 2 as F32 and the production scripts lock it out
    (``deepseek_export.py:53-79,196-198``; ``deepseek_native_engine.sh:342-355``).
    """
    from .safetensors import SafetensorsFile
    if str(quant).lower() != "q8":
        raise ValueError(f"unsupported quant={quant!r}: only q8 is supported")
    model_dir = Path(model_dir)
    cfg = ModelConfig.from_hf_dir(model_dir)
    files: Dict[str, SafetensorsFile] = {}
    opened = []
    try:
        for fn in sorted(model_dir.glob("*.safetensors")):
            f = SafetensorsFile(fn)
            opened.append(f)
            for key in f.keys():
                files[key] = f
        if not files:
            raise RuntimeError(f"no safetensors tensors found under {model_dir}")
        if cfg.qkv_bias and not any(key.endswith("q_proj.bias") for key in files):
            cfg = replace(cfg, qkv_bias=False)
        if LM_HEAD not in files and EMBED in files:
            cfg = replace(cfg, tie_embeddings=True)
        return write_dsi8(out_path, cfg, _ShardedExportWeights(files, cfg))
    finally:
        for f in opened:
            f.close()
