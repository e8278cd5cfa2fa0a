"""Sharded safetensors checkpoint reader with zero-copy tensors and row / column slices.

Counterpart of the reference's ``WeightLoader`` (``engine/weight_loader.py:28-96``): a model directory with either
``model.safetensors.index.json`` (``weight_map``: tensor name -> shard file) or a single ``model.safetensors``;
``get(key)``, ``get_slice(key, slices)``, ``rows(key, a, b)`` and ``cols(key, a, b)``.  Each shard file is mapped
copy-on-write once, on first use, and every returned tensor is a view into that mapping (no read, no copy; the
file itself is never modified).  A view keeps its mapping alive, also after :meth:`WeightLoader.close`.

File layout (the safetensors format): 8-byte little-endian header length N, N bytes of JSON
``{name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}}``, then the data section;
offsets are relative to the start of the data section.
"""
from __future__ import annotations

import json
import mmap
import struct
from pathlib import Path
from typing import Dict, Iterator, Optional, Sequence, Tuple, Union

import torch

DTYPES = {"F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
          "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
          "BOOL": torch.bool}


class SafetensorsFile:
    def __init__(self, path: Union[str, Path]):
        self.path = Path(path)
        self._f = self.path.open("rb")
        size = self.path.stat().st_size
        if size < 8:
            raise ValueError(f"{self.path}: not a safetensors file ({size} bytes)")
        (n,) = struct.unpack("<Q", self._f.read(8))
        if 8 + n > size:
            raise ValueError(f"{self.path}: header of {n} bytes runs past the end of the file ({size} bytes)")
        hdr = json.loads(self._f.read(n))
        self.metadata = hdr.pop("__metadata__", {}) or {}
        self.base = 8 + n
        self.entries: Dict[str, Tuple[torch.dtype, Tuple[int, ...], int, int]] = {}
        for k, m in hdr.items():
            if m["dtype"] not in DTYPES:
                raise ValueError(f"{self.path}:{k}: unsupported dtype {m['dtype']}")
            dt = DTYPES[m["dtype"]]
            shape = tuple(int(d) for d in m["shape"])
            b, e = (int(x) for x in m["data_offsets"])
            numel = 1
            for d in shape:
                numel *= d
            if e - b != numel * torch.empty((), dtype=dt).element_size() or self.base + e > size:
                raise ValueError(f"{self.path}:{k}: data_offsets {b}..{e} do not fit {m['dtype']}{list(shape)} "
                                 f"in a file of {size} bytes")
            self.entries[k] = (dt, shape, b, numel)
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_COPY) if size > self.base else None

    def keys(self):
        return self.entries.keys()

    def tensor(self, key: str) -> torch.Tensor:
        dt, shape, b, numel = self.entries[key]
        if numel == 0:
            return torch.empty(shape, dtype=dt)
        return torch.frombuffer(self._mm, dtype=dt, count=numel, offset=self.base + b).view(shape)

    def close(self) -> None:
        # The mapping is not unmapped here: every tensor view holds a reference to it (torch.frombuffer), so it is
        # released when the last view goes; unmapping now would leave live views pointing at nothing.
        self._mm = None
        self._f.close()


class WeightLoader:
    def __init__(self, model_dir: Union[str, Path]):
        self.model_dir = Path(model_dir)
        idx = self.model_dir / "model.safetensors.index.json"
        single = self.model_dir / "model.safetensors"
        self._files: Dict[str, SafetensorsFile] = {}
        if idx.is_file():
            self.weight_map: Dict[str, str] = dict(json.loads(idx.read_text())["weight_map"])
        elif single.is_file():
            f = self._files[single.name] = SafetensorsFile(single)
            self.weight_map = {k: single.name for k in f.keys()}
        else:
            raise FileNotFoundError(f"{self.model_dir}: no model.safetensors.index.json or model.safetensors")

    def _file_for_key(self, key: str) -> SafetensorsFile:
        fn = self.weight_map.get(key)
        if fn is None:
            raise KeyError(f"{key} is not in the checkpoint at {self.model_dir}")
        f = self._files.get(fn)
        if f is None:
            f = self._files[fn] = SafetensorsFile(self.model_dir / fn)
        return f

    def keys(self) -> Iterator[str]:
        return iter(self.weight_map)

    def __contains__(self, key: str) -> bool:
        return key in self.weight_map

    def get(self, key: str) -> torch.Tensor:
        return self._file_for_key(key).tensor(key)

    def get_slice(self, key: str, slices: Sequence[slice]) -> torch.Tensor:
        return self.get(key)[tuple(slices)]

    def rows(self, key: str, start: int, end: int) -> torch.Tensor:
        return self.get(key)[start:end]

    def cols(self, key: str, start: int, end: int) -> torch.Tensor:
        return self.get(key)[:, start:end]

    def close(self) -> None:
        for f in self._files.values():
            f.close()
        self._files.clear()

    def __enter__(self) -> "WeightLoader":
        return self

    def __exit__(self, *a) -> None:
        self.close()


def write_safetensors(path: Union[str, Path], tensors: Dict[str, torch.Tensor],
                      metadata: Optional[Dict[str, str]] = None) -> Path:
    """Write ``tensors`` as one safetensors file (header padded to 8 bytes, tensors in name order)."""
    inv = {v: k for k, v in DTYPES.items()}
    hdr, blobs, off = {}, [], 0
    for k in sorted(tensors):
        t = tensors[k].detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        hdr[k] = {"dtype": inv[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        hdr["__metadata__"] = {str(a): str(b) for a, b in metadata.items()}
    h = json.dumps(hdr, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    p = Path(path)
    with p.open("wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    return p
