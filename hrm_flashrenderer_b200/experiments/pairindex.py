"""Python binding of the PairIndex tokenizer (``hrm_core/build/libhrm_pairindex.so``, C++).

The tokenizer of the experiments plane: bytes keep ids 0..255, the K1 most frequent byte pairs get ids 256..256+K1-1,
and the K2 most frequent adjacent pairs of those ids get macro ids after that (see ``hrm_core/include/hrm/pairindex.h``
for the exact rules, identical to the reference's ``llm_engine.cu:141-336`` and its ``index_build_v7`` tool).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Iterable, Sequence

import numpy as np

REPO_ROOT = Path(__file__).resolve().parents[2]


def _find_lib() -> Path:
    cands = [os.environ.get("HRM_PAIRINDEX_LIB", ""), str(REPO_ROOT / "hrm_core" / "build" / "libhrm_pairindex.so")]
    for c in cands:
        if c and Path(c).is_file():
            return Path(c)
    raise FileNotFoundError("libhrm_pairindex.so not built (run: make -C hrm_core)")


_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        L = ctypes.CDLL(str(_find_lib()))
        vp, u8p = ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint8)
        u16p, u32p = ctypes.POINTER(ctypes.c_uint16), ctypes.POINTER(ctypes.c_uint32)
        L.hrm_pi_build_files.restype = vp
        L.hrm_pi_build_files.argtypes = [ctypes.POINTER(ctypes.c_char_p), ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.hrm_pi_build_bytes.restype = vp
        L.hrm_pi_build_bytes.argtypes = [u8p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
        L.hrm_pi_load.restype = vp
        L.hrm_pi_load.argtypes = [ctypes.c_char_p]
        L.hrm_pi_from_tables.restype = vp
        L.hrm_pi_from_tables.argtypes = [ctypes.c_int, ctypes.c_int, u16p, u32p, ctypes.c_uint32, u32p, u16p]
        L.hrm_pi_save.argtypes = [vp, ctypes.c_char_p]
        L.hrm_pi_info.argtypes = [vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), u32p]
        L.hrm_pi_tables.argtypes = [vp, u16p, u32p, u32p, u16p]
        L.hrm_pi_encode.restype = ctypes.c_size_t
        L.hrm_pi_encode.argtypes = [vp, u8p, ctypes.c_size_t, u16p, ctypes.c_size_t]
        L.hrm_pi_decode.restype = ctypes.c_size_t
        L.hrm_pi_decode.argtypes = [vp, u16p, ctypes.c_size_t, u8p, ctypes.c_size_t]
        L.hrm_pi_free.argtypes = [vp]
        L.hrm_pi_last_error.restype = ctypes.c_char_p
        _LIB = L
    return _LIB


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


class PairIndex:
    """Owning wrapper around a native PairIndex handle."""

    def __init__(self, handle):
        if not handle:
            raise RuntimeError("pairindex: " + lib().hrm_pi_last_error().decode())
        self._h = handle
        k1, k2, hs = ctypes.c_int(), ctypes.c_int(), ctypes.c_uint32()
        lib().hrm_pi_info(self._h, ctypes.byref(k1), ctypes.byref(k2), ctypes.byref(hs))
        self.k1, self.k2, self.hsize = k1.value, k2.value, hs.value

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _LIB is not None:
            _LIB.hrm_pi_free(h)

    # ---------------------------------------------------------------- construction
    @classmethod
    def build_files(cls, paths: Sequence[str], k1: int = 8192, k2: int = 8192) -> "PairIndex":
        arr = (ctypes.c_char_p * len(paths))(*[str(p).encode() for p in paths])
        return cls(lib().hrm_pi_build_files(arr, len(paths), k1, k2))

    @classmethod
    def build_bytes(cls, data: bytes, k1: int = 8192, k2: int = 8192) -> "PairIndex":
        b = np.frombuffer(data, dtype=np.uint8)
        return cls(lib().hrm_pi_build_bytes(_ptr(b, ctypes.c_uint8), b.size, k1, k2))

    @classmethod
    def load(cls, path: str) -> "PairIndex":
        return cls(lib().hrm_pi_load(str(path).encode()))

    @classmethod
    def from_tables(cls, k1: int, k2: int, id2pair: np.ndarray, id2pair2: np.ndarray, hkeys: np.ndarray,
                    hvals: np.ndarray) -> "PairIndex":
        id2pair = np.ascontiguousarray(id2pair, dtype=np.uint16)
        id2pair2 = np.ascontiguousarray(id2pair2, dtype=np.uint32)
        hkeys = np.ascontiguousarray(hkeys, dtype=np.uint32)
        hvals = np.ascontiguousarray(hvals, dtype=np.uint16)
        return cls(lib().hrm_pi_from_tables(k1, k2, _ptr(id2pair, ctypes.c_uint16), _ptr(id2pair2, ctypes.c_uint32),
                                            hkeys.size, _ptr(hkeys, ctypes.c_uint32), _ptr(hvals, ctypes.c_uint16)))

    def save(self, path: str) -> None:
        if not lib().hrm_pi_save(self._h, str(path).encode()):
            raise RuntimeError("pairindex save: " + lib().hrm_pi_last_error().decode())

    def tables(self):
        id2pair = np.zeros(self.k1, np.uint16)
        id2pair2 = np.zeros(self.k2, np.uint32)
        hkeys = np.zeros(self.hsize, np.uint32)
        hvals = np.zeros(self.hsize, np.uint16)
        lib().hrm_pi_tables(self._h, _ptr(id2pair, ctypes.c_uint16), _ptr(id2pair2, ctypes.c_uint32),
                            _ptr(hkeys, ctypes.c_uint32), _ptr(hvals, ctypes.c_uint16))
        return id2pair, id2pair2, hkeys, hvals

    # ---------------------------------------------------------------- use
    @property
    def vocab(self) -> int:
        return 256 + self.k1 + self.k2

    def encode(self, data) -> np.ndarray:
        if isinstance(data, str):
            data = data.encode("utf-8")
        b = np.frombuffer(data, dtype=np.uint8)
        n = lib().hrm_pi_encode(self._h, _ptr(b, ctypes.c_uint8), b.size, None, 0)
        out = np.zeros(n, dtype=np.uint16)
        lib().hrm_pi_encode(self._h, _ptr(b, ctypes.c_uint8), b.size, _ptr(out, ctypes.c_uint16), n)
        return out

    def decode_bytes(self, ids: Iterable[int]) -> bytes:
        a = np.ascontiguousarray(np.asarray(list(ids) if not isinstance(ids, np.ndarray) else ids, dtype=np.uint16))
        n = lib().hrm_pi_decode(self._h, _ptr(a, ctypes.c_uint16), a.size, None, 0)
        out = np.zeros(max(n, 1), dtype=np.uint8)
        lib().hrm_pi_decode(self._h, _ptr(a, ctypes.c_uint16), a.size, _ptr(out, ctypes.c_uint8), n)
        return out[:n].tobytes()

    def decode(self, ids: Iterable[int]) -> str:
        return self.decode_bytes(ids).decode("utf-8", errors="replace")
