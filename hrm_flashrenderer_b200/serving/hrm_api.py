"""ctypes binding of the HRM C ABI (``hrm_core/include/hrm/api.h``).

Library search order (reference ``hrm_flash/hrm_api.py:14-55``): ``$HRM_API_LIB``, ``<repo>/hrm_core/build/``,
``./hrm_core/build/``, ``/usr/local/lib``, ``/usr/lib``.  Handles are cached per model directory by
:func:`shared_handle` so a server opens each index once (the C++ engine loads the snippet table into memory at
open and queries are read-only, so one handle serves concurrent threads).
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Dict, List, Optional

REPO_ROOT = Path(__file__).resolve().parents[2]


class HRMError(RuntimeError):
    pass


HRMApiError = HRMError   # reference name


def _candidates(repo_root: Optional[Path]) -> List[Path]:
    c: List[Path] = []
    if os.environ.get("HRM_API_LIB"):
        c.append(Path(os.environ["HRM_API_LIB"]))
    for root in (repo_root, REPO_ROOT, Path.cwd()):
        if root is not None:
            c.append(Path(root) / "hrm_core" / "build" / "libhrm_api.so")
    c += [Path("/usr/local/lib/libhrm_api.so"), Path("/usr/lib/libhrm_api.so")]
    return c


_lib_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


def load_hrm_api(repo_root: Optional[Path] = None) -> ctypes.CDLL:
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        for p in _candidates(repo_root):
            if p.is_file():
                try:
                    lib = ctypes.CDLL(str(p))
                except OSError:
                    continue
                lib.hrm_open.argtypes = [ctypes.c_char_p]
                lib.hrm_open.restype = ctypes.c_void_p
                lib.hrm_close.argtypes = [ctypes.c_void_p]
                lib.hrm_close.restype = None
                lib.hrm_query_json.argtypes = [ctypes.c_void_p, ctypes.c_char_p] + [ctypes.c_int] * 5
                lib.hrm_query_json.restype = ctypes.c_void_p
                lib.hrm_free.argtypes = [ctypes.c_void_p]
                lib.hrm_free.restype = None
                lib.hrm_last_error.argtypes = []
                lib.hrm_last_error.restype = ctypes.c_char_p
                _lib = lib
                return lib
    raise HRMError("HRM API shared library not found: build it with `make -C hrm_core` "
                   "(expects hrm_core/build/libhrm_api.so) or set HRM_API_LIB")


class HRMHandle:
    def __init__(self, model_dir, repo_root: Optional[Path] = None):
        self.model_dir = Path(model_dir).resolve()
        self.lib = load_hrm_api(repo_root)
        h = self.lib.hrm_open(str(self.model_dir).encode("utf-8"))
        if not h:
            raise HRMError(f"hrm_open failed: {self._err()}")
        self._h = ctypes.c_void_p(h)

    def _err(self) -> str:
        e = self.lib.hrm_last_error()
        return e.decode("utf-8", errors="replace") if e else "unknown"

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.hrm_close(self._h)
            self._h = None

    def query_json(self, prompt: str, top_k: int = 8, top_m: int = 400, k: int = 8, lam_num: int = 7,
                   lam_den: int = 10) -> str:
        if not getattr(self, "_h", None):
            raise HRMError("handle closed")
        p = self.lib.hrm_query_json(self._h, prompt.encode("utf-8"), int(top_k), int(top_m), int(k), int(lam_num),
                                    int(lam_den))
        if not p:
            raise HRMError(f"hrm_query_json failed: {self._err()}")
        try:
            s = ctypes.cast(p, ctypes.c_char_p).value
            return s.decode("utf-8", errors="replace") if s else "{}"
        finally:
            self.lib.hrm_free(p)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_handles: Dict[str, HRMHandle] = {}
_handles_lock = threading.Lock()


def shared_handle(model_dir, repo_root: Optional[Path] = None) -> HRMHandle:
    """Process-wide cached handle for ``model_dir`` (reopened if the index files changed)."""
    key = str(Path(model_dir).resolve())
    stamp = tuple(os.stat(os.path.join(key, f)).st_mtime_ns for f in ("router_index.bin", "index.sqlite"))
    with _handles_lock:
        h = _handles.get(key)
        if h is not None and getattr(h, "_stamp", None) == stamp:
            return h
        if h is not None:
            h.close()
        h = HRMHandle(key, repo_root)
        h._stamp = stamp
        _handles[key] = h
        return h


def reset_handles() -> None:
    with _handles_lock:
        for h in _handles.values():
            h.close()
        _handles.clear()
