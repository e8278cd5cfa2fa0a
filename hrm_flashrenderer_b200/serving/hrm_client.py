"""HRM query client: in-process C ABI (cached handle) or the ``hrm`` CLI as a subprocess.

Reference ``hrm_flash/hrm_client.py:39-100``: without a timeout the ctypes API is used; with a timeout the reference
spawns ``hrm query --prompt-stdin`` so the timeout can kill it (1.8 s default in the service).  Here a timeout does
not force a process per query: the query runs on a worker thread against the process-wide cached handle and the
caller stops waiting after ``timeout_s`` (queries are read-only and bounded, so a late one just finishes in the
background).  ``prefer_api=False`` keeps the subprocess path available.
"""
from __future__ import annotations

import concurrent.futures
import json
import subprocess
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, Optional

from .utils import find_hrm_binary

_POOL = concurrent.futures.ThreadPoolExecutor(max_workers=4, thread_name_prefix="hrm-query")


@dataclass(frozen=True)
class HRMQueryResult:
    raw: Dict[str, Any]


def _files_ok(model_dir: Path) -> bool:
    return (model_dir / "router_index.bin").is_file() and (model_dir / "index.sqlite").is_file()


def run_hrm_query_via_api(repo_root: Optional[Path], model_dir: Path, prompt: str, top_k: int, top_m: int,
                          k: int) -> Optional[HRMQueryResult]:
    if not _files_ok(model_dir):
        return None
    try:
        from .hrm_api import shared_handle
        h = shared_handle(model_dir, repo_root)
    except Exception:
        return None
    return HRMQueryResult(raw=json.loads(h.query_json(prompt, top_k=top_k, top_m=top_m, k=k)))


def run_hrm_query(hrm_bin: Optional[Path], model_dir: Path, prompt: str, top_k: int = 16, top_m: int = 400,
                  k: int = 16, prefer_api: bool = True, repo_root: Optional[Path] = None,
                  timeout_s: Optional[float] = 1.8) -> HRMQueryResult:
    model_dir = Path(model_dir)
    enforce = timeout_s is not None and float(timeout_s) > 0.0
    if prefer_api:
        fut = _POOL.submit(run_hrm_query_via_api, repo_root, model_dir, prompt, top_k, top_m, k)
        try:
            r = fut.result(timeout=float(timeout_s) if enforce else None)
        except concurrent.futures.TimeoutError as e:
            raise RuntimeError(f"HRM query timed out after {float(timeout_s):.3f}s "
                               f"(prompt_bytes={len(prompt.encode('utf-8'))}, top_k={top_k}, k={k}, top_m={top_m})") from e
        if r is not None:
            return r
    binp = find_hrm_binary(repo_root=repo_root, explicit=str(hrm_bin) if hrm_bin is not None else None)
    if not binp.is_file():
        raise FileNotFoundError(f"HRM binary not found (set HRM_BIN or build with `make -C hrm_core`): {binp}")
    if not _files_ok(model_dir):
        raise FileNotFoundError(f"HRM model dir must contain router_index.bin and index.sqlite: {model_dir}")
    cmd = [str(binp), "query", "--model", str(model_dir), "--format", "json", "--top-k", str(int(top_k)),
           "--top-m", str(int(top_m)), "--k", str(int(k)), "--prompt-stdin"]
    try:
        p = subprocess.run(cmd, input=prompt.encode("utf-8"), stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                           timeout=float(timeout_s) if enforce else None)
    except subprocess.TimeoutExpired as e:
        raise RuntimeError(f"HRM query timed out after {float(timeout_s):.3f}s") from e
    if p.returncode != 0:
        raise RuntimeError(f"HRM query failed (code {p.returncode}):\n{p.stderr.decode('utf-8', 'replace')}")
    try:
        return HRMQueryResult(raw=json.loads(p.stdout.decode("utf-8")))
    except Exception as e:
        raise RuntimeError(f"HRM returned invalid JSON: {e}") from e
