"""GPU layout detection and lane placement for one 8xB200 NVSwitch node, plus lane start/stop/health.

Reference: ``scripts/start_native_topology.sh`` (``detect_gpu_layout`` :302-471 reads ``nvidia-smi
--query-gpu=index,memory.total`` and ``nvidia-smi topo -m``, scores pairs by NVLink + same memory tier, validates
manual overrides strictly, allows a PCIe pair only with ``ALLOW_PCIE_PAIR_FALLBACK=1``, fails on
``REQUIRE_NVLINK=1`` without NVLink; ``start_service`` :558-599 starts one ``serve`` per lane with
``CUDA_VISIBLE_DEVICES`` and pid/log files; ``wait_service`` :618-640 polls ``/v1/health``).

Retargeted semantics: GPUs qualify as B200 when ``memory.total >= 150000 MiB``; a lane of TP size N takes N GPUs that
are pairwise NVLink-connected (``NV<k>`` in the topology matrix; on HGX B200 every pair is ``NV18`` through
NVSwitch); lanes are packed on ascending indices, largest first.  Manual overrides ``LANE_GPUS_<lane>="i,j,..."``
must name distinct B200 indices of the right count, else the launch fails (``STRICT_GPU_TOPOLOGY=1``, default) or
the override is ignored with a warning.
"""
from __future__ import annotations

import json
import os
import re
import shlex
import signal
import subprocess
import sys
import time
import urllib.request
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, List, Optional, Tuple

from .hw import Derived, HWError

REPO_ROOT = Path(__file__).resolve().parents[2]
B200_MIN_MIB = 150000
LANE_PORTS = {"solo_22gb": 8081, "nvlink_pair": 8082, "solo_3080": 8083}


class TopologyError(RuntimeError):
    pass


@dataclass
class GPULayout:
    mem_mib: Dict[int, int]
    links: Dict[Tuple[int, int], str]

    @property
    def indices(self) -> List[int]:
        return sorted(self.mem_mib)

    def b200(self) -> List[int]:
        return [i for i in self.indices if self.mem_mib[i] >= B200_MIN_MIB]

    def link(self, i: int, j: int) -> str:
        return self.links.get((i, j)) or self.links.get((j, i)) or ""

    def nvlink(self, i: int, j: int) -> int:
        m = re.match(r"NV(\d+)", self.link(i, j))
        return int(m.group(1)) if m else 0


def _run(cmd: List[str]) -> str:
    return subprocess.check_output(cmd, text=True, stderr=subprocess.DEVNULL)


def detect_layout(smi: str = "nvidia-smi") -> GPULayout:
    try:
        mem_out = _run([smi, "--query-gpu=index,memory.total", "--format=csv,noheader,nounits"])
    except Exception as e:
        raise TopologyError(f"nvidia-smi query failed: {e}")
    mem = {}
    for ln in mem_out.splitlines():
        parts = [p.strip() for p in ln.split(",")]
        if len(parts) >= 2 and parts[0].isdigit():
            try:
                mem[int(parts[0])] = int(float(parts[1]))
            except ValueError:
                pass
    links: Dict[Tuple[int, int], str] = {}
    try:
        header = None
        for raw in _run([smi, "topo", "-m"]).splitlines():
            toks = raw.split()
            if not toks:
                continue
            if header is None and any(t.startswith("GPU") for t in toks):
                header = [int(t[3:]) for t in toks if re.fullmatch(r"GPU\d+", t)]
                continue
            if header and re.fullmatch(r"GPU\d+", toks[0]):
                row = int(toks[0][3:])
                for j, col in enumerate(header):
                    if j + 1 < len(toks):
                        links[(row, col)] = toks[j + 1]
    except Exception:
        links = {}
    if not mem:
        raise TopologyError("no GPUs reported by nvidia-smi")
    return GPULayout(mem, links)


def _all_nvlink(layout: GPULayout, gpus: List[int]) -> bool:
    return all(layout.nvlink(a, b) > 0 for i, a in enumerate(gpus) for b in gpus[i + 1:])


@dataclass
class LanePlan:
    lanes: Dict[str, List[int]] = field(default_factory=dict)
    link: Dict[str, str] = field(default_factory=dict)     # lane -> NVLINK | PCIE | SINGLE
    warnings: List[str] = field(default_factory=list)


def plan_lanes(layout: GPULayout, derived: Derived, env: Optional[Dict[str, str]] = None) -> LanePlan:
    env = dict(os.environ if env is None else env)
    strict = env.get("STRICT_GPU_TOPOLOGY", "1") == "1"
    require_nv = env.get("REQUIRE_NVLINK", str(derived.require_nvlink)) == "1"
    allow_pcie = env.get("ALLOW_PCIE_PAIR_FALLBACK", "0") == "1"
    pool = layout.b200()
    need = sum(derived.lanes.values())
    if len(pool) < need:
        raise TopologyError(f"selected pool needs {need} B200 GPUs, found {len(pool)} (memory >= {B200_MIN_MIB} MiB): "
                            f"{layout.mem_mib}")
    plan = LanePlan()
    free = list(pool)
    # manual overrides first
    for lane, tp in derived.lanes.items():
        ov = env.get(f"LANE_GPUS_{lane.upper()}") or env.get(f"LANE_GPUS_{lane}")
        if not ov:
            continue
        try:
            gpus = [int(x) for x in ov.split(",") if x.strip()]
        except ValueError:
            gpus = []
        ok = len(gpus) == tp and len(set(gpus)) == tp and all(g in free for g in gpus)
        if not ok:
            msg = f"manual override LANE_GPUS_{lane.upper()}={ov!r} invalid for TP={tp} (free B200: {free})"
            if strict:
                raise TopologyError(msg)
            plan.warnings.append(msg + "; ignored")
            continue
        plan.lanes[lane] = gpus
        for g in gpus:
            free.remove(g)
    for lane, tp in sorted(derived.lanes.items(), key=lambda kv: -kv[1]):
        if lane in plan.lanes:
            continue
        chosen = None
        for start in range(0, len(free) - tp + 1):       # contiguous, NVLink-connected windows first
            cand = free[start:start + tp]
            if tp == 1 or _all_nvlink(layout, cand):
                chosen = cand
                break
        if chosen is None:
            if tp > 1 and require_nv and not allow_pcie:
                raise TopologyError(f"REQUIRE_NVLINK=1 but no NVLink-connected set of {tp} GPUs for lane {lane}")
            chosen = free[:tp]
            plan.warnings.append(f"lane {lane}: no NVLink set of {tp} GPUs; PCIe fallback")
        plan.lanes[lane] = chosen
        for g in chosen:
            free.remove(g)
    for lane, gpus in plan.lanes.items():
        if len(gpus) == 1:
            plan.link[lane] = "SINGLE"
        else:
            plan.link[lane] = "NVLINK" if _all_nvlink(layout, gpus) else "PCIE"
            if plan.link[lane] == "PCIE" and require_nv and not allow_pcie:
                raise TopologyError(f"REQUIRE_NVLINK=1 but lane {lane} GPUs {gpus} are not NVLink-connected")
    return plan


# ------------------------------------------------------------------------------------------------ start / stop
RUN_DIR = REPO_ROOT / ".run" / "services"


# Per-lane context / prefill-chunk limits with the reference's environment overrides (names and fall-backs as
# scripts/start_native_topology.sh:52-61,278-285: MAX_SEQ_<LANE>, then MAX_SEQ_SOLO / MAX_SEQ_NVLINK; PREFILL_*
# alike).  The defaults are sized for B200 lanes (180 GB each), not the reference's 11-22 GB cards.
LANE_LIMITS = {"solo_22gb": (8192, 4096, "SOLO"), "nvlink_pair": (8192, 4096, "NVLINK"),
               "solo_3080": (8192, 4096, "SOLO")}


def lane_limits(lane: str, env: Optional[Dict[str, str]] = None) -> Tuple[int, int]:
    env = os.environ if env is None else env
    seq, pre, group = LANE_LIMITS.get(lane, (4096, 768, "SOLO"))
    up = lane.upper()
    seq = int(env.get(f"MAX_SEQ_{up}") or env.get(f"MAX_SEQ_{group}") or seq)
    pre = int(env.get(f"PREFILL_{up}") or env.get(f"PREFILL_{group}") or pre)
    return seq, pre


def lane_command(lane: str, tp: int, port: int, hrm_model: str, llm_model: str, extra: List[str],
                 env: Optional[Dict[str, str]] = None) -> List[str]:
    """The lane's ``serve`` command; ``HRM_FLASH_BIN`` replaces the interpreter + module prefix."""
    env = os.environ if env is None else env
    seq, pre = lane_limits(lane, env)
    prefix = shlex.split(env["HRM_FLASH_BIN"]) if env.get("HRM_FLASH_BIN") else \
        [sys.executable, "-m", "hrm_flashrenderer_b200.serving.cli"]
    return prefix + ["serve", "--hrm_model", hrm_model, "--llm_model", llm_model, "--world", str(tp), "--port",
                     str(port), "--max_seq_len", str(seq), "--prefill_chunk_size", str(pre)] + list(extra)


def start_lane(lane: str, gpus: List[int], port: int, cmd: List[str], run_dir: Path = RUN_DIR) -> int:
    run_dir.mkdir(parents=True, exist_ok=True)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=",".join(map(str, gpus)))
    log = open(run_dir / f"{lane}.log", "ab")
    p = subprocess.Popen(cmd, env=env, stdout=log, stderr=subprocess.STDOUT, start_new_session=True)
    (run_dir / f"{lane}.pid").write_text(str(p.pid))
    (run_dir / f"{lane}.port").write_text(str(port))
    return p.pid


def wait_health(url: str, timeout_s: float = 600.0, interval_s: float = 1.0, pid: Optional[int] = None) -> bool:
    t0 = time.time()
    while time.time() - t0 < timeout_s:
        if pid is not None:
            try:
                os.kill(pid, 0)
            except OSError:
                return False
        try:
            with urllib.request.urlopen(url.rstrip("/") + "/v1/health", timeout=2) as r:
                if json.loads(r.read().decode()).get("ok"):
                    return True
        except Exception:
            pass
        time.sleep(interval_s)
    return False


def stop_lanes(run_dir: Path = RUN_DIR, timeout_s: float = 20.0) -> List[str]:
    """Stop services recorded by pid files (signals the exact process group we started)."""
    stopped = []
    if not run_dir.is_dir():
        return stopped
    for pf in sorted(run_dir.glob("*.pid")):
        try:
            pid = int(pf.read_text().strip())
        except ValueError:
            pf.unlink()
            continue
        try:
            os.killpg(pid, signal.SIGTERM)
            t0 = time.time()
            while time.time() - t0 < timeout_s:
                os.kill(pid, 0)
                time.sleep(0.2)
            os.killpg(pid, signal.SIGKILL)
        except (OSError, ProcessLookupError):
            pass
        pf.unlink()
        stopped.append(pf.stem)
    return stopped


def main(argv=None) -> int:
    import argparse
    from .hw import load_selection, derive
    ap = argparse.ArgumentParser(prog="hrm-flash-topology")
    sub = ap.add_subparsers(dest="cmd", required=True)
    d = sub.add_parser("detect")
    d.add_argument("--smi", default=os.environ.get("NVIDIA_SMI", "nvidia-smi"))
    st = sub.add_parser("start")
    st.add_argument("--hrm_model", required=True)
    st.add_argument("--llm_model", required=True)
    st.add_argument("--smi", default=os.environ.get("NVIDIA_SMI", "nvidia-smi"))
    st.add_argument("--health_timeout_s", type=float, default=float(os.environ.get("LANE_HEALTH_TIMEOUT_S", "900")))
    st.add_argument("--dry_run", action="store_true")
    st.add_argument("extra", nargs=argparse.REMAINDER)
    sub.add_parser("stop")
    a = ap.parse_args(argv)
    try:
        if a.cmd == "stop":
            print("stopped:", " ".join(stop_lanes()) or "(none)")
            return 0
        sel = load_selection()
        der = derive(sel)
        layout = detect_layout(a.smi)
        plan = plan_lanes(layout, der)
        for w in plan.warnings:
            print(f"[topology] WARN {w}", file=sys.stderr)
        for lane, gpus in plan.lanes.items():
            print(f"LANE_{lane.upper()}_GPUS={','.join(map(str, gpus))}")
            print(f"LANE_{lane.upper()}_LINK={plan.link[lane]}")
        if a.cmd == "detect":
            return 0
        extra = [x for x in (a.extra or []) if x != "--"]
        for lane, gpus in plan.lanes.items():
            cmd = lane_command(lane, len(gpus), LANE_PORTS[lane], a.hrm_model, a.llm_model, extra)
            if a.dry_run:
                print(f"CUDA_VISIBLE_DEVICES={','.join(map(str, gpus))} {shlex.join(cmd)}")
                continue
            pid = start_lane(lane, gpus, LANE_PORTS[lane], cmd)
            ok = wait_health(f"http://127.0.0.1:{LANE_PORTS[lane]}", a.health_timeout_s, pid=pid)
            print(f"[topology] lane {lane} pid={pid} gpus={gpus} healthy={ok}")
            if not ok:
                return 3
        return 0
    except (HWError, TopologyError) as e:
        print(f"ERR: {e}", file=sys.stderr)
        return 2


if __name__ == "__main__":
    raise SystemExit(main())
