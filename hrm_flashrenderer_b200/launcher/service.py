"""Service wrappers around the stack: systemd unit, supervised run (restart-on-failure contract), router smoke.

    python -m hrm_flashrenderer_b200.launcher.service unit --workdir /opt/hrm --hrm_model /opt/hrm/model_index \
        --llm_model llama3.1-70b > /etc/systemd/system/hrm-flash.service
    python -m hrm_flashrenderer_b200.launcher.service supervise [--router_url URL] [--lane_url URL ...]
    python -m hrm_flashrenderer_b200.launcher.service smoke [--router_url URL]

* ``unit`` prints a oneshot systemd unit (``RemainAfterExit``) whose ExecStart starts the lanes through the
  topology launcher and then the router, and whose ExecStop stops them by pid file.  Counterpart of the
  reference's ``scripts/systemd/hrm-flash.service:1-22`` (same unit shape, timeouts 900 s / 30 s).
* ``supervise`` is the long-running foreground wrapper a process manager keeps alive (the reference's
  ``scripts/pm2_native_stack.sh:56-104``): one holder per lock file, health of the router and the primary lane polled
  every ``interval`` s, exit status 1 after ``fail_limit`` consecutive failures so the manager restarts the stack.
  It never kills processes by name; stopping goes through the pid files that the launcher wrote.
* ``smoke`` posts one prompt three times to the router - no hint, ``route_hint=fast``, ``route_hint=quality`` - and
  prints the lane that answered, the router's prompt-token estimate and the latency (the reference's
  ``scripts/smoke_router.sh:26-53``).
"""
from __future__ import annotations

import argparse
import fcntl
import json
import os
import shlex
import sys
import time
import urllib.request
from pathlib import Path
from typing import Callable, Dict, Iterable, List, Optional

from .topology import LANE_PORTS, REPO_ROOT

ROUTER_PORT = 8090
DEFAULT_LOCK = "/tmp/hrm_flashrenderer_b200_stack.lock"
SMOKE_PROMPT = "Summarize the key retrieval evidence in 5 concise bullets."


def systemd_unit(workdir: str, hrm_model: str, llm_model: str, python: str = "/usr/bin/env python3",
                 router_port: int = ROUTER_PORT) -> str:
    start = (f"{python} -m hrm_flashrenderer_b200.launcher.topology start --hrm_model {shlex.quote(hrm_model)} "
             f"--llm_model {shlex.quote(llm_model)} && "
             f"{python} -m hrm_flashrenderer_b200.launcher.service start-router --port {router_port}")
    stop = f"{python} -m hrm_flashrenderer_b200.launcher.topology stop"
    return "\n".join([
        "[Unit]",
        "Description=HRM FlashRenderer B200 stack (lane services + router)",
        "After=network-online.target",
        "Wants=network-online.target",
        "",
        "[Service]",
        "Type=oneshot",
        "RemainAfterExit=yes",
        f"WorkingDirectory={workdir}",
        "Environment=LOCAL_FILES_ONLY=1",
        f"Environment=HRM_MODEL_DIR={hrm_model}",
        f"ExecStart=/usr/bin/env bash -lc {shlex.quote(start)}",
        f"ExecStop=/usr/bin/env bash -lc {shlex.quote(stop)}",
        "TimeoutStartSec=900",
        "TimeoutStopSec=30",
        "",
        "[Install]",
        "WantedBy=multi-user.target",
        "",
    ])


def http_ok(url: str, timeout: float = 5.0) -> bool:
    try:
        with urllib.request.urlopen(url, timeout=timeout) as r:
            return 200 <= r.status < 300
    except Exception:
        return False


class LockHeld(RuntimeError):
    pass


def acquire_lock(path: str):
    """Exclusive non-blocking lock; returns the open file (keep it alive)."""
    f = open(path, "w")
    try:
        fcntl.flock(f.fileno(), fcntl.LOCK_EX | fcntl.LOCK_NB)
    except OSError:
        f.close()
        raise LockHeld(f"another stack wrapper holds {path}")
    return f


def supervise(urls: Iterable[str], interval_s: float = 20.0, fail_limit: int = 3,
              health: Callable[[str], bool] = http_ok, sleep: Callable[[float], None] = time.sleep,
              max_checks: Optional[int] = None, log: Callable[[str], None] = print) -> int:
    """Poll every health URL; return 1 after ``fail_limit`` consecutive failed rounds (0 if ``max_checks`` ran out)."""
    urls = list(urls)
    failures = checks = 0
    while max_checks is None or checks < max_checks:
        checks += 1
        if all(health(u) for u in urls):
            failures = 0
        else:
            failures += 1
            log(f"WARN: health check failed ({failures}/{fail_limit})")
            if failures >= fail_limit:
                log("ERR: health failed repeatedly; exiting for a supervisor restart")
                return 1
        sleep(interval_s)
    return 0


def _post(url: str, payload: Dict, timeout: float = 600.0) -> Dict:
    req = urllib.request.Request(url, data=json.dumps(payload).encode(), headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.loads(r.read().decode())


def smoke_router(router_url: str, prompt: str = SMOKE_PROMPT, max_new_tokens: int = 192,
                 log: Callable[[str], None] = print) -> List[Dict]:
    """Health + auto / fast / quality routing cases; returns one record per case."""
    router_url = router_url.rstrip("/")
    with urllib.request.urlopen(router_url + "/v1/health", timeout=10) as r:
        h = json.loads(r.read().decode())
    log("[smoke] router health: " + json.dumps({"ok": h.get("ok"), "backends": h.get("backends")}))
    out = []
    for label, hint in (("auto", None), ("fast", "fast"), ("quality", "quality")):
        payload = {"prompt": prompt, "max_new_tokens": int(max_new_tokens)}
        if hint:
            payload["route_hint"] = hint
        t0 = time.perf_counter()
        resp = _post(router_url + "/v1/generate", payload)
        ms = (time.perf_counter() - t0) * 1e3
        route = resp.get("route", {})
        rec = {"case": label, "selected": route.get("selected", "?"), "prompt_tokens": route.get("prompt_tokens", "?"),
               "latency_ms": round(ms, 1)}
        log(f"[smoke] {label} -> selected={rec['selected']} prompt_tokens={rec['prompt_tokens']} "
            f"latency_ms={rec['latency_ms']}")
        out.append(rec)
    log("[smoke] done")
    return out


def start_router(port: int, run_dir: Path) -> int:
    """Start the router in its own process group with a pid file next to the lanes' (stopped by ``topology stop``)."""
    import subprocess
    run_dir.mkdir(parents=True, exist_ok=True)
    log = open(run_dir / "router.log", "ab")
    p = subprocess.Popen([sys.executable, "-m", "hrm_flashrenderer_b200.serving.cli", "router", "--port", str(port)],
                         stdout=log, stderr=subprocess.STDOUT, start_new_session=True, cwd=str(REPO_ROOT))
    (run_dir / "router.pid").write_text(str(p.pid))
    return p.pid


def main(argv=None) -> int:
    from .topology import RUN_DIR
    ap = argparse.ArgumentParser(prog="hrm-flash-service")
    sub = ap.add_subparsers(dest="cmd", required=True)
    u = sub.add_parser("unit", help="print a systemd unit")
    u.add_argument("--workdir", default=str(REPO_ROOT))
    u.add_argument("--hrm_model", required=True)
    u.add_argument("--llm_model", required=True)
    u.add_argument("--python", default="/usr/bin/env python3")
    u.add_argument("--router_port", type=int, default=ROUTER_PORT)
    s = sub.add_parser("supervise", help="health loop; exit 1 after repeated failures")
    s.add_argument("--router_url", default=f"http://127.0.0.1:{ROUTER_PORT}")
    s.add_argument("--lane_url", action="append", default=None)
    s.add_argument("--interval_s", type=float, default=float(os.environ.get("HEALTH_INTERVAL_S", "20")))
    s.add_argument("--fail_limit", type=int, default=int(os.environ.get("HEALTH_FAIL_LIMIT", "3")))
    s.add_argument("--lock_file", default=os.environ.get("LOCK_FILE", DEFAULT_LOCK))
    m = sub.add_parser("smoke", help="router routing smoke test")
    m.add_argument("--router_url", default=f"http://127.0.0.1:{ROUTER_PORT}")
    m.add_argument("--prompt", default=os.environ.get("PROMPT", SMOKE_PROMPT))
    m.add_argument("--max_new_tokens", type=int, default=int(os.environ.get("MAX_NEW_TOKENS", "192")))
    r = sub.add_parser("start-router", help="start the router with a pid file")
    r.add_argument("--port", type=int, default=ROUTER_PORT)
    a = ap.parse_args(argv)
    if a.cmd == "unit":
        sys.stdout.write(systemd_unit(a.workdir, a.hrm_model, a.llm_model, a.python, a.router_port))
        return 0
    if a.cmd == "smoke":
        smoke_router(a.router_url, a.prompt, a.max_new_tokens)
        return 0
    if a.cmd == "start-router":
        print(f"router pid={start_router(a.port, RUN_DIR)}")
        return 0
    try:
        lock = acquire_lock(a.lock_file)
    except LockHeld as e:
        print(f"ERR: {e}", file=sys.stderr)
        return 1
    urls = [a.router_url.rstrip("/") + "/v1/health"]
    lanes = a.lane_url or [f"http://127.0.0.1:{LANE_PORTS['solo_22gb']}"]
    urls += [x.rstrip("/") + "/v1/health" for x in lanes]
    try:
        return supervise(urls, a.interval_s, a.fail_limit)
    finally:
        lock.close()


if __name__ == "__main__":
    raise SystemExit(main())
