"""Live end-to-end harness against a running router, and the mock stack used to test it without GPUs.

Reference: ``scripts/prod_live_e2e.sh:210-518`` (mode matrix x N determinism runs through the router, mixed-mode
forbidden phrases, ``hrm_active=false`` for deepseek_only, quick-latency SLO of 3.0 s at <= 32 new tokens, SHA-256
of ``(text, source_count)`` per mode, stable mixed-mode source fingerprint) and ``scripts/mock_stack_server.py``
(three lanes + a router on localhost; ``--empty-sources`` fault injection).

Structural checks always run.  Content checks that only make sense for a trained model (retrieval answers cite a
source id, mixed answers never mention sources) run with ``--content_checks``; with random-init weights the text is
noise and only determinism / structure / latency are meaningful.
"""
import argparse
import hashlib
import json
import re
import sys
import threading
import time
import urllib.request
from typing import Dict, Optional

BANNED_MIXED = ("quellen", "snippets", "laut den", "basierend auf", "according to the documents",
                "retrieved information")
MODES = ("mixed", "retrieval", "deepseek_only")
DEFAULT_PROMPTS = {"mixed": "Who guards the silver bridge at night?",
                   "retrieval": "What did the merchants promise the king?",
                   "deepseek_only": "Write one sentence about winter."}


def post_json(url: str, payload: Dict, timeout: float = 300.0) -> Dict:
    req = urllib.request.Request(url, data=json.dumps(payload).encode(), method="POST",
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.loads(r.read().decode())


def get_json(url: str, timeout: float = 10.0) -> Dict:
    with urllib.request.urlopen(url, timeout=timeout) as r:
        return json.loads(r.read().decode())


class E2EFailure(AssertionError):
    pass


def run_e2e(router_url: str, runs: int = 3, max_new_tokens: int = 32, route_hint: Optional[str] = None,
            allow_empty: bool = False, content_checks: bool = False, quick_limit_s: float = 3.0,
            prompts: Optional[Dict[str, str]] = None, log=print) -> Dict:
    prompts = dict(DEFAULT_PROMPTS, **(prompts or {}))
    router_url = router_url.rstrip("/")
    h = get_json(router_url + "/v1/health")
    if not h.get("ok"):
        raise E2EFailure(f"router unhealthy: {h}")
    quick = min(max_new_tokens, 32)

    def send(mode, prompt, show=None, n=quick):
        p = {"prompt": prompt, "route_hint": route_hint, "max_new_tokens": n, "allow_failover": True}
        if mode is not None:
            p["mode"] = mode
        if show is not None:
            p["show_sources"] = show
        t0 = time.perf_counter()
        r = post_json(router_url + "/v1/generate", p)
        return r, time.perf_counter() - t0

    report: Dict = {"quick": {}, "modes": {}}
    log("[fp] 1) mixed-silent-test")
    r, dt = send("mixed", prompts["mixed"], show=False)
    report["quick"]["mixed_s"] = dt
    if dt > quick_limit_s:
        raise E2EFailure(f"mixed-silent-test: exceeded {quick_limit_s:.1f}s ({dt:.3f}s)")
    if not str(r.get("text", "")).strip():
        raise E2EFailure("mixed-silent-test: empty response")
    if content_checks and any(b in r["text"].lower() for b in BANNED_MIXED):
        raise E2EFailure("mixed-silent-test: forbidden phrase found")
    log("[fp] 2) deepseek_only-no-hrm-test")
    r, dt = send("deepseek_only", prompts["deepseek_only"])
    report["quick"]["deepseek_only_s"] = dt
    if dt > quick_limit_s:
        raise E2EFailure(f"deepseek_only-no-hrm-test: exceeded {quick_limit_s:.1f}s ({dt:.3f}s)")
    if r.get("hrm_active") is not False or int(r.get("source_count", -1)) != 0 or "sources" in r:
        raise E2EFailure(f"deepseek_only-no-hrm-test: retrieval leaked into deepseek_only: {r}")
    log("[fp] 3) default-mode-test")
    r, dt = send(None, prompts["mixed"], show=False)
    if str(r.get("mode", "")).lower() != "mixed":
        raise E2EFailure("default-mode-test: default mode is not mixed")
    ref_re = re.compile(r"\[\d{4}#s\d{4}\]")
    for mode in MODES:
        hashes, fps = set(), set()
        for i in range(runs):
            resp = post_json(router_url + "/v1/generate", {"prompt": prompts[mode], "mode": mode,
                                                           "route_hint": route_hint, "max_new_tokens": max_new_tokens,
                                                           "allow_failover": True})
            if not resp.get("ok"):
                raise E2EFailure(f"{mode} run {i}: ok=false")
            text = str(resp.get("text", "")).strip()
            if not text:
                raise E2EFailure(f"{mode} run {i}: empty response text")
            sc = int(resp.get("source_count", 0))
            if mode == "mixed":
                if not allow_empty and sc <= 0:
                    raise E2EFailure(f"{mode} run {i}: source_count is 0 (expected retrieval + inference)")
                if isinstance(resp.get("sources"), list) and resp["sources"]:
                    raise E2EFailure(f"{mode} run {i}: mixed response exposed sources by default")
                if resp.get("hrm_active") is not True:
                    raise E2EFailure(f"{mode} run {i}: mixed must return hrm_active=true")
                if content_checks and (any(b in text.lower() for b in BANNED_MIXED) or "sources" in text.lower()):
                    raise E2EFailure(f"{mode} run {i}: mixed output leaked retrieval phrasing")
            elif mode == "retrieval":
                if not allow_empty:
                    if sc <= 0 or not isinstance(resp.get("sources"), list) or not resp["sources"]:
                        raise E2EFailure(f"{mode} run {i}: retrieval mode must use and expose sources")
                    fps.add(json.dumps([s.get("sid") for s in resp["sources"]]))
                if content_checks and not (ref_re.search(text) or "source" in text.lower()):
                    raise E2EFailure(f"{mode} run {i}: retrieval output did not reference sources")
            else:
                if resp.get("hrm_active") is not False or sc != 0:
                    raise E2EFailure(f"{mode} run {i}: deepseek_only must not retrieve")
            hashes.add(hashlib.sha256(json.dumps([text, sc]).encode()).hexdigest())
        if len(hashes) != 1:
            raise E2EFailure(f"{mode}: non-deterministic output over {runs} runs ({len(hashes)} distinct)")
        if len(fps) > 1:
            raise E2EFailure(f"{mode}: source fingerprint changed between runs")
        report["modes"][mode] = {"hash": next(iter(hashes)), "runs": runs}
        log(f"[mode] {mode}: deterministic over {runs} runs")
    return report


# ------------------------------------------------------------------------------------------------ mock stack
def mock_stack(empty_sources: bool = False, fail_lanes=()):
    """Three lane services (echo backend + an in-memory retrieval stub) and a router, all in this process.
    Returns (router_url, servers) where servers must be closed by the caller (``for s in servers: s.close()``)."""
    import uvicorn
    from ..serving import serve as sv
    from ..serving.backend import EchoBackend
    from ..serving import router as rt

    class _Srv:
        def __init__(self, app):
            import socket
            s = socket.socket()
            s.bind(("127.0.0.1", 0))
            self.port = s.getsockname()[1]
            s.close()
            self.server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=self.port, log_level="warning"))
            self.thread = threading.Thread(target=self.server.run, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.server.started and time.time() - t0 < 20:
                time.sleep(0.02)

        def close(self):
            self.server.should_exit = True
            self.thread.join(10)

    def fake_query(**kw):
        from ..serving.hrm_client import HRMQueryResult
        if empty_sources:
            return HRMQueryResult({"prompt": kw["prompt"], "cids": [], "chosen": []})
        return HRMQueryResult({"prompt": kw["prompt"], "cids": ["0001"],
                               "chosen": [{"sid": "0001#s0000", "cid": "0001", "rel": 9, "txt": "mock fact one",
                                           "txt_c": "mock fact one"},
                                          {"sid": "0001#s0001", "cid": "0001", "rel": 7, "txt": "mock fact two",
                                           "txt_c": "mock fact two"}]})

    servers, urls = [], {}
    for lane in rt.LANES:
        st = sv.ServiceState(backend=EchoBackend(fail=lane in fail_lanes), hrm_model=None, max_concurrent=8,
                             max_seq_len=4096, max_new_tokens=64, query_fn=fake_query)
        s = _Srv(sv.create_app(st))
        servers.append(s)
        urls[lane] = f"http://127.0.0.1:{s.port}"
    rst = rt.RouterState()
    rst.backends = {n: rt.Backend(n, u) for n, u in urls.items()}
    r = _Srv(rt.create_app(rst))
    servers.append(r)
    return f"http://127.0.0.1:{r.port}", servers


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="hrm-flash-e2e", description="live e2e harness (router URL) or --mock")
    ap.add_argument("--router_url", default="http://127.0.0.1:8090")
    ap.add_argument("--runs", type=int, default=3)
    ap.add_argument("--max_new_tokens", type=int, default=32)
    ap.add_argument("--route_hint", default=None)
    ap.add_argument("--allow_empty", action="store_true")
    ap.add_argument("--content_checks", action="store_true")
    ap.add_argument("--quick_limit_s", type=float, default=3.0)
    ap.add_argument("--mock", action="store_true")
    ap.add_argument("--mock_empty_sources", action="store_true")
    ap.add_argument("--report", default=None)
    a = ap.parse_args(argv)
    servers = []
    url = a.router_url
    if a.mock:
        url, servers = mock_stack(empty_sources=a.mock_empty_sources)
    try:
        rep = run_e2e(url, a.runs, a.max_new_tokens, a.route_hint, a.allow_empty, a.content_checks, a.quick_limit_s)
        if a.report:
            json.dump(rep, open(a.report, "w"), indent=1)
        print("[ok] e2e passed")
        return 0
    except E2EFailure as e:
        print(f"FAIL: {e}", file=sys.stderr)
        return 1
    finally:
        for s in servers:
            s.close()


if __name__ == "__main__":
    raise SystemExit(main())
