"""Multi-lane router: lane selection, failover, OpenAI-compatible endpoints with SSE keep-alive.

Semantics of the reference router (``hrm_flash/router.py:154-575``), retargeted to an 8xB200 box:

* logical lanes keep their public names: ``solo_22gb`` (the max-model lane, e.g. TP=8), ``nvlink_pair`` (the
  balanced lane, e.g. TP=4) and ``solo_3080`` (the fast lane, e.g. TP=2/1); aliases: quality/best -> solo_22gb,
  balanced/default/pair -> nvlink_pair, fast/latency -> solo_3080;
* primary lane: ``prefer_backend`` > ``route_hint`` > collapsed max-model mode (solo_22gb and nvlink_pair share an
  endpoint -> nvlink_pair) > size classes (prompt <= 256 tokens and max_new <= 192 -> fast; <= 1200 / <= 384 ->
  balanced; else max-model);
* per-lane max_new caps (192 / 384 / 768), failover order per primary, 503 ``{error, primary, attempted,
  backend_errors}`` when every candidate fails; prompts truncated to the last ``max_prompt_chars`` (3000) chars;
* OpenAI endpoints default to ``mode = deepseek_only``; streaming sends ``: keepalive`` every 5 s until the result,
  then one chunk, a stop chunk with usage, and ``[DONE]``.
"""
import argparse
import asyncio
import contextlib
import json
import os
import secrets
import sys
import threading
import time
import urllib.error
import urllib.request
from dataclasses import dataclass
from typing import Any, Dict, Iterator, List, Optional, Tuple, Union

from .prompt_builder import SUPPORTED_MODES, normalize_mode

LANES = ("solo_22gb", "nvlink_pair", "solo_3080")
ALIASES = {
    "22gb": "solo_22gb", "solo22": "solo_22gb", "solo_22": "solo_22gb", "solo_22gb": "solo_22gb",
    "quality": "solo_22gb", "best": "solo_22gb", "max": "solo_22gb", "tp8": "solo_22gb",
    "pair": "nvlink_pair", "nvlink": "nvlink_pair", "nvlink_pair": "nvlink_pair", "balanced": "nvlink_pair",
    "default": "nvlink_pair", "tp4": "nvlink_pair",
    "3080": "solo_3080", "solo_3080": "solo_3080", "fast": "solo_3080", "low_latency": "solo_3080",
    "latency": "solo_3080", "tp2": "solo_3080",
}
FAILOVER = {
    "solo_3080": ["solo_3080", "nvlink_pair", "solo_22gb"],
    "nvlink_pair": ["nvlink_pair", "solo_22gb", "solo_3080"],
    "solo_22gb": ["solo_22gb", "nvlink_pair", "solo_3080"],
}
USER_MARKERS = ["\nuser:", "\nUser:", "\nUSER:", "<｜User｜>", "<|User|>", "### User:", "\nHuman:"]
DEFAULT_MODEL_ID = "deepseek-r1-distill-llama-70b-b200"


@dataclass(frozen=True)
class Backend:
    name: str
    base_url: str


class RouterState:
    def __init__(self):
        self.backends: Dict[str, Backend] = {}
        self.short_prompt_tokens = 256
        self.medium_prompt_tokens = 1200
        self.short_max_new_tokens = 192
        self.medium_max_new_tokens = 384
        self.long_max_new_tokens = 768
        self.request_timeout_s = 180.0
        self.health_timeout_s = 1.5
        self.chars_per_token = 4.0
        self.max_concurrent = 8
        self.sem: Optional[asyncio.Semaphore] = None
        self.tokenizer: Any = None
        self.tokenizer_name: Optional[str] = None
        self.default_mode = "mixed"
        self.max_prompt_chars = 3000
        self.keepalive_s = 5.0
        self.model_id = DEFAULT_MODEL_ID
        self.post = http_json_post    # injectable transport (tests)
        self.post_stream = http_sse_post
        self.get = http_json_get
        # routing counters (GET /metrics)
        self.requests_total = 0
        self.routed: Dict[str, int] = {}        # answered requests per lane
        self.lane_errors: Dict[str, int] = {}   # failed attempts per lane
        self.failovers_total = 0                # answered by a lane other than the primary
        self.all_failed_total = 0               # 503: every candidate lane failed


class LaneCallError(RuntimeError):
    """A lane request that produced no usable JSON object; ``status`` is the lane's HTTP status when it answered
    with an error status, else None (no answer: refused, timed out, unreadable)."""

    def __init__(self, url: str, reason: str, status: Optional[int] = None):
        super().__init__(f"{url}: {reason}")
        self.url, self.status = url, status


def _lane_call(method: str, url: str, payload: Optional[Dict[str, Any]], timeout_s: float
               ) -> Tuple[Dict[str, Any], int]:
    """One JSON request to a lane.  Returns the decoded object and the round trip in whole milliseconds; every
    failure (error status with the lane's own explanation, transport error, non-object body) is a LaneCallError,
    which the router counts against the lane and answers by trying the next one."""
    body = None if payload is None else json.dumps(payload).encode("utf-8")
    headers = {} if body is None else {"Content-Type": "application/json"}
    started = time.perf_counter()
    try:
        with urllib.request.urlopen(urllib.request.Request(url, data=body, method=method, headers=headers),
                                    timeout=timeout_s) as resp:
            raw = resp.read()
    except urllib.error.HTTPError as e:
        why = ""
        with contextlib.suppress(Exception):
            why = e.read().decode("utf-8", errors="replace").strip()
        raise LaneCallError(url, f"status {e.code}" + (f" ({why})" if why else ""), status=e.code) from e
    except (OSError, ValueError) as e:   # refused, reset, timeout (socket.timeout is an OSError), bad URL
        raise LaneCallError(url, f"no answer: {type(e).__name__}: {e}") from e
    elapsed_ms = int((time.perf_counter() - started) * 1000)
    try:
        obj = json.loads(raw.decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise LaneCallError(url, f"answer is not JSON ({len(raw)} bytes)") from e
    if not isinstance(obj, dict):
        raise LaneCallError(url, f"answer is a JSON {type(obj).__name__}, expected an object")
    return obj, elapsed_ms


def http_sse_post(url: str, payload: Dict[str, Any], timeout_s: float) -> Iterator[Dict[str, Any]]:
    """POST to a lane's streaming endpoint and yield the JSON object of every ``data:`` event as it arrives (until
    ``[DONE]``).  Failures before or during the stream are LaneCallErrors."""
    body = json.dumps(payload).encode("utf-8")
    req = urllib.request.Request(url, data=body, method="POST", headers={"Content-Type": "application/json"})
    try:
        resp = urllib.request.urlopen(req, timeout=timeout_s)
    except urllib.error.HTTPError as e:
        why = ""
        with contextlib.suppress(Exception):
            why = e.read().decode("utf-8", errors="replace").strip()
        raise LaneCallError(url, f"status {e.code}" + (f" ({why})" if why else ""), status=e.code) from e
    except (OSError, ValueError) as e:
        raise LaneCallError(url, f"no answer: {type(e).__name__}: {e}") from e
    with resp:
        try:
            for raw in resp:
                line = raw.decode("utf-8", errors="replace").strip()
                if not line.startswith("data:"):
                    continue            # keepalive comments and blank separators
                data = line[5:].strip()
                if data == "[DONE]":
                    return
                try:
                    obj = json.loads(data)
                except json.JSONDecodeError as e:
                    raise LaneCallError(url, f"stream event is not JSON: {data[:80]!r}") from e
                if isinstance(obj, dict):
                    yield obj
        except OSError as e:
            raise LaneCallError(url, f"stream broken: {type(e).__name__}: {e}") from e


def http_json_get(url: str, timeout_s: float) -> Tuple[Dict[str, Any], int]:
    return _lane_call("GET", url, None, timeout_s)


def http_json_post(url: str, payload: Dict[str, Any], timeout_s: float) -> Tuple[Dict[str, Any], int]:
    return _lane_call("POST", url, payload, timeout_s)


def normalize_backend_name(v: Optional[str]) -> Optional[str]:
    if not v:
        return None
    s = v.strip().lower()
    return ALIASES.get(s, s)


def estimate_prompt_tokens(st: RouterState, prompt: str) -> Tuple[int, str]:
    if st.tokenizer is not None:
        try:
            ids = st.tokenizer(prompt, add_special_tokens=True).get("input_ids", [])
            return max(1, len(ids)), "tokenizer"
        except Exception:
            pass
    return max(1, int(len(prompt) / max(1e-6, st.chars_per_token) + 0.999)), "chars"


def collapsed_max_model_mode(st: RouterState) -> bool:
    s, p, f = (st.backends.get(n) for n in LANES)
    return s is not None and p is not None and f is not None and s.base_url == p.base_url


def primary_backend(st: RouterState, prompt_tokens: int, max_new: int, route_hint: Optional[str],
                    prefer_backend: Optional[str]) -> str:
    pref = normalize_backend_name(prefer_backend)
    if pref in st.backends:
        return pref
    hint = normalize_backend_name(route_hint)
    if hint in st.backends:
        return hint
    if collapsed_max_model_mode(st):
        return "nvlink_pair"
    if prompt_tokens <= st.short_prompt_tokens and max_new <= st.short_max_new_tokens:
        return "solo_3080"
    if prompt_tokens <= st.medium_prompt_tokens and max_new <= st.medium_max_new_tokens:
        return "nvlink_pair"
    return "solo_22gb"


def max_new_limit(st: RouterState, lane: str) -> int:
    return {"solo_3080": st.short_max_new_tokens, "nvlink_pair": st.medium_max_new_tokens}.get(
        lane, st.long_max_new_tokens)


def candidate_order(st: RouterState, primary: str, allow_failover: bool) -> List[str]:
    if not allow_failover:
        return [primary]
    order = ["nvlink_pair", "solo_22gb"] if collapsed_max_model_mode(st) else \
        FAILOVER.get(primary, [primary, "nvlink_pair", "solo_22gb", "solo_3080"])
    out: List[str] = []
    for n in order:
        if n in st.backends and n not in out:
            out.append(n)
    return out


def resolve_show_sources(show: Optional[bool], mode: str) -> bool:
    if mode == "deepseek_only":
        return False
    return mode == "retrieval" if show is None else bool(show)


def last_user_prompt(prompt: str) -> str:
    text = str(prompt or "").strip()
    best_at, best = -1, ""
    for m in USER_MARKERS:
        at = text.rfind(m)
        if at > best_at:
            best_at, best = at, m
    return text[best_at + len(best):].strip() if best_at >= 0 else text


def chat_messages_to_prompt(messages: Any) -> str:
    if not isinstance(messages, list):
        return ""
    parts = []
    for msg in messages:
        if not isinstance(msg, dict):
            continue
        c = msg.get("content")
        text = " ".join(str(p.get("text") or "") for p in c if isinstance(p, dict)) if isinstance(c, list) \
            else str(c or "")
        if text.strip() and str(msg.get("role") or "user").lower() == "user":
            parts.append(text.strip())
    return "\n".join(parts).strip()


def create_app(st: RouterState):
    from fastapi import FastAPI, HTTPException, Request
    from fastapi.responses import JSONResponse, StreamingResponse
    from pydantic import BaseModel

    app = FastAPI(title="hrm-flash-b200-router", version="0.1.0")

    class GenerateReq(BaseModel):
        prompt: str
        max_new_tokens: Optional[int] = None
        mode: Optional[str] = None
        show_sources: Optional[bool] = None
        route_hint: Optional[str] = None
        prefer_backend: Optional[str] = None
        allow_failover: bool = True
        temperature: Optional[float] = None   # forwarded to the lane only when given (absent: greedy)
        top_k: Optional[int] = None
        seed: Optional[int] = None
        stop: Optional[Union[str, List[str]]] = None
        stream: Optional[bool] = None           # server-sent events: the lane's deltas, then its payload + route

    def truncate(prompt: str) -> str:
        t = str(prompt or "").strip()
        return t if len(t) <= st.max_prompt_chars else t[-st.max_prompt_chars:]

    async def run_generate(req: GenerateReq) -> Dict[str, Any]:
        if not req.prompt or not req.prompt.strip():
            raise HTTPException(status_code=400, detail="prompt required")
        prompt = truncate(req.prompt)
        try:
            mode = normalize_mode(req.mode if req.mode is not None else st.default_mode)
        except ValueError as e:
            raise HTTPException(status_code=400, detail=str(e))
        st.requests_total += 1
        if st.sem is None:
            st.sem = asyncio.Semaphore(st.max_concurrent)
        async with st.sem:
            req_new = max(1, min(4096, int(req.max_new_tokens) if req.max_new_tokens is not None else 256))
            ptoks, estimator = estimate_prompt_tokens(st, prompt)
            if mode == "deepseek_only":
                print("[router] mode=deepseek_only HRM disabled (no retrieval)", file=sys.stderr, flush=True)
            primary = primary_backend(st, ptoks, req_new, req.route_hint, req.prefer_backend)
            attempted, errors = [], []
            show = resolve_show_sources(req.show_sources, mode)
            for lane in candidate_order(st, primary, bool(req.allow_failover)):
                be = st.backends[lane]
                lane_new = min(req_new, max_new_limit(st, lane))
                attempted.append(lane)
                try:
                    lane_req = {"prompt": prompt, "max_new_tokens": lane_new, "mode": mode, "show_sources": show}
                    lane_req.update({k: v for k, v in (("temperature", req.temperature), ("top_k", req.top_k),
                                                       ("seed", req.seed), ("stop", req.stop)) if v is not None})
                    body, ms = await asyncio.to_thread(st.post, be.base_url + "/v1/generate", lane_req,
                                                       st.request_timeout_s)
                    if not bool(body.get("ok", True)):
                        raise RuntimeError(str(body.get("detail") or body.get("error") or "backend returned ok=false"))
                    out = dict(body)
                    st.routed[lane] = st.routed.get(lane, 0) + 1
                    if lane != primary:
                        st.failovers_total += 1
                    out["route"] = {"primary": primary, "selected": lane, "attempted": attempted,
                                    "estimator": estimator, "prompt_tokens": ptoks,
                                    "requested_max_new_tokens": req_new, "backend_max_new_tokens": lane_new,
                                    "latency_ms": ms}
                    return out
                except Exception as e:
                    errors.append(f"{lane}: {e}")
                    st.lane_errors[lane] = st.lane_errors.get(lane, 0) + 1
            st.all_failed_total += 1
            raise HTTPException(status_code=503, detail={"error": "all backends failed", "primary": primary,
                                                         "attempted": attempted, "backend_errors": errors})

    def usage(prompt: str, text: str) -> Dict[str, int]:
        p, _ = estimate_prompt_tokens(st, prompt)
        c, _ = estimate_prompt_tokens(st, text)
        return {"prompt_tokens": p, "completion_tokens": c, "total_tokens": p + c}

    def chunk(cid: str, model: str, chat: bool, piece: Optional[str], finish: Optional[str] = None,
              extra: Optional[Dict[str, Any]] = None, role: bool = False) -> str:
        now = int(time.time())
        if chat:
            delta = {"role": "assistant"} if role else ({} if piece is None else {"content": piece})
            choice = {"index": 0, "delta": delta, "finish_reason": finish}
            obj = {"id": cid, "object": "chat.completion.chunk", "created": now, "model": model, "choices": [choice]}
        else:
            choice = {"index": 0, "text": piece or "", "finish_reason": finish}
            obj = {"id": cid, "object": "text_completion", "created": now, "model": model, "choices": [choice]}
        if extra:
            obj.update(extra)
        return f"data: {json.dumps(obj)}\n\n"

    async def relay(req: GenerateReq, model: str, prompt: str, chat: bool, native: bool = False):
        """OpenAI streaming: the selected lane streams text deltas, relayed as chunks while it generates.  A lane
        that fails before its first delta is replaced by the next candidate (as for non-streaming requests);
        after that, an error ends the stream with an error event.  Comment lines keep the connection alive while a
        lane is silent.  When the client goes away, the lane connection is closed, which cancels the request on
        the lane.  ``native``: the lane's own events are passed on (``{"delta": ...}``, then its payload with the
        router's ``route`` record) instead of OpenAI chunks."""
        cid = f"{'chatcmpl' if chat else 'cmpl'}-{int(time.time() * 1000)}"
        try:
            mode = normalize_mode(req.mode if req.mode is not None else st.default_mode)
        except ValueError as e:
            yield f"data: {json.dumps({'error': str(e)})}\n\n"
            yield "data: [DONE]\n\n"
            return
        st.requests_total += 1
        req_new = max(1, min(4096, int(req.max_new_tokens) if req.max_new_tokens is not None else 256))
        ptoks, _ = estimate_prompt_tokens(st, prompt)
        primary = primary_backend(st, ptoks, req_new, req.route_hint, req.prefer_backend)
        attempted, errors = [], []
        loop = asyncio.get_running_loop()
        for lane in candidate_order(st, primary, bool(req.allow_failover)):
            be = st.backends[lane]
            attempted.append(lane)
            lane_req = {"prompt": prompt, "max_new_tokens": min(req_new, max_new_limit(st, lane)), "mode": mode,
                        "show_sources": resolve_show_sources(req.show_sources, mode), "stream": True}
            lane_req.update({k: v for k, v in (("temperature", req.temperature), ("top_k", req.top_k),
                                               ("seed", req.seed), ("stop", req.stop)) if v is not None})
            q: "asyncio.Queue" = asyncio.Queue()
            gone = threading.Event()   # set when this relay stops reading: the pump then drops the lane stream

            def pump(url=be.base_url + "/v1/generate", payload=lane_req, gone=gone, q=q):
                events = None
                try:
                    events = st.post_stream(url, payload, st.request_timeout_s)
                    for ev in events:
                        if gone.is_set():
                            return
                        loop.call_soon_threadsafe(q.put_nowait, ("ev", ev))
                    loop.call_soon_threadsafe(q.put_nowait, ("end", None))
                except Exception as e:   # handed to the event loop
                    if not gone.is_set():
                        loop.call_soon_threadsafe(q.put_nowait, ("err", e))
                finally:
                    close = getattr(events, "close", None)
                    if close is not None:
                        close()          # closes the lane connection; the lane then cancels the request

            threading.Thread(target=pump, daemon=True).start()
            started, text = False, []
            try:
                while True:
                    try:
                        kind, ev = await asyncio.wait_for(q.get(), timeout=st.keepalive_s)
                    except asyncio.TimeoutError:
                        yield ": keepalive\n\n"
                        continue
                    failed = (kind == "err" or (kind == "ev" and ev.get("ok") is False)
                              or (kind == "end" and not started))
                    if failed:
                        why = ev if kind == "err" else (ev or {}).get("error", "stream ended without an answer")
                        st.lane_errors[lane] = st.lane_errors.get(lane, 0) + 1
                        if not started:
                            errors.append(f"{lane}: {why}")
                            break                              # next candidate lane
                        err = {"ok": False, "error": str(why)} if native else {"error": str(why)}
                        yield f"data: {json.dumps(err)}\n\n"
                        yield "data: [DONE]\n\n"
                        return
                    if kind == "end":
                        ev = {"text": "".join(text)}
                    if "delta" in ev:
                        if not started and chat and not native:
                            yield chunk(cid, model, chat, None, role=True)
                        started = True
                        text.append(str(ev["delta"]))
                        if native:
                            yield f"data: {json.dumps({'delta': str(ev['delta'])})}\n\n"
                        else:
                            yield chunk(cid, model, chat, str(ev["delta"]))
                        continue
                    full = str(ev.get("text", "".join(text)))   # the final payload closes the stream
                    st.routed[lane] = st.routed.get(lane, 0) + 1
                    if lane != primary:
                        st.failovers_total += 1
                    if native:
                        out = dict(ev)
                        out["route"] = {"primary": primary, "selected": lane, "attempted": attempted,
                                        "prompt_tokens": ptoks, "requested_max_new_tokens": req_new,
                                        "backend_max_new_tokens": lane_req["max_new_tokens"]}
                        yield f"data: {json.dumps(out)}\n\n"
                    else:
                        if not started and full:
                            yield chunk(cid, model, chat, full)
                        yield chunk(cid, model, chat, None, "stop", {"usage": usage(prompt, full)})
                    yield "data: [DONE]\n\n"
                    return
            finally:
                gone.set()
        st.all_failed_total += 1
        detail = {"error": "all backends failed", "primary": primary, "attempted": attempted, "backend_errors": errors}
        yield f"data: {json.dumps({'ok': False, 'detail': detail} if native else {'error': detail})}\n\n"
        yield "data: [DONE]\n\n"

    def check(lane: str) -> Dict[str, Any]:
        be = st.backends[lane]
        try:
            payload, ms = st.get(be.base_url + "/v1/health", st.health_timeout_s)
            return {"ok": bool(payload.get("ok", False)), "latency_ms": ms, "url": be.base_url}
        except Exception as e:
            return {"ok": False, "error": str(e), "url": be.base_url}

    @app.get("/metrics")
    async def prometheus():
        """Routing counters in the Prometheus text format."""
        from fastapi.responses import PlainTextResponse
        from .prom import exposition
        lanes = [n for n in LANES if n in st.backends]
        text = exposition([
            ("hrm_router_requests_total", "counter", "generate requests accepted", [({}, st.requests_total)]),
            ("hrm_router_routed_total", "counter", "requests answered, by lane",
             [({"lane": n}, st.routed.get(n, 0)) for n in lanes]),
            ("hrm_router_lane_errors_total", "counter", "failed attempts, by lane",
             [({"lane": n}, st.lane_errors.get(n, 0)) for n in lanes]),
            ("hrm_router_failovers_total", "counter", "requests answered by a lane other than the primary",
             [({}, st.failovers_total)]),
            ("hrm_router_all_failed_total", "counter", "requests for which every candidate lane failed (503)",
             [({}, st.all_failed_total)]),
        ])
        return PlainTextResponse(text, media_type="text/plain; version=0.0.4")

    @app.get("/v1/health")
    async def health():
        names = [n for n in LANES if n in st.backends]
        checks = await asyncio.gather(*[asyncio.to_thread(check, n) for n in names])
        bh = dict(zip(names, checks))
        return {"ok": any(c["ok"] for c in checks),
                "router": {"tokenizer": st.tokenizer_name, "collapsed_max_model_mode": collapsed_max_model_mode(st),
                           "request_timeout_s": st.request_timeout_s, "max_concurrent": st.max_concurrent,
                           "max_prompt_chars": st.max_prompt_chars, "default_mode": st.default_mode,
                           "supported_modes": sorted(SUPPORTED_MODES),
                           "thresholds": {"short_prompt_tokens": st.short_prompt_tokens,
                                          "medium_prompt_tokens": st.medium_prompt_tokens,
                                          "short_max_new_tokens": st.short_max_new_tokens,
                                          "medium_max_new_tokens": st.medium_max_new_tokens,
                                          "long_max_new_tokens": st.long_max_new_tokens}},
                "backends": bh}

    @app.post("/v1/generate")
    async def generate(request: Request):
        req = GenerateReq(**(await request.json()))
        if req.stream:
            if not req.prompt or not req.prompt.strip():
                raise HTTPException(status_code=400, detail="prompt required")
            return StreamingResponse(relay(req, st.model_id, truncate(req.prompt), chat=False, native=True),
                                     media_type="text/event-stream")
        return JSONResponse(await run_generate(req))

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": st.model_id, "object": "model", "created": 0,
                                            "owned_by": "hrm-flashrenderer-b200"}]}

    async def openai(body: Dict[str, Any], prompt: str, chat: bool):
        prompt = truncate(last_user_prompt(prompt))
        model = str(body.get("model") or st.model_id)
        req = GenerateReq(prompt=prompt, mode=str(body.get("mode") or "deepseek_only"),
                          max_new_tokens=body.get("max_tokens") or body.get("max_completion_tokens")
                          or body.get("max_new_tokens"),
                          route_hint=body.get("route_hint"), prefer_backend=body.get("prefer_backend"),
                          temperature=body.get("temperature"), top_k=body.get("top_k"), seed=body.get("seed"),
                          stop=body.get("stop"))
        n = int(body.get("n") or 1)
        if not 1 <= n <= 16:
            raise HTTPException(status_code=400, detail="n must be in 1..16")
        if bool(body.get("stream")):
            if n != 1:
                raise HTTPException(status_code=400, detail="stream supports n = 1")
            return StreamingResponse(relay(req, model, prompt, chat), media_type="text/event-stream")
        if n == 1 or not req.temperature:
            texts = [str((await run_generate(req)).get("text") or "")] * n   # greedy: every choice is the same
        else:
            # n independent draws: one request per choice, seeds seed, seed + 1, ... (random when no seed)
            base = int(req.seed) if req.seed is not None else secrets.randbits(62)
            reqs = [req.model_copy(update={"seed": base + i}) for i in range(n)]
            texts = [str(r.get("text") or "") for r in await asyncio.gather(*(run_generate(r) for r in reqs))]
        use = usage(prompt, texts[0])
        if n > 1:
            comp = sum(usage(prompt, t)["completion_tokens"] for t in texts)
            use = {"prompt_tokens": use["prompt_tokens"], "completion_tokens": comp,
                   "total_tokens": use["prompt_tokens"] + comp}
        if chat:
            return JSONResponse({"id": f"chatcmpl-{int(time.time() * 1000)}", "object": "chat.completion",
                                 "created": int(time.time()), "model": model,
                                 "choices": [{"index": i, "message": {"role": "assistant", "content": t},
                                              "finish_reason": "stop"} for i, t in enumerate(texts)],
                                 "usage": use})
        return JSONResponse({"id": f"cmpl-{int(time.time() * 1000)}", "object": "text_completion",
                             "created": int(time.time()), "model": model,
                             "choices": [{"index": i, "text": t, "finish_reason": "stop"} for i, t in enumerate(texts)],
                             "usage": use})

    @app.post("/v1/completions")
    async def completions(request: Request):
        body = await request.json()
        prompt = body.get("prompt", "")
        if isinstance(prompt, list):
            prompt = "\n".join(str(x) for x in prompt)
        return await openai(body, str(prompt), chat=False)

    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request):
        body = await request.json()
        return await openai(body, chat_messages_to_prompt(body.get("messages")), chat=True)

    return app


def build_arg_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="hrm-flash-router", description="Lane router for hrm-flash B200 services")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=8090)
    ap.add_argument("--endpoint_solo_22gb", default="http://127.0.0.1:8081")
    ap.add_argument("--endpoint_nvlink_pair", default="http://127.0.0.1:8082")
    ap.add_argument("--endpoint_solo_3080", default="http://127.0.0.1:8083")
    ap.add_argument("--short_prompt_tokens", type=int, default=256)
    ap.add_argument("--medium_prompt_tokens", type=int, default=1200)
    ap.add_argument("--short_max_new_tokens", type=int, default=192)
    ap.add_argument("--medium_max_new_tokens", type=int, default=384)
    ap.add_argument("--long_max_new_tokens", type=int, default=768)
    ap.add_argument("--request_timeout_s", type=float, default=180.0)
    ap.add_argument("--health_timeout_s", type=float, default=1.5)
    ap.add_argument("--max_concurrent", type=int, default=8)
    ap.add_argument("--tokenizer_model", default=None)
    ap.add_argument("--chars_per_token", type=float, default=4.0)
    ap.add_argument("--local_files_only", action="store_true")
    ap.add_argument("--disable_tokenizer", action="store_true")
    ap.add_argument("--default_mode", choices=["retrieval", "mixed", "deepseek_only"], default="mixed")
    ap.add_argument("--max_prompt_chars", type=int, default=int(os.environ.get("ROUTER_MAX_PROMPT_CHARS", "3000")))
    return ap


def state_from_args(args) -> RouterState:
    st = RouterState()
    st.backends = {n: Backend(n, str(getattr(args, f"endpoint_{n}")).strip().rstrip("/")) for n in LANES}
    st.short_prompt_tokens = max(16, int(args.short_prompt_tokens))
    st.medium_prompt_tokens = max(st.short_prompt_tokens + 1, int(args.medium_prompt_tokens))
    st.short_max_new_tokens = max(16, int(args.short_max_new_tokens))
    st.medium_max_new_tokens = max(st.short_max_new_tokens, int(args.medium_max_new_tokens))
    st.long_max_new_tokens = max(st.medium_max_new_tokens, int(args.long_max_new_tokens))
    st.request_timeout_s = max(1.0, float(args.request_timeout_s))
    st.health_timeout_s = max(0.2, float(args.health_timeout_s))
    st.chars_per_token = max(1.0, float(args.chars_per_token))
    st.max_concurrent = max(1, int(args.max_concurrent))
    st.default_mode = normalize_mode(args.default_mode)
    st.max_prompt_chars = max(1024, int(args.max_prompt_chars))
    if not args.disable_tokenizer and args.tokenizer_model:
        try:
            from transformers import AutoTokenizer
            st.tokenizer = AutoTokenizer.from_pretrained(args.tokenizer_model, local_files_only=args.local_files_only)
            st.tokenizer_name = str(args.tokenizer_model)
        except Exception as e:
            print(f"[router] tokenizer unavailable, using char-estimate: {e}", file=sys.stderr, flush=True)
    return st


def main(argv=None):
    args = build_arg_parser().parse_args(argv)
    st = state_from_args(args)
    import uvicorn
    uvicorn.run(create_app(st), host=args.host, port=args.port, log_level="info")


if __name__ == "__main__":
    main()
