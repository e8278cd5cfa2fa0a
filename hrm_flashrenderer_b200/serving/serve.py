"""HTTP service of one lane: ``POST /v1/generate``, ``GET /v1/health``, ``GET /v1/metrics`` (JSON) and ``GET /metrics``
(Prometheus text format).

Request/response contract of the reference service (``hrm_flash/serve.py:207-301``):

* request: ``prompt`` (required), ``max_new_tokens``, ``mode`` (retrieval | mixed | deepseek_only + aliases),
  ``show_sources``;
* response: ``ok``, ``text``, ``mode``, ``source_count``, ``hrm_active``, ``audit{mode_resolved, hrm_called,
  source_injected_count, prompt_template}`` and ``sources`` when shown (default: retrieval mode only; never for
  deepseek_only);
* no retrieved sources (or no fit in the token budget) in retrieval/mixed mode -> ``text = "I don't know."``;
* health: ``ok`` = generation backend alive, plus the audit counters.  This build adds scheduler metrics (TTFT,
  inter-token latency, tok/s, queue depth, batch size).

Retrieval runs in-process against the C++ HRM core (cached handle, 1.8 s budget) while other requests keep the GPU
busy; generation goes to the continuous-batching engine, so ``--max_concurrent`` can exceed 1.
"""
import argparse
import asyncio
import json
import os
import threading
import time
from pathlib import Path
from typing import Any, List, Optional, Tuple, Union

from .hrm_client import run_hrm_query
from .prompt_builder import build_prompt_for_mode, build_sources, fit_prompt_to_token_budget, normalize_mode
from .utils import find_hrm_binary
from ..runtime.sampling import sampling_from_request

REPO_ROOT = Path(__file__).resolve().parents[2]
TEMPLATES = {"mixed": "mixed_silent", "retrieval": "retrieval_explicit", "deepseek_only": "deepseek_only_raw"}


class ServiceState:
    def __init__(self, backend=None, hrm_model: Optional[Path] = None, hrm_bin: Optional[Path] = None,
                 max_seq_len: int = 8192, max_new_tokens: int = 256, max_sources: int = 16,
                 max_chars_per_source: int = 1200, reserve_prompt_tokens: int = 16, disable_token_budget: bool = False,
                 expose_sources: bool = False, max_concurrent: int = 1, request_timeout_s: float = 180.0,
                 hrm_timeout_s: float = 1.8, world: int = 1, backend_name: str = "b200_int8", query_fn=None):
        self.backend = backend
        self.query_fn = query_fn      # retrieval function (default: run_hrm_query); injectable for mock lanes
        self.hrm_model = Path(hrm_model) if hrm_model else None
        self.hrm_bin = hrm_bin
        self.max_seq_len = max_seq_len
        self.max_new_tokens = max_new_tokens
        self.max_sources = max_sources
        self.max_chars_per_source = max_chars_per_source
        self.reserve_prompt_tokens = reserve_prompt_tokens
        self.disable_token_budget = disable_token_budget
        self.expose_sources = expose_sources
        self.max_concurrent = max(1, int(max_concurrent))
        self.request_timeout_s = request_timeout_s
        self.hrm_timeout_s = hrm_timeout_s
        self.world = world
        self.backend_name = backend_name
        self.sem: Optional[asyncio.Semaphore] = None
        self.requests_total = 0
        self.mode_counts = {"mixed": 0, "retrieval": 0, "deepseek_only": 0}
        self.hrm_query_calls_total = 0
        self.hrm_query_calls_by_mode = {"mixed": 0, "retrieval": 0, "deepseek_only": 0}
        self.prompt_build_failures = 0

    @property
    def tokenizer(self):
        return getattr(self.backend, "tokenizer", None)


def build_prompt(state: ServiceState, prompt: str, mode: str) -> Tuple[str, List[Any], str, bool]:
    """(prompt_text, sources, resolved_mode, hrm_active).  Empty prompt_text means "I don't know."."""
    resolved = normalize_mode(mode)
    if resolved == "deepseek_only":
        return build_prompt_for_mode(prompt, [], resolved), [], resolved, False
    state.hrm_query_calls_total += 1
    state.hrm_query_calls_by_mode[resolved] = state.hrm_query_calls_by_mode.get(resolved, 0) + 1
    q = state.query_fn or run_hrm_query
    r = q(hrm_bin=state.hrm_bin, model_dir=state.hrm_model, prompt=prompt, top_k=16, top_m=400, k=16,
          prefer_api=True, repo_root=REPO_ROOT, timeout_s=state.hrm_timeout_s)
    sources = build_sources(r.raw, max_sources=state.max_sources, max_chars_per_source=state.max_chars_per_source)
    if not sources:
        return "", [], resolved, True
    q, srcs = prompt, sources
    if not state.disable_token_budget:
        tok = state.tokenizer
        if tok is None:
            return "", [], resolved, True
        budget = int(state.max_seq_len) - int(state.max_new_tokens) - int(state.reserve_prompt_tokens)
        q, srcs = fit_prompt_to_token_budget(q, srcs, tok, budget, mode=resolved)
        if not srcs:
            return "", [], resolved, True
    return build_prompt_for_mode(q, srcs, resolved), srcs, resolved, True


# engine metric -> (Prometheus name, type, help); values that are None are left out
_PROM_ENGINE = (
    ("queue_depth", "hrm_engine_queue_depth", "gauge", "requests waiting for admission"),
    ("batch_size", "hrm_engine_batch_size", "gauge", "sequences in the running decode batch"),
    ("completed", "hrm_engine_requests_completed_total", "counter", "finished generation requests"),
    ("generated_tokens", "hrm_engine_generated_tokens_total", "counter", "tokens generated"),
    ("tok_per_s", "hrm_engine_tokens_per_second", "gauge", "generated tokens per second since start"),
    ("ttft_p50_ms", "hrm_engine_ttft_p50_ms", "gauge", "median time to first token (ms)"),
    ("ttft_p99_ms", "hrm_engine_ttft_p99_ms", "gauge", "99th percentile time to first token (ms)"),
    ("itl_p50_ms", "hrm_engine_itl_p50_ms", "gauge", "median inter-token latency (ms)"),
    ("prefilling", "hrm_engine_prefilling", "gauge", "admitted requests whose prompt is still being prefilled"),
    ("prefix_cache_hit_blocks", "hrm_engine_prefix_cache_hit_blocks_total", "counter",
     "KV blocks shared from the prefix cache instead of recomputed"),
    ("cancelled", "hrm_engine_requests_cancelled_total", "counter", "requests cancelled (caller timed out)"),
)


def prometheus_text(state: "ServiceState", eng: dict, running: bool) -> str:
    """Prometheus text exposition of the lane's audit counters and its engine's metrics."""
    from .prom import exposition
    fam = [
        ("hrm_lane_up", "gauge", "1 while the generation backend runs", [({}, 1 if running else 0)]),
        ("hrm_lane_requests_total", "counter", "generate requests received", [({}, state.requests_total)]),
        ("hrm_lane_requests_by_mode_total", "counter", "generate requests by resolved mode",
         [({"mode": m}, n) for m, n in sorted(state.mode_counts.items())]),
        ("hrm_lane_hrm_queries_total", "counter", "HRM retrieval queries by mode",
         [({"mode": m}, n) for m, n in sorted(state.hrm_query_calls_by_mode.items())]),
        ("hrm_lane_prompt_build_failures_total", "counter", "prompts that could not be built",
         [({}, state.prompt_build_failures)]),
    ]
    for key, name, typ, help_ in _PROM_ENGINE:
        v = eng.get(key)
        if isinstance(v, (int, float)) and not isinstance(v, bool):
            fam.append((name, typ, help_, [({}, v)]))
    if "fatal" in eng:
        fam.append(("hrm_engine_fatal", "gauge", "1 after a fatal engine error (the lane needs a restart)",
                    [({}, 0 if eng.get("fatal") is None else 1)]))
    return exposition(fam)


def create_app(state: ServiceState):
    from fastapi import FastAPI, HTTPException, Request
    from fastapi.responses import JSONResponse
    from pydantic import BaseModel

    app = FastAPI(title="hrm-flash-b200", version="0.1.0")

    class GenerateReq(BaseModel):
        prompt: str
        max_new_tokens: Optional[int] = None
        mode: Optional[str] = None
        show_sources: Optional[bool] = None
        temperature: Optional[float] = None   # absent or 0: greedy (the default)
        top_k: Optional[int] = None
        seed: Optional[int] = None
        stream: Optional[bool] = None         # server-sent events: text deltas, then the full payload
        stop: Optional[Union[str, List[str]]] = None   # end the answer before the first of these strings

    def sem() -> asyncio.Semaphore:
        if state.sem is None:
            state.sem = asyncio.Semaphore(state.max_concurrent)
        return state.sem

    @app.get("/v1/health")
    async def health():
        running = False
        try:
            running = bool(state.backend is not None and state.backend.is_running())
        except Exception:
            running = False
        out = {
            "ok": running, "backend": state.backend_name, "deepseek_running": running, "world": state.world,
            "audit": {"requests_total": state.requests_total, "mode_counts": dict(state.mode_counts),
                      "hrm_query_calls_total": state.hrm_query_calls_total,
                      "hrm_query_calls_by_mode": dict(state.hrm_query_calls_by_mode),
                      "prompt_build_failures": state.prompt_build_failures},
        }
        try:
            out["engine"] = state.backend.metrics() if state.backend is not None else {}
        except Exception as e:
            out["engine"] = {"error": str(e)}
        return out

    @app.get("/v1/metrics")
    async def metrics():
        return state.backend.metrics() if state.backend is not None else {}

    @app.get("/metrics")
    async def prometheus():
        """The same counters and engine metrics in the Prometheus text exposition format."""
        from fastapi.responses import PlainTextResponse
        try:
            eng = state.backend.metrics() if state.backend is not None else {}
        except Exception:
            eng = {}
        try:
            running = bool(state.backend is not None and state.backend.is_running())
        except Exception:
            running = False
        return PlainTextResponse(prometheus_text(state, eng, running), media_type="text/plain; version=0.0.4")

    @app.post("/v1/generate")
    async def generate(request: Request):
        try:
            req = GenerateReq(**(await request.json()))
        except Exception as e:
            raise HTTPException(status_code=400, detail=f"bad request: {e}")
        if not req.prompt:
            raise HTTPException(status_code=400, detail="prompt required")
        try:
            mode = normalize_mode(req.mode)
            sampling = sampling_from_request(req.temperature, req.top_k, req.seed)
        except ValueError as e:
            raise HTTPException(status_code=400, detail=str(e))
        async with sem():
            state.requests_total += 1
            state.mode_counts[mode] = state.mode_counts.get(mode, 0) + 1
            try:
                prompt_text, sources, mode, hrm_active = await asyncio.to_thread(build_prompt, state, req.prompt, mode)
            except Exception as e:
                raise HTTPException(status_code=500, detail=f"prompt build failed: {e}")
            template = TEMPLATES[mode]
            show = bool(req.show_sources) if req.show_sources is not None else (mode == "retrieval")
            if not prompt_text:
                state.prompt_build_failures += 1
                payload = {"ok": True, "text": "I don't know.", "source_count": 0, "mode": mode,
                           "hrm_active": hrm_active,
                           "audit": {"mode_resolved": mode, "hrm_called": bool(hrm_active), "source_injected_count": 0,
                                     "prompt_template": template}}
                if show or state.expose_sources:
                    payload["sources"] = []
                if req.stream:
                    return _sse_response(iter(()), payload)
                return JSONResponse(payload)
            max_new = int(req.max_new_tokens) if req.max_new_tokens is not None else state.max_new_tokens
            if state.backend is None:
                raise HTTPException(status_code=500, detail="generation backend not initialized")
        base = {"ok": True, "source_count": len(sources), "mode": mode, "hrm_active": hrm_active,
                "audit": {"mode_resolved": mode, "hrm_called": bool(hrm_active),
                          "source_injected_count": len(sources), "prompt_template": template}}
        if (show or state.expose_sources) and mode != "deepseek_only":
            base["sources"] = [{"sid": s.sid, "txt": s.txt} for s in sources]
        stops = [req.stop] if isinstance(req.stop, str) else list(req.stop or [])
        if req.stream:
            stop = threading.Event()
            kw = {"cancel": stop} if sampling is None else {"cancel": stop, "sampling": sampling}
            if stops:
                kw["stop"] = stops
            try:
                pieces = state.backend.generate_stream(prompt_text, max_new, state.request_timeout_s, **kw)
            except AttributeError:
                raise HTTPException(status_code=400, detail="this backend does not stream")
            return _sse_response(pieces, base, stop, request)
        # generation runs outside the admission semaphore's prompt-build section: the engine batches requests
        try:
            kw = {}
            if sampling is not None:
                kw["sampling"] = sampling
            if stops:
                kw["stop"] = stops
            text = await asyncio.to_thread(state.backend.generate, prompt_text, max_new, state.request_timeout_s,
                                           **kw)
        except Exception as e:
            raise HTTPException(status_code=500, detail=str(e))
        payload = {"ok": True, "text": text}
        payload.update((k, v) for k, v in base.items() if k != "ok")
        return JSONResponse(payload)

    def _sse_response(pieces, payload, stop=None, request=None):
        """``data: {"delta": ...}`` per text piece, then the full payload (with ``text``), then ``[DONE]``; a
        generation error ends the stream with ``{"ok": false, "error": ...}``.  A client that goes away closes the
        piece iterator, which cancels the request."""
        from fastapi.responses import StreamingResponse
        it = iter(pieces)

        async def events():
            parts = []
            try:
                while True:
                    piece = await asyncio.to_thread(next, it, None)
                    if piece is None:
                        break
                    parts.append(piece)
                    yield f"data: {json.dumps({'delta': piece})}\n\n"
                    # the server does not close this generator when the client leaves (its next write just fails),
                    # so look for the disconnect between pieces
                    if request is not None and await request.is_disconnected():
                        return
                out = dict(payload)
                out.setdefault("text", "".join(parts))
                yield f"data: {json.dumps(out)}\n\n"
            except Exception as e:
                yield f"data: {json.dumps({'ok': False, 'error': str(e)})}\n\n"
            finally:
                if stop is not None:
                    stop.set()           # the piece iterator sees it between tokens and cancels the request
                close = getattr(it, "close", None)
                if close is not None:
                    try:
                        close()
                    except ValueError:
                        # a next() is still running in its worker thread: close the iterator as soon as it
                        # returns (its cleanup cancels the engine request)
                        def close_later():
                            for _ in range(2000):
                                try:
                                    close()
                                    return
                                except ValueError:
                                    time.sleep(0.01)
                        threading.Thread(target=close_later, daemon=True).start()
            yield "data: [DONE]\n\n"

        return StreamingResponse(events(), media_type="text/event-stream")

    @app.on_event("shutdown")
    def _shutdown():
        if state.backend is not None:
            try:
                state.backend.stop()
            except Exception:
                pass

    return app


def build_arg_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="hrm-flash-serve", description="HRM FlashRenderer B200 lane service")
    ap.add_argument("--hrm_model", required=True)
    ap.add_argument("--llm_model", required=True,
                    help="DSI8 model_q8.bin, a local HF safetensors dir (exported to DSI8), or synthetic:<preset>")
    ap.add_argument("--world", type=int, choices=[1, 2, 4, 8], default=1, help="tensor-parallel size of this lane")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=8080)
    ap.add_argument("--max_seq_len", type=int, default=8192)
    ap.add_argument("--prefill_chunk_size", type=int, default=4096)
    ap.add_argument("--max_new_tokens", type=int, default=256)
    ap.add_argument("--max_batch", type=int, default=64)
    ap.add_argument("--local_files_only", action="store_true")
    ap.add_argument("--max_sources", type=int, default=16)
    ap.add_argument("--max_chars_per_source", type=int, default=1200)
    ap.add_argument("--reserve_prompt_tokens", type=int, default=16)
    ap.add_argument("--disable_token_budget", action="store_true")
    ap.add_argument("--expose_sources", action="store_true")
    ap.add_argument("--hrm_bin", default=None)
    ap.add_argument("--max_concurrent", type=int, default=64)
    ap.add_argument("--backend", choices=["b200_int8", "deepseek_int8", "echo"], default="b200_int8")
    ap.add_argument("--model_quant", choices=["q8"], default="q8")
    ap.add_argument("--tokenizer_model", default=None, help="HF tokenizer dir; default: the model dir, else bytes")
    ap.add_argument("--max_prompt_tokens", type=int, default=int(os.environ.get("DSI8_MAX_PROMPT_TOKENS", "2048")))
    ap.add_argument("--native_request_timeout_s", type=float, default=180.0)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--no_prefix_cache", dest="prefix_cache", action="store_false",
                    help="recompute every prompt (default: share the KV blocks of prompt prefixes seen before, such as "
                         "the system prompt)")
    ap.add_argument("--nccl_collectives", action="store_true",
                    help="TP lane: all-reduce and argmax through NCCL calls instead of the fused peer-memory kernels")
    return ap


def resolve_model(llm_model: str, out_dir: Path) -> Tuple[str, Optional[str]]:
    """-> (model source for EngineBackend, tokenizer source).  HF dirs are exported to DSI8 once (cached)."""
    if llm_model.startswith("synthetic:"):
        return llm_model, None
    p = Path(llm_model)
    if p.is_file():
        return str(p), None
    if p.is_dir() and (p / "config.json").is_file():
        from ..formats.dsi8 import export_dsi8
        dst = out_dir / (p.name.replace("/", "--") + "_q8.bin")
        if not dst.is_file():
            export_dsi8(p, dst)
        return str(dst), str(p)
    raise SystemExit(f"ERR: cannot resolve model {llm_model!r} (no network: use a local dir, a DSI8 file or "
                     f"synthetic:<preset>)")


def main(argv=None):
    args = build_arg_parser().parse_args(argv)
    hrm_model = Path(args.hrm_model).resolve()
    if not (hrm_model / "router_index.bin").is_file() or not (hrm_model / "index.sqlite").is_file():
        raise SystemExit(f"ERR: HRM model directory must contain router_index.bin and index.sqlite: {hrm_model}")
    if args.backend != "echo" and args.world > 1:
        # TP lane: one process per GPU; rank 0 hosts HTTP + scheduler, the other ranks mirror its engine calls
        from .daemon import LaneArgs, spawn_lane
        src, tok = resolve_model(args.llm_model, REPO_ROOT / "llm_models")
        lane = LaneArgs(src, args.world, args.max_seq_len, args.prefill_chunk_size, args.max_batch, "cuda",
                        master_port=int(os.environ.get("HRM_LANE_MASTER_PORT", str(29600 + args.port % 1000))),
                        fused_collectives=not args.nccl_collectives, prefix_cache=args.prefix_cache)
        spawn_lane(lane, _HttpEntry(args, str(hrm_model), args.tokenizer_model or tok))
        return
    if args.backend == "echo":
        from .backend import EchoBackend
        backend = EchoBackend()
    else:
        from .backend import EngineBackend
        src, tok = resolve_model(args.llm_model, REPO_ROOT / "llm_models")
        backend = EngineBackend(src, tokenizer_source=args.tokenizer_model or tok, device=args.device,
                                max_seq_len=args.max_seq_len, max_batch=args.max_batch,
                                prefill_chunk=args.prefill_chunk_size, max_prompt_tokens=args.max_prompt_tokens,
                                local_files_only=args.local_files_only, prefix_cache=args.prefix_cache)
    state = ServiceState(backend=backend, hrm_model=hrm_model,
                         hrm_bin=find_hrm_binary(repo_root=REPO_ROOT, explicit=args.hrm_bin),
                         max_seq_len=args.max_seq_len, max_new_tokens=args.max_new_tokens,
                         max_sources=args.max_sources, max_chars_per_source=args.max_chars_per_source,
                         reserve_prompt_tokens=args.reserve_prompt_tokens,
                         disable_token_budget=args.disable_token_budget, expose_sources=args.expose_sources,
                         max_concurrent=args.max_concurrent, request_timeout_s=args.native_request_timeout_s,
                         world=args.world, backend_name=args.backend)
    app = create_app(state)
    import uvicorn
    uvicorn.run(app, host=args.host, port=args.port, log_level="info")


class _HttpEntry:
    """Rank-0 body of a TP lane (picklable for mp.spawn): HTTP service over the mirrored engine."""

    def __init__(self, args, hrm_model: str, tokenizer_source):
        self.args, self.hrm_model, self.tok = args, hrm_model, tokenizer_source

    def __call__(self, engine):
        from .backend import EngineBackend
        a = self.args
        backend = EngineBackend("", tokenizer_source=self.tok, max_prompt_tokens=a.max_prompt_tokens,
                                local_files_only=a.local_files_only, engine=engine)
        state = ServiceState(backend=backend, hrm_model=Path(self.hrm_model),
                             hrm_bin=find_hrm_binary(repo_root=REPO_ROOT, explicit=a.hrm_bin),
                             max_seq_len=a.max_seq_len, max_new_tokens=a.max_new_tokens, max_sources=a.max_sources,
                             max_chars_per_source=a.max_chars_per_source,
                             reserve_prompt_tokens=a.reserve_prompt_tokens, disable_token_budget=a.disable_token_budget,
                             expose_sources=a.expose_sources, max_concurrent=a.max_concurrent,
                             request_timeout_s=a.native_request_timeout_s, world=a.world, backend_name=a.backend)
        import uvicorn
        try:
            uvicorn.run(create_app(state), host=a.host, port=a.port, log_level="info")
        finally:
            backend.stop()


if __name__ == "__main__":
    main()
