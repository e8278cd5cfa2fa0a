"""Prompt modes, the lane service and the router (CPU; echo backend, real HRM core for retrieval)."""
import json
import os
import subprocess
import sys

import pytest

from hrm_flashrenderer_b200.serving import prompt_builder as pb
from hrm_flashrenderer_b200.serving.backend import EchoBackend, ByteTokenizer
from hrm_flashrenderer_b200.serving.serve import ServiceState, create_app, build_prompt
from hrm_flashrenderer_b200.serving import router as rt

sys.path.insert(0, os.path.dirname(__file__))
from _http import LiveServer, post, get  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HRM = os.path.join(ROOT, "hrm_core", "build", "hrm")


# ---------------------------------------------------------------------------------------------- prompt modes
def test_mode_aliases_and_default():
    assert pb.normalize_mode(None) == "mixed"
    for a, m in [("silent", "mixed"), ("default", "mixed"), ("deepseek", "deepseek_only"), ("full", "deepseek_only"),
                 ("llm_only", "deepseek_only"), (" Retrieval ", "retrieval")]:
        assert pb.normalize_mode(a) == m
    with pytest.raises(ValueError):
        pb.normalize_mode("nonsense")


def test_templates():
    srcs = [pb.Source("0001#s0002", "alpha"), pb.Source("0003#s0004", "beta")]
    mixed = pb.build_prompt_for_mode("Q?", srcs, "mixed")
    assert mixed.startswith("[SYSTEM]\n" + pb.MIXED_SYSTEM_PROMPT + "\n\n[BACKGROUND_KNOWLEDGE]\n<kb_01> alpha\n<kb_02> beta")
    assert mixed.endswith("[USER]\nQ?\n\n[ASSISTANT]\n")
    assert "0001#s0002" not in mixed                       # ids hidden in mixed mode
    ret = pb.build_prompt_for_mode("Q?", srcs, "retrieval")
    assert "[SOURCES]\n[0001#s0002] alpha\n[0003#s0004] beta" in ret
    assert pb.build_prompt_for_mode("Q?", srcs, "deepseek_only") == "Q?"
    assert pb.SILENT_SYSTEM_PROMPT == pb.MIXED_SYSTEM_PROMPT
    assert "Never mention \"sources\"" in pb.MIXED_SYSTEM_PROMPT


def test_build_sources_caps():
    raw = {"chosen": [{"sid": f"s{i}", "txt": "x" * 1300} for i in range(20)] + [{"sid": "", "txt": "y"}]}
    s = pb.build_sources(raw)
    assert len(s) == 16 and s[0].txt.endswith(" …") and len(s[0].txt) == 1202


def test_token_budget_fit():
    tok = ByteTokenizer()
    srcs = [pb.Source(f"s{i}", "w" * 200) for i in range(5)]
    q, s = pb.fit_prompt_to_token_budget("question?", srcs, tok, 900, mode="mixed")
    assert len(tok(pb.build_prompt_for_mode(q, s, "mixed"), add_special_tokens=False)["input_ids"]) <= 900
    assert 1 <= len(s) < 5
    q2, s2 = pb.fit_prompt_to_token_budget("question?", srcs, tok, 5, mode="mixed")
    assert (q2, s2) == ("", [])


# ---------------------------------------------------------------------------------------------- lane service
@pytest.fixture(scope="module")
def hrm_model(tmp_path_factory):
    subprocess.run(["make", "-C", os.path.join(ROOT, "hrm_core"), "-j4", "all"], check=True, capture_output=True)
    d = tmp_path_factory.mktemp("kb")
    lines = ["The silver bridge is guarded by the night watch.", "Merchants promised the king bread and wine.",
             "Winter makes the tower dark and cold.", "The river stone shines under the golden light."] * 3
    (d / "kb.txt").write_text("\n".join(lines) + "\n")
    subprocess.run([HRM, "prep", "--input", str(d / "kb.txt"), "--out", str(d / "p.jsonl"), "--cluster-size", "4"],
                   check=True, capture_output=True)
    subprocess.run([HRM, "build", "--payloads", str(d / "p.jsonl"), "--outdir", str(d / "m")], check=True,
                   capture_output=True)
    return d / "m"


def _state(hrm_model, backend=None, **kw):
    return ServiceState(backend=backend or EchoBackend(), hrm_model=hrm_model, max_seq_len=4096, max_new_tokens=64,
                        max_concurrent=4, **kw)


def test_deepseek_only_never_calls_hrm(hrm_model, monkeypatch):
    import hrm_flashrenderer_b200.serving.serve as serve
    monkeypatch.setattr(serve, "run_hrm_query", lambda **k: (_ for _ in ()).throw(AssertionError("HRM called")))
    st = _state(hrm_model)
    text, srcs, mode, active = build_prompt(st, "who guards the bridge", "deepseek")
    assert (text, srcs, mode, active) == ("who guards the bridge", [], "deepseek_only", False)
    assert st.hrm_query_calls_total == 0


def test_generate_modes_over_http(hrm_model):
    be = EchoBackend()
    st = _state(hrm_model, be)
    with LiveServer(create_app(st)) as srv:
        code, body = post(srv.url + "/v1/generate", {"prompt": "who guards the silver bridge", "mode": "retrieval"})
        r = json.loads(body)
        assert code == 200 and r["ok"] and r["mode"] == "retrieval" and r["hrm_active"] is True
        assert r["source_count"] > 0 and "sources" in r and r["audit"]["prompt_template"] == "retrieval_explicit"
        assert "[SOURCES]" in be.calls[-1]["prompt"]
        code, body = post(srv.url + "/v1/generate", {"prompt": "who guards the silver bridge"})
        r = json.loads(body)
        assert r["mode"] == "mixed" and "sources" not in r and r["audit"]["prompt_template"] == "mixed_silent"
        assert "<kb_01>" in be.calls[-1]["prompt"] and "#s" not in be.calls[-1]["prompt"]
        code, body = post(srv.url + "/v1/generate", {"prompt": "hello", "mode": "deepseek_only", "show_sources": True})
        r = json.loads(body)
        assert r["hrm_active"] is False and r["source_count"] == 0 and "sources" not in r
        assert be.calls[-1]["prompt"] == "hello"
        code, body = post(srv.url + "/v1/generate", {"prompt": "zzqx", "mode": "mixed"})
        r = json.loads(body)
        if r["source_count"] == 0:
            assert r["text"] == "I don't know."
        code, _ = post(srv.url + "/v1/generate", {"prompt": "x", "mode": "bogus"})
        assert code == 400
        code, h = get(srv.url + "/v1/health")
        assert h["ok"] and h["audit"]["requests_total"] >= 4
        assert h["audit"]["mode_counts"]["retrieval"] == 1 and h["audit"]["hrm_query_calls_by_mode"]["deepseek_only"] == 0


def test_deterministic_repeat(hrm_model):
    st = _state(hrm_model)
    with LiveServer(create_app(st)) as srv:
        outs = [post(srv.url + "/v1/generate", {"prompt": "what did the merchants promise", "mode": "mixed"})[1]
                for _ in range(3)]
    assert len(set(outs)) == 1


def test_missing_tokenizer_means_no_prompt(hrm_model):
    be = EchoBackend()
    be.tokenizer = None
    st = _state(hrm_model, be)
    text, srcs, mode, active = build_prompt(st, "who guards the silver bridge", "mixed")
    assert text == "" and srcs == [] and active is True


def test_sampling_fields_reach_the_backend(hrm_model):
    """``temperature`` / ``top_k`` / ``seed`` on /v1/generate become the backend's sampling parameters; absent or
    zero temperature keeps the greedy call unchanged; bad values are a 400."""
    from hrm_flashrenderer_b200.runtime.sampling import SamplingParams
    be = EchoBackend()
    st = _state(hrm_model, be)
    with LiveServer(create_app(st)) as srv:
        code, _ = post(srv.url + "/v1/generate", {"prompt": "hi", "mode": "deepseek_only", "temperature": 0.7,
                                                  "top_k": 40, "seed": 5})
        assert code == 200 and be.calls[-1]["sampling"] == SamplingParams(0.7, 40, 5)
        code, _ = post(srv.url + "/v1/generate", {"prompt": "hi", "mode": "deepseek_only", "temperature": 0})
        assert code == 200 and be.calls[-1]["sampling"] is None
        for bad in ({"temperature": -1}, {"temperature": 1, "top_k": -3}, {"temperature": 1, "top_k": 5000}):
            code, _ = post(srv.url + "/v1/generate", dict({"prompt": "hi", "mode": "deepseek_only"}, **bad))
            assert code == 400, bad


# ---------------------------------------------------------------------------------------------- router
def _stream_from(post_fn):
    """A lane's streaming answer built from a fake non-streaming one: two deltas, then the payload."""
    def post_stream(url, payload, timeout):
        body, _ = post_fn(url, dict(payload, stream=False), timeout)
        text = str(body.get("text", ""))
        yield {"delta": text[:1]}
        yield {"delta": text[1:]}
        yield body
    return post_stream


def _router(post_fn, endpoints=None):
    st = rt.RouterState()
    endpoints = endpoints or {"solo_22gb": "http://a", "nvlink_pair": "http://b", "solo_3080": "http://c"}
    st.backends = {n: rt.Backend(n, u) for n, u in endpoints.items()}
    st.post = post_fn
    st.post_stream = _stream_from(post_fn) if post_fn is not None else None
    st.get = lambda url, t: ({"ok": not url.startswith("http://c")}, 1)
    st.keepalive_s = 0.05
    return st


def test_router_primary_selection():
    st = _router(None)
    assert rt.primary_backend(st, 100, 100, None, None) == "solo_3080"
    assert rt.primary_backend(st, 1000, 300, None, None) == "nvlink_pair"
    assert rt.primary_backend(st, 5000, 100, None, None) == "solo_22gb"
    assert rt.primary_backend(st, 100, 100, "quality", None) == "solo_22gb"
    assert rt.primary_backend(st, 100, 100, "quality", "fast") == "solo_3080"
    collapsed = _router(None, {"solo_22gb": "http://a", "nvlink_pair": "http://a", "solo_3080": "http://c"})
    assert rt.primary_backend(collapsed, 10, 10, None, None) == "nvlink_pair"
    assert rt.candidate_order(collapsed, "nvlink_pair", True) == ["nvlink_pair", "solo_22gb"]
    assert rt.candidate_order(st, "solo_3080", True) == ["solo_3080", "nvlink_pair", "solo_22gb"]
    assert rt.resolve_show_sources(True, "deepseek_only") is False
    assert rt.resolve_show_sources(None, "retrieval") is True


def test_router_failover_and_503():
    calls = []

    def fake_post(url, payload, timeout):
        calls.append((url, payload))
        if url.startswith("http://c"):
            raise RuntimeError("lane down")
        return {"ok": True, "text": "t", "mode": payload["mode"]}, 3

    st = _router(fake_post)
    with LiveServer(rt.create_app(st)) as srv:
        code, body = post(srv.url + "/v1/generate", {"prompt": "short", "max_new_tokens": 50})
        r = json.loads(body)
        assert code == 200 and r["route"]["primary"] == "solo_3080" and r["route"]["selected"] == "nvlink_pair"
        assert r["route"]["attempted"] == ["solo_3080", "nvlink_pair"] and r["route"]["backend_max_new_tokens"] == 50
        code, body = post(srv.url + "/v1/generate", {"prompt": "short", "max_new_tokens": 50, "allow_failover": False})
        assert code == 503 and json.loads(body)["detail"]["error"] == "all backends failed"
        code, h = get(srv.url + "/v1/health")
        assert h["ok"] and h["backends"]["solo_3080"]["ok"] is False
        code, m = get(srv.url + "/v1/models")
        assert m["object"] == "list"
        code, body = post(srv.url + "/v1/chat/completions",
                          {"messages": [{"role": "system", "content": "s"}, {"role": "user", "content": "hi"}]})
        r = json.loads(body)
        assert r["object"] == "chat.completion" and r["choices"][0]["message"]["content"] == "t"
        assert calls[-1][1]["mode"] == "deepseek_only" and calls[-1][1]["prompt"] == "hi"
        code, body = post(srv.url + "/v1/completions", {"prompt": "x", "stream": True})
        assert code == 200 and body.rstrip().endswith("data: [DONE]") and '"text_completion"' in body
        assert "temperature" not in calls[-1][1]                    # greedy requests keep the lane body unchanged
        post(srv.url + "/v1/chat/completions", {"messages": [{"role": "user", "content": "hi"}], "temperature": 0.5,
                                                "top_k": 8, "seed": 3})
        assert (calls[-1][1]["temperature"], calls[-1][1]["top_k"], calls[-1][1]["seed"]) == (0.5, 8, 3)


def test_lane_call_errors_and_success():
    """The router's lane transport: JSON object answers pass, error statuses keep the lane's explanation, and a
    non-object body or an unreachable lane is a LaneCallError."""
    import http.server
    import threading
    from hrm_flashrenderer_b200.serving import router as RT

    class H(http.server.BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def _send(self, code, body):
            self.send_response(code)
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

        def do_GET(self):
            self._send(200, b"[1, 2]" if self.path == "/list" else b'{"ok": true}')

        def do_POST(self):
            n = int(self.headers.get("Content-Length", "0"))
            got = json.loads(self.rfile.read(n))
            if self.path == "/fail":
                self._send(503, b"lane busy")
            else:
                self._send(200, json.dumps({"echo": got}).encode())

    srv = http.server.ThreadingHTTPServer(("127.0.0.1", 0), H)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    base = f"http://127.0.0.1:{srv.server_address[1]}"
    try:
        obj, ms = RT.http_json_post(base + "/gen", {"a": 1}, 5.0)
        assert obj == {"echo": {"a": 1}} and ms >= 0
        assert RT.http_json_get(base + "/h", 5.0)[0] == {"ok": True}
        with pytest.raises(RT.LaneCallError) as ei:
            RT.http_json_post(base + "/fail", {}, 5.0)
        assert ei.value.status == 503 and "lane busy" in str(ei.value)
        with pytest.raises(RT.LaneCallError, match="expected an object"):
            RT.http_json_get(base + "/list", 5.0)
    finally:
        srv.shutdown()
    with pytest.raises(RT.LaneCallError, match="no answer") as ei:
        RT.http_json_get(base + "/h", 1.0)
    assert ei.value.status is None


def test_cli_generate_greedy_and_sampled_on_cpu(capsys):
    """``hrm-flash generate`` end to end on the CPU engine (synthetic tiny model, deepseek_only): the greedy answer
    repeats, a seeded sampled answer repeats, and an invalid sampling flag is refused."""
    from hrm_flashrenderer_b200.serving import cli
    base = ["generate", "--hrm_model", "unused", "--llm_model", "synthetic:tiny", "--prompt", "hello there",
            "--mode", "deepseek_only", "--device", "cpu", "--max_new_tokens", "6", "--max_seq_len", "128"]
    outs = []
    for extra in ([], [], ["--temperature", "0.9", "--sample_top_k", "20", "--seed", "5"],
                  ["--temperature", "0.9", "--sample_top_k", "20", "--seed", "5"]):
        assert cli.main(base + extra) == 0
        outs.append(capsys.readouterr().out)
    assert outs[0] == outs[1] and outs[2] == outs[3]
    with pytest.raises(SystemExit):
        cli.main(base + ["--temperature", "-1"])


def _sse_events(url, payload):
    import urllib.request
    req = urllib.request.Request(url, data=json.dumps(payload).encode(), headers={"Content-Type": "application/json"})
    out = []
    with urllib.request.urlopen(req, timeout=120) as r:
        for line in r:
            line = line.decode().strip()
            if line.startswith("data: "):
                out.append(line[6:])
    return out


def test_lane_streams_deltas_then_the_payload(hrm_model):
    """``stream: true`` on /v1/generate: server-sent text deltas that concatenate to the text of the same request
    without streaming, then the full payload, then [DONE]."""
    be = EchoBackend()
    st = _state(hrm_model, be)
    with LiveServer(create_app(st)) as srv:
        body = {"prompt": "who guards the silver bridge", "mode": "retrieval"}
        code, plain = post(srv.url + "/v1/generate", body)
        plain = json.loads(plain)
        ev = _sse_events(srv.url + "/v1/generate", dict(body, stream=True))
    assert ev[-1] == "[DONE]"
    final = json.loads(ev[-2])
    deltas = [json.loads(e)["delta"] for e in ev[:-2]]
    assert len(deltas) > 1 and "".join(deltas) == final["text"] == plain["text"]
    assert final == plain


def test_engine_backend_stream_matches_generate_on_cpu():
    from hrm_flashrenderer_b200.runtime.sampling import SamplingParams
    from hrm_flashrenderer_b200.serving.backend import EngineBackend
    be = EngineBackend("synthetic:tiny", device="cpu", max_seq_len=128, max_batch=2)
    try:
        for sp in (None, SamplingParams(0.9, 30, 4)):
            full = be.generate("hello there", 10, sampling=sp)
            parts = list(be.generate_stream("hello there", 10, sampling=sp))
            assert "".join(parts) == full and len(parts) >= 2
        it = be.generate_stream("stop early", 100)
        next(it)
        it.close()                                   # the consumer went away: the request is cancelled
        import time
        t0 = time.time()
        while be.metrics()["cancelled"] < 1 and time.time() - t0 < 30:
            time.sleep(0.01)
        assert be.metrics()["cancelled"] == 1
    finally:
        be.stop()


def test_router_relays_lane_stream_with_failover_before_first_delta(hrm_model):
    """OpenAI streaming through the router over real HTTP: the primary lane is down, the next lane (a live lane
    service) streams its deltas, which arrive as chat chunks that concatenate to the lane's non-streamed text."""
    lane_state = _state(hrm_model, EchoBackend())
    with LiveServer(create_app(lane_state)) as lane:
        st = rt.RouterState()
        st.backends = {"solo_3080": rt.Backend("solo_3080", "http://127.0.0.1:9"),      # nothing listens there
                       "nvlink_pair": rt.Backend("nvlink_pair", lane.url),
                       "solo_22gb": rt.Backend("solo_22gb", "http://127.0.0.1:7")}
        st.keepalive_s = 0.05
        with LiveServer(rt.create_app(st)) as router:
            ev = _sse_events(router.url + "/v1/chat/completions",
                             {"messages": [{"role": "user", "content": "hello lane"}], "stream": True,
                              "max_tokens": 50})                      # short request: the primary is solo_3080
            code, plain = post(lane.url + "/v1/generate", {"prompt": "hello lane", "mode": "deepseek_only",
                                                           "max_new_tokens": 50})
    assert ev[-1] == "[DONE]"
    chunks = [json.loads(e) for e in ev[:-1]]
    assert chunks[0]["choices"][0]["delta"] == {"role": "assistant"}
    content = "".join(c["choices"][0]["delta"].get("content", "") for c in chunks)
    assert content == json.loads(plain)["text"]
    assert sum(1 for c in chunks if c["choices"][0]["delta"].get("content")) > 1      # really streamed in pieces
    assert chunks[-1]["choices"][0]["finish_reason"] == "stop" and chunks[-1]["usage"]["completion_tokens"] > 0
    assert st.failovers_total == 1 and st.lane_errors["solo_3080"] == 1


def test_lane_stream_client_disconnect_cancels_the_request(hrm_model):
    """A streaming client that closes its connection after the first delta: the lane's engine request is cancelled
    (KV blocks and the batch slot given back) instead of generating to the end."""
    import http.client
    import time
    from hrm_flashrenderer_b200.serving.backend import EngineBackend
    be = EngineBackend("synthetic:tiny", device="cpu", max_seq_len=512, max_batch=2)
    step = be.engine.decode_step

    def slow_step(g):                                  # 400 steps take seconds: time to notice the disconnect
        time.sleep(0.01)
        return step(g)
    be.engine.decode_step = slow_step
    st = _state(hrm_model, be)
    try:
        with LiveServer(create_app(st)) as srv:
            conn = http.client.HTTPConnection("127.0.0.1", srv.port, timeout=60)
            conn.request("POST", "/v1/generate", body=json.dumps({"prompt": "tell me", "mode": "deepseek_only",
                                                                  "max_new_tokens": 400, "stream": True}),
                         headers={"Content-Type": "application/json"})
            resp = conn.getresponse()
            while True:
                line = resp.fp.readline().decode()
                if line.startswith("data: ") and "delta" in line:
                    break
            conn.close()
            t0 = time.time()
            while be.metrics()["cancelled"] < 1 and time.time() - t0 < 60:
                time.sleep(0.05)
            m = be.metrics()
            assert m["cancelled"] == 1 and m["batch_size"] == 0, m
            assert m["generated_tokens"] < 400
    finally:
        be.stop()


def test_stop_strings_cut_the_answer(hrm_model):
    """``stop`` on /v1/generate (and forwarded by the router): the answer ends before the first stop string, in the
    plain and the streamed form, and the engine request stops there."""
    from hrm_flashrenderer_b200.serving.backend import EngineBackend, cut_at_stop
    assert "".join(cut_at_stop(iter(["hel", "lo wo", "rld"]), ["o w"])) == "hell"
    assert "".join(cut_at_stop(iter(["xSTO", "Py"]), ["STOP", "Py"])) == "x"
    be = EchoBackend()
    st = _state(hrm_model, be)
    with LiveServer(create_app(st)) as srv:
        full = json.loads(post(srv.url + "/v1/generate", {"prompt": "hi", "mode": "deepseek_only"})[1])["text"]
        stop = full[5:7]
        cut = json.loads(post(srv.url + "/v1/generate", {"prompt": "hi", "mode": "deepseek_only",
                                                         "stop": stop})[1])["text"]
        assert cut == full[:full.find(stop)]
        ev = _sse_events(srv.url + "/v1/generate", {"prompt": "hi", "mode": "deepseek_only", "stop": [stop],
                                                    "stream": True})
        assert json.loads(ev[-2])["text"] == cut
    eng = EngineBackend("synthetic:tiny", device="cpu", max_seq_len=256, max_batch=2)
    try:
        full = eng.generate("hello", 40)
        stop = full[6:8]
        assert eng.generate("hello", 40, stop=[stop]) == full[:full.find(stop)]
        import time
        t0 = time.time()
        while eng.metrics()["cancelled"] < 1 and time.time() - t0 < 30:
            time.sleep(0.01)
        assert eng.metrics()["cancelled"] == 1              # generation stopped at the stop string
    finally:
        eng.stop()


def test_router_generate_stream_passes_lane_events_with_route(hrm_model):
    """``stream: true`` on the router's /v1/generate: the lane's deltas pass through and the final event is the
    lane's payload plus the router's route record."""
    lane_state = _state(hrm_model, EchoBackend())
    with LiveServer(create_app(lane_state)) as lane:
        st = rt.RouterState()
        st.backends = {"solo_3080": rt.Backend("solo_3080", lane.url),
                       "nvlink_pair": rt.Backend("nvlink_pair", "http://127.0.0.1:9"),
                       "solo_22gb": rt.Backend("solo_22gb", "http://127.0.0.1:7")}
        st.keepalive_s = 0.05
        with LiveServer(rt.create_app(st)) as router:
            body = {"prompt": "who guards the silver bridge", "mode": "retrieval", "max_new_tokens": 50}
            ev = _sse_events(router.url + "/v1/generate", dict(body, stream=True))
            plain = json.loads(post(router.url + "/v1/generate", body)[1])
    assert ev[-1] == "[DONE]"
    final = json.loads(ev[-2])
    deltas = [json.loads(e)["delta"] for e in ev[:-2]]
    assert "".join(deltas) == final["text"] == plain["text"]
    assert final["route"]["selected"] == "solo_3080" and final["sources"] == plain["sources"]


def test_openai_n_choices():
    """``n`` choices: one lane request per choice with seeds seed, seed + 1, ... when sampling; greedy requests are
    answered once and repeated; streaming accepts n = 1 only."""
    calls = []

    def fake_post(url, payload, timeout):
        calls.append(payload)
        return {"ok": True, "text": f"t{payload.get('seed', 'g')}", "mode": payload["mode"]}, 1

    st = _router(fake_post)
    with LiveServer(rt.create_app(st)) as srv:
        code, body = post(srv.url + "/v1/chat/completions", {"messages": [{"role": "user", "content": "hi"}],
                                                             "n": 3, "temperature": 0.7, "seed": 10})
        r = json.loads(body)
        assert code == 200 and [c["message"]["content"] for c in r["choices"]] == ["t10", "t11", "t12"]
        assert [c["index"] for c in r["choices"]] == [0, 1, 2]
        calls.clear()
        code, body = post(srv.url + "/v1/completions", {"prompt": "hi", "n": 2})
        r = json.loads(body)
        assert [c["text"] for c in r["choices"]] == ["tg", "tg"] and len(calls) == 1
        code, _ = post(srv.url + "/v1/completions", {"prompt": "hi", "n": 2, "stream": True})
        assert code == 400


def test_router_stream_error_after_first_delta_is_not_retried():
    """Once a lane has streamed a delta, a later failure ends the stream with an error event (no second lane, so
    the client never sees two answers)."""
    tried = []

    def post_stream(url, payload, timeout):
        tried.append(url)
        yield {"delta": "par"}
        raise rt.LaneCallError(url, "stream broken")

    st = _router(lambda u, p, t: ({"ok": True, "text": "x", "mode": p["mode"]}, 1))
    st.post_stream = post_stream
    with LiveServer(rt.create_app(st)) as srv:
        ev = _sse_events(srv.url + "/v1/chat/completions", {"messages": [{"role": "user", "content": "hi"}],
                                                            "stream": True, "max_tokens": 50})
    assert ev[-1] == "[DONE]" and "error" in json.loads(ev[-2]) and len(tried) == 1
    assert "".join(json.loads(e)["choices"][0]["delta"].get("content", "") for e in ev[:-2]) == "par"
