"""Lane service ``GET /metrics``: valid Prometheus text (checked with prometheus_client's parser), audit counters and
the engine metrics, None values left out, the fatal flag."""
import os
import sys
import urllib.request

from prometheus_client.parser import text_string_to_metric_families

from hrm_flashrenderer_b200.serving.backend import EchoBackend
from hrm_flashrenderer_b200.serving.serve import ServiceState, create_app, prometheus_text

sys.path.insert(0, os.path.dirname(__file__))
from _http import LiveServer, post  # noqa: E402


def _families(text):
    return {f.name: f for f in text_string_to_metric_families(text)}


def test_prometheus_text_from_engine_metrics():
    st = ServiceState(backend=EchoBackend())
    st.requests_total = 7
    st.mode_counts["mixed"] = 5
    eng = {"queue_depth": 2, "batch_size": 16, "completed": 40, "generated_tokens": 9000, "tok_per_s": 812.5,
           "ttft_p50_ms": 123.4, "ttft_p99_ms": None, "itl_p50_ms": 19.7, "last_error": None, "fatal": "boom"}
    fam = _families(prometheus_text(st, eng, running=False))
    val = lambda n, **lab: next(s.value for s in fam[n].samples if all(s.labels.get(k) == v for k, v in lab.items()))
    assert val("hrm_lane_up") == 0 and val("hrm_engine_fatal") == 1
    assert val("hrm_lane_requests") == 7 and val("hrm_lane_requests_by_mode", mode="mixed") == 5
    assert val("hrm_engine_batch_size") == 16 and val("hrm_engine_tokens_per_second") == 812.5
    assert val("hrm_engine_generated_tokens") == 9000 and val("hrm_engine_itl_p50_ms") == 19.7
    assert "hrm_engine_ttft_p99_ms" not in fam


def test_metrics_endpoint_over_http():
    st = ServiceState(backend=EchoBackend())
    with LiveServer(create_app(st)) as srv:
        post(srv.url + "/v1/generate", {"prompt": "hello", "mode": "deepseek_only", "max_new_tokens": 4})
        with urllib.request.urlopen(srv.url + "/metrics", timeout=10) as r:
            assert r.status == 200 and r.headers["Content-Type"].startswith("text/plain")
            fam = _families(r.read().decode())
    up = fam["hrm_lane_up"].samples[0].value
    req = fam["hrm_lane_requests"].samples[0].value
    by_mode = {s.labels["mode"]: s.value for s in fam["hrm_lane_requests_by_mode"].samples}
    assert up == 1 and req == 1 and by_mode["deepseek_only"] == 1


def test_router_metrics_count_failover_and_503():
    from hrm_flashrenderer_b200.serving import router as rt

    def fake_post(url, payload, timeout):
        if url.startswith("http://c"):
            raise RuntimeError("lane down")
        return {"ok": True, "text": "t", "mode": payload["mode"]}, 3

    st = rt.RouterState()
    st.backends = {"solo_22gb": rt.Backend("solo_22gb", "http://a:1"),
                   "nvlink_pair": rt.Backend("nvlink_pair", "http://b:2"),
                   "solo_3080": rt.Backend("solo_3080", "http://c:3")}
    st.post = fake_post
    with LiveServer(rt.create_app(st)) as srv:
        post(srv.url + "/v1/generate", {"prompt": "short", "max_new_tokens": 50})                  # fails over
        post(srv.url + "/v1/generate", {"prompt": "short", "max_new_tokens": 50, "allow_failover": False})  # 503
        with urllib.request.urlopen(srv.url + "/metrics", timeout=10) as r:
            fam = _families(r.read().decode())
    one = lambda n: fam[n].samples[0].value
    by_lane = lambda n: {s.labels["lane"]: s.value for s in fam[n].samples}
    assert one("hrm_router_requests") == 2 and one("hrm_router_failovers") == 1 and one("hrm_router_all_failed") == 1
    assert by_lane("hrm_router_routed")["nvlink_pair"] == 1 and by_lane("hrm_router_lane_errors")["solo_3080"] == 2
