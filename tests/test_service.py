"""Service wrappers: systemd unit text, supervised health loop, lock, router smoke against the mock stack."""
import pytest

from hrm_flashrenderer_b200.launcher import service
from hrm_flashrenderer_b200.launcher.e2e import mock_stack


def test_systemd_unit_shape():
    u = service.systemd_unit("/opt/hrm", "/opt/hrm/idx", "llama3.1-70b")
    for line in ("Type=oneshot", "RemainAfterExit=yes", "WorkingDirectory=/opt/hrm", "TimeoutStartSec=900",
                 "TimeoutStopSec=30", "WantedBy=multi-user.target", "Environment=HRM_MODEL_DIR=/opt/hrm/idx"):
        assert line in u.splitlines()
    assert "launcher.topology start" in u and "launcher.topology stop" in u and "start-router" in u


def test_supervise_exits_after_consecutive_failures():
    seq = iter([True, True, False, True, False, False, False, True])
    logs = []
    rc = service.supervise(["u"], interval_s=0, fail_limit=3, health=lambda u: next(seq), sleep=lambda s: None,
                           log=logs.append)
    assert rc == 1
    assert sum("WARN" in l for l in logs) == 4          # the success in between reset the count


def test_supervise_healthy_runs_until_budget():
    assert service.supervise(["a", "b"], 0, 2, health=lambda u: True, sleep=lambda s: None, max_checks=5) == 0


def test_lock_single_holder(tmp_path):
    p = str(tmp_path / "lock")
    f = service.acquire_lock(p)
    with pytest.raises(service.LockHeld):
        service.acquire_lock(p)
    f.close()
    service.acquire_lock(p).close()


def test_smoke_router_mock_stack():
    url, servers = mock_stack()
    try:
        recs = service.smoke_router(url, max_new_tokens=16, log=lambda s: None)
    finally:
        for s in servers:
            s.close()
    assert [r["case"] for r in recs] == ["auto", "fast", "quality"]
    assert recs[1]["selected"] == "solo_3080" and recs[2]["selected"] == "solo_22gb"
