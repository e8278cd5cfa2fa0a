"""Mock-stack e2e (reference: scripts/test_prod_live_e2e.sh): happy path, empty-sources fault injection,
failover when a lane is down."""
import pytest

from hrm_flashrenderer_b200.launcher.e2e import mock_stack, run_e2e, E2EFailure


def _run(**kw):
    url, servers = mock_stack(**kw)
    try:
        return run_e2e(url, runs=3, log=lambda *a: None)
    finally:
        for s in servers:
            s.close()


def test_e2e_mock_happy_path():
    rep = _run()
    assert set(rep["modes"]) == {"mixed", "retrieval", "deepseek_only"}


def test_e2e_mock_empty_sources_is_hard_failure():
    with pytest.raises(E2EFailure):
        _run(empty_sources=True)


def test_e2e_mock_lane_failover():
    rep = _run(fail_lanes=("solo_3080",))
    assert rep["modes"]["deepseek_only"]["runs"] == 3
