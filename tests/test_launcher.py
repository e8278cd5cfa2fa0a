"""Hardware selection + topology planning with a fake nvidia-smi (no GPU)."""
import os

import pytest

from hrm_flashrenderer_b200.launcher import hw, topology as topo

FAKE = os.path.join(os.path.dirname(__file__), "fixtures", "fake_nvidia_smi.py")


def test_select_roundtrip_and_derive(tmp_path):
    p = hw.write_selection(hw.HWSelection(b200_count=8), tmp_path / "hw.env")
    sel = hw.load_selection(p)
    assert sel.b200_count == 8 and sel.model_quant == "q8"
    d = hw.derive(sel)
    assert d.lanes == {"solo_22gb": 8} and d.cuda_arch == "100a"
    d = hw.derive(hw.HWSelection(b200_count=8, lane_layout="4,2,2"))
    assert d.lanes == {"solo_22gb": 4, "nvlink_pair": 2, "solo_3080": 2} and d.topology_mode == "hetero_3lane"
    assert hw.derive(hw.HWSelection(b200_count=1)).lanes == {"solo_22gb": 1}
    with pytest.raises(hw.HWError):
        hw.write_selection(hw.HWSelection(b200_count=8, model_quant="q4"), tmp_path / "x.env")
    with pytest.raises(hw.HWError):
        hw.HWSelection(b200_count=4, lane_layout="4,2,2") and hw.validate(hw.HWSelection(b200_count=4, lane_layout="4,2,2"))
    (tmp_path / "bad.env").write_text("HW_POOL_VERSION=2\n")
    with pytest.raises(hw.HWError):
        hw.load_selection(tmp_path / "bad.env")


def _layout(monkeypatch, mem=None, link="NV18"):
    if mem:
        monkeypatch.setenv("FAKE_GPU_MEM", ",".join(map(str, mem)))
    monkeypatch.setenv("FAKE_LINK", link)
    return topo.detect_layout(FAKE)


def test_detect_and_plan_nvswitch(monkeypatch):
    lay = _layout(monkeypatch)
    assert lay.indices == list(range(8)) and lay.nvlink(0, 7) == 18
    plan = topo.plan_lanes(lay, hw.derive(hw.HWSelection(8, lane_layout="4,2,2")), env={})
    assert plan.lanes == {"solo_22gb": [0, 1, 2, 3], "nvlink_pair": [4, 5], "solo_3080": [6, 7]}
    assert set(plan.link.values()) == {"NVLINK"}


def test_manual_override_strict(monkeypatch):
    lay = _layout(monkeypatch)
    der = hw.derive(hw.HWSelection(8, lane_layout="4,2,2"))
    plan = topo.plan_lanes(lay, der, env={"LANE_GPUS_NVLINK_PAIR": "6,7"})
    assert plan.lanes["nvlink_pair"] == [6, 7] and plan.lanes["solo_3080"] == [4, 5]
    with pytest.raises(topo.TopologyError):
        topo.plan_lanes(lay, der, env={"LANE_GPUS_NVLINK_PAIR": "6,6"})
    plan = topo.plan_lanes(lay, der, env={"LANE_GPUS_NVLINK_PAIR": "6,6", "STRICT_GPU_TOPOLOGY": "0"})
    assert plan.warnings


def test_require_nvlink_and_pcie_fallback(monkeypatch):
    lay = _layout(monkeypatch, link="PIX")
    der = hw.derive(hw.HWSelection(8, lane_layout="4,2,2"))
    with pytest.raises(topo.TopologyError):
        topo.plan_lanes(lay, der, env={"REQUIRE_NVLINK": "1"})
    plan = topo.plan_lanes(lay, der, env={"REQUIRE_NVLINK": "1", "ALLOW_PCIE_PAIR_FALLBACK": "1"})
    assert plan.link["solo_22gb"] == "PCIE" and plan.warnings


def test_too_few_b200(monkeypatch):
    lay = _layout(monkeypatch, mem=[183359, 183359, 80000])
    with pytest.raises(topo.TopologyError):
        topo.plan_lanes(lay, hw.derive(hw.HWSelection(4)), env={})


def test_cli_detect(monkeypatch, tmp_path, capsys):
    hw.write_selection(hw.HWSelection(8, lane_layout="4,2,2"), tmp_path / "hw.env")
    monkeypatch.setenv("HW_SELECTION_FILE", str(tmp_path / "hw.env"))
    monkeypatch.setenv("FAKE_LINK", "NV18")
    assert topo.main(["detect", "--smi", FAKE]) == 0
    out = capsys.readouterr().out
    assert "LANE_SOLO_22GB_GPUS=0,1,2,3" in out and "LANE_SOLO_3080_LINK=NVLINK" in out
    assert topo.main(["start", "--smi", FAKE, "--hrm_model", "m", "--llm_model", "synthetic:tiny", "--dry_run"]) == 0
    assert "CUDA_VISIBLE_DEVICES=4,5" in capsys.readouterr().out


def test_lane_limits_and_command_env():
    from hrm_flashrenderer_b200.launcher.topology import lane_limits, lane_command
    assert lane_limits("nvlink_pair", {}) == (8192, 4096)
    env = {"MAX_SEQ_SOLO": "3000", "PREFILL_SOLO_3080": "256", "MAX_SEQ_NVLINK_PAIR": "5000"}
    assert lane_limits("solo_3080", env) == (3000, 256)
    assert lane_limits("solo_22gb", env) == (3000, 4096)
    assert lane_limits("nvlink_pair", env) == (5000, 4096)
    cmd = lane_command("solo_3080", 1, 8083, "idx", "m.bin", ["--x"], env=dict(env, HRM_FLASH_BIN="/opt/bin/hrm-flash -v"))
    assert cmd[:3] == ["/opt/bin/hrm-flash", "-v", "serve"]
    assert cmd[cmd.index("--max_seq_len") + 1] == "3000" and cmd[cmd.index("--prefill_chunk_size") + 1] == "256"
    assert cmd[-1] == "--x"
