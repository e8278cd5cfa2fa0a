"""UDP telemetry packet: layout, projection similarity fields, and a real localhost round trip."""
import socket

import torch

from hrm_flashrenderer_b200.serving.telemetry import PACKET, Telemetry, unpack


def test_disabled_by_default():
    t = Telemetry(env={})
    assert not t.enabled
    t.send(1)   # no-op


def test_packet_layout_and_round_trip():
    assert PACKET.size == 180
    rx = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
    rx.bind(("127.0.0.1", 0))
    rx.settimeout(5)
    port = rx.getsockname()[1]
    t = Telemetry("tiny-model", hidden=8, env={"TELEM_ENABLE": "1", "TELEM_PORT": str(port)})
    v = torch.arange(8, dtype=torch.float32)
    t.send(1, 0.5, v, "hello prompt")
    a = unpack(rx.recv(1024))
    assert a["step"] == 1 and abs(a["loss"] - 0.5) < 1e-6 and a["model_id"] == "tiny-model"
    assert a["prompt"] == "hello prompt" and a["cos_sim"] == 1.0          # no previous projection
    t.send(2, 0.0, v, None)
    b = unpack(rx.recv(1024))
    assert b["prompt"] == "SYSTEM_IDLE" and abs(b["cos_sim"] - 1.0) < 1e-5 and b["euclid_dist"] < 1e-4
    t.send(3, 0.0, -v, "x" * 100)
    c = unpack(rx.recv(1024))
    assert abs(c["cos_sim"] + 1.0) < 1e-5 and len(c["prompt"]) == 63
