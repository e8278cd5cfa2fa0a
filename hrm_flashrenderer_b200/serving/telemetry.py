"""UDP telemetry packets in the reference native engine's layout (``scripts/deepseek_native_engine.sh:248-258``,
sender ``:690-761``), for dashboards written against it.

Enabled by ``TELEM_ENABLE=1``; destination ``TELEM_TARGET`` (default 127.0.0.1) : ``TELEM_PORT`` (default 9999).
Packet (little-endian, 180 bytes): u32 step, f32 loss, f32 cos_sim, f32 euclid_dist, f32 proj_x / proj_y / proj_z,
f32 gpu_util[3], f32 gpu_mem[3] (percent), char model_id[64], char prompt[64] (NUL-padded, 63 bytes kept).
``proj`` is a fixed random 3 x D projection of a hidden-state vector; cos_sim / euclid_dist compare it with the
previous packet's projection (cos_sim 1 when either is zero).  GPU utilisation and memory come from NVML for the
first three visible GPUs when it is available, else zeros.  The send never blocks the caller on a slow receiver.
"""
from __future__ import annotations

import math
import os
import socket
import struct
from typing import Optional

PACKET = struct.Struct("<I6f3f3f64s64s")


def _cstr(s: str) -> bytes:
    return s.encode("utf-8", errors="replace")[:63]


class Telemetry:
    def __init__(self, model_id: str = "Unknown Model", hidden: int = 0, env=None, seed: int = 0):
        env = os.environ if env is None else env
        self.enabled = env.get("TELEM_ENABLE", "") == "1"
        self.addr = (env.get("TELEM_TARGET") or "127.0.0.1", int(env.get("TELEM_PORT") or 9999))
        self.model_id = model_id
        self.last = (0.0, 0.0, 0.0)
        self.sock = None
        self.proj = None
        self.nvml = []
        if not self.enabled:
            return
        self.sock = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
        self.sock.setblocking(False)
        if hidden:
            import torch
            g = torch.Generator().manual_seed(seed)
            self.proj = torch.rand(3, hidden, generator=g) * 2 - 1
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in range(min(3, pynvml.nvmlDeviceGetCount()))]
            self._pynvml = pynvml
        except Exception:
            self.nvml = []

    def _gpu(self):
        util, mem = [0.0] * 3, [0.0] * 3
        for i, h in enumerate(self.nvml):
            try:
                util[i] = float(self._pynvml.nvmlDeviceGetUtilizationRates(h).gpu)
                m = self._pynvml.nvmlDeviceGetMemoryInfo(h)
                mem[i] = float(m.used) / float(m.total) * 100.0
            except Exception:
                pass
        return util, mem

    def packet(self, step: int, loss: float = 0.0, hidden_vec=None, prompt: Optional[str] = None) -> bytes:
        p = (0.0, 0.0, 0.0)
        if hidden_vec is not None and self.proj is not None:
            v = hidden_vec.detach().float().reshape(-1).cpu()
            p = tuple(float(x) for x in (self.proj[:, : v.numel()] @ v))
        dx, dy, dz = (p[i] - self.last[i] for i in range(3))
        dist = math.sqrt(dx * dx + dy * dy + dz * dz)
        m1 = math.sqrt(sum(x * x for x in p))
        m2 = math.sqrt(sum(x * x for x in self.last))
        cos = sum(a * b for a, b in zip(p, self.last)) / (m1 * m2) if m1 > 1e-9 and m2 > 1e-9 else 1.0
        self.last = p
        util, mem = self._gpu()
        return PACKET.pack(int(step) & 0xFFFFFFFF, float(loss), cos, dist, *p, *util, *mem, _cstr(self.model_id),
                           _cstr(prompt if prompt is not None else "SYSTEM_IDLE"))

    def send(self, step: int, loss: float = 0.0, hidden_vec=None, prompt: Optional[str] = None) -> None:
        if not self.enabled:
            return
        try:
            self.sock.sendto(self.packet(step, loss, hidden_vec, prompt), self.addr)
        except (BlockingIOError, OSError):
            pass


def unpack(data: bytes) -> dict:
    f = PACKET.unpack(data)
    return {"step": f[0], "loss": f[1], "cos_sim": f[2], "euclid_dist": f[3], "proj": f[4:7], "gpu_util": f[7:10],
            "gpu_mem": f[10:13], "model_id": f[13].rstrip(b"\0").decode(), "prompt": f[14].rstrip(b"\0").decode()}
