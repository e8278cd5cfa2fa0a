"""Failure detection on the GPU without a fault: a bounded wait runs out and the kernel reports it.

The fused tensor-parallel GEMM is given a two-rank peer table whose second "rank" is just another buffer on this GPU
that no kernel ever signals.  Its wait for that rank's per-tile epoch flags must give up after the 2 s limit (every
tile-owning CTA waits in parallel), record the error
code in the status word (read on the host by ``ops.check_status``), and leave the context usable: a normal GEMM
launched afterwards still gives correct results.
"""
import time

import pytest
import torch

from hrm_flashrenderer_b200 import ops

pytestmark = pytest.mark.gpu

K_ERR_TIMEOUT_PEER = 5


class _SilentPeerWorkspace:
    """Same fields as ``SymmetricWorkspace`` for world = 2, both buffers local; rank 1 never runs."""

    def __init__(self, dev, max_tiles=64, max_bn=64):
        C = ops.ext()
        tile_bytes = max_bn * 128 * 4
        al = lambda x: (x + 255) // 256 * 256
        self.rank, self.world, self.max_tiles, self.max_bn = 0, 2, max_tiles, max_bn
        self.off_partials = 0
        self.off_final = al(2 * 2 * max_tiles * tile_bytes)
        self.off_flags = al(self.off_final + max_tiles * tile_bytes)
        self.off_tile_flags = al(self.off_flags + 2 * max_tiles * 4)
        self.off_scalars = al(self.off_tile_flags + 2 * max_tiles * 128)
        size = al(self.off_scalars + 4096)
        self.off_ll = size                     # epoch-tagged words of the flag-free variant
        size = al(size + 2 * 2 * max_tiles * max_bn * 128 * 8)
        with torch.cuda.device(dev):
            self.ptrs = [C.symm_alloc(size)[0], C.symm_alloc(size)[0]]
        self.peers = torch.tensor(self.ptrs, dtype=torch.int64, device=dev)
        self.epoch_ptr = self.ptrs[0] + self.off_scalars
        self.ticket = C.tensor_from_ptr(self.ptrs[0] + self.off_scalars + 128, [2], torch.int32, dev.index or 0)

    def close(self):
        for p in self.ptrs:
            ops.ext().symm_free(p)


def test_peer_wait_times_out_and_context_survives():
    dev = torch.device("cuda", 0)
    N, K, M = 1024, 512, 4
    w = ops.tile_w8(torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev))
    s = torch.rand(N, device=dev) * 1e-3
    x = torch.randn(M, K, device=dev).half()
    resid = torch.zeros(M, N, device=dev)
    xg = torch.empty(M, N, dtype=torch.float16, device=dev)
    ssq = torch.empty(N // 128, M, device=dev)
    ws = _SilentPeerWorkspace(dev)
    ops.check_status(dev)                      # clean status word before
    t0 = time.time()
    ops.w8a16_residual_ar_(x, w, s, resid, ws, torch.ones(N, device=dev), xg, ssq)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert 1.5 < dt < 30.0, dt                 # gave up after the bounded wait, did not hang
    with pytest.raises(RuntimeError, match=f"code {K_ERR_TIMEOUT_PEER}"):
        ops.check_status(dev)
    ops.check_status(dev)                      # the check re-armed the status word
    y = ops.w8a16_linear(x, w, s, out_dtype=torch.float32)
    ref = x.float() @ (ops.untile_w8(w, N).float() * s[:, None]).t()
    assert (y - ref).abs().max().item() < 1e-2
    ws.close()
