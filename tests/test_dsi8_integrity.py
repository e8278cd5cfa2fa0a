"""Corrupt DSI8 files fail at open with a message that says what is wrong: truncation anywhere (header, a record
header, a payload), a missing tensor, a wrong shape or a wrong tensor type.  The failure is made on the host (a
corrupted weight file); nothing reaches a device."""
import struct

import torch

import pytest

from hrm_flashrenderer_b200.config import TINY
from hrm_flashrenderer_b200.formats.dsi8 import DSI8File, read_dsi8, write_dsi8
from hrm_flashrenderer_b200.models.weights import QTensor, synth_weights

CFG = TINY.with_layers(2)


@pytest.fixture(scope="module")
def good(tmp_path_factory):
    d = tmp_path_factory.mktemp("dsi8")
    return write_dsi8(d / "m.bin", CFG, synth_weights(CFG, seed=0))


def _records(path):
    with DSI8File(path) as f:
        return dict(f.records)


def test_good_file_passes(good):
    cfg, w = read_dsi8(good)
    assert cfg.layers == 2 and "model.layers.1.mlp.down_proj.weight" in w


@pytest.mark.parametrize("cut", ["header", "record_header", "payload", "last_byte"])
def test_truncation_is_reported(good, tmp_path, cut):
    raw = good.read_bytes()
    recs = _records(good)
    first_off = min(off for _, _, off in recs.values())
    n = {"header": 30, "record_header": 60 + 6, "payload": first_off + 100, "last_byte": len(raw) - 1}[cut]
    p = tmp_path / "t.bin"
    p.write_bytes(raw[:n])
    with pytest.raises(ValueError, match="truncated"):
        read_dsi8(p)


def test_missing_tensor_is_named(tmp_path):
    w = synth_weights(CFG, seed=0)
    del w["model.layers.1.self_attn.k_proj.weight"]
    del w["model.layers.0.post_attention_layernorm.weight"]
    p = write_dsi8(tmp_path / "m.bin", CFG, w)
    with pytest.raises(ValueError) as e:
        read_dsi8(p)
    msg = str(e.value)
    assert "2 missing" in msg and "layers.1.self_attn.k_proj.weight" in msg and "post_attention_layernorm" in msg


def test_header_and_tensor_shapes_disagree(tmp_path):
    """Tensors written for intermediate 704 under a header that says 688: the FFN matrices are named."""
    from dataclasses import replace
    big = replace(CFG, intermediate=704)
    p = write_dsi8(tmp_path / "m.bin", big, synth_weights(big, seed=0))
    raw = bytearray(p.read_bytes())
    assert struct.unpack_from("<I", raw, 24)[0] == 704      # header field F (intermediate size)
    struct.pack_into("<I", raw, 24, 688)
    p.write_bytes(bytes(raw))
    with pytest.raises(ValueError) as e:
        read_dsi8(p)
    msg = str(e.value)
    assert "mlp.up_proj.weight" in msg and "(688, 256)" in msg


def test_bad_magic_and_ndim(good, tmp_path):
    raw = bytearray(good.read_bytes())
    p = tmp_path / "m.bin"
    p.write_bytes(b"XXXX" + bytes(raw[4:]))
    with pytest.raises(ValueError, match="magic"):
        read_dsi8(p)
    nl = struct.unpack_from("<I", raw, 60)[0]
    struct.pack_into("<I", raw, 60 + 4 + nl + 4, 9)        # first record: 9 dimensions
    p.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="dimensions"):
        read_dsi8(p)


def test_engine_load_fails_cleanly(good, tmp_path):
    from hrm_flashrenderer_b200.models.llama import LlamaW8
    p = tmp_path / "short.bin"
    p.write_bytes(good.read_bytes()[:-1000])
    with pytest.raises(ValueError, match="truncated"):
        LlamaW8.from_dsi8(str(p), device="cpu", max_pos=64)


def test_views_share_the_mapping_and_outlive_close(good):
    f = DSI8File(good)
    name = "model.layers.0.mlp.gate_proj.weight"
    v = f.get(name)
    c = f.get(name, copy=True)
    assert f.get(name).q.data_ptr() == v.q.data_ptr() != c.q.data_ptr()   # views share the mapping
    assert torch.equal(v.q, c.q) and torch.equal(v.scale, c.scale)
    f.close()                                  # views keep the mapping alive
    assert torch.equal(v.q, c.q)
    c.q[0, 0] += 1                             # a copy is independent of the file's contents
    assert not torch.equal(v.q, c.q)


def test_misaligned_fp32_records_come_back_aligned(good):
    """Payloads follow names of any length, so fp32 data (row scales, norm vectors) can start at an offset that is
    not a multiple of 4 -- the architecture's own names already produce such offsets.  Those arrays come back as
    aligned copies with the right values; int8 matrices stay views."""
    ref = synth_weights(CFG, seed=0)
    with DSI8File(good) as f:
        offs = {k: f.records[k][2] for k in f.names()}
        assert any(o % 4 for o in offs.values()), "no misaligned payload in this file"
        for k in f.names():
            t = f.get(k)
            for arr in ((t.scale,) if isinstance(t, QTensor) else (t,)):
                assert arr.data_ptr() % 4 == 0, k
            if isinstance(t, QTensor):
                assert torch.equal(t.q, ref[k].q) and torch.equal(t.scale, ref[k].scale), k
            else:
                assert torch.equal(t, ref[k].float()), k
