"""Layout of one rank's symmetric buffer (host-side): every region the fused kernels address is 256-byte aligned,
inside the buffer, and disjoint from every other region, for the tensor-parallel sizes and tile counts in use."""
import pytest

from hrm_flashrenderer_b200 import ops
from hrm_flashrenderer_b200.parallel.symm import ALIGN, FLAG_LINE, symm_layout


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("max_tiles,max_bn", [(64, 64), (40, 64), (1024, 64), (64, 16)])
def test_regions_aligned_disjoint_and_inside(world, max_tiles, max_bn):
    L = symm_layout(world, max_tiles, max_bn)
    regs = sorted(L["regions"].items(), key=lambda kv: kv[1][0])
    for name, (off, length) in regs:
        assert off % ALIGN == 0 and length > 0 and off + length <= L["bytes"], name
    for (n1, (o1, l1)), (n2, (o2, l2)) in zip(regs, regs[1:]):
        assert o1 + l1 <= o2, (n1, n2)
    # the scalars (launch epoch, CTA tickets, argmax epoch / row ticket at +0 / +128 / +256 / +384) fit their region
    assert 384 + 4 <= L["regions"]["scalars"][1]
    assert 1 <= L["argmax_rows"] <= ops.ARGMAX_XCHG_MAX_ROWS
    assert L["regions"]["tile_flags"][1] == world * max_tiles * FLAG_LINE
