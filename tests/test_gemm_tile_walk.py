"""Host-side check of the GEMM's output-tile walk (``TileWalk`` in ``csrc/gemm_w8a16.h``, inlined by the kernel's
producer and epilogue): for both tile numberings the incremental walk over any unit range equals the direct decode
of every unit, stays in range, and the whole unit space visits every (n_tile, m_tile, kt) exactly once."""
import pytest

from hrm_flashrenderer_b200 import ops

pytestmark = pytest.mark.skipif(not ops.has_ext(), reason="extension not built")


def _decode(u, n_tiles, m_tiles, k_tiles, m_fastest):
    tile, kt = divmod(u, k_tiles)
    if m_fastest:
        n, m = divmod(tile, m_tiles)
    else:
        m, n = divmod(tile, n_tiles)
    return n, m, kt


def _walk(n_tiles, m_tiles, k_tiles, u0, u1, m_fastest):
    f = ops.ext().gemm_tile_walk(n_tiles, m_tiles, k_tiles, u0, u1, m_fastest)
    return [tuple(f[i:i + 3]) for i in range(0, len(f), 3)]


@pytest.mark.parametrize("m_fastest", [False, True])
@pytest.mark.parametrize("n_tiles,m_tiles,k_tiles", [(1, 1, 1), (3, 1, 7), (1, 5, 4), (8, 3, 2), (448, 64, 32),
                                                     (7, 13, 1)])
def test_walk_matches_direct_decode(n_tiles, m_tiles, k_tiles, m_fastest):
    total = n_tiles * m_tiles * k_tiles
    full = _walk(n_tiles, m_tiles, k_tiles, 0, total, m_fastest)
    assert len(full) == total
    assert len(set(full)) == total
    assert all(0 <= n < n_tiles and 0 <= m < m_tiles and 0 <= kt < k_tiles for n, m, kt in full)
    step = max(1, total // 37)
    for u0 in range(0, total, step):     # ranges that start inside a tile, as stream-K segments do
        u1 = min(total, u0 + step + 3)
        got = _walk(n_tiles, m_tiles, k_tiles, u0, u1, m_fastest)
        assert got == [_decode(u, n_tiles, m_tiles, k_tiles, m_fastest) for u in range(u0, u1)]


def test_m_fastest_keeps_one_weight_tile_per_run():
    """m-fastest: consecutive tiles share the weight tile (n_tile) for all m_tiles token blocks."""
    walk = _walk(4, 6, 2, 0, 4 * 6 * 2, True)
    ns = [n for n, _, _ in walk]
    assert ns == sorted(ns)
    walk = _walk(4, 6, 2, 0, 4 * 6 * 2, False)
    ms = [m for _, m, _ in walk]
    assert ms == sorted(ms)


def test_walk_rejects_bad_ranges():
    with pytest.raises(ValueError):
        ops.ext().gemm_tile_walk(2, 2, 2, 0, 9, False)
    with pytest.raises(ValueError):
        ops.ext().gemm_tile_walk(0, 2, 2, 0, 0, False)


def test_toggle_round_trip():
    C = ops.ext()
    was = C.gemm_m_fastest()
    try:
        C.set_gemm_m_fastest(True)
        assert C.gemm_m_fastest()
        C.set_gemm_m_fastest(False)
        assert not C.gemm_m_fastest()
    finally:
        C.set_gemm_m_fastest(was)


@pytest.mark.parametrize("tiles,k_tiles,ctas", [(8, 4, 148), (10, 32, 148), (64, 4, 148), (3, 1, 148),
                                                (1, 200, 148), (40, 5, 148), (16, 16, 148), (5, 7, 16)])
def test_stream_k_segments_cover_every_tile_once(tiles, k_tiles, ctas):
    """The segment count / index of every tile (``tile_segments`` in ``csrc/gemm_w8a16.h``, used by the multi-phase
    chain, which runs every phase on all SMs even when a phase has fewer units than CTAs): the CTAs holding part of a
    tile number their segments 0..nseg-1 exactly once, so the last ticket is always taken and re-armed."""
    f = ops.ext().stream_k_segments(tiles, k_tiles, ctas)
    segs = [tuple(f[i:i + 4]) for i in range(0, len(f), 4)]
    by_tile = {}
    for c, t, nseg, idx in segs:
        by_tile.setdefault(t, []).append((nseg, idx, c))
    assert sorted(by_tile) == list(range(tiles))
    for t, lst in by_tile.items():
        nsegs = {n for n, _, _ in lst}
        assert len(nsegs) == 1, (t, lst)
        n = nsegs.pop()
        assert sorted(i for _, i, _ in lst) == list(range(n)), (t, lst)
        assert [i for _, i, _ in sorted(lst, key=lambda x: x[2])] == list(range(n))   # k order follows CTA order
