"""Geometry pins restated from the reference's tests/test_shrimp_geometry.py."""

from __future__ import annotations

import random

from hexo_bot_b200 import constants as K
from hexo_bot_b200 import geometry as G


def test_pack_roundtrip_and_order():
    rng = random.Random(7)
    coords = [(rng.randint(-300, 300), rng.randint(-300, 300)) for _ in range(500)]
    for q, r in coords:
        assert G.unpack_action_id(G.pack_action_id(q, r)) == (q, r)
    assert sorted(coords, key=lambda c: G.pack_action_id(*c)) == sorted(coords)


def test_hex_dist_forms():
    rng = random.Random(13)
    for _ in range(2000):
        dq, dr = rng.randint(-30, 30), rng.randint(-30, 30)
        assert G.hex_dist(dq, dr) == (abs(dq) + abs(dr) + abs(dq + dr)) // 2


def test_direction_algebra():
    d = K.DIRECTIONS
    for i in range(6):
        assert G.rot60(*d[i]) == d[(i + 1) % 6]
        assert G.reflect(*d[i]) == d[5 - i]


def test_d6_group():
    rng = random.Random(17)
    for sym in range(12):
        inv = G.d6_inverse(sym)
        for _ in range(50):
            q, r = rng.randint(-50, 50), rng.randint(-50, 50)
            tq, tr = G.apply_d6(sym, q, r)
            assert G.apply_d6(inv, tq, tr) == (q, r)
            assert G.hex_dist(tq, tr) == G.hex_dist(q, r)
            assert G.on_win_axis(tq, tr) == G.on_win_axis(q, r)


def test_exact_rows_bijection():
    offs = G.disk_offsets(K.BIAS_DISK_RADIUS)
    assert len(offs) == 217 and offs == sorted(offs)
    assert sorted(G.rel_bias_index(*o) for o in offs) == list(range(217))


def test_ring_and_far_rows():
    for d in range(9, 17):
        assert G.rel_bias_index(d, 0) == K.BIAS_ON_AXIS_BASE + d - 9
        assert G.rel_bias_index(0, d) == K.BIAS_ON_AXIS_BASE + d - 9
        assert G.rel_bias_index(d, -d) == K.BIAS_ON_AXIS_BASE + d - 9
        assert G.rel_bias_index(d, -1) == K.BIAS_OFF_AXIS_BASE + d - 9
    assert G.rel_bias_index(17, 0) == K.BIAS_FAR_ROW
    assert G.rel_bias_index(40, -11) == K.BIAS_FAR_ROW


def test_lut_clamps_to_far_row():
    lut = G.cell_bias_lut()
    m, w = K.LUT_M, K.LUT_W
    assert lut.shape == (w * w,)
    assert lut[(0 + m) * w + (0 + m)] == G.rel_bias_index(0, 0)
    assert lut[(m + m) * w + (0 + m)] == K.BIAS_FAR_ROW
    assert int(lut.max()) == K.BIAS_FAR_ROW
