"""The reference's wall extraction (walls.cpp, compiled into the oracle) on grids whose walls are
known: a rectangular room gives its four centre lines, ignore rectangles remove what they cover,
and a room drawn at 20 degrees gives that direction and segments along it (CPU)."""
import math

import numpy as np
import pytest


def _ref():
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")
    return ref


def _room(w=120, h=100, x0=10, y0=15, x1=90, y1=75, t=2):
    g = np.full((h, w), -1, np.int8)
    g[y0:y1, x0:x1] = 0
    g[y0:y0 + t, x0:x1] = 100
    g[y1 - t:y1, x0:x1] = 100
    g[y0:y1, x0:x0 + t] = 100
    g[y0:y1, x1 - t:x1] = 100
    return g


def test_rectangular_room_centre_lines():
    ref = _ref()
    res, ox, oy = 0.05, -1.0, -2.0
    segs = ref.wall_segments_grid(_room(), res, ox, oy, mode=0)
    assert len(segs) == 4
    horiz = sorted([s for s in segs if s[1] == s[3]], key=lambda s: s[1])
    vert = sorted([s for s in segs if s[0] == s[2]], key=lambda s: s[0])
    assert len(horiz) == 2 and len(vert) == 2
    # a 2-cell-thick wall's centre line lies on the boundary between its two cell rows
    assert abs(horiz[0][1] - (oy + 16 * res)) < 1e-9 and abs(horiz[1][1] - (oy + 74 * res)) < 1e-9
    assert abs(vert[0][0] - (ox + 11 * res)) < 1e-9 and abs(vert[1][0] - (ox + 89 * res)) < 1e-9
    assert ref.wall_segments_grid(_room(), res, ox, oy, mode=1) == 0.0   # axis-aligned


def test_ignore_rectangle_removes_a_wall():
    ref = _ref()
    res, ox, oy = 0.05, 0.0, 0.0
    # a rectangle over the whole bottom wall
    rect = [(0.0, 14 * res, 120 * res, 18 * res)]
    segs = ref.wall_segments_grid(_room(), res, ox, oy, rects=rect, mode=0)
    ys = [s[1] for s in segs if s[1] == s[3]]
    assert len(segs) == 3 and all(y > 20 * res for y in ys)


def test_tilted_room_direction_and_segments():
    ref = _ref()
    res, th = 0.05, math.radians(20.0)
    h, w = 160, 160
    g = np.full((h, w), 0, np.int8)
    c, s = math.cos(th), math.sin(th)
    # walls of a 5 x 4 m room turned by 20 degrees about the grid centre, 2 cells thick
    for y in range(h):
        for x in range(w):
            px, py = (x + 0.5 - w / 2) * res, (y + 0.5 - h / 2) * res
            u, v = c * px + s * py, -s * px + c * py
            if (abs(abs(u) - 2.5) < res and abs(v) < 2.0) or (abs(abs(v) - 2.0) < res and abs(u) < 2.5):
                g[y, x] = 100
    a = ref.wall_segments_grid(g, res, -w / 2 * res, -h / 2 * res, mode=1)
    assert abs(a - th) < math.radians(0.3)
    segs = ref.wall_segments_grid(g, res, -w / 2 * res, -h / 2 * res, mode=2, th=a)
    assert len(segs) >= 4
    for sg in segs:   # every segment runs along the room's direction or across it
        ang = math.atan2(sg[3] - sg[1], sg[2] - sg[0])
        d = (ang - th) % (math.pi / 2)
        assert min(d, math.pi / 2 - d) < math.radians(0.5)
