"""Wall extraction from the map's own occupancy grid before every object update (GPU):
smg_set_walls vs the reference's sm_push_image glue (refreshWalls + the window bridges,
capi.cpp:646-698, 866-890) over walls.cpp, both on the same grid window.

Runs the structure room (walls, floor and ceiling come back as detections) with a text model,
so confirmed named objects give ignore footprints, and compares every keyframe as the default
parity test does (the wall-line rules and the see-through drop then act on the extracted
segments), plus the extracted segments themselves (bit for bit) and the wall state vector at the
base pose.  The tilted case turns the whole map frame by 20 degrees: the dominant-direction
measurement, the rotated extraction and its refit to the original grid.
"""
import math

import numpy as np
import pytest

from conftest import has_gpu
from parity_util import compare_frame
import variants

pytestmark = pytest.mark.gpu

GRID = (512, 512, -256 + 60, -256 + 50)


def _need():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")


def _turn(fr: dict, th: float) -> dict:
    """The frame with the map frame turned by th about the origin (camera pose and base pose)."""
    if th == 0.0:
        return fr
    c, s = math.cos(th), math.sin(th)
    Rz = np.array([[c, -s, 0.0], [s, c, 0.0], [0.0, 0.0, 1.0]])
    T = np.asarray(fr["T_mc"], np.float64).reshape(3, 4)
    T2 = np.concatenate([Rz @ T[:, :3], (Rz @ T[:, 3])[:, None]], axis=1)
    b = np.asarray(fr["base"], np.float64)
    out = dict(fr)
    out["T_mc"] = T2.reshape(-1)
    out["base"] = np.array([c * b[0] - s * b[1], s * b[0] + c * b[1], b[2] + th])
    eef = np.asarray(fr["eef"], np.float64).reshape(2, 3)
    out["eef"] = (Rz @ eef.T).T.copy()
    return out


def _run(th_deg: float, n_frames: int, seed_base: int, bridge: float = 0.0):
    from oracle import ref
    from scenemap_b200 import smg, synth
    D = 1152
    v = variants.structure(n_frames)
    v["gen"] = dict(v["gen"], seed_base=seed_base)
    g = variants.make_gen(v, D=D)
    t = synth.text_model(g)
    kv = v["kv"] + (f",ap_bridge_max={bridge}" if bridge else "")
    R = ref.RefMap(kv)
    R.set_text_model(t)
    R.set_walls(GRID)
    B = smg.Batch(1, max_objects=256, emb_dim=D, max_det=32, grid=GRID, params=smg.Params(kv))
    B.set_text_model(t)
    B.set_walls(True)
    th = math.radians(th_deg)
    n_seen = 0
    for f in range(n_frames):
        fr = _turn(g.frame(f), th)
        R.frame(fr)
        B.push([fr], smg.SMG_MEM_HOST, smg.SMG_EMB_F32)
        errs = compare_frame(R, B, 0, D, deep=(f % 10 == 0 or f == n_frames - 1))
        assert not errs, f"frame {f}: " + "\n".join(errs[:20])
        wr, wg = R.wall_segments(), B.wall_segments(0)
        assert (wr is None) == (wg is None), f"frame {f}: walls ref {wr is not None} gpu {wg is not None}"
        if wr is not None:
            assert wr.shape == wg.shape, f"frame {f}: {len(wr)} ref segments, {len(wg)} gpu"
            assert np.array_equal(wr, wg), f"frame {f}: segments differ by {np.abs(wr - wg).max()}"
            n_seen = max(n_seen, len(wr))
            pose = fr["base"]
            sr, sg = R.wall_state(pose), B.wall_state(0, pose)
            # rays exactly; the nearest segments as a set: std::partial_sort leaves the order of
            # segments at equal distance (two walls meeting at the nearest corner) unspecified,
            # the device takes them in segment order
            assert np.array_equal(sr[:16], sg[:16]), f"frame {f}: wall rays differ: {np.abs(sr[:16] - sg[:16]).max()}"
            a, b = sr[16:].reshape(8, 5), sg[16:].reshape(8, 5)
            assert np.array_equal(np.array(sorted(map(tuple, a))), np.array(sorted(map(tuple, b)))), \
                f"frame {f}: nearest wall segments differ"
    assert B.error_word() == 0
    st = R.stats()
    B.close()
    return st, n_seen


def test_walls_axis_aligned():
    _need()
    st, n_seen = _run(0.0, 50, 12)
    assert n_seen >= 4 and st["n_wall"] + st["n_through"] > 0


def test_walls_bridged():
    """ap_bridge_max > 0: gaps between collinear segments join the keyframe's list."""
    _need()
    st, n_seen = _run(0.0, 30, 13, bridge=1.5)
    assert n_seen >= 4


def test_walls_tilted_map():
    _need()
    st, n_seen = _run(20.0, 50, 12)
    assert n_seen >= 2
