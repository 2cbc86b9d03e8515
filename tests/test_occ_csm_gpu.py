"""Config 3 on the B200: standalone OccGrid::insert and the correlative scan matcher (GPU).

Insert (smg_occ_insert) is compared with the reference's OccGrid::insert compiled in place
(oracle/_ref): the returned changed-cell count and every cell's log-odds, seen flag, export8
value and quantised probability must be identical.  The matcher (smg_occ_match/_track) is
compared with the C restatement (oracle/port/csm_port.c) run on the reference grid: the best
candidate index, its score and pose must be identical (integer sums; the same double
operations on both sides).  The matcher's parity to Cartographer itself is unpinned:
Cartographer is not part of the reference tree.
"""
import math

import numpy as np
import pytest

from conftest import has_gpu

pytestmark = pytest.mark.gpu
GRID = (1024, 1024, -100, -100)


def _need():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not (ref.available() and ref.port_available()):
        pytest.skip("oracle libraries not built")


def _compare_cells(dev: dict, refc: dict, q_unseen: int):
    W, H, X0, Y0 = GRID
    x0, y0 = refc["x0"] - X0, refc["y0"] - Y0
    h, w = refc["L"].shape
    assert x0 >= 0 and y0 >= 0 and x0 + w <= W and y0 + h <= H, "reference grid grew outside the device window"
    for k in ("L", "seen", "c8", "q"):
        d = dev[k][y0:y0 + h, x0:x0 + w]
        assert np.array_equal(d, refc[k]), f"{k}: {np.count_nonzero(d != refc[k])} cells differ"
    mask = np.ones((H, W), bool)
    mask[y0:y0 + h, x0:x0 + w] = False
    assert not dev["seen"][mask].any() and (dev["q"][mask] == q_unseen).all() and (dev["c8"][mask] == -1).all()


def test_insert_matches_reference():
    _need()
    from oracle import ref
    from scenemap_b200.floorplan import FloorPlan
    from scenemap_b200.occ import OccBatch
    fp = FloorPlan(seed=11, n_scans=80)
    G = OccBatch(1, GRID, max_points=4096)
    R = ref.RefOcc()
    rng = np.random.default_rng(5)
    for k in range(0, 80, 2):
        sc = fp.scan(k)
        pose = sc["pose"]
        extra = {}
        if k % 10 == 0:   # match points with normals go first and win their cells
            m = sc["hits"][::7] + rng.normal(0, 0.02, (len(sc["hits"][::7]), 2)).astype(np.float32)
            nrm = rng.normal(size=m.shape).astype(np.float32)
            extra = dict(match=m, normals=nrm)
        ch_d = G.insert([dict(hits=sc["hits"], free=sc["free"], **extra)], [pose])[0]
        ch_r = R.insert(sc["hits"], sc["free"], pose, match=extra.get("match"), normals=extra.get("normals"))
        assert ch_d == ch_r, f"scan {k}: changed {ch_d} vs {ch_r}"
    _compare_cells(G.cells(0), R.cells(), int(ref._lround(np.array([float(np.float32(0.1)) * 65535.0]))[0]))


def test_match_matches_restatement():
    _need()
    from oracle import ref
    from scenemap_b200.floorplan import FloorPlan
    from scenemap_b200.occ import OccBatch, config3_csm
    fp = FloorPlan(seed=12, n_scans=120)
    G = OccBatch(1, GRID, max_points=4096)
    R = ref.RefOcc()
    csm = config3_csm()
    for k in range(0, 40):          # build a map from true poses
        sc = fp.scan(k)
        G.insert([sc], [sc["pose"]])
        R.insert(sc["hits"], sc["free"], sc["pose"])
    cells = R.cells()
    for k in range(40, 120, 4):
        sc = fp.scan(k)
        po, idx, score = G.match([sc], [sc["pose0"]], csm)
        bi, bs, bp = ref.csm(cells, sc["hits"], sc["pose0"])
        assert idx[0] == bi and score[0] == bs and np.array_equal(po[0], bp), f"scan {k}: {idx[0]} {score[0]} vs {bi} {bs}"


def test_track_loop_matches_oracle_and_batches():
    _need()
    from oracle import ref
    from scenemap_b200.floorplan import FloorPlan
    from scenemap_b200.occ import OccBatch, config3_csm
    plans = [FloorPlan(seed=20 + i, n_scans=90) for i in range(3)]
    G = OccBatch(3, GRID, max_points=4096)
    Rs = [ref.RefOcc() for _ in plans]
    csm = config3_csm()
    for k in range(90):
        scans = [p.scan(k) for p in plans]
        if k == 30:
            scans[1] = dict(scans[1], hits=np.zeros((0, 2), np.float32))   # no returns: centre candidate
        po, idx, score, ch = G.track(scans, [s["pose0"] for s in scans], csm)
        for m, (s, R) in enumerate(zip(scans, Rs)):
            bi, bs, bp = ref.csm(R.cells(), s["hits"], s["pose0"])
            assert idx[m] == bi and score[m] == bs, f"map {m} scan {k}: {idx[m]} {score[m]} vs {bi} {bs}"
            assert np.array_equal(po[m], bp)
            assert ch[m] == R.insert(s["hits"], s["free"], bp), f"map {m} scan {k}: changed"
    q_unseen = int(ref._lround(np.array([float(np.float32(0.1)) * 65535.0]))[0])
    for m in range(3):
        _compare_cells(G.cells(m), Rs[m].cells(), q_unseen)


def test_scan_outside_window_is_rejected_and_leaves_grid():
    _need()
    from scenemap_b200.occ import OccBatch
    G = OccBatch(1, (64, 64, 0, 0), max_points=64)
    hits = np.array([[1.0, 0.5], [100.0, 0.0]], np.float32)   # second point far outside
    ch = G.insert([dict(hits=hits, free=np.zeros((0, 2), np.float32))], [[1.0, 1.0, 0.0]])
    assert ch[0] == -1
    assert not G.cells(0)["seen"].any()
    ch = G.insert([dict(hits=hits[:1], free=np.zeros((0, 2), np.float32))], [[1.0, 1.0, 0.0]])
    assert ch[0] > 0


def test_bad_matcher_parameters():
    _need()
    from scenemap_b200.occ import CsmParams, OccBatch
    from scenemap_b200.smg import SmgError
    G = OccBatch(1, GRID)
    sc = dict(hits=np.ones((4, 2), np.float32))
    with pytest.raises(SmgError):   # linear step must be the grid resolution
        G.match([sc], [[1, 1, 0]], CsmParams(0.3, 0.1, 0.04, 0.01, 10.0, 0.1))
    with pytest.raises(SmgError):   # too many offsets
        G.match([sc], [[1, 1, 0]], CsmParams(0.5, 0.1, 0.05, 0.01, 10.0, 0.1))
