"""The CPU restatement (oracle/port) pinned to the reference (CPU only).

1. The reference's own known-answer tests for apPlaneFit and apContact
   (src/scene_graph/scenemap/tests/test_objprob.cpp:96-163) hold on the restatement.
2. The restatement reproduces the reference's apPlaneFit outputs bit for bit on every KAT and
   edge-case cloud (golden outputs in tests/golden/plane_fit.json, written by
   tests/golden/make_golden.py from the reference compiled here).
3. Where the compiled reference (oracle/_ref/libscenemap_ref.so) is present, the primitives
   (apSeed, fp16 rounding, voxelKey, apContact, apPlaneFit) agree on seeded random inputs.
"""
import json
import os

import numpy as np
import pytest

import plane_clouds

HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    from oracle import ref
    if not ref.port_available():
        pytest.skip("oracle/_ref/libport.so not built (make -C oracle _ref/libport.so)")
    return ref


def _golden():
    g = json.load(open(os.path.join(HERE, "golden", "plane_fit.json")))
    return {k: np.array([float.fromhex(v) for v in c["out"]]) for k, c in g["cases"].items()}


def test_plane_fit_kats_on_port():
    ref = _port()
    for name, xyz, tau, seed, check in plane_clouds.kat_cases():
        o = ref.plane_fit(xyz, tau, seed, 64)
        assert check(o), f"{name}: {o}"
    # same seed, same answer (test_objprob.cpp:128-129)
    name, xyz, tau, seed, _ = plane_clouds.kat_cases()[2]
    assert np.array_equal(ref.plane_fit(xyz, tau, seed), ref.plane_fit(xyz, tau, seed))


def test_plane_fit_port_matches_reference_golden():
    ref = _port()
    gold = _golden()
    cases = plane_clouds.all_cases()
    assert len(cases) == len(gold)
    for name, xyz, tau, seed in cases:
        o = ref.plane_fit(xyz, tau, seed, 64)
        assert np.array_equal(o, gold[name]), f"{name}: {o} vs {gold[name]}"


def test_golden_properties():
    gold = _golden()
    assert gold["n7"][0] == 0 and gold["collinear"][0] == 0          # < 8 points, degenerate
    assert np.array_equal(gold["n7"], [0, 0, 0, 1, 1, 0, 0, 0, 0, 0])  # ApPlane defaults
    assert gold["plane_n20000"][0] == 1 and gold["n8"][0] == 1


def test_contact_kat_on_port():
    ref = _port()
    A = np.array([[0, 0, 0], [0.1, 0, 0]], np.float32)
    B = np.array([[0.03, 0, 0], [0.5, 0, 0]], np.float32)
    assert abs(ref.contact(A, B, 0.04) - 0.5) < 1e-9      # test_objprob.cpp:156-162
    assert ref.contact(A, B[:0], 0.04) == 0.0


def test_f16_edges_on_port():
    ref = _port()
    x = np.array([0.0, -0.0, 1.0, -2.5, 65504.0, 65520.0, 1e9, 6.1e-5, 5.96e-8, 2.98e-8, 1e-9, 0.1, 1.0 + 2**-11,
                  1.0 + 3 * 2**-12], np.float32)
    h = ref.to_f16(x)
    assert list(h[:5]) == [0x0000, 0x8000, 0x3C00, 0xC100, 0x7BFF]
    assert h[5] == 0x7C00 and h[6] == 0x7C00                  # overflow -> inf
    assert h[10] == 0                                          # flushed
    assert h[12] == 0x3C01                                     # half-way rounds up (reference rule)
    back = [ref.port_lib().op_h2f(int(v)) for v in h[:5]]
    assert back == [0.0, -0.0, 1.0, -2.5, 65504.0]


def test_primitives_port_vs_reference():
    ref = _port()
    if not ref.available():
        pytest.skip("compiled reference not present")
    rng = np.random.default_rng(7)
    for _ in range(200):
        a, b = (int(v) for v in rng.integers(0, 2**63, 2))
        assert ref.ap_seed(a, b) == ref.ap_seed(a, b, impl="ref")
    x = (rng.normal(size=20000) * rng.choice([1e-6, 1e-3, 1, 1e3, 7e4], 20000)).astype(np.float32)
    assert np.array_equal(ref.to_f16(x), ref.to_f16(x, impl="ref"))
    for _ in range(2000):
        p = rng.uniform(-50, 50, 3).astype(np.float32)
        assert ref.voxel_key(*p, 50.0) == ref.voxel_key(*p, 50.0, impl="ref")
    for _ in range(30):
        c = rng.uniform(-0.5, 0.5, (int(rng.integers(1, 400)), 3)).astype(np.float32)
        q = rng.uniform(-0.6, 0.6, (int(rng.integers(1, 200)), 3)).astype(np.float32)
        assert ref.contact(c, q, 0.04) == ref.contact(c, q, 0.04, impl="ref")
    for k in range(40):
        n = int(rng.integers(8, 2500))
        xyz = plane_clouds._plane_cloud(rng, n, float(rng.uniform(0.001, 0.05)), float(rng.uniform(0, 0.7)))
        tau, seed = float(rng.uniform(0.01, 0.06)), int(rng.integers(1, 2**62))
        assert np.array_equal(ref.plane_fit(xyz, tau, seed), ref.plane_fit(xyz, tau, seed, impl="ref")), k


def _csm_numpy(q, x0, y0, q_out, res, hits, pose0, lh, ah, step, wt, wr):
    """Direct statement of the matcher's definition (independent of oracle/port/csm_port.c)."""
    import math
    h, w = q.shape
    n = len(hits)
    best, bi = -1.0, -1
    rd = float(np.float32(res))
    for j in range(2 * ah + 1):
        th = pose0[2] + (j - ah) * step
        c, s = math.cos(th), math.sin(th)
        cells = [(math.floor((pose0[0] + c * float(px) - s * float(py)) / rd),
                  math.floor((pose0[1] + s * float(px) + c * float(py)) / rd)) for px, py in hits]
        for kx in range(-lh, lh + 1):
            for ky in range(-lh, lh + 1):
                tot = 0
                for ix, iy in cells:
                    X, Y = ix + kx - x0, iy + ky - y0
                    tot += int(q[Y, X]) if 0 <= X < w and 0 <= Y < h else q_out
                e = math.hypot(kx * rd, ky * rd) * wt + abs((j - ah) * step) * wr
                v = (tot / (n * 65535.0)) * math.exp(-(e * e))
                if v > best:
                    best, bi = v, (j * (2 * lh + 1) + kx + lh) * (2 * lh + 1) + ky + lh
    return bi, best


def test_csm_port_matches_definition():
    ref = _port()
    rng = np.random.default_rng(3)
    for trial in range(6):
        q = rng.integers(0, 65536, (40, 50)).astype(np.uint16)
        if trial == 0:
            q[:] = 6554                       # flat grid: every offset ties, the weights decide
        hits = rng.uniform(-0.8, 0.8, (int(rng.integers(1, 30)), 2)).astype(np.float32)
        pose0 = np.array([float(rng.uniform(0.8, 1.5)), float(rng.uniform(0.8, 1.2)), float(rng.uniform(-3, 3))])
        cells = {"q": q, "x0": -3, "y0": -2}
        bi, bs, bp = ref.csm(cells, hits, pose0, lin_half=2, ang_half=3, ang_step=0.02, w_t=10.0, w_r=0.1)
        want = _csm_numpy(q, -3, -2, 6554, 0.05, hits, pose0, 2, 3, 0.02, 10.0, 0.1)
        assert (bi, bs) == want, (trial, bi, bs, want)
        if trial == 0:
            assert bi == (3 * 5 + 2) * 5 + 2  # centre candidate
