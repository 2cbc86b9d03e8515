"""Batched plane fit on the B200 (smg_plane_fit) vs the reference's apPlaneFit (GPU).

Inputs: the reference's own known-answer clouds (test_objprob.cpp:96-153) and the edge cases
of tests/plane_clouds.py, all fitted in ONE call (one CTA per set).  Expected outputs are the
reference's, stored in tests/golden/plane_fit.json.  The RANSAC hypotheses, inlier counts and
percentile selections are exact, so ok, inl, zmed, zlo and zhi must be identical; the PCA
sums are tree reductions on the device instead of the reference's sequential sums, so the
normal and horizontal span are compared within 1e-9 absolute and the thickness (a square root
of the smallest eigenvalue) within 1e-7.
"""
import json
import os

import numpy as np
import pytest

import plane_clouds
from conftest import has_gpu

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
ATOL_FP = 1e-9   # n, thick, hspan: re-associated double sums


def _golden():
    g = json.load(open(os.path.join(HERE, "golden", "plane_fit.json")))
    return {k: np.array([float.fromhex(v) for v in c["out"]]) for k, c in g["cases"].items()}


ATOL_THICK = 1e-7   # thick = sqrt(ev0): for exactly planar points ev0 ~ 1e-17 and the square root
                    # turns a 1e-16 difference of the covariance sums into ~1e-8


def _compare(name, o, g):
    assert o[0] == g[0], f"{name}: ok {o[0]} vs {g[0]}"
    exact = [5, 6, 7, 8]           # inl, zmed, zlo, zhi
    assert np.array_equal(o[exact], g[exact]), f"{name}: {o[exact]} vs {g[exact]}"
    fp = [1, 2, 3, 9]              # n0..n2, hspan
    assert np.allclose(o[fp], g[fp], rtol=0, atol=ATOL_FP), f"{name}: {o[fp]} vs {g[fp]}"
    assert abs(o[4] - g[4]) <= ATOL_THICK, f"{name}: thick {o[4]} vs {g[4]}"


def test_plane_fit_batch_matches_reference():
    if not has_gpu():
        pytest.skip("no GPU")
    from scenemap_b200 import smg
    gold = _golden()
    cases = plane_clouds.all_cases()
    # one call per distinct tau (the entry point takes one tau per call), all sets of that tau batched
    for tau in sorted({c[2] for c in cases}):
        sel = [c for c in cases if c[2] == tau]
        out = smg.plane_fit([c[1] for c in sel], tau, [c[3] for c in sel], 64)
        for (name, _, _, _), o in zip(sel, out):
            _compare(name, o, gold[name])


def test_plane_fit_kats_on_gpu():
    if not has_gpu():
        pytest.skip("no GPU")
    from scenemap_b200 import smg
    for name, xyz, tau, seed, check in plane_clouds.kat_cases():
        o = smg.plane_fit([xyz], tau, [seed], 64)[0]
        assert check(o), f"{name}: {o}"


def test_plane_fit_bad_arguments():
    if not has_gpu():
        pytest.skip("no GPU")
    from scenemap_b200 import smg
    with pytest.raises(smg.SmgError):
        smg.plane_fit([np.zeros((10, 3), np.float32)], 0.02, [1], 257)   # above the 256-hypothesis limit
