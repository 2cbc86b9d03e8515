"""Correlative scan matching against the floor plan's ground truth.

No reference test or golden output fixes the matcher's results (the reference configures
Cartographer's real-time correlative matcher, which is not in the tree).  The floor-plan
generator knows the true pose of every scan, so the matcher is checked against that: a map is
built by inserting every even scan at its true pose, and every odd scan is matched from its
perturbed initial pose (errors up to 0.25 m and 8 degrees).  With the search's pose-prior
weights off (translation_weight = rotation_weight = 0: the pure correlative argmax), the best
candidate must lie within one linear step (0.05 m) and one angular step (0.5 degrees) of the
true pose on at least 95 % of the scans.  With the configured weights (10 and 0.1) the prior
pulls the estimate toward the initial pose by design, so those runs are compared with the
restatement instead (tests/test_occ_csm_gpu.py).

The CPU test holds the restatement (oracle/port/csm_port.c) to this; the GPU test holds the
device matcher (smg_occ_match) to it.
"""
import math

import numpy as np
import pytest

from conftest import has_gpu

N_SCANS = 120


def _within_one_step(pose, truth):
    d = np.abs(np.asarray(pose, np.float64) - truth)
    d[2] = abs((pose[2] - truth[2] + math.pi) % (2 * math.pi) - math.pi)
    return d[0] <= 0.05 + 1e-9 and d[1] <= 0.05 + 1e-9 and d[2] <= math.radians(0.5) + 1e-9


@pytest.mark.parametrize("seed", [7, 11])
def test_restated_matcher_recovers_true_poses(seed):
    from oracle import ref
    if not (ref.available() and ref.port_available()):
        pytest.skip("oracle libraries not built")
    from scenemap_b200.floorplan import FloorPlan
    P = FloorPlan(seed=seed, n_scans=N_SCANS)
    R = ref.RefOcc()
    ok = tot = 0
    for k in range(N_SCANS):
        s = P.scan(k)
        if k % 2 == 0:
            R.insert(s["hits"], s["free"], s["pose"])
            continue
        _, _, bp = ref.csm(R.cells(), s["hits"], s["pose0"], w_t=0.0, w_r=0.0)
        ok += _within_one_step(bp, s["pose"])
        tot += 1
    assert ok >= 0.95 * tot, f"{ok} of {tot} scans within one step of the true pose"


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [7, 11])
def test_device_matcher_recovers_true_poses(seed):
    if not has_gpu():
        pytest.skip("no GPU")
    from scenemap_b200.floorplan import FloorPlan
    from scenemap_b200.occ import OccBatch, config3_csm
    P = FloorPlan(seed=seed, n_scans=N_SCANS)
    G = OccBatch(1, (1024, 1024, -100, -100), max_points=4096)
    csm = config3_csm()
    csm.translation_weight = 0.0
    csm.rotation_weight = 0.0
    ok = tot = 0
    for k in range(N_SCANS):
        s = P.scan(k)
        if k % 2 == 0:
            G.insert([s], [s["pose"]])
            continue
        po, _, _ = G.match([s], [s["pose0"]], csm)
        ok += _within_one_step(po[0], s["pose"])
        tot += 1
    G.close()
    assert ok >= 0.95 * tot, f"{ok} of {tot} scans within one step of the true pose"
