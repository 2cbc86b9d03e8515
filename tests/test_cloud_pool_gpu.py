"""Object clouds in a per-map pool smaller than the object slots (smg_create_pooled, GPU).

A map reserves object slots (scalars and vectors) and, separately, cloud slots (a full-capacity
cloud, its voxel index and contact cells each).  With a pool large enough for the live
objects the results must equal those of a batch with one cloud per object slot, field for
field; with a pool too small the map must say so in its error word, not drop objects silently.
"""
import numpy as np
import pytest

from conftest import has_gpu

pytestmark = pytest.mark.gpu


def _need():
    if not has_gpu():
        pytest.skip("no GPU")


def test_pooled_clouds_match_one_cloud_per_slot():
    _need()
    from scenemap_b200 import smg, synth
    D, N, M = 1152, 30, 3
    gens = [synth.BoxRoom(seed=synth.map_seed(3131, i), n_frames=N, D=D, bf16=True) for i in range(M)]
    A = smg.Batch(M, max_objects=256, emb_dim=D, max_det=32)
    P = smg.Batch(M, max_objects=256, emb_dim=D, max_det=32, max_clouds=96)
    for f in range(N):
        frs = [g.frame(f) for g in gens]
        A.push(frs, smg.SMG_MEM_HOST, smg.SMG_EMB_BF16)
        P.push(frs, smg.SMG_MEM_HOST, smg.SMG_EMB_BF16)
        for m in range(M):
            oa, op = A.objects(m), P.objects(m)
            assert oa == op, f"map {m} frame {f}"
            if f % 10 == 9:
                for i in range(len(oa)):
                    ca, cp = A.object_cloud(m, i), P.object_cloud(m, i)
                    assert np.array_equal(ca[0], cp[0]) and np.array_equal(ca[1], cp[1])
            ra, rp = A.reencode(m), P.reencode(m)
            assert np.array_equal(ra["id"], rp["id"]) and np.array_equal(ra["bits"], rp["bits"])
    assert A.error_word() == 0 and P.error_word() == 0
    A.close()
    P.close()


def test_exhausted_cloud_pool_is_reported():
    _need()
    from scenemap_b200 import smg, synth
    D = 1152
    g = synth.BoxRoom(seed=synth.map_seed(3132, 0), n_frames=12, D=D, bf16=True)
    P = smg.Batch(1, max_objects=256, emb_dim=D, max_det=32, max_clouds=4)
    for f in range(12):
        P.push([g.frame(f)], smg.SMG_MEM_HOST, smg.SMG_EMB_BF16)
    assert P.error_word() & 1, "capacity bit of the error word"
    assert len(P.objects(0)) <= 4
    P.close()
