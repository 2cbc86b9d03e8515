"""The re-encode restatement (oracle/reenc_oracle.py) pinned to the reference (CPU only).

The compiled reference runs the keyframe glue including ObjectMap::buildReencode
(scenemap src/objmap.cpp:1371-1458, called as capi.cpp:1002-1005 does); after every frame the
numpy restatement, given the reference's own objects and clouds, must produce the same
requests: ids in order, boxes, kappa, cameras and every mask bit.  The device kernel k_reenc
follows the same steps and is compared with the reference directly in the GPU parity tests.
"""
import numpy as np
import pytest


def _ref():
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built (make -C oracle)")
    return ref


@pytest.mark.parametrize("seed,frames", [(1234, 14), (9090, 12)])
def test_reenc_restatement_matches_reference(seed, frames):
    ref = _ref()
    from oracle import reenc_oracle
    from scenemap_b200 import synth
    g = synth.BoxRoom(seed=synth.map_seed(seed, 0), n_frames=frames, D=1152, bf16=True)
    R = ref.RefMap()
    n_req = 0
    for f in range(frames):
        fr = g.frame(f)
        R.frame(fr)
        objs = R.objects()
        clouds = [R.object_cloud(i)[0] for i in range(len(objs))]
        want = R.reenc()
        got = reenc_oracle.build_reencode(fr, objs, clouds)
        assert want["id"].tolist() == got["id"].tolist(), f"frame {f}"
        for k in ("box", "kappa", "cam", "bits"):
            assert np.array_equal(want[k], got[k]), f"frame {f}: {k}"
        n_req += len(want["id"])
    assert n_req > 0                                   # the run exercised the requests
    assert R.stats()["n_reenc_req"] == n_req           # ApStats counts what was handed out
