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


def test_whole_view_answer_semantics():
    """The answer side (sm_set_object_embeddings -> ObjectMap::addWholeView, objmap.cpp:1361-1369,
    apAddView with whole = true, objprob.cpp:312-356) as the reference applies it: each answered
    object gains one whole view with its request's kappa (tempered at most), stops needing a
    whole view, and from then on is asked again only behind the objects that still need one."""
    ref = _ref()
    from scenemap_b200 import synth
    g = synth.BoxRoom(seed=synth.map_seed(1234, 0), n_frames=16, D=1152, bf16=True)
    R = ref.RefMap()
    rng = np.random.default_rng(7)
    answered = {}
    for f in range(16):
        fr = g.frame(f)
        R.frame(fr)
        req = R.reenc()
        if len(req["id"]) == 0:
            continue
        need_first = [int(i) not in answered for i in req["id"]]
        # objects that still need a whole view come first (priority 1e6 + kappa)
        assert need_first == sorted(need_first, reverse=True), f"frame {f}"
        if f % 3 == 0:
            emb = rng.standard_normal((len(req["id"]), 1152)).astype(np.float32)
            emb /= np.linalg.norm(emb, axis=1, keepdims=True)
            before = R.stats()["n_reenc_done"]
            kw0 = {o["id"]: o["k_whole"] for o in R.objects()}
            assert R.add_whole_views(req["id"], emb, fr["stamp"]) == len(req["id"])
            assert R.stats()["n_reenc_done"] == before + len(req["id"])
            objs = {o["id"]: o for o in R.objects()}
            for i, k in zip(req["id"].tolist(), req["kappa"].tolist()):
                o = objs[i]
                assert o["need_whole"] == 0
                assert o["n_whole"] == answered.get(i, 0) + 1
                answered[i] = o["n_whole"]
                dk = o["k_whole"] - kw0[i]   # the request's kappa, or tempered (x 0.3) from a similar view
                assert any(abs(dk - k * t) <= 1e-9 * max(1.0, k) for t in (1.0, 0.3)), (i, dk, k)
    assert answered, "no request was answered"
    assert R.add_whole_views([0xFFFFFFF], np.ones((1, 1152), np.float32), 0.0) == 0   # no such request
