"""Whole-object views: the answer side of the re-encode requests (GPU).

After every keyframe the caller encodes the requested whole-object crops and hands the
embeddings back (sm_set_object_embeddings -> ObjectMap::addWholeView, objmap.cpp:1361-1369).
Here the "encoder" is a deterministic stand-in: each requested object's fragment sum direction
plus seeded noise, renormalised (fp32).  Both sides get the same answers after every keyframe,
plus one answer for an object that was not requested and one repeated answer (both must follow
the reference: ignored / applied twice).  Every later keyframe is compared as in the default
parity test, deep comparisons include r_whole, k_whole and n_whole; the whole views then drive
association (apCosMax over r_whole), the whole-first view order, mu, and the merge fold.
"""
import numpy as np
import pytest

from conftest import has_gpu
from parity_util import compare_frame

pytestmark = pytest.mark.gpu


def _answers(R, f: int, D: int):
    rr = R.reenc()
    ids = [int(i) for i in rr["id"]]
    if not ids:
        return np.zeros(0, np.uint32), np.zeros((0, D), np.float32)
    objs = {o["id"]: i for i, o in enumerate(R.objects())}
    ids = ids + [ids[0]] + [987654]   # a repeated answer and one for an object never requested
    Z = np.zeros((len(ids), D), np.float32)
    for k, oid in enumerate(ids):
        rng = np.random.default_rng(1000003 * f + oid)
        base = R.object_vectors(objs[oid], D)[0].astype(np.float64) if oid in objs else rng.normal(size=D)
        v = base / max(np.linalg.norm(base), 1e-12) + 0.05 * rng.normal(size=D) / np.sqrt(D)
        Z[k] = (v / np.linalg.norm(v)).astype(np.float32)
    return np.asarray(ids, np.uint32), Z


def test_parity_whole_view_answers():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")
    from scenemap_b200 import smg, synth
    D, N = 1152, 45
    g = synth.BoxRoom(seed=synth.map_seed(808, 0), n_frames=N, D=D, bf16=True)
    R = ref.RefMap()
    B = smg.Batch(1, max_objects=256, emb_dim=D, max_det=32)
    n_done = 0
    for f in range(N):
        fr = g.frame(f)
        R.frame(fr)
        B.push([fr], smg.SMG_MEM_HOST, smg.SMG_EMB_BF16)
        errs = compare_frame(R, B, 0, D, deep=(f % 5 == 0 or f == N - 1))
        assert not errs, f"frame {f}: " + "\n".join(errs[:20])
        ids, Z = _answers(R, f, D)
        if len(ids):
            n_done += R.add_whole_views(ids, Z, fr["stamp"])
            B.set_object_embeddings(np.zeros(len(ids), np.int32), ids, Z)
    assert n_done > 20 and R.stats()["n_reenc_done"] == B.stats(0)["n_reenc_done"] > 20
    assert any(o["n_whole"] > 0 for o in R.objects())
    assert B.error_word() == 0
    B.close()
