"""Object-memory snapshot (GPU): smg_snapshot vs the reference's sm_snapshot object list
(capi.cpp:1051-1067) and dsg_save's per-object point files (dsg_save.cpp:70-89 plyBytes).

Four box rooms run with a text model (so objects get names and become exportable); after chosen
keyframes the batch's one-call snapshot of all maps must list, per map, the same exportable
objects in the same order with identical fields, and the PLY bytes (header + packed vertex
records) of every object must equal the reference's file byte for byte.
"""
import numpy as np
import pytest

from conftest import has_gpu

pytestmark = pytest.mark.gpu


def _need():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")


def test_snapshot_objects_and_ply():
    _need()
    from oracle import ref
    from scenemap_b200 import smg, synth
    D, M, n_frames = 1152, 4, 30
    gens = [synth.BoxRoom(seed=synth.map_seed(81, m), n_frames=n_frames, D=D, rgb=(m % 2 == 0)) for m in range(M)]
    B = smg.Batch(M, max_objects=128, emb_dim=D, max_det=32)
    t = synth.text_model(gens[0])   # one text model for the batch (and every reference map)
    B.set_text_model(t)
    refs = []
    for _ in gens:
        R = ref.RefMap("")
        R.set_text_model(t)
        refs.append(R)
    n_checked = 0
    for f in range(n_frames):
        frs = [g.frame(f) for g in gens]
        for R, fr in zip(refs, frs):
            R.frame(fr)
        B.push(frs, smg.SMG_MEM_HOST, smg.SMG_EMB_F32)
        if f % 7 != 6 and f != n_frames - 1:
            continue
        snap = B.snapshot()
        for m, R in enumerate(refs):
            ro = R.snapshot()
            a, b = int(snap["map_off"][m]), int(snap["map_off"][m + 1])
            go = snap["objects"][a:b]
            assert [o["id"] for o in ro] == [o["id"] for o in go], f"frame {f} map {m}: ids differ"
            for r, g in zip(ro, go):
                for k in r:
                    assert r[k] == g[k], f"frame {f} map {m} object {r['id']}: {k} ref {r[k]} gpu {g[k]}"
            for i in range(len(ro)):
                p0, p1 = int(snap["point_off"][a + i]), int(snap["point_off"][a + i + 1])
                ply = B.ply_header(p1 - p0) + snap["points"][15 * p0:15 * p1]
                assert ply == R.snapshot_ply(i), f"frame {f} map {m} object {i}: PLY bytes differ"
            n_checked += len(ro)
    assert n_checked >= 20
    assert B.error_word() == 0
    B.close()
