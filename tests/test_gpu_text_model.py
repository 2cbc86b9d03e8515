"""The text model inside the keyframe chain (GPU): ObjectMap with setTextModel / setClassKinds.

Both sides get the same synthetic text model (synth.text_model: rows near the rooms' own
embeddings; labels with the reference's kinds, shape groups, flat-object flags, hypernyms,
priors and size statistics).  With it the chain runs apObsStructural's label part (structure
probabilities feeding the wall rules), the association's structure guards and blocked pairs,
apAddView's label evidence, apRename after the update, after merges and after whole-view
answers (posterior, name, class = name, so isBig reads the class kinds), the merge pass's
guards and name-distribution overlap, and apStructObject's named-structure rules.

Every keyframe is compared as in the default parity test (objects include cls, so names that
differ show up at once); deep frames also compare every object's name state: the posterior
within 1e-5 (device exp / log round within an ulp of the host's), name, top label and roll-up
flag exactly.
"""
import numpy as np
import pytest

from conftest import has_gpu
from parity_util import compare_frame
import variants

pytestmark = pytest.mark.gpu


def _compare_names(R, B, m: int) -> list:
    errs = []
    n = len(R.objects())
    for i in range(n):
        a, b = R.object_name(i), B.object_name(m, i)
        if a["has_post"] != b["has_post"]:
            errs.append(f"object {i} has_post ref {a['has_post']} gpu {b['has_post']}")
            continue
        for k in ("name_lab", "top_lab", "rolled"):
            if a[k] != b[k]:
                errs.append(f"object {i} {k}: ref {a[k]} gpu {b[k]}")
        for k, tol in (("name_p", 1e-5), ("top_p", 1e-5), ("name_H", 1e-4)):
            if abs(a[k] - b[k]) > tol:
                errs.append(f"object {i} {k}: ref {a[k]} gpu {b[k]}")
        d = float(np.max(np.abs(a["post"] - b["post"]))) if len(a["post"]) else 0.0
        if d > 1e-5:
            errs.append(f"object {i} post differs by {d}")
    return errs


def _run(gen_kw: dict, kv: str, n_frames: int, bf16: bool = False, answers: bool = False, deep_every: int = 5):
    from oracle import ref
    from scenemap_b200 import smg, synth
    D = 1152
    kw = dict(gen_kw)
    seed = synth.map_seed(kw.pop("seed_base"), 0)
    g = synth.BoxRoom(seed=seed, n_frames=n_frames, D=D, bf16=bf16, **kw)
    t = synth.text_model(g)
    R = ref.RefMap(kv)
    R.set_text_model(t)
    B = smg.Batch(1, max_objects=256, emb_dim=D, max_det=32, params=smg.Params(kv))
    B.set_text_model(t)
    n_named = 0
    for f in range(n_frames):
        fr = g.frame(f)
        R.frame(fr)
        B.push([fr], smg.SMG_MEM_HOST, smg.SMG_EMB_BF16 if bf16 else smg.SMG_EMB_F32)
        deep = f % deep_every == 0 or f == n_frames - 1
        errs = compare_frame(R, B, 0, D, deep=deep)
        assert not errs, f"frame {f}: " + "\n".join(errs[:20])
        if deep:
            errs = _compare_names(R, B, 0)
            assert not errs, f"frame {f}: " + "\n".join(errs[:20])
        if answers:   # whole-view answers after every keyframe: L_whole and renames
            rr = R.reenc()
            ids = np.asarray([int(i) for i in rr["id"]], np.uint32)
            if len(ids):
                objs = {o["id"]: i for i, o in enumerate(R.objects())}
                Z = np.zeros((len(ids), D), np.float32)
                for k, oid in enumerate(ids):
                    rng = np.random.default_rng(7919 * f + int(oid))
                    v = R.object_vectors(objs[int(oid)], D)[0].astype(np.float64) + 0.05 * rng.normal(size=D) / np.sqrt(D)
                    Z[k] = (v / np.linalg.norm(v)).astype(np.float32)
                R.add_whole_views(ids, Z, fr["stamp"])
                B.set_object_embeddings(np.zeros(len(ids), np.int32), ids, Z)
    n_named = sum(R.object_name(i)["has_post"] for i in range(len(R.objects())))
    assert B.error_word() == 0
    B.close()
    return R, n_named


def _need():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")


def test_text_model_box_room():
    _need()
    R, n_named = _run(dict(seed_base=71), "", 40)
    assert n_named >= 10


def test_text_model_structure():
    """Walls, floor and ceiling as detections: structure probabilities, wall rules, guards."""
    _need()
    v = variants.structure(60)
    R, n_named = _run(v["gen"], v["kv"], v["n_frames"], deep_every=10)
    st = R.stats()
    assert st["n_obj_struct"] > 0 and n_named >= 10


def test_text_model_whole_views():
    """Whole-view answers every keyframe: whole-view label evidence and renames."""
    _need()
    R, n_named = _run(dict(seed_base=73), "", 35, bf16=True, answers=True)
    assert R.stats()["n_reenc_done"] > 10 and n_named >= 10


def test_text_model_hands():
    """Class kinds in isBig: what the gripper may hold, how absence counts."""
    _need()
    h = variants.hands(90)
    R, n_named = _run(h["gen"], h["kv"], h["n_frames"], deep_every=10)
    assert n_named >= 10
