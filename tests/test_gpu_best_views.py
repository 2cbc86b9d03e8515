"""Best views and cloud-point colours (GPU): the RGB side of the reference's keyframe glue.

With an RGBA image per frame, the reference glue (scenemap src/capi.cpp:903-998) colours the
observation cloud points from the image (gatherRgbHost) and keeps one best view per object:
moved / put-down events reset a view's quality, views of objects that are gone are dropped,
a detection attached to an object replaces its view when valid mask area x score is >= the
view's quality, and the crop is the detection box + 10 % (cropGeometry), area-averaged RGB
(cropRgbHost), nearest millimetre depth (cropDepthMm) and the detection mask (cropMask).

The oracle driver runs that glue around the reference's own bestview.cpp functions and keeps
its views map.  The device returns the views each keyframe replaced (smg_get_views); the test
keeps them the way a caller would (drop the views of objects that are gone, then install the
keyframe's views in order) and compares that map with the reference's after every keyframe:
ids, versions, qualities, boxes, metadata and every image byte.  Cloud colours are compared
point for point on every object.
"""
import numpy as np
import pytest

from conftest import has_gpu
from parity_util import compare_frame
import variants

pytestmark = pytest.mark.gpu

META = ("version", "q", "stamp", "box", "det_box", "mask_area", "depth_m", "score", "cam_T", "w", "h")


def _mirror_update(mirror: dict, B, m: int) -> None:
    live = {o["id"] for o in B.objects(m)}
    for oid in [i for i in mirror if i not in live]:
        del mirror[oid]
    for v in B.views(m):
        mirror[v["id"]] = v


def _compare_views(ref_views: dict, mirror: dict) -> list:
    errs = []
    if sorted(ref_views) != sorted(mirror):
        return [f"view ids: ref {sorted(ref_views)} gpu {sorted(mirror)}"]
    for oid, r in ref_views.items():
        g = mirror[oid]
        for k in META:
            if r[k] != g[k]:
                errs.append(f"view {oid} {k}: ref {r[k]} gpu {g[k]}")
        for k in ("rgb", "depth", "mask"):
            if r[k].shape != g[k].shape or not np.array_equal(r[k], g[k]):
                bad = int(np.sum(r[k] != g[k])) if r[k].shape == g[k].shape else -1
                errs.append(f"view {oid} {k}: {bad} values differ (shape ref {r[k].shape} gpu {g[k].shape})")
    return errs


def _compare_colours(R, B, m: int) -> list:
    errs = []
    n = len(R.objects())
    for i in range(n):
        a, b = R.object_cloud_rgb(i), B.object_cloud_rgb(m, i)
        if a.shape != b.shape or not np.array_equal(a, b):
            errs.append(f"object {i} colours differ ({a.shape} vs {b.shape}, "
                        f"{int(np.sum(a != b)) if a.shape == b.shape else -1} values)")
    return errs


def _run(gen_kw: dict, kv: str, n_frames: int, bf16: bool = False, deep_every: int = 5):
    from oracle import ref
    from scenemap_b200 import smg, synth
    D = 1152
    kw = dict(gen_kw)
    seed = synth.map_seed(kw.pop("seed_base"), 0)
    g = synth.BoxRoom(seed=seed, n_frames=n_frames, D=D, bf16=bf16, rgb=True, **kw)
    R = ref.RefMap(kv)
    B = smg.Batch(1, max_objects=256, emb_dim=D, max_det=32, params=smg.Params(kv))
    mirror = {}
    n_views = n_reset = 0
    prev_q = {}
    for f in range(n_frames):
        fr = g.frame(f)
        R.frame(fr)
        B.push([fr], smg.SMG_MEM_HOST, smg.SMG_EMB_BF16 if bf16 else smg.SMG_EMB_F32)
        deep = f % deep_every == 0 or f == n_frames - 1
        errs = compare_frame(R, B, 0, D, deep=deep)
        assert not errs, f"frame {f}: " + "\n".join(errs[:20])
        _mirror_update(mirror, B, 0)
        rv = R.views()
        errs = _compare_views(rv, mirror)
        assert not errs, f"frame {f}: " + "\n".join(errs[:20])
        if deep:
            errs = _compare_colours(R, B, 0)
            assert not errs, f"frame {f}: " + "\n".join(errs[:20])
        n_views = max(n_views, len(rv))
        for oid, v in rv.items():   # a view replaced at a lower quality: an event reset it
            if oid in prev_q and v["version"] != prev_q[oid][0] and v["q"] < prev_q[oid][1]:
                n_reset += 1
        prev_q = {oid: (v["version"], v["q"]) for oid, v in rv.items()}
    assert B.error_word() == 0
    B.close()
    return n_views, n_reset


def _need():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")


def test_best_views_box_room():
    _need()
    n_views, _ = _run(dict(seed_base=71), "", 40)
    assert n_views >= 8


def test_best_views_events():
    """Moved boxes (event 2) and a put-down box (event 5) reset view qualities."""
    _need()
    v = variants.moving(90)
    _, n_reset_m = _run(v["gen"], v["kv"], v["n_frames"], deep_every=10)
    h = variants.hands(100)
    _, n_reset_h = _run(h["gen"], h["kv"], h["n_frames"], deep_every=10)
    assert n_reset_m + n_reset_h >= 1


def test_best_views_coarse_masks():
    """Detector bit masks on a 4-pixel grid: cropMask reads the coarse cells."""
    _need()
    v = variants.coarse_masks(30)
    n_views, _ = _run(v["gen"], v["kv"], v["n_frames"], bf16=True)
    assert n_views >= 8
