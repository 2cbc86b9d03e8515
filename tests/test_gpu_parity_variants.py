"""B200 objprob update vs the reference on the generator variants (GPU).

The default box room never reaches the structural drops (ceiling, floor, tall wall,
apStructObject), the absence/gone/relink rules, or non-default parameters.  These runs feed
byte-identical variant frames to both sides, compare every frame as the default parity test
does, and check that the targeted counters and events really occurred (equal on both sides).
"""
import numpy as np
import pytest

import variants
from conftest import has_gpu
from parity_util import compare_frame

pytestmark = pytest.mark.gpu


def _need():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")


def _run_variant(v: dict, bf16: bool = False, deep_every: int = 10, D: int = 1152):
    from oracle import ref
    from scenemap_b200 import smg
    bf16 = bf16 or v.get("bf16", False)
    g = variants.make_gen(v, D=D, bf16=bf16)
    R = ref.RefMap(v["kv"])
    B = smg.Batch(1, max_objects=256, emb_dim=D, max_det=32, params=smg.Params(v["kv"]))
    dtype = smg.SMG_EMB_BF16 if bf16 else smg.SMG_EMB_F32
    n = v["n_frames"]
    for f in range(n):
        fr = g.frame(f)
        R.frame(fr)
        B.push([fr], smg.SMG_MEM_HOST, dtype)
        errs = compare_frame(R, B, 0, D, deep=(f % deep_every == 0 or f == n - 1))
        assert not errs, f"frame {f}: " + "\n".join(errs[:20])
    assert B.error_word() == 0
    st = B.stats(0)
    for k in v["stats"]:
        assert st[k] > 0, f"{k} never fired ({st})"
    seen = {e[2] for e in R.events()}
    for k in v["events"]:
        assert k in seen, f"no event of kind {k} (seen {sorted(seen)})"
    B.close()


def test_parity_structure_variant():
    """Walls/floor/ceiling as detections: ceiling, floor and tall-wall drops, apStructObject."""
    _need()
    _run_variant(variants.structure())


def test_parity_wall_segments():
    """Keyframes with wall segments: wall-line drops and wall-like fragments, the see-through
    drop, the wall share and flat-plane test of apStructObject, stored vs per-keyframe sets."""
    _need()
    _run_variant(variants.walls(), deep_every=8)


def test_parity_moving_boxes():
    """Boxes that slide, jump, vanish and appear: absence, gone, relink, seen again."""
    _need()
    _run_variant(variants.moving(), deep_every=20)


def test_parity_engine_params():
    """The reference's engine parameter file (yolo26n-seg-obj-416 obj_params), bf16 embeddings."""
    _need()
    _run_variant(variants.engine_params(), bf16=True)


def test_parity_hands():
    """A gripper picks up a small box, carries it, puts it on a larger one that is then pushed:
    grasp, hold, release, support link and the supported object following (updateHands)."""
    _need()
    _run_variant(variants.hands(), deep_every=5)


def test_parity_coarse_detector_masks():
    """Bit masks on a 4-pixel grid (sm_detections with mask_sx = mask_sy = 4)."""
    _need()
    _run_variant(variants.coarse_masks(), deep_every=8)


def test_parity_depth_millimetres():
    """uint16 millimetre depth (ObjFrame::depth_mm), read as mm * 1e-3f everywhere."""
    _need()
    _run_variant(variants.depth_millimetres(), deep_every=8)


def test_bit_masks_on_the_image_grid_equal_the_label_image():
    """The two input forms of the same detections (label image, or bit masks with scale 1)
    give the same results, field for field."""
    _need()
    from scenemap_b200 import smg, synth
    import numpy as np
    D = 1152
    g = synth.BoxRoom(seed=synth.map_seed(71, 0), n_frames=20, D=D, bf16=True)
    A = smg.Batch(1, max_objects=128, emb_dim=D, max_det=32)
    Bm = smg.Batch(1, max_objects=128, emb_dim=D, max_det=32)
    for f in range(20):
        fr = g.frame(f)
        frb = dict(fr, mask_bits=synth.label_masks(fr["label"], fr["det_label"], 1), mask_w=fr["w"], mask_h=fr["h"],
                   mask_affine=(1.0, 1.0, 0.0, 0.0))
        A.push([fr], smg.SMG_MEM_HOST, smg.SMG_EMB_BF16)
        Bm.push([frb], smg.SMG_MEM_HOST, smg.SMG_EMB_BF16)
        assert A.objects(0) == Bm.objects(0), f"frame {f}"
        ra, rb = A.reencode(0), Bm.reencode(0)
        for k in ("id", "box", "kappa", "bits"):
            assert np.array_equal(ra[k], rb[k]), (f, k)
        assert np.array_equal(A.assoc(0)["obj_id"], Bm.assoc(0)["obj_id"])
    A.close()
    Bm.close()
