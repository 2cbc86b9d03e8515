"""The generator variants reach the rules they are meant for, on the reference (CPU).

The GPU parity tests run the same variants through both sides; this test keeps the variants
honest: if a generator change stopped them from firing the targeted counters and events, the
parity tests would silently stop covering those rules.
"""
import pytest

import variants


def _need():
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")


@pytest.mark.parametrize("name", ["structure", "moving", "hands"])
def test_variant_fires_its_rules_on_the_reference(name):
    _need()
    from oracle import ref
    v = getattr(variants, name)()
    g = variants.make_gen(v)
    R = ref.RefMap(v["kv"])
    for f in range(v["n_frames"]):
        R.frame(g.frame(f))
    st = R.stats()
    for k in v["stats"]:
        assert st[k] > 0, f"{name}: {k} is 0 on the reference ({st})"
    seen = {e[2] for e in R.events()}   # the reference keeps every event of the run
    for k in v["events"]:
        assert k in seen, f"{name}: no event of kind {k} on the reference (seen {sorted(seen)})"


def test_bit_masks_on_the_image_grid_equal_the_label_image_on_the_reference():
    """The reference gets the same result from the label image (turned into bit masks on the
    image grid by the oracle driver) and from bit masks with scale 1 given directly."""
    _need()
    from oracle import ref
    from scenemap_b200 import synth
    g = synth.BoxRoom(seed=synth.map_seed(71, 0), n_frames=12, bf16=True)
    A, Bm = ref.RefMap(), ref.RefMap()
    for f in range(12):
        fr = g.frame(f)
        A.frame(fr)
        Bm.frame(dict(fr, mask_bits=synth.label_masks(fr["label"], fr["det_label"], 1), mask_w=fr["w"], mask_h=fr["h"],
                      mask_affine=(1.0, 1.0, 0.0, 0.0)))
        assert A.objects() == Bm.objects()
        assert A.stats() == Bm.stats()


def test_text_model_reaches_its_rules():
    """With the synthetic text model the reference names objects (some through the hypernym /
    fallback roll-up), blocks wall-looking fragments from non-structure objects, and drops
    structure: the rules the device text model is compared on are reached."""
    from oracle import ref
    from scenemap_b200 import synth
    if not ref.available():
        pytest.skip("reference oracle library not built")
    v = variants.structure(60)
    kw = dict(v["gen"])
    g = synth.BoxRoom(seed=synth.map_seed(kw.pop("seed_base"), 0), n_frames=v["n_frames"], D=1152, **kw)
    R = ref.RefMap(v["kv"])
    R.set_text_model(synth.text_model(g))
    for f in range(v["n_frames"]):
        R.frame(g.frame(f))
    names = [R.object_name(i) for i in range(len(R.objects()))]
    assert sum(n["has_post"] for n in names) >= 10
    assert sum(n["rolled"] for n in names) >= 1
    st = R.stats()
    assert st["n_blocked"] > 0 and st["n_obj_struct"] > 0
