"""Every optional part of the keyframe at once (GPU): the hands variant (grasp, carry, put down,
push) with an RGB image (best views, cloud colours), a text model (names, guards, structural
rules), wall extraction before every update (ignore footprints of named objects) and the
snapshot, against the reference with the same glue.  Each part has its own parity test; this one
checks they compose: every keyframe is compared as the default parity test does, plus the views,
names, extracted wall segments, and every few keyframes the snapshot's object lists.
"""
import numpy as np
import pytest

from conftest import has_gpu
from parity_util import compare_frame
from test_gpu_best_views import _compare_colours, _compare_views, _mirror_update
from test_gpu_text_model import _compare_names
import variants

pytestmark = pytest.mark.gpu

GRID = (512, 512, -256 + 60, -256 + 50)


def test_all_features_compose():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")
    from scenemap_b200 import smg, synth
    D = 1152
    v = variants.hands(90)
    kw = dict(v["gen"])
    g = synth.BoxRoom(seed=synth.map_seed(kw.pop("seed_base"), 0), n_frames=v["n_frames"], D=D, rgb=True, **kw)
    t = synth.text_model(g)
    R = ref.RefMap(v["kv"])
    R.set_text_model(t)
    R.set_walls(GRID)
    B = smg.Batch(1, max_objects=256, emb_dim=D, max_det=32, grid=GRID, params=smg.Params(v["kv"]))
    B.set_text_model(t)
    B.set_walls(True)
    mirror = {}
    n_named = n_walls = n_views = 0
    for f in range(v["n_frames"]):
        fr = g.frame(f)
        R.frame(fr)
        B.push([fr], smg.SMG_MEM_HOST, smg.SMG_EMB_F32)
        deep = f % 10 == 0 or f == v["n_frames"] - 1
        errs = compare_frame(R, B, 0, D, deep=deep)
        assert not errs, f"frame {f}: " + "\n".join(errs[:20])
        _mirror_update(mirror, B, 0)
        rv = R.views()
        errs = _compare_views(rv, mirror)
        assert not errs, f"frame {f}: " + "\n".join(errs[:20])
        n_views = max(n_views, len(rv))
        wr, wg = R.wall_segments(), B.wall_segments(0)
        assert (wr is None) == (wg is None) and (wr is None or np.array_equal(wr, wg)), f"frame {f}: wall segments differ"
        n_walls = max(n_walls, 0 if wr is None else len(wr))
        if deep:
            errs = _compare_colours(R, B, 0) + _compare_names(R, B, 0)
            assert not errs, f"frame {f}: " + "\n".join(errs[:20])
            ro, go = R.snapshot(), B.snapshot(points=False)["objects"]
            assert [o["id"] for o in ro] == [o["id"] for o in go], f"frame {f}: snapshot ids differ"
            for a, b in zip(ro, go):
                assert a == b, f"frame {f}: snapshot object {a['id']} differs"
    n_named = sum(R.object_name(i)["has_post"] for i in range(len(R.objects())))
    # (with names, the carried box's class can be a static kind, which the hand does not take:
    # the grasp itself is covered by the hands variant without a text model)
    assert n_named >= 5 and n_walls >= 2 and n_views >= 5
    assert B.error_word() == 0
    B.close()
