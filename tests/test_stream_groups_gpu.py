"""Stream groups: the maps of a batch split into ranges whose chains run on separate streams
(and whose host inputs arrive on a copy stream group by group) must give exactly the results of
one chain over all maps: the maps are independent, so every output is compared for equality.
"""
import os

import numpy as np
import pytest

from conftest import has_gpu

pytestmark = pytest.mark.gpu


def _pinned(fr: dict) -> dict:
    """The frame with its images in pinned host memory (the device reads them in place)."""
    import torch
    out = dict(fr)
    for k in ("depth", "label"):
        a = np.ascontiguousarray(fr[k])
        t = torch.empty(a.shape, dtype=torch.float32 if a.dtype == np.float32 else torch.int16, pin_memory=True)
        v = t.numpy().view(a.dtype)
        v[...] = a
        out[k] = v
        out["_keep_" + k] = t
    return out


def _run(groups: int, M: int, N: int, D: int, pinned: bool = False, walls: bool = False):
    from scenemap_b200 import smg, synth
    os.environ["SMG_STREAM_GROUPS"] = str(groups)
    try:
        B = smg.Batch(M, max_objects=128, emb_dim=D, max_det=32)
    finally:
        del os.environ["SMG_STREAM_GROUPS"]
    gens = [synth.BoxRoom(seed=synth.map_seed(9090, i), n_frames=N, D=D, bf16=True) for i in range(M)]
    if walls:   # wall extraction on each group's grid stream, the object streams waiting for it
        B.set_text_model(synth.text_model(gens[0]))
        B.set_walls(True)
    trace = []
    for f in range(N):
        frs = [g.frame(f) for g in gens]
        if pinned:
            frs = [_pinned(fr) for fr in frs]
        B.push(frs, smg.SMG_MEM_HOST, smg.SMG_EMB_BF16)   # host inputs: copied group by group
        trace.append(B.assoc_all().copy())
        trace.append([B.reencode(m) for m in range(M)])   # re-encode masks read host depth when gathered
    out = {"assoc": trace, "err": B.error_word()}
    for m in range(M):
        out[f"obj{m}"] = B.objects(m)
        out[f"stats{m}"] = B.stats(m)
        out[f"events{m}"] = B.events(m)
        out[f"grid{m}"] = B.grid_cells(m)
        out[f"kf{m}"] = B.keyframe(m)
        if walls:
            out[f"walls{m}"] = B.wall_segments(m)
    B.close()
    return out


def _same(a, b, path="out"):
    if isinstance(a, dict):
        assert set(a) == set(b), path
        for k in a:
            _same(a[k], b[k], f"{path}.{k}")
    elif isinstance(a, (list, tuple)):
        assert len(a) == len(b), path
        for i, (x, y) in enumerate(zip(a, b)):
            _same(x, y, f"{path}[{i}]")
    elif isinstance(a, np.ndarray):
        assert a.shape == b.shape and a.dtype == b.dtype, path
        assert np.array_equal(a, b, equal_nan=a.dtype.kind == "f"), path
    else:
        assert a == b or (a != a and b != b), f"{path}: {a!r} != {b!r}"


def test_stream_groups_match_one_chain():
    if not has_gpu():
        pytest.skip("no GPU")
    M, N, D = 8, 24, 1152
    one = _run(1, M, N, D)
    four = _run(4, M, N, D)
    assert one["err"] == 0 and four["err"] == 0
    _same(one, four)
    three = _run(3, M, N, D)   # uneven ranges (3, 2, 3 maps)
    _same(one, three)


def test_pinned_host_frames_gathered():
    """Pinned host frames are read in place, only the pixels the chain reads (k_gather); the
    results must equal those of whole-frame copies of pageable frames."""
    if not has_gpu():
        pytest.skip("no GPU")
    M, N, D = 8, 24, 1152
    paged = _run(4, M, N, D)
    pinned = _run(4, M, N, D, pinned=True)
    assert paged["err"] == 0 and pinned["err"] == 0
    _same(paged, pinned)


def test_stream_groups_with_walls():
    """Wall extraction on every group's grid stream gives what one chain gives."""
    if not has_gpu():
        pytest.skip("no GPU")
    M, N, D = 8, 24, 1152
    one = _run(1, M, N, D, walls=True)
    four = _run(4, M, N, D, walls=True)
    assert one["err"] == 0 and four["err"] == 0
    assert any(one[f"walls{m}"] is not None and len(one[f"walls{m}"]) for m in range(M))
    _same(one, four)
