"""The benchmarked configuration itself against the reference (GPU).

bench.py times config 1 on frames rendered on the device (RoomBatch) with 1024 object slots, a
512x512 grid at (-196, -206) and 24 detections per frame, from keyframe 105 on.  Here the same
settings run for 130 keyframes over 8 maps, device frames into the library and their host
copies into one reference instance per map, compared after every keyframe.  A second test
checks that the device renderer produces the host generator's frames byte for byte, so the
host-generated parity runs and the device-generated benchmark see the same inputs.
"""
import threading

import numpy as np
import pytest

from conftest import has_gpu
from parity_util import compare_frame

pytestmark = pytest.mark.gpu

BENCH_GRID = (512, 512, -256 + 60, -256 + 50)


def _need():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")


def test_device_renderer_matches_host_generator():
    if not has_gpu():
        pytest.skip("no GPU")
    from scenemap_b200 import synth
    from scenemap_b200.workload import RoomBatch
    M, N = 4, 3
    wl = RoomBatch(M, 1000, 40, D=1152, bf16=True, max_det=24)
    for f0 in (0, 37):
        R = wl.render(f0, N)
        for fi in range(N):
            hf = wl.host_frames(R, fi)
            for m in range(M):
                ref_fr = wl.rooms[m].frame(f0 + fi)
                d = hf[m]
                assert np.array_equal(d["depth"].view(np.uint32), ref_fr["depth"].view(np.uint32)), (m, f0 + fi)
                assert np.array_equal(d["label"], ref_fr["label"]), (m, f0 + fi)
                assert d["n_det"] == ref_fr["n_det"]
                for k in ("det_label", "box", "cls", "score"):
                    assert np.array_equal(np.asarray(d[k]), np.asarray(ref_fr[k])), (k, m, f0 + fi)
                assert np.array_equal(d["emb"].view(np.uint32), ref_fr["emb"].view(np.uint32)), (m, f0 + fi)
    # detector bit masks on a 4-pixel grid, built on the device from the rendered labels
    wl4 = RoomBatch(M, 1000, 40, D=1152, bf16=True, max_det=24, mask_grid=4)
    R = wl4.render(5, 2)
    for fi in range(2):
        hf = wl4.host_frames(R, fi)
        for m in range(M):
            ref_fr = wl4.rooms[m].frame(5 + fi)
            want = synth.label_masks(ref_fr["label"], ref_fr["det_label"], 4)
            assert np.array_equal(hf[m]["mask_bits"], want), (m, 5 + fi)


def test_parity_bench_configuration():
    _need()
    from oracle import ref
    from scenemap_b200 import smg
    from scenemap_b200.workload import RoomBatch
    M, N, D = 8, 130, 1152
    wl = RoomBatch(M, 1000, N, D=D, bf16=True, max_det=24)
    B = smg.Batch(M, max_objects=1024, emb_dim=D, max_w=640, max_h=480, max_det=24, grid=BENCH_GRID)
    refs = [ref.RefMap() for _ in range(M)]
    for f0 in range(0, N, 10):
        nf = min(10, N - f0)
        R = wl.render(f0, nf)
        for fi in range(nf):
            f = f0 + fi
            hf = wl.host_frames(R, fi)
            ths = [threading.Thread(target=refs[m].frame, args=(hf[m],)) for m in range(M)]
            for t in ths:
                t.start()
            keep = []
            B.push(None, smg.SMG_MEM_DEVICE, structs=wl.structs(R, fi, keep), stream=0)
            for t in ths:
                t.join()
            deep = f % 25 == 0 or f == N - 1
            for m in range(M):
                errs = compare_frame(refs[m], B, m, D, deep=deep)
                assert not errs, f"map {m} frame {f}: " + "\n".join(errs[:20])
    assert B.error_word() == 0
    B.close()
