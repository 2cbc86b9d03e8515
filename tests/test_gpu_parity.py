"""B200 objprob update vs the reference scenemap code, frame by frame (GPU).

Both sides get byte-identical synthetic frames (config-0 generator).  Decisions and integer
state (association, object ids/counts/states, cloud points, voxel keys via the clouds, grid
log-odds per global cell, events, stats) must be identical; positions and boxes within 1e-5
relative (the reference's double sums are re-associated on the device).
"""
import os

import numpy as np
import pytest

from conftest import has_gpu
from parity_util import compare_frame

pytestmark = pytest.mark.gpu


def _need():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")


def _run(n_frames: int, seed: int, bf16: bool, deep_every: int, D: int = 1152, **gen_kw):
    from oracle import ref
    from scenemap_b200 import smg, synth
    g = synth.BoxRoom(seed=synth.map_seed(seed, 0), n_frames=n_frames, D=D, bf16=bf16, **gen_kw)
    R = ref.RefMap()
    B = smg.Batch(1, max_objects=256, emb_dim=D, max_det=32)
    dtype = smg.SMG_EMB_BF16 if bf16 else smg.SMG_EMB_F32
    for f in range(n_frames):
        fr = g.frame(f)
        R.frame(fr)
        B.push([fr], smg.SMG_MEM_HOST, dtype)
        deep = deep_every > 0 and (f % deep_every == 0 or f == n_frames - 1)
        errs = compare_frame(R, B, 0, D, deep=deep)
        assert not errs, f"frame {f}: " + "\n".join(errs[:20])
    assert B.error_word() == 0
    B.close()


def test_parity_config0_short():
    _need()
    _run(40, 1234, bf16=False, deep_every=5)


def test_parity_config0_bf16():
    _need()
    _run(30, 77, bf16=True, deep_every=10)


@pytest.mark.slow
def test_parity_config0_full():
    _need()
    n = int(os.environ.get("SMG_PARITY_FRAMES", "300"))
    _run(n, 1234, bf16=False, deep_every=25)


def test_parity_batch_maps():
    """Several maps in one batch: each map must match its own reference instance."""
    _need()
    from oracle import ref
    from scenemap_b200 import smg, synth
    M, N, D = 4, 25, 1152
    gens = [synth.BoxRoom(seed=synth.map_seed(4242, i), n_frames=N, D=D, bf16=True) for i in range(M)]
    refs = [ref.RefMap() for _ in range(M)]
    B = smg.Batch(M, max_objects=128, emb_dim=D, max_det=32)
    for f in range(N):
        frs = [g.frame(f) for g in gens]
        for R, fr in zip(refs, frs):
            R.frame(fr)
        B.push(frs, smg.SMG_MEM_HOST, smg.SMG_EMB_BF16)
        for m in range(M):
            errs = compare_frame(refs[m], B, m, D, deep=(f % 8 == 0 or f == N - 1))
            assert not errs, f"map {m} frame {f}: " + "\n".join(errs[:20])
    assert B.error_word() == 0
    B.close()
