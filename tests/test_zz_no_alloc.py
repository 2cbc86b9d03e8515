"""smg_plane_fit_noalloc: the plane fit for callers that cannot allocate device memory (GPU).

Some callers of this library must not allocate GPU memory once they are running, for example
a robot's real-time frame loop that reserves its whole memory budget at start-up, where a
cudaMalloc in mid-frame could block, synchronise the device or fail.  For them the library
offers one entry point whose scratch is a static device array of the library (at most 65536
points per call).  This test calls it twice in a row through the C ABI, with different point
sets each time, and checks each result against smg_plane_fit (which allocates its scratch per
call).  Both run the same kernel with the same arithmetic, so the results must be identical
(tolerance zero, tighter than the 1e-9 the reference comparisons use); the second call also
shows that scratch left over from the first call does not leak into the next result.

This file is collected last so that a run stopping at the first failure has run every other
test; it passes alone in a fresh process as well.
"""
import numpy as np
import pytest

import plane_clouds
from conftest import has_gpu

pytestmark = pytest.mark.gpu


def _sets(which):
    cases = plane_clouds.all_cases()
    sel = cases[0::2] if which == 0 else cases[1::2]
    return [c[1] for c in sel], [c[3] for c in sel]


def test_noalloc_matches_allocating_entry_point_twice():
    if not has_gpu():
        pytest.skip("no GPU")
    from scenemap_b200 import smg
    for call, tau in ((0, 0.02), (1, 0.03)):
        clouds, seeds = _sets(call)
        assert sum(len(c) for c in clouds) <= 65536
        want = smg.plane_fit(clouds, tau, seeds, 64, entry="smg_plane_fit")
        got = smg.plane_fit(clouds, tau, seeds, 64, entry="smg_plane_fit_noalloc")
        assert np.array_equal(got, want), f"call {call}: max diff {np.nanmax(np.abs(got - want))}"
        assert (got[:, 0] >= 0).all()


def test_noalloc_rejects_oversize_call():
    if not has_gpu():
        pytest.skip("no GPU")
    from scenemap_b200 import smg
    big = np.zeros((65537, 3), np.float32)
    big[:, 0] = np.arange(65537, dtype=np.float32) * 1e-3
    with pytest.raises(smg.SmgError, match="exceeds the static scratch limit"):
        smg.plane_fit([big], 0.02, [1], 64, entry="smg_plane_fit_noalloc")
