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
