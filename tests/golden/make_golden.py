"""Writes tests/golden/plane_fit.json: apPlaneFit outputs of the REFERENCE itself.

Run in a container where the reference sources are present and oracle/_ref/libscenemap_ref.so
has been built (`make -C oracle`):

    python tests/golden/make_golden.py

Inputs are rebuilt by tests/plane_clouds.py (deterministic), so only the outputs are stored.
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, ".."))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

from oracle import ref  # noqa: E402
import plane_clouds  # noqa: E402

assert ref.available(), "oracle/_ref/libscenemap_ref.so is missing"
out = {}
for name, xyz, tau, seed in plane_clouds.all_cases():
    r = ref.plane_fit(xyz, tau, seed, 64, impl="ref")
    out[name] = {"n": int(len(xyz)), "tau": tau, "seed": seed, "out": [float(v).hex() for v in r]}
with open(os.path.join(HERE, "plane_fit.json"), "w") as f:
    json.dump({"generator": "tests/golden/make_golden.py", "max_iters": 64,
               "fields": ["ok", "n0", "n1", "n2", "thick", "inl", "zmed", "zlo", "zhi", "hspan"], "cases": out}, f, indent=1)
print("wrote", len(out), "cases")
