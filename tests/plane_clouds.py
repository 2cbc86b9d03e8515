"""Point clouds for the plane-fit parity tests (apPlaneFit, scenemap objprob.cpp:130-209).

`kat_cases()` rebuilds the inputs of the reference's own known-answer test
(src/scene_graph/scenemap/tests/test_objprob.cpp:96-153: a thin vertical plane, a horizontal
plane, a noisy ceiling with outliers, a wall with furniture in front, a half cylinder and a
sphere) with its float32 arithmetic and its 64-bit LCG; each case carries the properties that
test asserts.  `edge_cases()` adds seeded clouds around the algorithm's boundaries (fewer than
8 points, collinear points, the 256-point subsample stride, large clouds, duplicates).
"""
from __future__ import annotations

import math

import numpy as np

F = np.float32


class _Lcg:
    """u01/gau of test_objprob.cpp:112-113 (Knuth MMIX LCG, 53-bit uniforms, Box-Muller)."""

    def __init__(self, seed: int):
        self.r = seed

    def u01(self) -> float:
        self.r = (self.r * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        return float(self.r >> 11) * (1.0 / 9007199254740992.0)

    def gau(self) -> float:
        a = math.sqrt(-2 * math.log(max(1e-12, self.u01())))
        return a * math.cos(6.283185307 * self.u01())


def _ap_seed(a: int, b: int) -> int:
    """apSeed (objprob.cpp:125-128)."""
    M = 0xFFFFFFFFFFFFFFFF
    s = ((a * 0x9E3779B97F4A7C15) & M) ^ ((b + 0x632BE59BD9B4E019) & M)
    s = (s + 0x9E3779B97F4A7C15) & M
    z = s
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    return z ^ (z >> 31)


def kat_cases():
    """[(name, xyz float32 (n,3), tau, seed, check(out) -> bool)] from test_objprob.cpp."""
    out = []
    P = [(F(1.0) + F(0.001) * F((i * 7 + j) % 3), F(0.05) * F(i), F(0.05) * F(j)) for i in range(40) for j in range(40)]
    out.append(("vertical", np.array(P, F), 0.02, 1,
                lambda o: o[0] == 1 and o[4] < 0.005 and abs(o[3]) < 0.1 and o[9] > 1.5 and o[5] > 0.99))
    P = [(F(0.05) * F(i), F(0.05) * F(j), F(2.4)) for i in range(40) for j in range(40)]
    out.append(("horizontal", np.array(P, F), 0.02, 2, lambda o: o[0] == 1 and abs(o[3]) > 0.99 and abs(o[6] - 2.4) < 1e-3))
    g = _Lcg(12345)
    P = []
    for _ in range(1200):
        P.append((F(3 * g.u01()), F(2 * g.u01()), F(2.5 + 0.01 * g.gau())))
    for _ in range(300):
        P.append((F(3 * g.u01()), F(2.0 + 0.01 * g.gau()), F(1.5 + g.u01())))
    for _ in range(300):
        P.append((F(3 * g.u01()), F(2 * g.u01()), F(3 * g.u01())))
    out.append(("noisy_ceiling", np.array(P, F), 0.03, _ap_seed(7, 1),
                lambda o: o[0] == 1 and abs(o[3]) > 0.99 and abs(o[6] - 2.5) < 0.01 and 0.6 < o[5] < 0.8 and o[4] < 0.015))
    P = []
    for _ in range(800):
        P.append((F(2 * g.u01()), F(0.015 * g.gau()), F(2.4 * g.u01())))
    for _ in range(200):
        P.append((F(0.5 + 0.5 * g.u01()), F(0.1 + 0.5 * g.u01()), F(0.8 * g.u01())))
    out.append(("wall", np.array(P, F), 0.04, _ap_seed(8, 2),
                lambda o: o[0] == 1 and abs(o[2]) > 0.99 and o[5] > 0.75 and o[9] > 1.5 and o[8] - o[7] > 1.5))
    P = []
    for i in range(60):
        for j in range(20):
            t = 3.14159265 * i / 59
            P.append((F(0.4 * math.cos(t)), F(0.4 * math.sin(t)), F(0.04 * j)))
    out.append(("half_cylinder", np.array(P, F), 0.02, _ap_seed(9, 3), lambda o: o[0] == 1 and o[5] < 0.7))
    P = []
    for i in range(30):
        for j in range(30):
            th, ph = 3.14159265 * (i + 0.5) / 30, 6.2831853 * j / 30
            P.append((F(0.3 * math.sin(th) * math.cos(ph)), F(0.3 * math.sin(th) * math.sin(ph)), F(1 + 0.3 * math.cos(th))))
    out.append(("sphere", np.array(P, F), 0.02, _ap_seed(9, 4), lambda o: o[5] < 0.7))
    return out


def _plane_cloud(rng, n, noise, outl):
    nrm = rng.normal(size=3)
    nrm /= np.linalg.norm(nrm)
    u = np.cross(nrm, [0.0, 0.0, 1.0] if abs(nrm[2]) < 0.9 else [1.0, 0.0, 0.0])
    u /= np.linalg.norm(u)
    v = np.cross(nrm, u)
    a, b = rng.uniform(-1, 1, n), rng.uniform(-1, 1, n)
    p = rng.uniform(-3, 3, 3) + a[:, None] * u + b[:, None] * v + rng.normal(0, noise, n)[:, None] * nrm
    k = int(outl * n)
    if k:
        p[:k] = rng.uniform(-3, 3, (k, 3))
    return p.astype(F)


def edge_cases():
    """[(name, xyz, tau, seed)] around the boundaries of apPlaneFit."""
    rng = np.random.default_rng(20240601)
    cases = [("n7", _plane_cloud(rng, 7, 0.005, 0.0), 0.02, 11),
             ("n8", _plane_cloud(rng, 8, 0.005, 0.0), 0.02, 12),
             ("collinear", np.stack([np.linspace(0, 1, 50)] * 3, 1).astype(F), 0.02, 13),
             ("duplicates", np.repeat(_plane_cloud(rng, 20, 0.002, 0.0), 5, axis=0), 0.02, 14)]
    for n in (255, 256, 257, 511, 512, 513, 1000, 4096, 20000):
        cases.append((f"plane_n{n}", _plane_cloud(rng, n, 0.01, 0.3), 0.03, int(rng.integers(1, 2**62))))
    for k in range(6):
        n = int(rng.integers(30, 3000))
        cases.append((f"random{k}", _plane_cloud(rng, n, float(rng.uniform(0.001, 0.05)), float(rng.uniform(0, 0.6))),
                      float(rng.uniform(0.01, 0.06)), int(rng.integers(1, 2**62))))
    cases.append(("cube_noise", rng.uniform(-1, 1, (900, 3)).astype(F), 0.02, 99))
    return cases


def all_cases():
    """[(name, xyz, tau, seed)] of every KAT and edge case."""
    return [(n, x, t, s) for n, x, t, s, _ in kat_cases()] + edge_cases()
