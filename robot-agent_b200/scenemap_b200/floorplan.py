"""Seeded synthetic 2D laser workload.

A floor plan of 12 rooms (4 x 3, random column widths and row heights, one door on every
shared wall, a few box obstacles in room corners) is ray cast with 720 beams over 360 degrees,
8 m maximum range and sigma = 0.01 m range noise, along a trajectory that visits the rooms in
a serpentine order through their doors and turns back at the end.  Each scan comes with its
true pose and an initial pose estimate (true pose plus odometry-like noise inside the
matcher's search window).  Points are in the base frame (sensor at the base origin); beams
without a return become free rays that end at the maximum range.
"""
from __future__ import annotations

import math

import numpy as np


class FloorPlan:
    def __init__(self, seed: int, n_scans: int = 5000, beams: int = 720, max_range: float = 8.0, sigma: float = 0.01,
                 step_m: float = 0.05, pose_noise=(0.05, math.radians(2.0)), pose_clip=(0.25, math.radians(8.0))):
        self.rng = np.random.default_rng(seed)
        self.beams, self.max_range, self.sigma = beams, max_range, sigma
        self._walls()
        self._path(n_scans, step_m)
        r = self.rng
        dx = np.clip(r.normal(0, pose_noise[0], (n_scans, 2)), -pose_clip[0], pose_clip[0])
        dth = np.clip(r.normal(0, pose_noise[1], n_scans), -pose_clip[1], pose_clip[1])
        self.pose0 = self.poses.copy()
        self.pose0[:, :2] += dx
        self.pose0[:, 2] += dth
        self.phi = 2 * math.pi * np.arange(beams) / beams
        self._noise_seed = int(r.integers(1, 2**62))

    # ------------------------------------------------------------ geometry
    def _walls(self):
        r = self.rng
        cw = r.uniform(4.0, 7.0, 4)
        rh = r.uniform(4.0, 6.0, 3)
        xs = np.concatenate([[0.0], np.cumsum(cw)])
        ys = np.concatenate([[0.0], np.cumsum(rh)])
        self.xs, self.ys = xs, ys
        segs = []
        door = 1.0

        def wall_with_door(a, b, fixed, horizontal, with_door):
            if not with_door:
                segs.append((a, fixed, b, fixed) if horizontal else (fixed, a, fixed, b))
                return None
            c = r.uniform(a + 0.5 + door / 2, b - 0.5 - door / 2)
            for lo, hi in ((a, c - door / 2), (c + door / 2, b)):
                segs.append((lo, fixed, hi, fixed) if horizontal else (fixed, lo, fixed, hi))
            return c

        self.doors = {}
        # outer boundary
        wall_with_door(xs[0], xs[-1], ys[0], True, False)
        wall_with_door(xs[0], xs[-1], ys[-1], True, False)
        wall_with_door(ys[0], ys[-1], xs[0], False, False)
        wall_with_door(ys[0], ys[-1], xs[-1], False, False)
        # internal vertical walls (between columns), one door per room pair
        for ci in range(1, 4):
            for ri in range(3):
                c = wall_with_door(ys[ri], ys[ri + 1], xs[ci], False, True)
                self.doors[((ri, ci - 1), (ri, ci))] = (xs[ci], c)
        # internal horizontal walls (between rows)
        for ri in range(1, 3):
            for ci in range(4):
                c = wall_with_door(xs[ci], xs[ci + 1], ys[ri], True, True)
                self.doors[((ri - 1, ci), (ri, ci))] = (c, ys[ri])
        # box obstacles in room corners
        for ri in range(3):
            for ci in range(4):
                for corner in r.choice(4, size=int(r.integers(1, 4)), replace=False):
                    w, h = r.uniform(0.3, 0.9, 2)
                    x0 = xs[ci] + 0.25 if corner in (0, 2) else xs[ci + 1] - 0.25 - w
                    y0 = ys[ri] + 0.25 if corner in (0, 1) else ys[ri + 1] - 0.25 - h
                    segs += [(x0, y0, x0 + w, y0), (x0 + w, y0, x0 + w, y0 + h), (x0 + w, y0 + h, x0, y0 + h),
                             (x0, y0 + h, x0, y0)]
        self.segs = np.asarray(segs, np.float64)

    def _path(self, n_scans, step_m):
        order = []
        for ri in range(3):
            cols = range(4) if ri % 2 == 0 else range(3, -1, -1)
            order += [(ri, ci) for ci in cols]
        center = lambda rc: ((self.xs[rc[1]] + self.xs[rc[1] + 1]) / 2, (self.ys[rc[0]] + self.ys[rc[0] + 1]) / 2)
        pts = [center(order[0])]
        for a, b in zip(order[:-1], order[1:]):
            key = (a, b) if (a, b) in self.doors else (b, a)
            dx, dy = self.doors[key]
            if key[0][0] == key[1][0]:          # vertical wall: approach along x
                pts += [(dx - 0.6 * np.sign(center(b)[0] - center(a)[0]), dy), (dx + 0.6 * np.sign(center(b)[0] - center(a)[0]), dy)]
            else:
                pts += [(dx, dy - 0.6 * np.sign(center(b)[1] - center(a)[1])), (dx, dy + 0.6 * np.sign(center(b)[1] - center(a)[1]))]
            pts.append(center(b))
        pts = np.asarray(pts)
        loop = np.concatenate([pts, pts[::-1][1:]])
        seg_len = np.hypot(*np.diff(loop, axis=0).T)
        cum = np.concatenate([[0.0], np.cumsum(seg_len)])
        total = cum[-1]
        s = (np.arange(n_scans) * step_m) % total
        i = np.clip(np.searchsorted(cum, s, side="right") - 1, 0, len(seg_len) - 1)
        t = (s - cum[i]) / np.maximum(seg_len[i], 1e-9)
        xy = loop[i] + (loop[i + 1] - loop[i]) * t[:, None]
        head = np.arctan2(loop[i + 1, 1] - loop[i, 1], loop[i + 1, 0] - loop[i, 0])
        th = head + 0.3 * np.sin(np.arange(n_scans) * 0.05)
        self.poses = np.column_stack([xy, th])

    # ------------------------------------------------------------ scans
    def ranges(self, k: int) -> np.ndarray:
        """True ranges of scan k (inf = no wall within max range)."""
        x, y, th = self.poses[k]
        ang = th + self.phi
        d = np.stack([np.cos(ang), np.sin(ang)], 1)                     # beams x 2
        a = self.segs[:, :2]
        e = self.segs[:, 2:] - a                                          # segs x 2
        den = d[:, None, 0] * e[None, :, 1] - d[:, None, 1] * e[None, :, 0]
        w = a[None, :, :] - np.array([x, y])[None, None, :]
        with np.errstate(divide="ignore", invalid="ignore"):
            t = (w[..., 0] * e[None, :, 1] - w[..., 1] * e[None, :, 0]) / den
            u = (w[..., 0] * d[:, None, 1] - w[..., 1] * d[:, None, 0]) / den
        ok = (np.abs(den) > 1e-12) & (t > 1e-6) & (u >= 0) & (u <= 1)
        t = np.where(ok, t, np.inf).min(1)
        return np.where(t <= self.max_range, t, np.inf)

    def scan(self, k: int) -> dict:
        """Scan k: hits (n, 2) float32 and free-ray ends (m, 2) float32 in the base frame."""
        r = self.ranges(k)
        g = np.random.default_rng(self._noise_seed + k)
        rn = r + g.normal(0, self.sigma, len(r))
        hit = np.isfinite(r) & (rn > 0.05) & (rn < self.max_range)
        c, s = np.cos(self.phi), np.sin(self.phi)
        hits = np.stack([rn[hit] * c[hit], rn[hit] * s[hit]], 1).astype(np.float32)
        free = np.stack([self.max_range * c[~hit], self.max_range * s[~hit]], 1).astype(np.float32)
        return {"hits": hits, "free": free, "pose": self.poses[k].copy(), "pose0": self.pose0[k].copy()}
