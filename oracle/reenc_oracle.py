"""CPU restatement of the whole-object re-encode requests (TEST INFRASTRUCTURE ONLY).

Restates ObjectMap::buildReencode (scenemap src/objmap.cpp:1371-1458) for the mask grid equal
to the image grid (mask scale 1, offset 0), the form the batch library runs:

- candidates (objmap.cpp:1383): confirmed, not gone, seen this keyframe (last_kf == stamp),
  at least 30 cloud points, in list order;
- every stp-th cloud point, stp = max(1, n // 3000) (:1385-1391); the point in the map frame
  is (org + p) - cam in double, rotated by T_mc's columns (:1392-1394);
- z < 0.15: skipped; a projection outside the image sets trunc (:1395-1397); visible when the
  depth at (int(u), int(v)) is > 0 and >= z - 0.08 (:1398-1400);
- a visible point paints the cells [floor(u - r), floor(u + r)] x [floor(v - r), floor(v + r)],
  r = 0.6 * voxel * fx / z, clipped to the grid (:1403-1409), updates the u/v extremes and sets
  trunc within 2 px of the border (:1410-1411);
- at least 12 visible points and a visible fraction >= reenc_min_vis (:1413-1416);
- closing: an empty cell with >= 3 painted cells among its 8 neighbours is filled (:1418-1430);
  size = sqrt(area) must reach reenc_min_px (:1431-1433);
- kappa = viewKappa(float size, trunc, float median depth, float visible fraction, camera rate)
  (bestview.cpp:77-81, objprob_math.h:78-87); objects that still need a whole view always ask,
  others when kappa >= reenc_gain * whole_kappa (:1436-1443);
- priority (need ? 1e6 : 0) + kappa / max(1, whole_kappa); the reenc_max best are kept, equal
  priorities in list order (:1444-1457).

The painting is a 2-D difference array (exactly the union of the squares) and the closing a
neighbour count on the painted grid.
"""
from __future__ import annotations

import numpy as np


def view_kappa(size_px: float, trunc: bool, depth: float, vis: float, cam_w: float, k0=4369.0, s0=40.0,
               trunc_k=1.0, d0=100.0, occ=1.0, blur_w=0.0) -> float:
    """objprob_math.h:78-87 in the reference's operation order (double)."""
    s, d = max(0.0, size_px), max(0.0, depth)
    k = k0 * s / (s + s0)
    if trunc:
        k *= trunc_k
    k /= 1.0 + (d / d0) * (d / d0)
    v = 0.0 if vis < 0 else (1.0 if vis > 1 else vis)
    k *= v if occ == 1.0 else v ** occ
    if blur_w > 0:
        k *= float(np.exp(-max(0.0, cam_w) / blur_w))
    return max(k, 1e-3)


def build_reencode(frame: dict, objects: list, clouds: list, voxel: float = 0.02, reenc_max: int = 8,
                   reenc_gain: float = 1.3, reenc_min_vis: float = 0.5, reenc_min_px: int = 24,
                   cam_w: float = 0.0, kappa_params: dict | None = None) -> dict:
    """Requests of one keyframe, best first.

    frame: stamp, depth (h x w float32), fx, fy, cx, cy (float32 values), T_mc (12 doubles).
    objects: dicts in list order with id, confirmed, state, last_kf, cloud_org, need_whole and
    whole_kappa (0 when absent: no whole view was ever added).  clouds[i]: float32 (n, 3)
    points of object i relative to its cloud_org.
    """
    kp = kappa_params or {}
    depth = np.asarray(frame["depth"], np.float32)
    h, w = depth.shape
    T = np.asarray(frame["T_mc"], np.float64)
    fx, fy = float(np.float32(frame["fx"])), float(np.float32(frame["fy"]))
    cx0, cy0 = float(np.float32(frame["cx"])), float(np.float32(frame["cy"]))
    words = (w * h + 31) // 32
    cands = []
    for o, xyz in zip(objects, clouds):
        if not o["confirmed"] or o["state"] == 1 or o["last_kf"] != frame["stamp"] or len(xyz) < 30:
            continue
        n = len(xyz)
        stp = max(1, n // 3000)
        pts = np.asarray(xyz, np.float32)[::stp].astype(np.float64)
        tot = len(pts)
        org = np.asarray(o["cloud_org"], np.float64)
        p = (org + pts) - T[[3, 7, 11]]
        cx = T[0] * p[:, 0] + T[4] * p[:, 1] + T[8] * p[:, 2]
        cy = T[1] * p[:, 0] + T[5] * p[:, 1] + T[9] * p[:, 2]
        cz = T[2] * p[:, 0] + T[6] * p[:, 1] + T[10] * p[:, 2]
        front = cz >= 0.15
        cx, cy, cz = cx[front], cy[front], cz[front]
        ud = fx * cx / cz + cx0
        vd = fy * cy / cz + cy0
        inside = (ud >= 0) & (vd >= 0) & (ud < w) & (vd < h)
        trunc = bool((~inside).any())
        ud, vd, cz = ud[inside], vd[inside], cz[inside]
        d = depth[vd.astype(np.int64), ud.astype(np.int64)].astype(np.float64)
        vis = (d > 0) & ~(d < cz - 0.08)
        ud, vd, cz = ud[vis], vd[vis], cz[vis]
        nvis = len(cz)
        if tot == 0 or nvis < 12:
            continue
        vfrac = nvis / tot
        if vfrac < reenc_min_vis:
            continue
        rpx = 0.6 * voxel * fx / cz
        i0 = np.maximum(0, np.floor(ud - rpx).astype(np.int64))
        i1 = np.minimum(w - 1, np.floor(ud + rpx).astype(np.int64))
        j0 = np.maximum(0, np.floor(vd - rpx).astype(np.int64))
        j1 = np.minimum(h - 1, np.floor(vd + rpx).astype(np.int64))
        ok = (i0 <= i1) & (j0 <= j1)
        diff = np.zeros((h + 1, w + 1), np.int64)
        np.add.at(diff, (j0[ok], i0[ok]), 1)
        np.add.at(diff, (j0[ok], i1[ok] + 1), -1)
        np.add.at(diff, (j1[ok] + 1, i0[ok]), -1)
        np.add.at(diff, (j1[ok] + 1, i1[ok] + 1), 1)
        grid = (diff.cumsum(0).cumsum(1)[:h, :w] > 0).astype(np.uint8)
        if ((ud <= 2) | (vd <= 2) | (ud >= w - 3) | (vd >= h - 3)).any():
            trunc = True
        pad = np.pad(grid, 1)
        nb = sum(pad[1 + dy:1 + dy + h, 1 + dx:1 + dx + w].astype(np.int32)
                 for dy in (-1, 0, 1) for dx in (-1, 0, 1) if dy or dx)
        g2 = grid | ((grid == 0) & (nb >= 3)).astype(np.uint8)
        area = int(g2.sum())
        size_px = float(np.sqrt(float(area)))
        if size_px < reenc_min_px:
            continue
        zs = cz.astype(np.float32)
        zmed = float(np.partition(zs, nvis // 2)[nvis // 2])
        kap = view_kappa(float(np.float32(size_px)), trunc, zmed, float(np.float32(vfrac)), float(np.float32(cam_w)), **kp)
        need = bool(o["need_whole"])
        wk = float(o.get("whole_kappa", 0.0))
        if not need and kap < reenc_gain * wk:
            continue
        bits = np.packbits(g2.reshape(-1), bitorder="little")
        bits = np.pad(bits, (0, words * 4 - len(bits))).view(np.uint32)
        box = np.array([max(0.0, ud.min() - 2), max(0.0, vd.min() - 2), min(float(w), ud.max() + 2),
                        min(float(h), vd.max() + 2)], np.float32)
        cam = np.array([T[3], T[7], T[11], T[2], T[6], T[10]], np.float64)
        cands.append(((1e6 if need else 0.0) + kap / max(1.0, wk), o["id"], box, np.float32(kap), cam, bits))
    order = sorted(range(len(cands)), key=lambda i: (-cands[i][0], i))[:max(0, reenc_max)]
    sel = [cands[i] for i in order]
    return dict(id=np.array([c[1] for c in sel], np.uint32), box=np.array([c[2] for c in sel], np.float32).reshape(-1, 4),
                kappa=np.array([c[3] for c in sel], np.float32), cam=np.array([c[4] for c in sel]).reshape(-1, 6),
                bits=np.array([c[5] for c in sel], np.uint32).reshape(-1, words))
