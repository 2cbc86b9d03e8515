"""ctypes binding of the standalone occupancy grid + correlative scan matcher (smg_occ_*).

Mirrors scenemap's OccGrid (grid.hpp) for the insert and the reference's configured
real-time correlative scan matcher for the search; see include/smg.h.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .smg import SmgError, _check, lib

_ready = False


class OccParams(C.Structure):
    _fields_ = [("res", C.c_float), ("l_hit", C.c_float), ("l_miss", C.c_float), ("l_min", C.c_float),
                ("l_max", C.c_float), ("pmin", C.c_float), ("pmax", C.c_float)]


class Scan2(C.Structure):
    _fields_ = [("ox", C.c_float), ("oy", C.c_float), ("n_match", C.c_int32),
                ("mx", C.POINTER(C.c_float)), ("my", C.POINTER(C.c_float)), ("mnx", C.POINTER(C.c_float)),
                ("mny", C.POINTER(C.c_float)), ("n_hit", C.c_int32), ("hx", C.POINTER(C.c_float)),
                ("hy", C.POINTER(C.c_float)), ("n_free", C.c_int32), ("fx", C.POINTER(C.c_float)),
                ("fy", C.POINTER(C.c_float))]


class CsmParams(C.Structure):
    _fields_ = [("linear_window", C.c_double), ("angular_window", C.c_double), ("linear_step", C.c_double),
                ("angular_step", C.c_double), ("translation_weight", C.c_double), ("rotation_weight", C.c_double)]


def config3_csm(res: float = 0.05) -> CsmParams:
    """Config-3 search: +-0.3 m x +-0.3 m x +-10 deg at 0.05 m / 0.5 deg (13 x 13 x 41), with the
    reference's delta-cost weights (carto_2d.lua:19-20: translation 10, rotation 0.1)."""
    import math
    return CsmParams(0.3, math.radians(10.0), res, math.radians(0.5), 10.0, 0.1)


def _lib():
    global _ready
    L = lib()
    if not _ready:
        vp = C.c_void_p
        P = C.POINTER
        L.smg_occ_create.argtypes = [P(OccParams), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P(vp)]
        L.smg_occ_destroy.argtypes = [vp]
        L.smg_occ_insert.argtypes = [vp, P(Scan2), P(C.c_double), C.c_int, P(C.c_int32), vp]
        L.smg_occ_match.argtypes = [vp, P(Scan2), P(C.c_double), P(CsmParams), C.c_int, P(C.c_double), P(C.c_int32),
                                    P(C.c_double), vp]
        L.smg_occ_track.argtypes = [vp, P(Scan2), P(C.c_double), P(CsmParams), C.c_int, P(C.c_double), P(C.c_int32),
                                    P(C.c_double), P(C.c_int32), vp]
        L.smg_occ_get_cells.argtypes = [vp, C.c_int, P(C.c_int16), P(C.c_uint8), P(C.c_int8), P(C.c_uint16)]
        _ready = True
    return L


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float)) if a is not None and len(a) else None


def make_scan(hits=None, free=None, match=None, normals=None, origin=(0.0, 0.0), keep=None) -> Scan2:
    """Scan2 from (n, 2) float32 arrays; `keep` collects the arrays that must outlive the call."""
    keep = keep if keep is not None else []
    s = Scan2()
    s.ox, s.oy = origin
    cols = []
    for arr in (match, normals, hits, free):
        if arr is None or len(arr) == 0:
            cols.append((None, None, 0))
            continue
        a = np.ascontiguousarray(arr, np.float32).reshape(-1, 2)
        x, y = np.ascontiguousarray(a[:, 0]), np.ascontiguousarray(a[:, 1])
        keep += [x, y]
        cols.append((x, y, len(a)))
    (mx, my, nm), (nx, ny, _), (hx, hy, nh), (fx, fy, nf) = cols
    s.n_match, s.mx, s.my, s.mnx, s.mny = nm, _fp(mx), _fp(my), _fp(nx), _fp(ny)
    s.n_hit, s.hx, s.hy = nh, _fp(hx), _fp(hy)
    s.n_free, s.fx, s.fy = nf, _fp(fx), _fp(fy)
    return s


class OccBatch:
    """n_maps independent fixed-window grids on one GPU."""

    def __init__(self, n_maps: int = 1, grid=(1024, 1024, -100, -100), res=0.05, l_hit=0.85, l_miss=-0.4, l_min=-5.0,
                 l_max=5.0, pmin=0.1, pmax=0.9, max_points=4096, dev=0):
        L = _lib()
        self.p = OccParams(res, l_hit, l_miss, l_min, l_max, pmin, pmax)
        self.M, (self.W, self.H, self.X0, self.Y0) = n_maps, grid
        h = C.c_void_p()
        _check(L.smg_occ_create(C.byref(self.p), n_maps, self.W, self.H, self.X0, self.Y0, max_points, dev, C.byref(h)),
               "smg_occ_create")
        self.h = h

    def close(self):
        if self.h:
            _lib().smg_occ_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _scans(scans):
        keep = []
        arr = (Scan2 * len(scans))()
        for i, sc in enumerate(scans):
            arr[i] = make_scan(sc.get("hits"), sc.get("free"), sc.get("match"), sc.get("normals"),
                               sc.get("origin", (0.0, 0.0)), keep)
        return arr, keep

    def insert(self, scans, poses, stream=0):
        arr, keep = self._scans(scans)
        P = np.ascontiguousarray(poses, np.float64).reshape(-1, 3)
        ch = np.zeros(len(scans), np.int32)
        _check(_lib().smg_occ_insert(self.h, arr, P.ctypes.data_as(C.POINTER(C.c_double)), len(scans),
                                     ch.ctypes.data_as(C.POINTER(C.c_int32)), C.c_void_p(stream)), "smg_occ_insert")
        return ch

    def match(self, scans, pose0, csm: CsmParams, stream=0):
        arr, keep = self._scans(scans)
        n = len(scans)
        P = np.ascontiguousarray(pose0, np.float64).reshape(-1, 3)
        po, idx, sc = np.zeros((n, 3)), np.zeros(n, np.int32), np.zeros(n)
        _check(_lib().smg_occ_match(self.h, arr, P.ctypes.data_as(C.POINTER(C.c_double)), C.byref(csm), n,
                                    po.ctypes.data_as(C.POINTER(C.c_double)), idx.ctypes.data_as(C.POINTER(C.c_int32)),
                                    sc.ctypes.data_as(C.POINTER(C.c_double)), C.c_void_p(stream)), "smg_occ_match")
        return po, idx, sc

    def track(self, scans, pose0, csm: CsmParams, stream=0):
        arr, keep = self._scans(scans)
        n = len(scans)
        P = np.ascontiguousarray(pose0, np.float64).reshape(-1, 3)
        po, idx, sc, ch = np.zeros((n, 3)), np.zeros(n, np.int32), np.zeros(n), np.zeros(n, np.int32)
        _check(_lib().smg_occ_track(self.h, arr, P.ctypes.data_as(C.POINTER(C.c_double)), C.byref(csm), n,
                                    po.ctypes.data_as(C.POINTER(C.c_double)), idx.ctypes.data_as(C.POINTER(C.c_int32)),
                                    sc.ctypes.data_as(C.POINTER(C.c_double)), ch.ctypes.data_as(C.POINTER(C.c_int32)),
                                    C.c_void_p(stream)), "smg_occ_track")
        return po, idx, sc, ch

    def cells(self, m=0):
        n = self.W * self.H
        L, seen, c8, q = np.zeros(n, np.int16), np.zeros(n, np.uint8), np.zeros(n, np.int8), np.zeros(n, np.uint16)
        _check(_lib().smg_occ_get_cells(self.h, m, L.ctypes.data_as(C.POINTER(C.c_int16)),
                                        seen.ctypes.data_as(C.POINTER(C.c_uint8)), c8.ctypes.data_as(C.POINTER(C.c_int8)),
                                        q.ctypes.data_as(C.POINTER(C.c_uint16))), "smg_occ_get_cells")
        sh = (self.H, self.W)
        return {"L": L.reshape(sh), "seen": seen.reshape(sh), "c8": c8.reshape(sh), "q": q.reshape(sh),
                "x0": self.X0, "y0": self.Y0}
