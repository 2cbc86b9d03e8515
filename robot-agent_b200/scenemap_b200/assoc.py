"""Config-2 association stress workload and the ctypes binding of smg_assoc_* (include/smg.h).

Memory bank: 4096 cluster centres ~ N(0, 1)^D, each memory = centre + N(0, 0.1)^D,
L2-normalised, stored bf16; boxes with centres U over 20 x 20 x 2.5 m and extents U(0.05, 0.6)
m per axis.  Detections per frame: half are perturbed memory vectors (noise N(0, 0.015)^D,
renormalised, box = the memory's box jittered by N(0, 0.03) m and scaled by U(0.9, 1.1)),
half are fresh draws with random boxes.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .smg import _check, lib

_ready = False


def _lib():
    global _ready
    L = lib()
    if not _ready:
        vp = C.c_void_p
        L.smg_assoc_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(vp)]
        L.smg_assoc_destroy.argtypes = [vp]
        L.smg_assoc_match.argtypes = [vp, vp, vp, C.c_int, vp, vp, C.c_int, C.c_float, C.c_double, vp, vp, vp, vp, vp]
        L.smg_assoc_error.argtypes = [vp]
        L.smg_assoc_stamps.argtypes = [vp, C.c_int, C.POINTER(C.c_int64)]
        _ready = True
    return L


def to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bits (uint16)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def _norm(v):
    return v / np.linalg.norm(v, axis=1, keepdims=True)


def _boxes(rng, c, ext):
    return np.concatenate([c - ext / 2, c + ext / 2], 1).astype(np.float32)


class AssocWorkload:
    def __init__(self, seed: int, n_mem: int = 16384, n_det: int = 256, dim: int = 1152, n_centres: int = 4096):
        rng = np.random.default_rng(seed)
        self.rng, self.n_mem, self.n_det, self.dim = rng, n_mem, n_det, dim
        centres = rng.standard_normal((n_centres, dim), dtype=np.float32)
        cid = rng.integers(0, n_centres, n_mem)
        mem = _norm(centres[cid] + 0.1 * rng.standard_normal((n_mem, dim), dtype=np.float32))
        self.mem = to_bf16(mem)
        self.mem_f = mem.astype(np.float32)
        cen = rng.uniform([0, 0, 0], [20, 20, 2.5], (n_mem, 3))
        self.mem_box = _boxes(rng, cen, rng.uniform(0.05, 0.6, (n_mem, 3)))

    def frame(self, k: int):
        rng = np.random.default_rng((hash((k, 77)) & 0xFFFFFFFF) ^ self.n_mem)
        n = self.n_det
        npert = n // 2
        src = rng.integers(0, self.n_mem, npert)
        z = np.empty((n, self.dim), np.float32)
        z[:npert] = _norm(self.mem_f[src] + 0.015 * rng.standard_normal((npert, self.dim), dtype=np.float32))
        z[npert:] = _norm(rng.standard_normal((n - npert, self.dim), dtype=np.float32))
        mb = self.mem_box[src]
        c = (mb[:, :3] + mb[:, 3:]) / 2 + rng.normal(0, 0.03, (npert, 3))
        ext = (mb[:, 3:] - mb[:, :3]) * rng.uniform(0.9, 1.1, (npert, 3))
        box = np.empty((n, 6), np.float32)
        box[:npert] = _boxes(rng, c, ext)
        box[npert:] = _boxes(rng, rng.uniform([0, 0, 0], [20, 20, 2.5], (n - npert, 3)),
                             rng.uniform(0.05, 0.6, (n - npert, 3)))
        return to_bf16(z), box, src


class AssocGPU:
    """Device-resident bank + per-frame matching through smg_assoc_match."""

    def __init__(self, max_det: int, max_mem: int, dim: int, dev: int = 0):
        h = C.c_void_p()
        _check(_lib().smg_assoc_create(max_det, max_mem, dim, dev, C.byref(h)), "smg_assoc_create")
        self.h = h

    def close(self):
        if self.h:
            _lib().smg_assoc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def match(self, det, det_box, mem, mem_box, iou_min=0.1, cos_min=0.8, scores=None, stream=0):
        """All arguments are torch device tensors (bf16 bits as int16/uint16, boxes float32);
        returns device tensors (match int32, score float64, certified int32)."""
        import torch
        n_det, n_mem = det.shape[0], mem.shape[0]
        dev = det.device
        m = torch.empty(n_det, dtype=torch.int32, device=dev)
        s = torch.empty(n_det, dtype=torch.float64, device=dev)
        c = torch.empty(n_det, dtype=torch.int32, device=dev)
        vp = C.c_void_p
        _check(_lib().smg_assoc_match(self.h, vp(det.data_ptr()), vp(det_box.data_ptr()), n_det, vp(mem.data_ptr()),
                                      vp(mem_box.data_ptr()), n_mem, iou_min, cos_min, vp(m.data_ptr()), vp(s.data_ptr()),
                                      vp(c.data_ptr()), vp(scores.data_ptr() if scores is not None else 0), vp(stream)),
               "smg_assoc_match")
        return m, s, c

    def stamps(self, enable: bool):
        """Enable phase timestamps; returns the last record (8 x ns, %globaltimer)."""
        out = (C.c_int64 * 16)()
        _check(_lib().smg_assoc_stamps(self.h, 1 if enable else 0, out), "smg_assoc_stamps")
        return [int(v) for v in out]

    def error(self) -> int:
        return _check(_lib().smg_assoc_error(self.h), "smg_assoc_error")
