"""ctypes binding of the text-model entry points (smg_label_loglik, smg_name; include/smg.h)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from .smg import _check, lib

_ready = False


class SmgText(C.Structure):
    _fields_ = [("dim", C.c_int32), ("n_labels", C.c_int32), ("rows", C.c_int32), ("text", C.c_void_p),
                ("row_label", C.c_void_p), ("scale", C.c_float), ("bias", C.c_float), ("log_prior", C.c_void_p),
                ("ls_mu", C.c_void_p), ("ls_sd", C.c_void_p), ("parent", C.c_void_p), ("object_label", C.c_int32)]


class NameParams(C.Structure):
    _fields_ = [("whole_w", C.c_double), ("name_wmax", C.c_double), ("size_w", C.c_double), ("name_tau", C.c_double)]


def _lib():
    global _ready
    L = lib()
    if not _ready:
        vp = C.c_void_p
        L.smg_label_loglik.argtypes = [C.POINTER(SmgText), vp, C.c_int, vp, vp]
        L.smg_name.argtypes = [C.POINTER(SmgText), C.POINTER(NameParams), C.c_int] + [vp] * 10 + [vp]
        _ready = True
    return L


class TextModel:
    """ApText on the device (objprob.hpp:40-54)."""

    def __init__(self, text, row_label, n_labels, scale=111.83257, bias=-16.766876, log_prior=None, ls_mu=None,
                 ls_sd=None, parent=None, object_label=-1, device="cuda:0"):
        import torch
        t = lambda a, dt: None if a is None else torch.from_numpy(np.ascontiguousarray(a, dt)).to(device)
        self.text = t(text, np.float32)
        self.row_label = t(row_label, np.int32)
        self.log_prior, self.ls_mu, self.ls_sd = t(log_prior, np.float32), t(ls_mu, np.float32), t(ls_sd, np.float32)
        self.parent = t(parent, np.int32)
        ptr = lambda x: x.data_ptr() if x is not None else None
        self.s = SmgText(self.text.shape[1], n_labels, self.text.shape[0], ptr(self.text), ptr(self.row_label), scale, bias,
                         ptr(self.log_prior), ptr(self.ls_mu), ptr(self.ls_sd), ptr(self.parent), object_label)
        self.n_labels, self.device = n_labels, device

    def loglik(self, z):
        import torch
        zz = torch.from_numpy(np.ascontiguousarray(z, np.float32).reshape(-1, self.s.dim)).to(self.device)
        out = torch.empty((zz.shape[0], self.n_labels), dtype=torch.float32, device=self.device)
        _check(_lib().smg_label_loglik(C.byref(self.s), C.c_void_p(zz.data_ptr()), zz.shape[0], C.c_void_p(out.data_ptr()),
                                       None), "smg_label_loglik")
        torch.cuda.synchronize()
        return out.cpu().numpy()

    def name(self, params: NameParams, size, L_frag=None, lw_frag=None, L_whole=None, lw_whole=None, L_ext=None,
             L_geo=None):
        """Batched apName: every array has a leading object axis; returns (post, lab3, val3)."""
        import torch
        n = len(size)
        d = lambda a, dt: None if a is None else torch.from_numpy(np.ascontiguousarray(a, dt)).to(self.device)
        ins = [d(L_frag, np.float32), d(lw_frag, np.float64), d(L_whole, np.float32), d(lw_whole, np.float64),
               d(L_ext, np.float32), d(L_geo, np.float32), d(size, np.float64)]
        post = torch.empty((n, self.n_labels), dtype=torch.float32, device=self.device)
        lab = torch.empty((n, 3), dtype=torch.int32, device=self.device)
        val = torch.empty((n, 3), dtype=torch.float32, device=self.device)
        ptrs = [C.c_void_p(x.data_ptr()) if x is not None else None for x in ins]
        _check(_lib().smg_name(C.byref(self.s), C.byref(params), n, *ptrs, C.c_void_p(post.data_ptr()),
                               C.c_void_p(lab.data_ptr()), C.c_void_p(val.data_ptr()), None), "smg_name")
        torch.cuda.synchronize()
        return post.cpu().numpy(), lab.cpu().numpy(), val.cpu().numpy()
