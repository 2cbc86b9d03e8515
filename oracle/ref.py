"""ctypes binding of the oracle libraries (TEST INFRASTRUCTURE ONLY).

``_ref/libscenemap_ref.so`` is the reference scenemap code compiled in place by
``oracle/Makefile`` plus ``ref_driver.cpp``; ``_ref/libport.so`` is the C restatement in
``port/``.  Only tests, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use this
module, as the checker or the timed CPU baseline; the product never imports it.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "libscenemap_ref.so")
PORT_SO = os.path.join(HERE, "_ref", "libport.so")


class RfSnap(C.Structure):
    _fields_ = [("id", C.c_uint32), ("name_lab", C.c_int32), ("score", C.c_float), ("pos", C.c_double * 3),
                ("extent", C.c_double * 3), ("first_pos", C.c_double * 3), ("n_obs", C.c_uint32), ("last_seen", C.c_double),
                ("state", C.c_int32), ("structural", C.c_int32), ("movable", C.c_int32), ("n_points", C.c_int32),
                ("cloud_stamp", C.c_double)]


class RfFrame(C.Structure):
    _fields_ = [("stamp", C.c_double), ("w", C.c_int), ("h", C.c_int), ("depth", C.POINTER(C.c_float)),
                ("label", C.POINTER(C.c_uint16)), ("fx", C.c_float), ("fy", C.c_float), ("cx", C.c_float),
                ("cy", C.c_float), ("T_mc", C.c_double * 12), ("T_bc", C.c_float * 12), ("base", C.c_double * 3),
                ("eef", C.c_double * 6), ("eef_base", C.c_float * 6), ("n_det", C.c_int),
                ("det_label", C.POINTER(C.c_uint16)), ("box", C.POINTER(C.c_float)), ("cls", C.POINTER(C.c_int32)),
                ("score", C.POINTER(C.c_float)), ("emb", C.POINTER(C.c_float)), ("emb_dim", C.c_int),
                ("grid_only", C.c_int), ("grip", C.c_float * 2), ("mask_bits", C.POINTER(C.c_uint32)),
                ("mask_w", C.c_int), ("mask_h", C.c_int), ("mask_sx", C.c_float), ("mask_sy", C.c_float),
                ("mask_ox", C.c_float), ("mask_oy", C.c_float), ("img_w", C.c_int), ("img_h", C.c_int),
                ("depth_mm", C.POINTER(C.c_uint16)), ("rgba", C.POINTER(C.c_uint8)),
                ("wall_segs", C.POINTER(C.c_double)), ("n_wall_segs", C.c_int)]


class RfView(C.Structure):
    _fields_ = [("id", C.c_uint32), ("version", C.c_uint32), ("q", C.c_double), ("stamp", C.c_double),
                ("box", C.c_int32 * 4), ("det_box", C.c_int32 * 4), ("mask_area", C.c_float), ("depth_m", C.c_float),
                ("score", C.c_float), ("cam_T", C.c_double * 12), ("w", C.c_int32), ("h", C.c_int32)]


class RfObj(C.Structure):
    _fields_ = [("id", C.c_uint32), ("cls", C.c_int32), ("pos", C.c_double * 3), ("ext", C.c_double * 3),
                ("first_pos", C.c_double * 3), ("lo", C.c_double * 3), ("hi", C.c_double * 3), ("n_obs", C.c_uint32),
                ("first_seen", C.c_double), ("last_seen", C.c_double), ("state", C.c_int32), ("confirmed", C.c_int32),
                ("moved", C.c_int32), ("misses", C.c_int32), ("n_vis_miss", C.c_uint32), ("score", C.c_float),
                ("max_det_z", C.c_double), ("last_kf", C.c_double), ("gone_t", C.c_double), ("appeared", C.c_int32),
                ("mv_cnt", C.c_int32), ("trk_pos", C.c_double * 3), ("trk_t", C.c_double), ("trk_step", C.c_double * 2),
                ("moving_t", C.c_double), ("move_from_t", C.c_double), ("first_miss", C.c_double),
                ("miss_cam", C.c_double * 3), ("last_miss_cam", C.c_double * 3), ("last_miss_fwd", C.c_double * 3),
                ("cloud_n", C.c_int32), ("cloud_version", C.c_uint32), ("cloud_org", C.c_double * 3),
                ("ap_ver", C.c_uint32), ("k_frag", C.c_double), ("k_whole", C.c_double), ("n_views", C.c_int32),
                ("n_ap_obs", C.c_int32), ("n_wall_obs", C.c_int32), ("n_struct_look", C.c_int32),
                ("need_whole", C.c_int32), ("n_whole", C.c_int32), ("P", C.c_double * 3), ("n_cams", C.c_int32),
                ("geo", C.c_int32), ("drop", C.c_int32), ("hide", C.c_int32), ("held_by", C.c_int32),
                ("parent", C.c_uint32), ("parent_rel", C.c_double * 3), ("wall_like", C.c_int32), ("fw", C.c_float)]


STAT_FIELDS = ["n_through", "n_obs", "n_wall", "n_wall_name", "n_ceil", "n_floor", "n_assoc", "n_new", "n_merge",
               "n_obj_struct", "n_reenc_req", "n_reenc_done", "n_blocked", "n_wall_tall", "n_so_big", "n_bridge"]


class RfStats(C.Structure):
    _fields_ = [(n, C.c_long) for n in STAT_FIELDS]


_ref = None


def available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib():
    global _ref
    if _ref is None:
        if not available():
            raise RuntimeError(f"reference oracle not built: {REF_SO}")
        L = C.CDLL(REF_SO)
        P = C.POINTER
        L.ref_create.restype = C.c_void_p
        L.ref_create.argtypes = [C.c_char_p, C.c_double, C.c_int, C.c_int, P(C.c_float), C.c_int]
        L.ref_destroy.argtypes = [C.c_void_p]
        L.ref_set_reencode.argtypes = [C.c_void_p, C.c_int]
        L.ref_frame.argtypes = [C.c_void_p, P(RfFrame)]
        L.ref_n_objects.argtypes = [C.c_void_p]
        L.ref_objects.argtypes = [C.c_void_p, P(RfObj), C.c_int]
        L.ref_object_vectors.argtypes = [C.c_void_p, C.c_int, P(C.c_float), C.c_int, P(C.c_uint16), P(C.c_float),
                                         P(C.c_double), C.c_int]
        L.ref_object_cloud.argtypes = [C.c_void_p, C.c_int, P(C.c_float), P(C.c_uint32), C.c_int]
        L.ref_object_cloud_rgb.argtypes = [C.c_void_p, C.c_int, P(C.c_uint8), C.c_int]
        L.ref_set_text_model.argtypes = [C.c_void_p, P(C.c_float), P(C.c_int32), C.c_int, C.c_int, C.c_float, C.c_float, C.c_int,
                                         P(C.c_float), P(C.c_float), P(C.c_float), P(C.c_int32), C.c_int, P(C.c_uint8),
                                         P(C.c_uint8), P(C.c_uint8)]
        L.ref_object_name.argtypes = [C.c_void_p, C.c_int, P(C.c_float), C.c_int, P(C.c_int32), P(C.c_float)]
        L.ref_views.argtypes = [C.c_void_p, P(RfView), P(C.c_uint8), P(C.c_uint16), P(C.c_uint8), C.c_int]
        L.ref_assoc.argtypes = [C.c_void_p, P(C.c_uint32), P(C.c_int32), P(C.c_float), P(C.c_float), C.c_int]
        L.ref_n_points.argtypes = [C.c_void_p]
        L.ref_points.argtypes = [C.c_void_p, C.c_int, P(C.c_uint32), P(C.c_int32), P(C.c_float), P(C.c_int32), C.c_int]
        L.ref_stats.argtypes = [C.c_void_p, P(RfStats)]
        L.ref_n_events.argtypes = [C.c_void_p]
        L.ref_events.argtypes = [C.c_void_p, P(C.c_double), P(C.c_uint32), P(C.c_int32), C.c_int]
        L.ref_kf.argtypes = [C.c_void_p, P(C.c_int32)]
        L.ref_reenc.argtypes = [C.c_void_p, P(C.c_uint32), P(C.c_float), P(C.c_float), P(C.c_double), P(C.c_uint32),
                                C.c_int]
        L.ref_reenc_words.argtypes = [C.c_void_p]
        L.ref_add_whole_views.argtypes = [C.c_void_p, P(C.c_uint32), P(C.c_float), C.c_int, C.c_int, C.c_double]
        L.ref_object_whole.argtypes = [C.c_void_p, C.c_int, P(C.c_float), C.c_int, P(C.c_double)]
        L.ref_grid_geom.argtypes = [C.c_void_p, P(C.c_int32)]
        L.ref_grid_cells.argtypes = [C.c_void_p, P(C.c_int16), P(C.c_uint8), P(C.c_int8)]
        L.ref_occ_create.restype = C.c_void_p
        L.ref_occ_create.argtypes = [P(C.c_float)]
        L.ref_occ_destroy.argtypes = [C.c_void_p]
        L.ref_occ_insert.argtypes = [C.c_void_p, C.c_float, C.c_float, P(C.c_float), P(C.c_float), C.c_int,
                                     P(C.c_float), P(C.c_float), C.c_int, P(C.c_float), P(C.c_float), P(C.c_float),
                                     P(C.c_float), C.c_int, P(C.c_double)]
        L.ref_occ_geom.argtypes = [C.c_void_p, P(C.c_int32)]
        L.ref_occ_cells.argtypes = [C.c_void_p, P(C.c_int16), P(C.c_uint8), P(C.c_int8), P(C.c_float)]
        L.ref_make_scan.argtypes = [C.c_int, C.c_int, P(C.c_float), C.c_float, C.c_float, C.c_float, C.c_float,
                                    P(C.c_float), P(C.c_float)] + [P(C.c_float)] * 8 + [P(C.c_int16), C.c_float,
                                                                                          P(C.c_int32), P(C.c_float)]
        L.ref_plane_fit.argtypes = [P(C.c_float), C.c_int, C.c_double, C.c_uint64, C.c_int, P(C.c_double)]
        L.ref_ap_seed.restype = C.c_uint64
        L.ref_ap_seed.argtypes = [C.c_uint64, C.c_uint64]
        L.ref_to_f16.argtypes = [P(C.c_float), P(C.c_uint16), C.c_int]
        L.ref_voxel_key.restype = C.c_uint64
        L.ref_voxel_key.argtypes = [C.c_float, C.c_float, C.c_float, C.c_float]
        L.ref_contact.restype = C.c_double
        L.ref_contact.argtypes = [P(C.c_float), C.c_int, P(C.c_float), C.c_int, C.c_double]
        L.ref_set_walls.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        L.ref_snapshot.argtypes = [C.c_void_p, P(RfSnap), C.c_int]
        L.ref_snapshot_ply.restype = C.c_long
        L.ref_snapshot_ply.argtypes = [C.c_void_p, C.c_int, P(C.c_uint8), C.c_long]
        L.ref_wall_segments.argtypes = [C.c_void_p, P(C.c_double), C.c_int]
        L.ref_wall_state.argtypes = [C.c_void_p, P(C.c_double), P(C.c_float)]
        L.ref_wall_segments_grid.argtypes = [P(C.c_int8), C.c_int, C.c_int, C.c_double, C.c_double, C.c_double, P(C.c_double),
                                             C.c_int, C.c_int, C.c_double, P(C.c_double), P(C.c_double), C.c_int]
        _ref = L
    return _ref


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t))


def make_rf_frame(fr: dict, keep: list) -> RfFrame:
    """Fill an RfFrame from a synth frame dict; `keep` holds the arrays alive."""
    f = RfFrame()
    f.stamp = fr["stamp"]
    f.w, f.h = fr["w"], fr["h"]
    if fr.get("depth_mm") is not None:   # millimetre depth instead of metres
        dmm = np.ascontiguousarray(fr["depth_mm"], np.uint16)
        keep.append(dmm)
        f.depth_mm = _p(dmm, C.c_uint16)
    else:
        depth = np.ascontiguousarray(fr["depth"], np.float32)
        keep.append(depth)
        f.depth = _p(depth, C.c_float)
    if fr.get("label") is not None:
        label = np.ascontiguousarray(fr["label"], np.uint16)
        keep.append(label)
        f.label = _p(label, C.c_uint16)
    if fr.get("mask_bits") is not None:   # the detector's bit masks on their own grid
        mb = np.ascontiguousarray(fr["mask_bits"], np.uint32)
        keep.append(mb)
        f.mask_bits = _p(mb, C.c_uint32)
        f.mask_w, f.mask_h = fr["mask_w"], fr["mask_h"]
        f.mask_sx, f.mask_sy, f.mask_ox, f.mask_oy = fr["mask_affine"]
    f.img_w, f.img_h = fr.get("img_w", 0), fr.get("img_h", 0)
    if fr.get("rgba") is not None:
        rgba = np.ascontiguousarray(fr["rgba"], np.uint8)
        keep.append(rgba)
        f.rgba = _p(rgba, C.c_uint8)
    if fr.get("wall_segs") is not None:   # ObjFrame::wall_segs; an empty set is still a set
        ws = np.ascontiguousarray(fr["wall_segs"], np.float64).reshape(-1, 4)
        buf = ws if len(ws) else np.zeros(4)
        keep.append(buf)
        f.wall_segs, f.n_wall_segs = _p(buf, C.c_double), len(ws)
    f.fx, f.fy, f.cx, f.cy = fr["fx"], fr["fy"], fr["cx"], fr["cy"]
    for i in range(12):
        f.T_mc[i] = fr["T_mc"][i]
        f.T_bc[i] = fr["T_bc"][i]
    for i in range(3):
        f.base[i] = fr["base"][i]
    eef = np.asarray(fr["eef"], np.float64).reshape(-1)
    eefb = np.asarray(fr["eef_base"], np.float32).reshape(-1)
    for i in range(6):
        f.eef[i] = eef[i]
        f.eef_base[i] = eefb[i]
    n = int(fr["n_det"])
    f.n_det = n
    if n:
        dl = np.ascontiguousarray(fr["det_label"], np.uint16)
        bx = np.ascontiguousarray(fr["box"], np.float32)
        cl = np.ascontiguousarray(fr["cls"], np.int32)
        sc = np.ascontiguousarray(fr["score"], np.float32)
        em = np.ascontiguousarray(fr["emb"], np.float32)
        keep += [dl, bx, cl, sc, em]
        f.det_label = _p(dl, C.c_uint16)
        f.box = _p(bx, C.c_float)
        f.cls = _p(cl, C.c_int32)
        f.score = _p(sc, C.c_float)
        f.emb = _p(em, C.c_float)
        f.emb_dim = int(fr["emb_dim"])
    f.grid_only = 0
    grip = np.asarray(fr.get("grip", (1.0, 1.0)), np.float32).reshape(-1)
    f.grip[0], f.grip[1] = float(grip[0]), float(grip[1])
    return f


class RefMap:
    """One reference scenemap (ObjectMap + Mapper2D) driven frame by frame."""

    def __init__(self, obj_kv: str = "", voxel: float = 0.02, cloud_cap: int = 8000, grid=(0.05, 0.85, -0.4, -4.0, 4.0),
                 grid_on: bool = True, attach_on: bool = False):
        L = ref_lib()
        g = np.asarray(grid, np.float32)
        self._h = L.ref_create(obj_kv.encode(), voxel, cloud_cap, 1 if grid_on else 0, _p(g, C.c_float),
                               1 if attach_on else 0)

    def __del__(self):
        if getattr(self, "_h", None):
            ref_lib().ref_destroy(self._h)
            self._h = None

    def set_reencode(self, on: bool) -> None:
        ref_lib().ref_set_reencode(self._h, 1 if on else 0)

    def frame(self, fr: dict) -> None:
        keep = []
        f = make_rf_frame(fr, keep)
        rc = ref_lib().ref_frame(self._h, C.byref(f))
        if rc != 0:
            raise RuntimeError(f"ref_frame rc={rc}")

    def objects(self) -> list:
        L = ref_lib()
        n = L.ref_n_objects(self._h)
        arr = (RfObj * max(n, 1))()
        L.ref_objects(self._h, arr, n)
        out = []
        for i in range(n):
            o = arr[i]
            d = {}
            for name, _ in RfObj._fields_:
                v = getattr(o, name)
                d[name] = list(v) if hasattr(v, "__len__") else v
            out.append(d)
        return out

    def object_vectors(self, i: int, D: int):
        L = ref_lib()
        r = np.zeros(D, np.float32)
        views = np.zeros((5, D), np.uint16)
        vk = np.zeros(5, np.float32)
        vs = np.zeros(5, np.float64)
        nv = L.ref_object_vectors(self._h, i, _p(r, C.c_float), D, _p(views, C.c_uint16), _p(vk, C.c_float),
                                  _p(vs, C.c_double), 5)
        return r, views[:nv], vk[:nv], vs[:nv]

    def object_whole(self, i: int, D: int):
        """r_whole (zeros when empty), k_whole and n_whole of object i."""
        r = np.zeros(D, np.float32)
        k = C.c_double(0)
        n = ref_lib().ref_object_whole(self._h, i, _p(r, C.c_float), D, C.byref(k))
        return r, k.value, n

    def object_cloud(self, i: int):
        L = ref_lib()
        n = L.ref_object_cloud(self._h, i, None, None, 0)
        xyz = np.zeros((max(n, 1), 3), np.float32)
        seq = np.zeros(max(n, 1), np.uint32)
        L.ref_object_cloud(self._h, i, _p(xyz, C.c_float), _p(seq, C.c_uint32), n)
        return xyz[:n], seq[:n]

    def snapshot(self) -> list:
        """sm_snapshot's object list (exportable objects, object order) as dicts."""
        L = ref_lib()
        n = L.ref_snapshot(self._h, None, 0)
        recs = (RfSnap * max(n, 1))()
        L.ref_snapshot(self._h, recs, n)
        out = []
        for k in range(n):
            r = recs[k]
            out.append({name: (list(getattr(r, name)) if isinstance(getattr(r, name), C.Array) else getattr(r, name))
                        for name, _ in RfSnap._fields_})
        return out

    def snapshot_ply(self, n: int) -> bytes:
        """dsg_save's point file (plyBytes) of the n-th exportable object."""
        L = ref_lib()
        k = L.ref_snapshot_ply(self._h, n, None, 0)
        buf = np.zeros(max(k, 1), np.uint8)
        L.ref_snapshot_ply(self._h, n, _p(buf, C.c_uint8), k)
        return buf[:k].tobytes()

    def set_walls(self, grid) -> None:
        """Wall extraction before every object update (sm_push_image's refreshWalls and bridges),
        on the reference grid laid over the window grid = (w, h, x0, y0) cells."""
        w, h, x0, y0 = grid
        assert ref_lib().ref_set_walls(self._h, 1, int(x0), int(y0), int(w), int(h)) == 0

    def wall_segments(self):
        """sm_snap_wall_segments: (n, 4) extracted segments, or None before the first extraction."""
        L = ref_lib()
        n = L.ref_wall_segments(self._h, None, 0)
        if n < 0:
            return None
        out = np.zeros((max(n, 1), 4), np.float64)
        L.ref_wall_segments(self._h, _p(out, C.c_double), n)
        return out[:n]

    def wall_state(self, pose) -> np.ndarray | None:
        """sm_snap_wall_state at pose (x, y, yaw): the wall state vector (56 floats)."""
        p = np.ascontiguousarray(pose, np.float64)
        out = np.zeros(56, np.float32)
        if ref_lib().ref_wall_state(self._h, _p(p, C.c_double), _p(out, C.c_float)) != 0:
            return None
        return out

    def set_text_model(self, t: dict) -> None:
        """ObjectMap::setTextModel + setClassKinds from a synth.text_model dict."""
        self._text = {k: (np.ascontiguousarray(v) if isinstance(v, np.ndarray) else v) for k, v in t.items()}
        x = self._text
        rows = x["text"].shape[0]
        dim = x["text"].shape[1] if rows else 0
        opt = lambda k, ct: _p(x[k], ct) if x.get(k) is not None else None
        rc = ref_lib().ref_set_text_model(self._h, _p(x["text"], C.c_float), _p(x["row_label"], C.c_int32), rows, dim, x["scale"],
                                          x["bias"], x["n_labels"], opt("log_prior", C.c_float), opt("ls_mu", C.c_float),
                                          opt("ls_sd", C.c_float), opt("parent", C.c_int32), x["object_label"],
                                          opt("kinds", C.c_uint8), opt("so_shape", C.c_uint8), opt("flat_ok", C.c_uint8))
        assert rc == 0
        self._nlab = x["n_labels"]

    def object_name(self, i: int) -> dict:
        n = self._nlab
        post = np.zeros(n, np.float32)
        lab = np.zeros(3, np.int32)
        val = np.zeros(3, np.float32)
        k = ref_lib().ref_object_name(self._h, i, _p(post, C.c_float), n, _p(lab, C.c_int32), _p(val, C.c_float))
        return dict(has_post=k > 0, post=post, name_lab=int(lab[0]), top_lab=int(lab[1]), rolled=int(lab[2]), name_p=float(val[0]),
                    top_p=float(val[1]), name_H=float(val[2]))

    def object_cloud_rgb(self, i: int):
        L = ref_lib()
        n = L.ref_object_cloud_rgb(self._h, i, None, 0)
        rgb = np.zeros((max(n, 1), 3), np.uint8)
        L.ref_object_cloud_rgb(self._h, i, _p(rgb, C.c_uint8), n)
        return rgb[:n]

    def views(self) -> dict:
        """The glue's views map after the last frame: id -> view dict with its images."""
        L = ref_lib()
        n = L.ref_views(self._h, None, None, None, None, 0)
        arr = (RfView * max(n, 1))()
        S = 256 * 256
        rgb = np.zeros((max(n, 1), S * 3), np.uint8)
        dep = np.zeros((max(n, 1), S), np.uint16)
        msk = np.zeros((max(n, 1), S), np.uint8)
        L.ref_views(self._h, arr, _p(rgb, C.c_uint8), _p(dep, C.c_uint16), _p(msk, C.c_uint8), n)
        out = {}
        for v in range(n):
            o = arr[v]
            d = {}
            for name, _ in RfView._fields_:
                x = getattr(o, name)
                d[name] = list(x) if hasattr(x, "__len__") else x
            w, h = o.w, o.h
            d["rgb"] = rgb[v, :w * h * 3].reshape(h, w, 3).copy()
            d["depth"] = dep[v, :w * h].reshape(h, w).copy()
            d["mask"] = msk[v, :w * h].reshape(h, w).copy()
            out[o.id] = d
        return out

    def assoc(self):
        L = ref_lib()
        cap = 256
        oid = np.zeros(cap, np.uint32)
        nv = np.zeros(cap, np.int32)
        ar = np.zeros(cap, np.float32)
        dm = np.zeros(cap, np.float32)
        n = L.ref_assoc(self._h, _p(oid, C.c_uint32), _p(nv, C.c_int32), _p(ar, C.c_float), _p(dm, C.c_float), cap)
        return dict(obj_id=oid[:n], n_valid=nv[:n], area_px=ar[:n], depth_med=dm[:n])

    def points(self) -> list:
        L = ref_lib()
        out = []
        for j in range(L.ref_n_points(self._h)):
            n = L.ref_points(self._h, j, None, None, None, None, 0)
            oid = C.c_uint32()
            det = C.c_int32()
            xyz = np.zeros((max(n, 1), 3), np.float32)
            px = np.zeros((max(n, 1), 2), np.int32)
            L.ref_points(self._h, j, C.byref(oid), C.byref(det), _p(xyz, C.c_float), _p(px, C.c_int32), n)
            out.append(dict(obj_id=oid.value, det=det.value, xyz=xyz[:n], px=px[:n]))
        return out

    def stats(self) -> dict:
        s = RfStats()
        ref_lib().ref_stats(self._h, C.byref(s))
        return {n: getattr(s, n) for n in STAT_FIELDS}

    def events(self):
        L = ref_lib()
        n = L.ref_n_events(self._h)
        t = np.zeros(max(n, 1), np.float64)
        i = np.zeros(max(n, 1), np.uint32)
        k = np.zeros(max(n, 1), np.int32)
        L.ref_events(self._h, _p(t, C.c_double), _p(i, C.c_uint32), _p(k, C.c_int32), n)
        return list(zip(t[:n].tolist(), i[:n].tolist(), k[:n].tolist()))

    def reenc(self) -> dict:
        """Re-encode requests of the last keyframe (ObjectMap::buildReencode), best first."""
        L = ref_lib()
        n = L.ref_reenc(self._h, None, None, None, None, None, 0)
        nw = L.ref_reenc_words(self._h)
        k = max(n, 1)
        ids = np.zeros(k, np.uint32)
        box = np.zeros((k, 4), np.float32)
        kap = np.zeros(k, np.float32)
        cam = np.zeros((k, 6), np.float64)
        bits = np.zeros((k, max(nw, 1)), np.uint32)
        L.ref_reenc(self._h, _p(ids, C.c_uint32), _p(box, C.c_float), _p(kap, C.c_float), _p(cam, C.c_double),
                    _p(bits, C.c_uint32), n)
        return dict(id=ids[:n], box=box[:n], kappa=kap[:n], cam=cam[:n], bits=bits[:n, :nw])

    def add_whole_views(self, ids, emb, stamp: float) -> int:
        """Answer the last keyframe's requests (sm_set_object_embeddings): one L2 embedding per id."""
        ids = np.ascontiguousarray(ids, np.uint32)
        emb = np.ascontiguousarray(emb, np.float32)
        return ref_lib().ref_add_whole_views(self._h, _p(ids, C.c_uint32), _p(emb, C.c_float), len(ids),
                                             emb.shape[1] if emb.ndim == 2 else 0, stamp)

    def kf(self):
        o = np.zeros(3, np.int32)
        ref_lib().ref_kf(self._h, _p(o, C.c_int32))
        return dict(inserted=int(o[0]), changed=int(o[1]), n_hits=int(o[2]))

    def grid(self):
        L = ref_lib()
        g = np.zeros(4, np.int32)
        if L.ref_grid_geom(self._h, _p(g, C.c_int32)) != 0:
            return None
        x0, y0, w, h = (int(v) for v in g)
        Lq = np.zeros((h, w), np.int16)
        seen = np.zeros((h, w), np.uint8)
        c8 = np.zeros((h, w), np.int8)
        L.ref_grid_cells(self._h, _p(Lq, C.c_int16), _p(seen, C.c_uint8), _p(c8, C.c_int8))
        return dict(x0=x0, y0=y0, w=w, h=h, L=Lq, seen=seen, c8=c8)


# ---------------------------------------------------------------- C restatement (port/)
_port = None


def port_available() -> bool:
    return os.path.exists(PORT_SO)


def port_lib():
    global _port
    if _port is None:
        L = C.CDLL(PORT_SO)
        P = C.POINTER
        L.op_ap_seed.restype = C.c_uint64
        L.op_ap_seed.argtypes = [C.c_uint64, C.c_uint64]
        L.op_f2h.restype = C.c_uint16
        L.op_f2h.argtypes = [C.c_float]
        L.op_h2f.restype = C.c_float
        L.op_h2f.argtypes = [C.c_uint16]
        L.op_to_f16.argtypes = [P(C.c_float), P(C.c_uint16), C.c_int]
        L.op_voxel_key.restype = C.c_uint64
        L.op_voxel_key.argtypes = [C.c_float, C.c_float, C.c_float, C.c_float]
        L.op_contact.restype = C.c_double
        L.op_contact.argtypes = [P(C.c_float), C.c_int, P(C.c_float), C.c_int, C.c_double]
        L.op_plane_fit.argtypes = [P(C.c_float), C.c_int, C.c_double, C.c_uint64, C.c_int, P(C.c_double)]
        L.op_fast_atan2.restype = C.c_float
        L.op_fast_atan2.argtypes = [C.c_float, C.c_float]
        _port = L
    return _port


def plane_fit(xyz, tau: float, seed: int, max_iters: int = 64, impl: str = "port") -> np.ndarray:
    """apPlaneFit of an (n, 3) float32 cloud: 10 doubles (ok, n0, n1, n2, thick, inl, zmed, zlo,
    zhi, hspan) from the restatement (impl="port") or the compiled reference (impl="ref")."""
    a = np.ascontiguousarray(xyz, np.float32).reshape(-1, 3)
    out = np.zeros(10, np.float64)
    if impl == "port":
        port_lib().op_plane_fit(_p(a, C.c_float), len(a), tau, seed, max_iters, _p(out, C.c_double))
    else:
        ref_lib().ref_plane_fit(_p(a, C.c_float), len(a), tau, seed, max_iters, _p(out, C.c_double))
    return out


def ap_seed(a: int, b: int, impl: str = "port") -> int:
    return int(port_lib().op_ap_seed(a, b) if impl == "port" else ref_lib().ref_ap_seed(a, b))


def contact(cloud, pts, cell: float, impl: str = "port") -> float:
    c = np.ascontiguousarray(cloud, np.float32).reshape(-1, 3)
    p = np.ascontiguousarray(pts, np.float32).reshape(-1, 3)
    fn = port_lib().op_contact if impl == "port" else ref_lib().ref_contact
    return float(fn(_p(c, C.c_float), len(c), _p(p, C.c_float), len(p), cell))


def to_f16(x, impl: str = "port") -> np.ndarray:
    a = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = np.zeros(len(a), np.uint16)
    fn = port_lib().op_to_f16 if impl == "port" else ref_lib().ref_to_f16
    fn(_p(a, C.c_float), _p(out, C.c_uint16), len(a))
    return out


def voxel_key(x: float, y: float, z: float, inv: float, impl: str = "port") -> int:
    fn = port_lib().op_voxel_key if impl == "port" else ref_lib().ref_voxel_key
    return int(fn(x, y, z, inv))


# ---------------------------------------------------------------- config 3: grid + matcher
def _lround(x: np.ndarray) -> np.ndarray:
    """C lround for x >= 0 (halves away from zero), exact: floor, then compare the remainder."""
    r = np.floor(x)
    return (r + (x - r >= 0.5)).astype(np.int64)


class RefOcc:
    """The reference OccGrid (grid.cpp), compiled in place, with the config-3 parameters."""

    def __init__(self, res=0.05, l_hit=0.85, l_miss=-0.4, l_min=-5.0, l_max=5.0):
        g5 = np.array([res, l_hit, l_miss, l_min, l_max], np.float32)
        self.res = res
        self.g = ref_lib().ref_occ_create(_p(g5, C.c_float))

    def __del__(self):
        if getattr(self, "g", None):
            ref_lib().ref_occ_destroy(self.g)
            self.g = None

    def insert(self, hits, free, pose, match=None, normals=None, origin=(0.0, 0.0)) -> int:
        def xy(a):
            a = np.zeros((0, 2), np.float32) if a is None else np.ascontiguousarray(a, np.float32).reshape(-1, 2)
            return np.ascontiguousarray(a[:, 0]), np.ascontiguousarray(a[:, 1]), len(a)
        hx, hy, nh = xy(hits)
        fx, fy, nf = xy(free)
        mx, my, nm = xy(match)
        mnx, mny, _ = xy(normals) if normals is not None else (None, None, 0)
        P = np.ascontiguousarray(pose, np.float64)
        fp = lambda a: _p(a, C.c_float) if a is not None else None
        return int(ref_lib().ref_occ_insert(self.g, origin[0], origin[1], fp(hx), fp(hy), nh, fp(fx), fp(fy), nf, fp(mx),
                                            fp(my), fp(mnx), fp(mny), nm, _p(P, C.c_double)))

    def cells(self) -> dict:
        g4 = np.zeros(4, np.int32)
        ref_lib().ref_occ_geom(self.g, _p(g4, C.c_int32))
        x0, y0, w, h = (int(v) for v in g4)
        n = w * h
        L, seen, c8, prob = np.zeros(n, np.int16), np.zeros(n, np.uint8), np.zeros(n, np.int8), np.zeros(n, np.float32)
        if n:
            ref_lib().ref_occ_cells(self.g, _p(L, C.c_int16), _p(seen, C.c_uint8), _p(c8, C.c_int8), _p(prob, C.c_float))
        q = _lround(prob.astype(np.float64) * 65535.0).astype(np.uint16)
        sh = (h, w)
        return {"L": L.reshape(sh), "seen": seen.reshape(sh), "c8": c8.reshape(sh), "prob": prob.reshape(sh),
                "q": q.reshape(sh), "x0": x0, "y0": y0}


def csm(cells: dict, hits, pose0, lin_half=6, ang_half=20, ang_step=None, w_t=10.0, w_r=0.1, res=0.05, pmin=0.1):
    """Restated correlative scan match (oracle/port/csm_port.c) on a grid snapshot from
    RefOcc.cells(): (best index, best score, best pose)."""
    import math
    L = port_lib()
    P = C.POINTER
    if not getattr(L, "_csm_ready", False):
        L.op_csm.argtypes = [P(C.c_uint16), C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint16, C.c_float, P(C.c_float),
                             P(C.c_float), C.c_int, P(C.c_double), C.c_int, C.c_int, C.c_double, C.c_double, C.c_double,
                             P(C.c_int32), P(C.c_double), P(C.c_double)]
        L._csm_ready = True
    ang_step = math.radians(0.5) if ang_step is None else ang_step
    q = np.ascontiguousarray(cells["q"], np.uint16)
    h, w = q.shape
    a = np.ascontiguousarray(hits, np.float32).reshape(-1, 2)
    hx, hy = np.ascontiguousarray(a[:, 0]), np.ascontiguousarray(a[:, 1])
    p0 = np.ascontiguousarray(pose0, np.float64)
    bi, bs, bp = np.zeros(1, np.int32), np.zeros(1), np.zeros(3)
    q_out = int(_lround(np.array([float(np.float32(pmin)) * 65535.0]))[0])
    L.op_csm(_p(q, C.c_uint16) if q.size else None, w, h, cells["x0"], cells["y0"], q_out, res, _p(hx, C.c_float),
             _p(hy, C.c_float), len(a), _p(p0, C.c_double), lin_half, ang_half, ang_step, w_t, w_r, _p(bi, C.c_int32),
             _p(bs, C.c_double), _p(bp, C.c_double))
    return int(bi[0]), float(bs[0]), bp


# ---------------------------------------------------------------- text model (apLabelLogLik, apName)
def label_loglik(text, row_label, n_labels, scale, bias, z):
    L = ref_lib()
    P = C.POINTER
    L.ref_label_loglik.argtypes = [C.c_int, C.c_int, C.c_int, P(C.c_float), P(C.c_int32), C.c_float, C.c_float,
                                   P(C.c_float), C.c_int, P(C.c_float)]
    t = np.ascontiguousarray(text, np.float32)
    rl = np.ascontiguousarray(row_label, np.int32)
    zz = np.ascontiguousarray(z, np.float32).reshape(-1, t.shape[1])
    out = np.zeros((len(zz), n_labels), np.float32)
    L.ref_label_loglik(t.shape[1], n_labels, len(t), _p(t, C.c_float), _p(rl, C.c_int32), scale, bias, _p(zz, C.c_float),
                       len(zz), _p(out, C.c_float))
    return out


def name(text, row_label, n_labels, scale, bias, log_prior, ls_mu, ls_sd, parent, object_label, whole_w, name_wmax,
         size_w, name_tau, L_frag, lw_frag, L_whole, lw_whole, L_ext, L_geo, size):
    """apName of one object (ref_name): (post, name_lab, name_p, top_lab, top_p, name_H, rolled, named)."""
    L = ref_lib()
    P = C.POINTER
    L.ref_name.argtypes = [C.c_int, C.c_int, C.c_int, P(C.c_float), P(C.c_int32), C.c_float, C.c_float, P(C.c_float),
                           P(C.c_float), P(C.c_float), P(C.c_int32), C.c_int, C.c_double, C.c_double, C.c_double,
                           C.c_double, P(C.c_float), C.c_double, P(C.c_float), C.c_double, P(C.c_float), P(C.c_float),
                           C.c_double, P(C.c_float), P(C.c_double)]
    f = lambda a: None if a is None else _p(np.ascontiguousarray(a, np.float32), C.c_float)
    keep = [np.ascontiguousarray(a, np.float32) for a in (text, log_prior, ls_mu, ls_sd, L_frag, L_whole, L_ext, L_geo)
            if a is not None]
    t = np.ascontiguousarray(text, np.float32)
    rl = np.ascontiguousarray(row_label, np.int32)
    par = None if parent is None else np.ascontiguousarray(parent, np.int32)
    arrs = {}
    for k, a in (("lp", log_prior), ("mu", ls_mu), ("sd", ls_sd), ("lf", L_frag), ("lwh", L_whole), ("le", L_ext), ("lg", L_geo)):
        arrs[k] = None if a is None else np.ascontiguousarray(a, np.float32)
    fp = lambda k: None if arrs[k] is None else _p(arrs[k], C.c_float)
    post = np.zeros(n_labels, np.float32)
    f6 = np.zeros(6)
    named = L.ref_name(t.shape[1], n_labels, len(t), _p(t, C.c_float), _p(rl, C.c_int32), scale, bias, fp("lp"), fp("mu"),
                       fp("sd"), None if par is None else _p(par, C.c_int32), object_label, whole_w, name_wmax, size_w,
                       name_tau, fp("lf"), lw_frag, fp("lwh"), lw_whole, fp("le"), fp("lg"), size, _p(post, C.c_float),
                       _p(f6, C.c_double))
    del keep
    return post, int(f6[0]), float(f6[1]), int(f6[2]), float(f6[3]), float(f6[4]), int(f6[5]), bool(named)


def wall_segments_grid(cells: np.ndarray, res: float, ox: float, oy: float, rects=(), mode: int = 0, th: float = 0.0):
    """walls.hpp on a caller's export8 grid (h, w): mode 0 wallSegments -> (n, 4); 1 wallAngle ->
    float; 2 wallSegmentsAtAngle(th) -> (n, 4).  rects: ignore areas (x0, y0, x1, y1)."""
    L = ref_lib()
    c = np.ascontiguousarray(cells, np.int8)
    h, w = c.shape
    rv = np.ascontiguousarray(np.asarray(rects, np.float64).reshape(-1, 4))
    rp = _p(rv, C.c_double) if len(rv) else None
    ang = C.c_double(0.0)
    n = L.ref_wall_segments_grid(_p(c, C.c_int8), w, h, res, ox, oy, rp, len(rv), mode, th, C.byref(ang), None, 0)
    if mode == 1:
        return ang.value
    out = np.zeros((max(n, 1), 4), np.float64)
    L.ref_wall_segments_grid(_p(c, C.c_int8), w, h, res, ox, oy, rp, len(rv), mode, th, None, _p(out, C.c_double), n)
    return out[:n]
