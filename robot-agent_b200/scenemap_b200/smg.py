"""Host-side binding of the B200 scenemap objprob update (ctypes over libsmg.so).

Mirrors the reference's C++ surface for one batch of independent maps: create the maps
(``ObjectMap(p)`` + ``Mapper2D``), push one keyframe per map (``Mapper2D::keyframe`` +
``ObjectMap::update`` + ``addPoints``), read objects / association / grid back.  The compute
runs only in the CUDA library; if it is missing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("SMG_LIB") or os.path.join(os.path.dirname(_HERE), "libsmg.so")

SMG_MEM_DEVICE, SMG_MEM_HOST = 0, 1
SMG_EMB_F32, SMG_EMB_BF16 = 0, 1
SMG_OK, SMG_ERR_ARGS, SMG_ERR_PARAM, SMG_ERR_CAPACITY, SMG_ERR_DEVICE, SMG_ERR_UNSUPPORTED = 0, -1, -2, -3, -4, -5
STAT_FIELDS = ["n_through", "n_obs", "n_wall", "n_wall_name", "n_ceil", "n_floor", "n_assoc", "n_new", "n_merge",
               "n_obj_struct", "n_reenc_req", "n_reenc_done", "n_blocked", "n_wall_tall", "n_so_big", "n_bridge"]


class SmgFrame(C.Structure):
    _fields_ = [("stamp", C.c_double), ("w", C.c_int32), ("h", C.c_int32), ("depth", C.c_void_p), ("label", C.c_void_p),
                ("fx", C.c_float), ("fy", C.c_float), ("cx", C.c_float), ("cy", C.c_float), ("T_mc", C.c_double * 12),
                ("T_bc", C.c_float * 12), ("base", C.c_double * 3), ("eef", C.c_double * 6), ("eef_base", C.c_float * 6),
                ("n_det", C.c_int32), ("det_label", C.c_void_p), ("box", C.c_void_p), ("cls", C.c_void_p),
                ("score", C.c_void_p), ("emb", C.c_void_p), ("emb_dtype", C.c_int32), ("grip", C.c_float * 2),
                ("mask_bits", C.c_void_p), ("mask_w", C.c_int32), ("mask_h", C.c_int32), ("mask_sx", C.c_float),
                ("mask_sy", C.c_float), ("mask_ox", C.c_float), ("mask_oy", C.c_float), ("img_w", C.c_int32),
                ("img_h", C.c_int32), ("depth_mm", C.c_void_p), ("rgba", C.c_void_p), ("wall_segs", C.c_void_p),
                ("n_wall_segs", C.c_int32)]


class SmgSnapObject(C.Structure):
    _fields_ = [("id", C.c_uint32), ("name_lab", C.c_int32), ("score", C.c_float), ("pos", C.c_double * 3),
                ("extent", C.c_double * 3), ("first_pos", C.c_double * 3), ("n_obs", C.c_uint32), ("last_seen", C.c_double),
                ("state", C.c_int32), ("structural", C.c_int32), ("movable", C.c_int32), ("n_points", C.c_int32),
                ("cloud_stamp", C.c_double)]


class SmgView(C.Structure):
    _fields_ = [("id", C.c_uint32), ("version", C.c_uint32), ("q", C.c_double), ("stamp", C.c_double),
                ("box", C.c_int32 * 4), ("det_box", C.c_int32 * 4), ("mask_area", C.c_float), ("depth_m", C.c_float),
                ("score", C.c_float), ("cam_T", C.c_double * 12), ("w", C.c_int32), ("h", C.c_int32)]


VIEW_MAX_SIDE = 256


class SmgReencReq(C.Structure):
    _fields_ = [("id", C.c_uint32), ("box", C.c_float * 4), ("kappa", C.c_float), ("cam", C.c_double * 6),
                ("mask_w", C.c_int32), ("mask_h", C.c_int32)]


class SmgObject(C.Structure):
    _fields_ = [("id", C.c_uint32), ("cls", C.c_int32), ("pos", C.c_double * 3), ("ext", C.c_double * 3),
                ("first_pos", C.c_double * 3), ("lo", C.c_double * 3), ("hi", C.c_double * 3), ("n_obs", C.c_uint32),
                ("first_seen", C.c_double), ("last_seen", C.c_double), ("state", C.c_int32), ("confirmed", C.c_int32),
                ("moved", C.c_int32), ("misses", C.c_int32), ("n_vis_miss", C.c_uint32), ("score", C.c_float),
                ("max_det_z", C.c_double), ("last_kf", C.c_double), ("appeared", C.c_int32), ("cloud_n", C.c_int32),
                ("cloud_version", C.c_uint32), ("cloud_org", C.c_double * 3), ("ap_ver", C.c_uint32),
                ("k_frag", C.c_double), ("n_views", C.c_int32), ("n_ap_obs", C.c_int32), ("need_whole", C.c_int32),
                ("P", C.c_double * 3), ("n_cams", C.c_int32), ("geo", C.c_int32), ("k_whole", C.c_double),
                ("n_whole", C.c_int32), ("held_by", C.c_int32),
                ("parent", C.c_uint32), ("parent_rel", C.c_double * 3), ("wall_like", C.c_int32), ("hide", C.c_int32),
                ("n_wall_obs", C.c_int32), ("fw", C.c_float)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"CUDA library not built: {LIB_PATH} (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        P, vp = C.POINTER, C.c_void_p
        L.smg_params_size.restype = C.c_int
        L.smg_params_default.argtypes = [vp]
        L.smg_params_apply.argtypes = [vp, C.c_char_p]
        L.smg_params_set_cloud.argtypes = [vp, C.c_double, C.c_int]
        L.smg_create.argtypes = [vp] + [C.c_int] * 11 + [P(vp)]
        L.smg_create_pooled.argtypes = [vp] + [C.c_int] * 12 + [P(vp)]
        L.smg_destroy.argtypes = [vp]
        L.smg_push_frames.argtypes = [vp, P(SmgFrame), C.c_int, C.c_int, vp]
        L.smg_get_objects.argtypes = [vp, C.c_int, P(SmgObject), C.c_int]
        L.smg_get_object_vectors.argtypes = [vp, C.c_int, C.c_int, vp, vp, vp, vp, C.c_int]
        L.smg_get_object_cloud.argtypes = [vp, C.c_int, C.c_int, vp, vp, C.c_int]
        L.smg_get_assoc.argtypes = [vp, C.c_int, vp, vp, vp, vp, C.c_int]
        L.smg_get_object_cloud_rgb.argtypes = [vp, C.c_int, C.c_int, vp, C.c_int]
        L.smg_get_views.argtypes = [vp, C.c_int, vp, vp, vp, vp, C.c_int]
        L.smg_get_assoc_all_async.argtypes = [vp, vp, C.POINTER(C.c_int64)]
        L.smg_set_text_model.argtypes = [vp, vp, vp, vp, vp]
        L.smg_get_object_name.argtypes = [vp, C.c_int, C.c_int, vp, vp, vp]
        L.smg_wait_read.argtypes = [vp, C.c_int64]
        L.smg_set_walls.argtypes = [vp, C.c_int]
        L.smg_snapshot.argtypes = [vp, vp, vp, C.c_int, vp, vp, C.c_int64, C.POINTER(C.c_int64)]
        L.smg_ply_header.argtypes = [C.c_int64, vp, C.c_int]
        L.smg_get_wall_segments.argtypes = [vp, C.c_int, vp, C.c_int]
        L.smg_wall_state.argtypes = [vp, C.c_int, vp, vp]
        L.smg_get_stats.argtypes = [vp, C.c_int, vp]
        L.smg_get_events.argtypes = [vp, C.c_int, vp, vp, vp, C.c_int]
        L.smg_get_grid.argtypes = [vp, C.c_int, vp, vp, vp]
        L.smg_get_keyframe.argtypes = [vp, C.c_int, vp]
        L.smg_error_word.argtypes = [vp]
        L.smg_last_error.restype = C.c_char_p
        L.smg_get_assoc_all.argtypes = [vp, vp]
        L.smg_get_reencode.argtypes = [vp, C.c_int, vp, vp, C.c_int]
        L.smg_debug_check.argtypes = [vp, vp]
        L.smg_timing_enable.argtypes = [vp, C.c_int]
        L.smg_timing_read.argtypes = [vp, vp, vp, vp]
        L.smg_kernel_launches.restype = C.c_int64
        L.smg_kernel_launches.argtypes = [vp]
        L.smg_get_work.argtypes = [vp, C.POINTER(C.c_int64), C.c_int]
        L.smg_set_reencode.argtypes = [vp, C.c_int]
        L.smg_set_object_embeddings.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, vp]
        L.smg_get_object_whole.argtypes = [vp, C.c_int, C.c_int, vp, P(C.c_double)]
        L.smg_plane_fit.argtypes = [vp, vp, C.c_int, C.c_int, C.c_double, vp, C.c_int, vp, vp]
        L.smg_plane_fit_noalloc.argtypes = [vp, vp, C.c_int, C.c_int, C.c_double, vp, C.c_int, vp, vp]
        _lib = L
    return _lib


EXPORTED = ["smg_params_set_cloud", "smg_params_size", "smg_params_default", "smg_params_apply", "smg_create", "smg_create_pooled", "smg_destroy", "smg_push_frames",
            "smg_get_objects", "smg_get_object_vectors", "smg_get_object_cloud", "smg_get_assoc", "smg_get_stats",
            "smg_get_events", "smg_get_grid", "smg_get_keyframe", "smg_error_word", "smg_last_error",
            "smg_kernel_launches", "smg_get_assoc_all", "smg_debug_check", "smg_timing_enable", "smg_timing_read",
           "smg_get_work", "smg_set_reencode", "smg_set_object_embeddings", "smg_get_object_whole", "smg_plane_fit", "smg_plane_fit_noalloc", "smg_occ_create", "smg_occ_destroy",
           "smg_occ_insert", "smg_occ_match", "smg_occ_track", "smg_occ_get_cells", "smg_assoc_create", "smg_assoc_destroy",
           "smg_assoc_match", "smg_assoc_error", "smg_assoc_stamps", "smg_label_loglik", "smg_name", "smg_get_reencode",
           "smg_get_object_cloud_rgb", "smg_get_views", "smg_get_assoc_all_async", "smg_wait_read",
           "smg_set_text_model", "smg_get_object_name", "smg_set_walls", "smg_get_wall_segments", "smg_wall_state",
           "smg_snapshot", "smg_ply_header"]

NUM_KERNELS = 18


def _ptr(a):
    return None if a is None else a.ctypes.data


class SmgError(RuntimeError):
    pass


def _check(rc, what):
    if rc < 0:
        raise SmgError(f"{what} rc={rc}: {lib().smg_last_error().decode()}")
    return rc


class Params:
    """smg_params as an opaque buffer (defaults of the reference structs + applyParams keys)."""

    def __init__(self, kv: str = ""):
        L = lib()
        self.buf = C.create_string_buffer(L.smg_params_size())
        _check(L.smg_params_default(self.buf), "smg_params_default")
        if kv:
            rc = L.smg_params_apply(self.buf, kv.encode())
            if rc > 0:
                raise SmgError(f"unknown parameter keys in {kv!r}")
            _check(rc, "smg_params_apply")


class Batch:
    def __init__(self, n_maps: int, max_objects: int = 256, emb_dim: int = 1152, max_w: int = 640, max_h: int = 480,
                 max_det: int = 32, grid=(512, 512, -256 + 60, -256 + 50), params: Params | None = None, dev: int = 0,
                 cloud_cap: int | None = None, max_clouds: int | None = None):
        L = lib()
        self.params = params or Params()
        if cloud_cap is not None:   # ObjectMap::setCloudParams (objmap.hpp:255-258)
            _check(L.smg_params_set_cloud(self.params.buf, 0.0, int(cloud_cap)), "smg_params_set_cloud")
        self.n_maps, self.max_objects, self.D, self.max_det = n_maps, max_objects, emb_dim, max_det
        self.max_w, self.max_h = max_w, max_h
        self.grid = grid
        h = C.c_void_p()
        self.max_clouds = max_clouds or max_objects
        _check(L.smg_create_pooled(self.params.buf, n_maps, max_objects, self.max_clouds, emb_dim, max_w, max_h, max_det,
                                   grid[0], grid[1], grid[2], grid[3], dev, C.byref(h)), "smg_create_pooled")
        self.h = h

    def close(self):
        if getattr(self, "h", None) and self.h.value:
            lib().smg_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def frame_struct(fr: dict, keep: list, emb_dtype: int = SMG_EMB_F32, ptrs: dict | None = None) -> SmgFrame:
        """smg_frame from a synth frame dict (host numpy arrays, or device pointers in `ptrs`)."""
        f = SmgFrame()
        f.stamp = fr["stamp"]
        f.w, f.h = fr["w"], fr["h"]
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
        dl = np.ascontiguousarray(fr["det_label"], np.uint16)
        bx = np.ascontiguousarray(fr["box"], np.float32)
        cl = np.ascontiguousarray(fr["cls"], np.int32)
        sc = np.ascontiguousarray(fr["score"], np.float32)
        keep += [dl, bx, cl, sc]
        f.det_label, f.box, f.cls, f.score = _ptr(dl), _ptr(bx), _ptr(cl), _ptr(sc)
        f.emb_dtype = emb_dtype
        grip = np.asarray(fr.get("grip", (1.0, 1.0)), np.float32).reshape(-1)
        f.grip[0], f.grip[1] = float(grip[0]), float(grip[1])
        f.img_w, f.img_h = fr.get("img_w", 0), fr.get("img_h", 0)
        if fr.get("mask_w"):
            f.mask_w, f.mask_h = fr["mask_w"], fr["mask_h"]
            f.mask_sx, f.mask_sy, f.mask_ox, f.mask_oy = fr["mask_affine"]
        if fr.get("wall_segs") is not None:   # n x (ax, ay, bx, by) map metres, host memory
            ws = np.ascontiguousarray(fr["wall_segs"], np.float64).reshape(-1, 4)
            buf = ws if len(ws) else np.zeros(4)   # an empty set is still a set: a non-null pointer
            keep.append(buf)
            f.wall_segs, f.n_wall_segs = buf.ctypes.data, len(ws)
        if ptrs is not None:
            f.depth, f.label, f.emb = ptrs["depth"], ptrs["label"], ptrs["emb"]
            f.mask_bits = ptrs.get("mask_bits")
            f.rgba = ptrs.get("rgba")
        else:
            if fr.get("rgba") is not None:
                rgba = np.ascontiguousarray(fr["rgba"], np.uint8)
                keep.append(rgba)
                f.rgba = _ptr(rgba)
            if fr.get("mask_bits") is not None:
                mb = np.ascontiguousarray(fr["mask_bits"], np.uint32)
                keep.append(mb)
                f.mask_bits = _ptr(mb)
            if fr.get("depth_mm") is not None:
                dmm = np.ascontiguousarray(fr["depth_mm"], np.uint16)
                keep.append(dmm)
                f.depth_mm = _ptr(dmm)
            depth = np.ascontiguousarray(fr["depth"], np.float32) if fr.get("depth_mm") is None else None
            label = np.ascontiguousarray(fr["label"], np.uint16)
            if emb_dtype == SMG_EMB_BF16:
                e32 = np.ascontiguousarray(fr["emb"], np.float32)
                emb = (e32.view(np.uint32) >> 16).astype(np.uint16)
            else:
                emb = np.ascontiguousarray(fr["emb"], np.float32)
            keep += [depth, label, emb]
            f.depth, f.label, f.emb = _ptr(depth), _ptr(label), (_ptr(emb) if n else None)
        return f

    def push(self, frames: list, where: int = SMG_MEM_HOST, emb_dtype: int = SMG_EMB_F32, stream: int = 0,
             structs=None):
        keep = []
        if structs is None:
            arr = (SmgFrame * len(frames))(*[self.frame_struct(fr, keep, emb_dtype) for fr in frames])
        else:
            arr = structs
        _check(lib().smg_push_frames(self.h, arr, len(arr), where, C.c_void_p(stream)), "smg_push_frames")
        self._keep = keep

    def objects(self, m: int = 0) -> list:
        L = lib()
        n = _check(L.smg_get_objects(self.h, m, None, 0), "smg_get_objects")
        arr = (SmgObject * max(n, 1))()
        L.smg_get_objects(self.h, m, arr, n)
        out = []
        for i in range(n):
            o = arr[i]
            d = {}
            for name, _ in SmgObject._fields_:
                v = getattr(o, name)
                d[name] = list(v) if hasattr(v, "__len__") else v
            out.append(d)
        return out

    def object_vectors(self, m: int, i: int):
        r = np.zeros(self.D, np.float32)
        views = np.zeros((8, self.D), np.uint16)
        vk = np.zeros(8, np.float32)
        vs = np.zeros(8, np.float64)
        nv = _check(lib().smg_get_object_vectors(self.h, m, i, _ptr(r), _ptr(views), _ptr(vk), _ptr(vs), 8),
                    "smg_get_object_vectors")
        return r, views[:nv], vk[:nv], vs[:nv]

    def object_cloud(self, m: int, i: int):
        n = _check(lib().smg_get_object_cloud(self.h, m, i, None, None, 0), "smg_get_object_cloud")
        xyz = np.zeros((max(n, 1), 3), np.float32)
        seq = np.zeros(max(n, 1), np.uint32)
        lib().smg_get_object_cloud(self.h, m, i, _ptr(xyz), _ptr(seq), n)
        return xyz[:n], seq[:n]

    def object_cloud_rgb(self, m: int, i: int):
        n = _check(lib().smg_get_object_cloud_rgb(self.h, m, i, None, 0), "smg_get_object_cloud_rgb")
        rgb = np.zeros((max(n, 1), 3), np.uint8)
        lib().smg_get_object_cloud_rgb(self.h, m, i, _ptr(rgb), n)
        return rgb[:n]

    def views(self, m: int = 0) -> list:
        """Best views the last keyframe of map m installed (smg_get_views), with their images."""
        L = lib()
        cap = self.max_det
        arr = (SmgView * cap)()
        S = VIEW_MAX_SIDE * VIEW_MAX_SIDE
        rgb = np.zeros((cap, S * 3), np.uint8)
        dep = np.zeros((cap, S), np.uint16)
        msk = np.zeros((cap, S), np.uint8)
        n = _check(L.smg_get_views(self.h, m, arr, _ptr(rgb), _ptr(dep), _ptr(msk), cap), "smg_get_views")
        out = []
        for v in range(n):
            o = arr[v]
            d = {}
            for name, _ in SmgView._fields_:
                x = getattr(o, name)
                d[name] = list(x) if hasattr(x, "__len__") else x
            w, h = o.w, o.h
            d["rgb"] = rgb[v, :w * h * 3].reshape(h, w, 3).copy()
            d["depth"] = dep[v, :w * h].reshape(h, w).copy()
            d["mask"] = msk[v, :w * h].reshape(h, w).copy()
            out.append(d)
        return out

    def assoc(self, m: int = 0):
        cap = self.max_det
        oid = np.zeros(cap, np.uint32)
        nv = np.zeros(cap, np.int32)
        ar = np.zeros(cap, np.float32)
        dm = np.zeros(cap, np.float32)
        n = _check(lib().smg_get_assoc(self.h, m, _ptr(oid), _ptr(nv), _ptr(ar), _ptr(dm), cap), "smg_get_assoc")
        return dict(obj_id=oid[:n], n_valid=nv[:n], area_px=ar[:n], depth_med=dm[:n])

    def stats(self, m: int = 0) -> dict:
        s = np.zeros(16, np.int64)
        _check(lib().smg_get_stats(self.h, m, _ptr(s)), "smg_get_stats")
        return {k: int(v) for k, v in zip(STAT_FIELDS, s)}

    def events(self, m: int = 0):
        cap = 1024
        t = np.zeros(cap, np.float64)
        i = np.zeros(cap, np.uint32)
        k = np.zeros(cap, np.int32)
        n = _check(lib().smg_get_events(self.h, m, _ptr(t), _ptr(i), _ptr(k), cap), "smg_get_events")
        return list(zip(t[:n].tolist(), i[:n].tolist(), k[:n].tolist()))

    def grid_cells(self, m: int = 0):
        gw, gh, x0, y0 = self.grid
        L = np.zeros((gh, gw), np.int16)
        seen = np.zeros((gh, gw), np.uint8)
        c8 = np.zeros((gh, gw), np.int8)
        _check(lib().smg_get_grid(self.h, m, _ptr(L), _ptr(seen), _ptr(c8)), "smg_get_grid")
        return dict(x0=x0, y0=y0, w=gw, h=gh, L=L, seen=seen, c8=c8)

    def keyframe(self, m: int = 0):
        o = np.zeros(3, np.int32)
        _check(lib().smg_get_keyframe(self.h, m, _ptr(o)), "smg_get_keyframe")
        return dict(inserted=int(o[0]), changed=int(o[1]), n_hits=int(o[2]))

    def reencode(self, m: int = 0) -> dict:
        """Whole-object re-encode requests of map m's last keyframe (smg_get_reencode), best first:
        id, box, kappa, cam and the row-major mask bits (ceil(w * h / 32) words per request)."""
        L = lib()
        n = _check(L.smg_get_reencode(self.h, m, None, None, 0), "smg_get_reencode")
        k = max(n, 1)
        stride = (self.max_w * self.max_h + 31) // 32
        reqs = (SmgReencReq * k)()
        bits = np.zeros((k, stride), np.uint32)
        _check(L.smg_get_reencode(self.h, m, reqs, _ptr(bits), n), "smg_get_reencode")
        nw = (reqs[0].mask_w * reqs[0].mask_h + 31) // 32 if n else 0
        return dict(id=np.array([reqs[r].id for r in range(n)], np.uint32),
                    box=np.array([list(reqs[r].box) for r in range(n)], np.float32).reshape(n, 4),
                    kappa=np.array([reqs[r].kappa for r in range(n)], np.float32),
                    cam=np.array([list(reqs[r].cam) for r in range(n)], np.float64).reshape(n, 6),
                    bits=bits[:n, :nw])

    def assoc_all(self) -> np.ndarray:
        out = np.zeros(self.n_maps * self.max_det, np.uint32)
        _check(lib().smg_get_assoc_all(self.h, _ptr(out)), "smg_get_assoc_all")
        return out.reshape(self.n_maps, self.max_det)

    def set_text_model(self, t: dict) -> None:
        """smg_set_text_model from a synth.text_model dict (host arrays, copied)."""
        x = {k: (np.ascontiguousarray(v) if isinstance(v, np.ndarray) else v) for k, v in t.items()}
        self._text_keep = x
        rows = x["text"].shape[0]
        from .text import SmgText
        st = SmgText()
        st.dim = x["text"].shape[1] if rows else self.D
        st.n_labels = x["n_labels"]
        st.rows = rows
        st.text = _ptr(x["text"]) if rows else None
        st.row_label = _ptr(x["row_label"]) if rows else None
        st.scale, st.bias = x["scale"], x["bias"]
        for k in ("log_prior", "ls_mu", "ls_sd", "parent"):
            setattr(st, k, _ptr(x[k]) if x.get(k) is not None else None)
        st.object_label = x["object_label"]
        opt = lambda k: _ptr(x[k]) if x.get(k) is not None else None
        _check(lib().smg_set_text_model(self.h, C.byref(st), opt("kinds"), opt("so_shape"), opt("flat_ok")), "smg_set_text_model")
        self._nlab = x["n_labels"]

    def object_name(self, m: int, i: int) -> dict:
        n = self._nlab
        post = np.zeros(n, np.float32)
        lab = np.zeros(3, np.int32)
        val = np.zeros(3, np.float32)
        k = _check(lib().smg_get_object_name(self.h, m, i, _ptr(post), _ptr(lab), _ptr(val)), "smg_get_object_name")
        return dict(has_post=k > 0, post=post, name_lab=int(lab[0]), top_lab=int(lab[1]), rolled=int(lab[2]), name_p=float(val[0]),
                    top_p=float(val[1]), name_H=float(val[2]))

    def set_walls(self, on: bool = True) -> None:
        """Extract wall segments from every map's grid before each object update (sm_push_image)."""
        _check(lib().smg_set_walls(self.h, 1 if on else 0), "smg_set_walls")

    def wall_segments(self, m: int):
        """(n, 4) segments of map m's last extraction, or None before the first one."""
        L = lib()
        n = L.smg_get_wall_segments(self.h, m, None, 0)
        if n == -1:
            return None
        _check(n, "smg_get_wall_segments")
        out = np.zeros((max(n, 1), 4), np.float64)
        L.smg_get_wall_segments(self.h, m, _ptr(out), n)
        return out[:n]

    def wall_state(self, m: int, pose) -> np.ndarray | None:
        """The wall state vector (56 floats) of map m at pose (x, y, yaw), or None."""
        p = np.ascontiguousarray(pose, np.float64)
        out = np.zeros(56, np.float32)
        rc = lib().smg_wall_state(self.h, m, _ptr(p), _ptr(out))
        if rc == -1:
            return None
        _check(rc, "smg_wall_state")
        return out

    def snapshot(self, points: bool = True) -> dict:
        """The object-memory snapshot of every map: map_off (n_maps + 1), objects (list of dicts,
        map after map), point_off and the packed 15-byte PLY vertex records (bytes)."""
        L = lib()
        moff = np.zeros(self.n_maps + 1, np.int32)
        tot = C.c_int64(0)
        n = _check(L.smg_snapshot(self.h, _ptr(moff), None, 0, None, None, 0, C.byref(tot)), "smg_snapshot")
        recs = (SmgSnapObject * max(n, 1))()
        poff = np.zeros(n + 1, np.int64)
        pts = np.zeros(max(int(tot.value), 1) * 15, np.uint8)
        _check(L.smg_snapshot(self.h, _ptr(moff), recs, n, _ptr(poff), _ptr(pts) if points else None, int(tot.value) if points else 0,
                              C.byref(tot)), "smg_snapshot")
        objs = []
        for k in range(n):
            r = recs[k]
            objs.append({name: (list(getattr(r, name)) if isinstance(getattr(r, name), C.Array) else getattr(r, name))
                         for name, _ in SmgSnapObject._fields_})
        return dict(map_off=moff, objects=objs, point_off=poff, points=pts[:int(tot.value) * 15].tobytes() if points else None)

    @staticmethod
    def ply_header(n: int) -> bytes:
        L = lib()
        k = L.smg_ply_header(n, None, 0)
        buf = C.create_string_buffer(k)
        L.smg_ply_header(n, buf, k)
        return buf.raw[:k]

    def assoc_all_async(self, out_ptr: int) -> int:
        """Enqueue the read of every map's association into host memory at out_ptr (n_maps x
        max_det uint32, pinned for an asynchronous copy); returns a ticket for wait_read."""
        t = C.c_int64(0)
        _check(lib().smg_get_assoc_all_async(self.h, C.c_void_p(out_ptr), C.byref(t)), "smg_get_assoc_all_async")
        return t.value

    def wait_read(self, ticket: int) -> None:
        _check(lib().smg_wait_read(self.h, ticket), "smg_wait_read")

    def set_object_embeddings(self, maps, ids, emb, stream: int = 0):
        """Whole-object embeddings answering the last keyframe's re-encode requests (host arrays)."""
        maps = np.ascontiguousarray(maps, np.int32)
        ids = np.ascontiguousarray(ids, np.uint32)
        emb = np.ascontiguousarray(emb, np.float32).reshape(len(ids), self.D)
        _check(lib().smg_set_object_embeddings(self.h, _ptr(maps), _ptr(ids), _ptr(emb), len(ids), self.D, SMG_MEM_HOST,
                                                C.c_void_p(stream)), "smg_set_object_embeddings")

    def object_whole(self, m: int, i: int):
        r = np.zeros(self.D, np.float32)
        k = C.c_double(0)
        n = _check(lib().smg_get_object_whole(self.h, m, i, _ptr(r), C.byref(k)), "smg_get_object_whole")
        return r, k.value, n

    def set_reencode(self, on: bool):
        _check(lib().smg_set_reencode(self.h, 1 if on else 0), "smg_set_reencode")

    def timing(self, on: bool = True):
        _check(lib().smg_timing_enable(self.h, 1 if on else 0), "smg_timing_enable")

    def timing_read(self) -> dict:
        ms = np.zeros(NUM_KERNELS, np.float64)
        n = np.zeros(NUM_KERNELS, np.int64)
        names = (C.c_char_p * NUM_KERNELS)()
        _check(lib().smg_timing_read(self.h, _ptr(ms), _ptr(n), names), "smg_timing_read")
        return {names[k].decode(): (float(ms[k]), int(n[k])) for k in range(NUM_KERNELS)}

    def debug_check(self):
        out = np.zeros(3, np.uint64)
        _check(lib().smg_debug_check(self.h, _ptr(out)), "smg_debug_check")
        return [int(v) for v in out]

    def error_word(self) -> int:
        return _check(lib().smg_error_word(self.h), "smg_error_word")

    def launches(self) -> int:
        return int(lib().smg_kernel_launches(self.h))

    WORK_KEYS = ("obs_px", "det", "vec16", "upd", "cloud_pts", "scan_px", "scan_pts", "cells", "h2d")

    def work(self) -> dict:
        """Cumulative work counters (smg_get_work) as a dict keyed by WORK_KEYS."""
        out = (C.c_int64 * len(self.WORK_KEYS))()
        _check(lib().smg_get_work(self.h, out, len(self.WORK_KEYS)), "smg_get_work")
        return dict(zip(self.WORK_KEYS, (int(v) for v in out)))


def plane_fit(clouds, tau, seeds, max_iters=64, device="cuda:0", entry="smg_plane_fit"):
    """apPlaneFit on a list of (n, 3) float32 point sets through the batched C entry point.

    Returns an (n_sets, 10) float64 array: ok, n0, n1, n2, thick, inl, zmed, zlo, zhi, hspan.
    `entry` names the C entry point: "smg_plane_fit" (stream-ordered scratch allocation) or
    "smg_plane_fit_noalloc" (static scratch, no device allocation, <= 65536 points)."""
    import numpy as np
    import torch
    dev = torch.device(device)
    pts = [np.ascontiguousarray(c, dtype=np.float32).reshape(-1, 3) for c in clouds]
    off = np.zeros(len(pts) + 1, np.int32)
    off[1:] = np.cumsum([len(p) for p in pts])
    xyz = torch.from_numpy(np.concatenate(pts) if pts else np.zeros((0, 3), np.float32)).to(dev)
    off_d = torch.from_numpy(off).to(dev)
    seeds_d = torch.from_numpy(np.asarray(seeds, np.uint64).view(np.int64)).to(dev)
    out = torch.empty((len(pts), 10), dtype=torch.float64, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    fn = getattr(lib(), entry)
    _check(fn(C.c_void_p(xyz.data_ptr()), C.c_void_p(off_d.data_ptr()), len(pts), int(off[-1]), float(tau),
              C.c_void_p(seeds_d.data_ptr()), int(max_iters), C.c_void_p(out.data_ptr()), C.c_void_p(st)), entry)
    torch.cuda.synchronize(dev)
    return out.cpu().numpy()
