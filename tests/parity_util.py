"""Shared comparison of the B200 batch against the reference oracle (tests only)."""
from __future__ import annotations

import numpy as np

EXACT_FIELDS = ["id", "cls", "n_obs", "state", "confirmed", "moved", "misses", "n_vis_miss", "appeared", "cloud_n",
                "cloud_version", "ap_ver", "n_views", "n_ap_obs", "need_whole", "n_cams", "geo", "held_by", "parent",
                "n_whole", "wall_like", "hide", "n_wall_obs", "fw"]
FLOAT_FIELDS = ["pos", "ext", "first_pos", "lo", "hi", "first_seen", "last_seen", "max_det_z", "last_kf", "k_frag",
                "P", "cloud_org", "parent_rel", "k_whole"]


def compare_objects(ref_objs: list, gpu_objs: list, rel: float = 1e-5) -> list:
    """Differences between two object lists (reference order); empty list when they agree."""
    errs = []
    if len(ref_objs) != len(gpu_objs):
        errs.append(f"object count ref={len(ref_objs)} gpu={len(gpu_objs)}")
        return errs
    for i, (r, g) in enumerate(zip(ref_objs, gpu_objs)):
        for f in EXACT_FIELDS:
            if r[f] != g[f]:
                errs.append(f"obj[{i}] id={r['id']} {f}: ref={r[f]} gpu={g[f]}")
        for f in FLOAT_FIELDS:
            a = np.asarray(r[f], np.float64)
            b = np.asarray(g[f], np.float64)
            tol = rel * np.maximum(1.0, np.abs(a))
            if np.any(np.abs(a - b) > tol):
                errs.append(f"obj[{i}] id={r['id']} {f}: ref={a.tolist()} gpu={b.tolist()}")
    return errs


def compare_grid(ref_g: dict, gpu_g: dict) -> list:
    """Per global cell index: log-odds, seen flag and export8 value must be identical."""
    errs = []
    if ref_g is None:
        return errs
    gx0, gy0, gw, gh = gpu_g["x0"], gpu_g["y0"], gpu_g["w"], gpu_g["h"]
    rx0, ry0, rw, rh = ref_g["x0"], ref_g["y0"], ref_g["w"], ref_g["h"]
    # every seen reference cell must lie in the GPU window
    rs = ref_g["seen"].astype(bool)
    ys, xs = np.nonzero(rs)
    gxs, gys = xs + rx0 - gx0, ys + ry0 - gy0
    if len(xs) and (gxs.min() < 0 or gys.min() < 0 or gxs.max() >= gw or gys.max() >= gh):
        errs.append("reference grid reaches outside the GPU window")
        return errs
    # overlap region
    ox0, oy0 = max(gx0, rx0), max(gy0, ry0)
    ox1, oy1 = min(gx0 + gw, rx0 + rw), min(gy0 + gh, ry0 + rh)
    R = lambda a: a[oy0 - ry0:oy1 - ry0, ox0 - rx0:ox1 - rx0]
    G = lambda a: a[oy0 - gy0:oy1 - gy0, ox0 - gx0:ox1 - gx0]
    for k in ("L", "seen", "c8"):
        a, b = R(ref_g[k]), G(gpu_g[k])
        if not np.array_equal(a, b):
            d = np.argwhere(a != b)
            errs.append(f"grid {k}: {len(d)} cells differ, first at {d[0].tolist()} ref={a[tuple(d[0])]} gpu={b[tuple(d[0])]}")
    # GPU cells outside the reference grid must be untouched
    seen_out = gpu_g["seen"].sum() - G(gpu_g["seen"]).sum()
    if seen_out:
        errs.append(f"grid: {seen_out} GPU cells seen outside the reference grid")
    return errs


def compare_frame(ref, gpu, m: int, D: int, deep: bool = False) -> list:
    errs = []
    ra, ga = ref.assoc(), gpu.assoc(m)
    if not np.array_equal(ra["obj_id"], ga["obj_id"]):
        errs.append(f"assoc obj_id ref={ra['obj_id'].tolist()} gpu={ga['obj_id'].tolist()}")
    if not np.array_equal(ra["n_valid"], ga["n_valid"]):
        errs.append(f"assoc n_valid ref={ra['n_valid'].tolist()} gpu={ga['n_valid'].tolist()}")
    if not np.array_equal(ra["area_px"], ga["area_px"]) or not np.array_equal(ra["depth_med"], ga["depth_med"]):
        errs.append("assoc area/depth differ")
    rs, gs = ref.stats(), gpu.stats(m)
    if rs != gs:
        errs.append(f"stats ref={rs} gpu={gs}")
    re, ge = ref.events(), gpu.events(m)
    n_prev = getattr(ref, "_ev_seen", 0)
    re_new = re[n_prev:]
    ref._ev_seen = len(re)
    if [(e[1], e[2]) for e in re_new] != [(e[1], e[2]) for e in ge]:
        errs.append(f"events ref={re_new} gpu={ge}")
    ro, go = ref.objects(), gpu.objects(m)
    errs += compare_objects(ro, go)
    rr, gr = ref.reenc(), gpu.reencode(m)   # buildReencode requests, best first
    if not np.array_equal(rr["id"], gr["id"]):
        errs.append(f"reencode ids ref={rr['id'].tolist()} gpu={gr['id'].tolist()}")
    else:
        for k in ("box", "kappa", "cam", "bits"):
            if len(rr["id"]) and not np.array_equal(rr[k], gr[k]):
                errs.append(f"reencode {k} differs")
    rk, gk = ref.kf(), gpu.keyframe(m)
    if rk != gk:
        errs.append(f"keyframe ref={rk} gpu={gk}")
    if deep and not errs:
        for i in range(len(ro)):
            r1, v1, k1, s1 = ref.object_vectors(i, D)
            r2, v2, k2, s2 = gpu.object_vectors(m, i)
            if not np.array_equal(r1, r2):
                errs.append(f"obj[{i}] r_frag max diff {np.abs(r1 - r2).max()}")
            if not (np.array_equal(v1, v2) and np.array_equal(k1, k2) and np.array_equal(s1, s2)):
                errs.append(f"obj[{i}] views differ")
            w1, kw1, nw1 = ref.object_whole(i, D)
            w2, kw2, nw2 = gpu.object_whole(m, i)
            if not (np.array_equal(w1, w2) and kw1 == kw2 and nw1 == nw2):
                errs.append(f"obj[{i}] r_whole differs (n_whole {nw1} vs {nw2})")
            c1, q1 = ref.object_cloud(i)
            c2, q2 = gpu.object_cloud(m, i)
            if not (np.array_equal(c1, c2) and np.array_equal(q1, q2)):
                errs.append(f"obj[{i}] cloud differs (n {len(c1)} vs {len(c2)})")
        errs += compare_grid(ref.grid(), gpu.grid_cells(m))
    return errs
