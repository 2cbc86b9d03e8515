"""Seeded synthetic frames for the scenemap objprob configurations (ctypes over libsynth.so).

The generator itself is C (``synth/synth.h``, ``synth/synth_host.cpp``); this module only
wraps it and assembles per-frame input dictionaries that both the B200 path and the CPU
reference consume, so that both see byte-identical inputs.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(os.path.dirname(_HERE), "synth", "libsynth.so")

SY_MAX_BOXES = 64
SY_SHELL_LABEL0 = 1 + 3 * SY_MAX_BOXES   # first room-face label (synth.h)


class SyBox(C.Structure):
    _fields_ = [("lo", C.c_double * 3), ("hi", C.c_double * 3)]


class SyScene(C.Structure):
    _fields_ = [("seed", C.c_uint64), ("room", C.c_double * 3), ("n_boxes", C.c_int),
                ("box", SyBox * SY_MAX_BOXES), ("noise_k", C.c_float), ("shell_labels", C.c_int32)]


def obj_of_label(label):
    """The object a label belongs to (synth.h sy_obj_of_label): box b for its three face labels,
    SY_MAX_BOXES + face for the room faces.  Works on ints and integer numpy arrays."""
    label = np.asarray(label, np.int64)
    return np.where(label < SY_SHELL_LABEL0, (label - 1) // 3, SY_MAX_BOXES + (label - SY_SHELL_LABEL0))


class SyCamera(C.Structure):
    _fields_ = [("w", C.c_int), ("h", C.c_int), ("fx", C.c_float), ("fy", C.c_float),
                ("cx", C.c_float), ("cy", C.c_float)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(f"libsynth.so not built ({_LIB_PATH}); run __graft_entry__.build()")
        L = C.CDLL(_LIB_PATH)
        P = C.POINTER
        L.sy_scene_make.argtypes = [C.c_uint64, C.c_int, C.c_double, C.c_double, C.c_double, C.c_float,
                                    C.c_double, C.c_double, C.c_double, C.c_double, P(SyScene)]
        L.sy_traj.argtypes = [P(SyScene), C.c_int, C.c_double, C.c_double, C.c_double, P(C.c_double)]
        L.sy_rig_T_bc.argtypes = [C.c_float, C.c_float, C.c_float, P(C.c_float)]
        L.sy_T_mc.argtypes = [P(C.c_double), P(C.c_float), P(C.c_double)]
        L.sy_render.argtypes = [P(SyScene), P(SyCamera), P(C.c_double), C.c_uint64, P(C.c_float), P(C.c_uint16)]
        L.sy_dets.argtypes = [P(C.c_uint16), C.c_int, C.c_int, C.c_int, C.c_int, P(C.c_uint16), P(C.c_float),
                              P(C.c_int32), P(C.c_float)]
        L.sy_dets.restype = C.c_int
        L.sy_embed.argtypes = [P(SyScene), C.c_uint64, C.c_int, P(C.c_uint16), C.c_int, C.c_double, C.c_int, P(C.c_float)]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t))


def label_masks(label: np.ndarray, det_label, s: int) -> np.ndarray:
    """Detector bit masks on an s-pixel grid (the sm_detections form): cell (i, j) covers pixels
    [s i, s i + s) x [s j, s j + s) and is set when the label at its centre pixel (s i + s/2,
    s j + s/2) is the detection's; (w // s) x (h // s) cells, LSB-first row-major words."""
    h, w = label.shape
    MW, MH = w // s, h // s
    samp = label[s // 2::s, s // 2::s][:MH, :MW]
    words = (MW * MH + 31) // 32
    out = np.zeros((max(len(det_label), 1), words), np.uint32)
    for k, l in enumerate(det_label):
        flat = np.zeros(words * 32, bool)
        flat[:MW * MH] = (samp == l).reshape(-1)
        out[k] = np.packbits(flat, bitorder="little").view("<u4")
    return out[:len(det_label)]


def map_seed(base: int, index: int) -> int:
    """Per-map seed: splitmix64 of base xor map index."""
    z = (base ^ index) & 0xFFFFFFFFFFFFFFFF
    z = (z + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return z ^ (z >> 31)


def rgba_image(label: np.ndarray, depth: np.ndarray) -> np.ndarray:
    """A colour image for a rendered frame: a base colour per label plus a pixel texture and
    depth shading, so crops average distinct values (deterministic; alpha 255)."""
    h, w = label.shape
    v, u = np.mgrid[0:h, 0:w].astype(np.uint32)
    lab = label.astype(np.uint32)
    dq = (np.clip(depth, 0.0, 10.0) * 20.0).astype(np.uint32)
    r = (lab * 73 + 3 * u + v + dq) & 255
    g = (lab * 151 + u + 5 * v) & 255
    b = (lab * 29 + 7 * (u ^ v) + 2 * dq) & 255
    a = np.full_like(r, 255)
    return np.stack([r, g, b, a], axis=-1).astype(np.uint8)


class BoxRoom:
    """Config 0/1/4 generator: 6x5x2.6 m room, 20 boxes, pinhole camera on a moving base.

    Variants (parity cases for rules the default room never reaches):
      shell_labels  the room's walls, floor and ceiling come back as detections of their own;
      box_moves     [(frame, box, (dx, dy, dz)), ...]: from that frame on the box is translated
                    (cumulatively); a translation far outside the room makes it vanish;
      box_extra     [(lo, hi), ...]: boxes added after the seeded ones (their placement is the
                    caller's, e.g. small graspable boxes or boxes that only enter through a move);
      hands         callable f -> (eef (2, 3) map frame, grip (2,)): the robot hand's point and
                    gripper value per frame (default: far away, open);
      mask_grid     s > 0: detections also carry bit masks on an s-pixel grid (label_masks), the
                    form the reference's detector produces; both sides then read those;
      depth_mm      depth also as uint16 millimetres (rounded), which both sides then read;
      rgb           an RGBA colour image registered with the depth (rgba_image), which both sides
                    use for best views and cloud-point colours;
      walls         callable f -> (n, 4) wall segments (ax, ay, bx, by, map metres) the keyframe
                    carries, or None for none (ObjFrame::wall_segs).
    """

    def __init__(self, seed: int, n_boxes: int = 20, room=(6.0, 5.0, 2.6), noise_k: float = 0.005,
                 size=(0.2, 0.6), height=(0.15, 0.9), w: int = 640, h: int = 480, fx: float = 525.0,
                 fy: float = 525.0, cx: float = 319.5, cy: float = 239.5, dt: float = 0.1, speed: float = 0.3,
                 n_frames: int = 300, D: int = 1152, bf16: bool = False, emb_sigma: float = 0.05,
                 min_px: int = 64, max_det: int = 24, cam_height: float = 0.9, pitch_deg: float = 20.0,
                 shell_labels: bool = False, box_moves=(), box_extra=(), hands=None, mask_grid: int = 0,
                 depth_mm: bool = False, rgb: bool = False, walls=None):
        L = lib()
        self.seed = seed
        self.scene = SyScene()
        L.sy_scene_make(seed, n_boxes, room[0], room[1], room[2], noise_k, size[0], size[1], height[0], height[1],
                        C.byref(self.scene))
        for lo, hi in box_extra:
            b = self.scene.n_boxes
            assert b < SY_MAX_BOXES
            for k in range(3):
                self.scene.box[b].lo[k] = lo[k]
                self.scene.box[b].hi[k] = hi[k]
            self.scene.n_boxes = b + 1
        self.scene.shell_labels = 1 if shell_labels else 0
        self.mask_grid, self.depth_mm, self.rgb, self.walls = mask_grid, depth_mm, rgb, walls
        self.box_moves = sorted(box_moves, key=lambda e: e[0])
        self.hands = hands
        self.cam = SyCamera(w, h, fx, fy, cx, cy)
        self.w, self.h, self.fx, self.fy, self.cx, self.cy = w, h, fx, fy, cx, cy
        self.dt, self.n_frames, self.D, self.bf16, self.emb_sigma = dt, n_frames, D, bf16, emb_sigma
        self.min_px, self.max_det = min_px, max_det
        self.poses = np.zeros((n_frames, 3), np.float64)
        L.sy_traj(C.byref(self.scene), n_frames, dt, speed, 0.5, _p(self.poses, C.c_double))
        self.T_bc = np.zeros(12, np.float32)
        L.sy_rig_T_bc(0.1, cam_height, pitch_deg, _p(self.T_bc, C.c_float))
        # hands: far from everything (the synthetic rig has no arm)
        self.eef = np.full((2, 3), 1000.0, np.float64)
        self.eef_base = np.tile(np.array([-0.05, 0.0, 0.25], np.float32), (2, 1))

    def T_mc(self, f: int) -> np.ndarray:
        out = np.zeros(12, np.float64)
        pose = np.ascontiguousarray(self.poses[f])
        lib().sy_T_mc(_p(pose, C.c_double), _p(self.T_bc, C.c_float), _p(out, C.c_double))
        return out

    def scene_at(self, f: int) -> SyScene:
        """The scene of frame f: the seeded boxes with every move of frames <= f applied."""
        if not self.box_moves:
            return self.scene
        S = SyScene.from_buffer_copy(self.scene)
        for fm, b, d in self.box_moves:
            if fm > f:
                break
            for k in range(3):
                S.box[b].lo[k] += d[k]
                S.box[b].hi[k] += d[k]
        return S

    def frame(self, f: int) -> dict:
        L = lib()
        T = self.T_mc(f)
        depth = np.zeros((self.h, self.w), np.float32)
        label = np.zeros((self.h, self.w), np.uint16)
        key = f + 1
        S = self.scene_at(f)
        L.sy_render(C.byref(S), C.byref(self.cam), _p(T, C.c_double), key, _p(depth, C.c_float),
                    _p(label, C.c_uint16))
        md = self.max_det
        det_label = np.zeros(md, np.uint16)
        box = np.zeros((md, 4), np.float32)
        cls = np.zeros(md, np.int32)
        score = np.zeros(md, np.float32)
        n = L.sy_dets(_p(label, C.c_uint16), self.w, self.h, self.min_px, md, _p(det_label, C.c_uint16),
                      _p(box, C.c_float), _p(cls, C.c_int32), _p(score, C.c_float))
        emb = np.zeros((max(n, 1), self.D), np.float32)
        if n:
            L.sy_embed(C.byref(S), key, n, _p(det_label, C.c_uint16), self.D, self.emb_sigma,
                       1 if self.bf16 else 0, _p(emb, C.c_float))
        eef, grip = (self.eef, np.ones(2, np.float32)) if self.hands is None else self.hands(f)
        extra = {}
        if self.mask_grid > 0:
            s = self.mask_grid
            extra.update(mask_bits=label_masks(label, det_label[:n], s), mask_w=self.w // s, mask_h=self.h // s,
                         mask_affine=(float(s), float(s), 0.0, 0.0), img_w=self.w, img_h=self.h)
        if self.rgb:
            extra["rgba"] = rgba_image(label, depth)
        if self.depth_mm:
            extra["depth_mm"] = np.clip(np.rint(depth * 1000.0), 0, 65535).astype(np.uint16)
        if self.walls is not None:
            ws = self.walls(f)
            if ws is not None:
                extra["wall_segs"] = np.asarray(ws, np.float64).reshape(-1, 4)
        return dict(stamp=f * self.dt, w=self.w, h=self.h, depth=depth, label=label, fx=self.fx, fy=self.fy,
                    cx=self.cx, cy=self.cy, T_mc=T, T_bc=self.T_bc, base=self.poses[f].copy(),
                    eef=np.asarray(eef, np.float64), grip=np.asarray(grip, np.float32), eef_base=self.eef_base,
                    n_det=n, det_label=det_label[:n].copy(), box=box[:n].copy(), cls=cls[:n].copy(),
                    score=score[:n].copy(), emb=emb[:n].copy(), emb_dim=self.D, **extra)


# ---- a synthetic text model for the box rooms (label table, text rows, statistics) ----
# Labels 0..15 are the detector classes (a box's class is its index mod 16); 16-19 room structure
# and stairs; 20 "furniture" (hypernym of chair / table / sofa / cabinet, no text row) and 21
# "object" (the fallback name, no text row).  Kinds: 0 object, 1 structure, 2 static, 3
# structural object (the reference's kKind* values).
TEXT_LABELS = ["box", "chair", "table", "sofa", "cabinet", "door", "window", "pillar", "picture", "tv", "cup", "bottle", "book",
               "bag", "lamp", "plant", "wall", "floor", "ceiling", "stairs", "furniture", "object"]
TEXT_KINDS = [0, 0, 2, 2, 2, 3, 3, 3, 0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 3, 0, 0]
TEXT_SO_SHAPE = [0, 0, 0, 0, 0, 1, 1, 3, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 2, 0, 0]
TEXT_FLAT = [0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0]
TEXT_PARENT = [-1, 20, 20, 20, 20, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1]
TEXT_LOGSIZE = [(-0.9, 0.5), (-0.5, 0.4), (-0.2, 0.5), (0.0, 0.5), (-0.1, 0.5), (0.6, 0.4), (0.2, 0.5), (0.8, 0.6), (-0.9, 0.5),
                (-0.7, 0.5), (-2.3, 0.4), (-1.9, 0.4), (-1.8, 0.4), (-1.0, 0.5), (-0.8, 0.5), (-0.9, 0.6), (1.2, 0.5), (1.4, 0.5),
                (1.4, 0.5), (0.9, 0.5), (0.0, 0.0), (0.0, 0.0)]


def text_model(room: "BoxRoom", scale: float = 20.0, bias: float = -6.0, seed: int = 7) -> dict:
    """A text model whose rows sit near the rooms' own embeddings: the row of class c is the
    normalised sum of the base directions (the noise-free embedding) of the boxes of class c,
    walls / floor / ceiling rows come from the room faces' bases, and labels without boxes get a
    seeded random row; "furniture" and "object" have none (a hypernym and the fallback name)."""
    L = lib()
    nl, D = len(TEXT_LABELS), room.D
    rng = np.random.default_rng(seed)
    base = np.zeros(D, np.float32)

    def base_of(label_value: int) -> np.ndarray:
        dl = np.array([label_value], np.uint16)
        L.sy_embed(C.byref(room.scene), 1, 1, _p(dl, C.c_uint16), D, 0.0, 0, _p(base, C.c_float))
        return base.astype(np.float64).copy()

    acc = [np.zeros(D) for _ in range(nl)]
    for b in range(room.scene.n_boxes):
        acc[b % 16] += base_of(1 + 3 * b)
    for face in range(6):
        lab = 16 if face < 4 else (17 if face == 4 else 18)
        acc[lab] += base_of(SY_SHELL_LABEL0 + face)
    rows, row_label = [], []
    for c in range(nl):
        if c in (20, 21):
            continue
        v = acc[c] if np.any(acc[c]) else rng.normal(size=D)
        rows.append((v / np.linalg.norm(v)).astype(np.float32))
        row_label.append(c)
    lp = np.log(np.full(nl, 1.0 / nl)) + rng.normal(scale=0.1, size=nl)
    return dict(text=np.ascontiguousarray(np.stack(rows), np.float32), row_label=np.asarray(row_label, np.int32), scale=scale,
                bias=bias, n_labels=nl, log_prior=lp.astype(np.float32),
                ls_mu=np.asarray([m for m, _ in TEXT_LOGSIZE], np.float32), ls_sd=np.asarray([s for _, s in TEXT_LOGSIZE], np.float32),
                parent=np.asarray(TEXT_PARENT, np.int32), object_label=21, kinds=np.asarray(TEXT_KINDS, np.uint8),
                so_shape=np.asarray(TEXT_SO_SHAPE, np.uint8), flat_ok=np.asarray(TEXT_FLAT, np.uint8))
