"""Generator variants that reach rules the default box room never does (tests only).

Each variant is a BoxRoom configuration plus the reference parameter string both sides get,
the frame count, and the ApStats counters / event kinds it must produce on the reference.
"""
from __future__ import annotations

# engine parameter file of the reference (tools/realbag/objprob_params/yolo26n-seg-obj-416.json,
# its "obj_params" string)
YOLO26N_OBJ_PARAMS = ("ap_w0=-4.235,ap_w1=5.063,ap_w2=-5.289,ap_w3=-0.3241,ap_w4=5.02,ap_w5=1.417,ap_w6=-0.013,ap_w7=0,"
                      "ap_wm0=-2.671,ap_wm1=1.209,ap_wm2=-4.964,ap_wm3=-0.3121,ap_wm4=6.248,ap_wm5=1.648,ap_wm6=-0.5892,"
                      "ap_wm7=2.04,ap_same_p=0.5,ap_merge_p=0.7,ap_cos0=0.75,kap_k0=4369,kap_s0=40,kap_trunc=1,kap_d0=100")


def structure(n_frames: int = 80) -> dict:
    """Walls, floor and ceiling come back as detections (a segmenter that also segments the room
    shell); a wide-angle camera pitched up sees them within the 3 m depth cut.  Reaches the
    ceiling and floor drops, the tall-wall rule (its width lowered by a parameter, since a wall
    within 3 m rarely spans the default 3 m) and apStructObject on merged clouds."""
    return dict(gen=dict(seed_base=12, shell_labels=True, pitch_deg=-5.0, noise_k=0.0005, fx=280.0, fy=280.0,
                         room=(5.0, 4.5, 2.5)),
                kv="ap_tall_w_any=1.0", n_frames=n_frames,
                stats=("n_ceil", "n_floor", "n_obj_struct", "n_wall_tall"), events=())


def moving(n_frames: int = 160) -> dict:
    """Boxes that slide, jump, vanish and appear mid-run: absence evidence, gone objects,
    relinking of a moved object and objects seen again."""
    slide = [(30 + i, 0, (0.04, 0.0, 0.0)) for i in range(15)]
    moves = slide + [(40, 1, (1.2, 0.8, 0.0)), (30, 2, (0.0, 0.0, 100.0)), (25, 3, (0.0, 0.0, 100.0)),
                     (70, 3, (0.5, 0.3, -100.0))]
    return dict(gen=dict(seed_base=21, box_moves=moves), kv="", n_frames=n_frames, stats=(), events=(2, 3))


def engine_params(n_frames: int = 40) -> dict:
    """The reference's engine parameter file (logistic weights, same_p, cos0, kappa)."""
    return dict(gen=dict(seed_base=31), kv=YOLO26N_OBJ_PARAMS, n_frames=n_frames, stats=(), events=())


def coarse_masks(n_frames: int = 40) -> dict:
    """Detections as bit masks on a 4-pixel grid (the form the reference's detector emits, and
    the grid of its own object-memory test), bf16 embeddings: the mask-cell arithmetic of the
    back-projection and of the re-encode requests on a grid coarser than the image."""
    return dict(gen=dict(seed_base=51, mask_grid=4), kv="", n_frames=n_frames, stats=(), events=(), bf16=True)


def depth_millimetres(n_frames: int = 30) -> dict:
    """Depth as uint16 millimetres (ObjFrame::depth_mm) instead of float metres."""
    return dict(gen=dict(seed_base=61, depth_mm=True), kv="", n_frames=n_frames, stats=(), events=(), bf16=True)


def walls(n_frames: int = 80) -> dict:
    """The structure variant with wall segments on the keyframes (ObjFrame::wall_segs): the room's
    four walls, a collinear gap (a window) in one, and an interior segment the camera sees boxes
    behind.  Reaches the wall-line rules of apObsStructural (wall planes dropped, wall-like
    fragments kept), the see-through drop, and apStructObject's wall share and flat-plane test.
    Every fourth keyframe carries no set (the stored one stays), one carries an empty set."""
    rx, ry = 5.0, 4.5
    segs = [(0.0, 0.0, rx, 0.0), (rx, 0.0, rx, 1.6), (rx, 2.4, rx, ry), (rx, ry, 0.0, ry), (0.0, ry, 0.0, 0.0),
            (2.5, 0.4, 2.5, 2.2)]

    def ws(f: int):
        if f % 4 == 3:
            return None
        if f == 10:
            return []
        return segs

    v = structure(n_frames)
    v["gen"] = dict(v["gen"], seed_base=14, walls=ws)
    v["stats"] = ("n_wall", "n_through")
    return v


def make_gen(v: dict, D: int = 1152, bf16: bool = False):
    from scenemap_b200 import synth
    kw = dict(v["gen"])
    seed = synth.map_seed(kw.pop("seed_base"), 0)
    return synth.BoxRoom(seed=seed, n_frames=v["n_frames"], D=D, bf16=bf16, **kw)


def hands(n_frames: int = 110, seed_base: int = 41, support: int = 2) -> dict:
    """A robot hand picks a small box off a larger one, carries it, puts it back on top (the
    support link), and the larger box is then pushed: grasp, hold (the object follows the hand),
    release, and an object that follows its support.  The small box is rendered where the hand
    carries it; the hand's gripper closes at frame 40 and opens at frame 66."""
    import numpy as np
    from scenemap_b200 import synth
    g0 = synth.BoxRoom(seed=synth.map_seed(seed_base, 0), n_frames=1)
    S = g0.scene
    b = S.box[support]
    cx, cy, top = 0.5 * (b.lo[0] + b.hi[0]), 0.5 * (b.lo[1] + b.hi[1]), b.hi[2]
    small = ((cx - 0.02, cy - 0.025, top), (cx + 0.02, cy + 0.025, top + 0.10))
    k_small = S.n_boxes   # index of the added box
    far = np.full((2, 3), 1000.0)
    path = {}
    p = np.array([cx, cy, top + 0.05])
    for f in range(40, 66):
        if 45 <= f < 50:
            p = p + np.array([0.0, 0.0, 0.03])      # lift
        elif 50 <= f < 58:
            p = p + np.array([0.02, 0.0, 0.0])      # carry
        elif 58 <= f < 63:
            p = p + np.array([0.0, 0.0, -0.03])     # put down on the support, offset in x
        path[f] = p.copy()
    moves = []
    prev = np.array([cx, cy, top + 0.05])
    for f in range(40, 66):
        d = path[f] - prev
        if np.any(d != 0):
            moves.append((f, k_small, tuple(float(x) for x in d)))
        prev = path[f]
    for f in range(80, 92):   # push the support, with the small box on it
        moves.append((f, support, (0.03, 0.0, 0.0)))
        moves.append((f, k_small, (0.03, 0.0, 0.0)))

    def hand(f):
        if f in path:
            eef = far.copy()
            eef[0] = path[f]
            return eef, np.array([0.35 if f < 66 else 1.0, 1.0], np.float32)
        return far, np.ones(2, np.float32)

    return dict(gen=dict(seed_base=seed_base, box_extra=[small], box_moves=moves, hands=hand), kv="", n_frames=n_frames,
                stats=(), events=(4, 5))
