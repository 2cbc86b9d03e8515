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


def make_gen(v: dict, D: int = 1152, bf16: bool = False):
    from scenemap_b200 import synth
    kw = dict(v["gen"])
    seed = synth.map_seed(kw.pop("seed_base"), 0)
    return synth.BoxRoom(seed=seed, n_frames=v["n_frames"], D=D, bf16=bf16, **kw)
