"""The C ABI library loads without a GPU and exports every function include/smg.h declares;
host-only entry points (parameters) behave like the reference's applyParams (CPU only)."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "smg.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(smg_[a-z0-9_]+)\s*\(", src)))


def _lib():
    so = os.path.join(ROOT, "robot-agent_b200", "libsmg.so")
    if not os.path.exists(so):
        pytest.skip("libsmg.so not built (python __graft_entry__.py build)")
    return C.CDLL(so)


def test_exports_every_declared_symbol():
    L = _lib()
    names = _declared()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_python_binding_lists_the_exports():
    from scenemap_b200 import smg
    assert set(smg.EXPORTED) <= set(_declared())


def test_params_default_and_apply():
    from scenemap_b200 import smg
    L = smg.lib()
    p = smg.Params()
    before = p.buf.raw
    assert L.smg_params_apply(p.buf, b"ap_same_p=0.7") == 0
    assert p.buf.raw != before                       # a known key changes the struct
    assert L.smg_params_apply(p.buf, b"no_such_key=1,ap_same_p=0.7") == 1
    q = smg.Params()
    assert q.buf.raw == before                       # defaults are reproducible
    with pytest.raises(smg.SmgError):
        smg.Params("no_such_key=1")


# engine parameter file of the reference (tools/realbag/objprob_params/yolo26n-seg-obj-416.json,
# its "obj_params" string): every key it sets is implemented on the device
YOLO26N_OBJ_PARAMS = ("ap_w0=-4.235,ap_w1=5.063,ap_w2=-5.289,ap_w3=-0.3241,ap_w4=5.02,ap_w5=1.417,ap_w6=-0.013,ap_w7=0,"
                      "ap_wm0=-2.671,ap_wm1=1.209,ap_wm2=-4.964,ap_wm3=-0.3121,ap_wm4=6.248,ap_wm5=1.648,ap_wm6=-0.5892,"
                      "ap_wm7=2.04,ap_same_p=0.5,ap_merge_p=0.7,ap_cos0=0.75,kap_k0=4369,kap_s0=40,kap_trunc=1,kap_d0=100")


def test_params_unsupported_keys_are_not_silent():
    """Keys of features the device does not run (the inspect pass, the export filter) are
    accepted at the reference default only; the text-model and wall-line keys are real fields."""
    from scenemap_b200 import smg
    L = smg.lib()
    p = smg.Params()
    assert L.smg_params_apply(p.buf, YOLO26N_OBJ_PARAMS.encode()) == 0
    # the reference defaults of inert keys are accepted (a full parameter dump stays loadable)
    assert L.smg_params_apply(p.buf, b"ap_through_d=0.2,ap_wall_big=1,ap_export_named=1,inspect=0,ap_so_dw_w=2.2") == 0
    before = p.buf.raw
    rc = L.smg_params_apply(p.buf, b"ap_same_p=0.55,ap_through_d=0.5,ap_export_named=0,ap_bridge_max=3,inspect=1")
    assert rc == smg.SMG_ERR_UNSUPPORTED
    msg = L.smg_last_error().decode()
    assert "ap_export_named" in msg and "inspect" in msg
    assert "ap_same_p" not in msg and "ap_through_d" not in msg and "ap_bridge_max" not in msg
    assert p.buf.raw != before                      # the supported key was still applied
    with pytest.raises(smg.SmgError):
        smg.Params("inspect=1")


def test_bad_arguments_fail_cleanly_without_gpu():
    from scenemap_b200 import smg
    L = smg.lib()
    assert L.smg_destroy(None) == -1
    assert L.smg_plane_fit(None, None, 0, 0, 0.02, None, 64, None, None) == -1
    assert b"bad arguments" in L.smg_last_error()


def test_ply_header_is_the_reference_format():
    """smg_ply_header writes plyBytes' header (dsg_save.cpp:70-76): binary little-endian, float
    x y z, uchar red green blue; a buffer too small gets the needed size and no bytes."""
    from scenemap_b200 import smg
    want = (b"ply\nformat binary_little_endian 1.0\nelement vertex 1234\nproperty float x\nproperty float y\n"
            b"property float z\nproperty uchar red\nproperty uchar green\nproperty uchar blue\nend_header\n")
    assert smg.Batch.ply_header(1234) == want
    assert smg.lib().smg_ply_header(1234, None, 0) == len(want)
