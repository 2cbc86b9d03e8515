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


def test_bad_arguments_fail_cleanly_without_gpu():
    from scenemap_b200 import smg
    L = smg.lib()
    assert L.smg_destroy(None) == -1
    assert L.smg_plane_fit(None, None, 0, 0, 0.02, None, 64, None, None) == -1
    assert b"bad arguments" in L.smg_last_error()
