"""Text-model label posterior on the B200: smg_label_loglik (apLabelLogLik) and smg_name
(apName) against the reference compiled in place (GPU).

1. The reference's own naming known-answer test (tests/test_objprob.cpp:72-98): an
   ambiguous cup/mug view rolls up to the hypernym "container" with high entropy; strong
   external "mug" evidence then names it "mug".
2. Random text models (label trees, priors, size Gaussians) and objects: log-likelihoods
   within 1e-5, posteriors within 1e-6, entropies within 1e-5 of the reference; name, top
   label and roll-up identical.  (Device exp/log/log1p may differ from the host libm in the
   last bit, so floating results are compared with these tolerances.)
"""
import math

import numpy as np
import pytest

from conftest import has_gpu

pytestmark = pytest.mark.gpu


def _need():
    if not has_gpu():
        pytest.skip("no GPU")
    from oracle import ref
    if not ref.available():
        pytest.skip("reference oracle library not built")


def _label_term(w, ll):   # objprob_math.h:93-95 (weight * max(log p, -60)), accumulated as float
    return np.float32(w * np.maximum(ll.astype(np.float64), -60.0))


def test_naming_kat():
    _need()
    from scenemap_b200.text import NameParams, TextModel
    rows = np.array([[1, 0, 0, 0], [0.8, 0.6, 0, 0], [0, 0, 1, 0]], np.float32)
    T = TextModel(rows, [0, 1, 3], 4, scale=10.0, bias=-5.0, parent=[2, 2, -1, -1])
    zc = np.array([[0.9, 0.3, 0, 0]], np.float32)
    ll = T.loglik(zc)[0]
    w = 100.0 / 100.0                     # label_weight(kappa 100, kappa_ref 100)
    L = _label_term(w, ll)[None, :]
    p = NameParams(1.0, 6.0, 1.0, 0.8)
    post, lab, val = T.name(p, [0.1], L_frag=L, lw_frag=[w])
    assert lab[0, 2] == 1 and lab[0, 0] == 2, (lab, val)   # rolled to "container"
    assert val[0, 2] > 0.5                                    # entropy
    ext = np.zeros((1, 4), np.float32)
    ext[0, 1] = 8.0                                           # apObserveName(mug, 8)
    post, lab, val = T.name(p, [0.1], L_frag=L, lw_frag=[w], L_ext=ext)
    assert lab[0, 0] == 1 and lab[0, 2] == 0


def test_loglik_and_names_match_reference():
    _need()
    from oracle import ref
    from scenemap_b200.text import NameParams, TextModel
    rng = np.random.default_rng(4)
    for trial in range(4):
        C, D, rows = int(rng.integers(5, 60)), int(rng.choice([16, 64, 768])), int(rng.integers(5, 120))
        text = rng.standard_normal((rows, D)).astype(np.float32)
        text /= np.linalg.norm(text, axis=1, keepdims=True)
        row_label = rng.integers(0, C, rows).astype(np.int32)
        row_label[rng.random(rows) < 0.1] = -1
        parent = np.where(rng.random(C) < 0.6, rng.integers(0, C, C), -1).astype(np.int32)
        parent = np.where(parent >= np.arange(C), -1, parent).astype(np.int32)   # a forest (parents earlier)
        log_prior = rng.normal(0, 0.5, C).astype(np.float32) if trial % 2 else None
        ls_mu = rng.normal(-1, 0.5, C).astype(np.float32) if trial >= 2 else None
        ls_sd = np.where(rng.random(C) < 0.7, rng.uniform(0.2, 1.0, C), 0.0).astype(np.float32) if trial >= 2 else None
        obj_label = int(rng.integers(0, C)) if trial == 3 else -1
        scale, bias = 111.83257, -16.766876
        T = TextModel(text, row_label, C, scale, bias, log_prior, ls_mu, ls_sd, parent, obj_label)
        z = rng.standard_normal((40, D)).astype(np.float32)
        z[:20] = text[rng.integers(0, rows, 20)] + 0.3 * z[:20] / np.sqrt(D)
        z /= np.linalg.norm(z, axis=1, keepdims=True)
        ll = T.loglik(z)
        want = ref.label_loglik(text, row_label, C, scale, bias, z)
        dead = want < -1e29
        assert np.array_equal(ll < -1e29, dead)
        assert np.abs(ll[~dead] - want[~dead]).max() < 1e-5
        # objects: fragment sums of 1-6 views, optional whole views, external and geometric terms
        n = 64
        Lf = np.zeros((n, C), np.float32)
        lwf = np.zeros(n)
        for o in range(n):
            for _ in range(int(rng.integers(0, 7))):
                wv = float(rng.uniform(0.05, 2.0))
                Lf[o] += _label_term(wv, want[int(rng.integers(0, len(z)))])
                lwf[o] += wv
        Lw = (Lf * rng.uniform(0, 1.5, (n, 1))).astype(np.float32) if trial % 2 == 0 else None
        lww = rng.uniform(0, 2, n) if Lw is not None else None
        Le = np.where(rng.random((n, C)) < 0.03, rng.normal(0, 4, (n, C)), 0).astype(np.float32)
        Lg = np.where(rng.random((n, C)) < 0.05, 3.0, 0).astype(np.float32) if trial >= 1 else None
        size = rng.uniform(0.01, 3.0, n)
        p = NameParams(1.0, 6.0, 1.0, float(rng.choice([0.5, 0.6, 0.8])))
        post, lab, val = T.name(p, size, L_frag=Lf, lw_frag=lwf, L_whole=Lw, lw_whole=lww, L_ext=Le, L_geo=Lg)
        for o in range(n):
            r = ref.name(text, row_label, C, scale, bias, log_prior, ls_mu, ls_sd, parent, obj_label, 1.0, 6.0, 1.0,
                         p.name_tau, Lf[o], lwf[o], None if Lw is None else Lw[o], 0.0 if lww is None else lww[o], Le[o],
                         None if Lg is None else Lg[o], size[o])
            rpost, rlab, rname_p, rtop, rtop_p, rH, rrolled, named = r
            if not named:
                assert lab[o, 0] == -2
                continue
            assert np.abs(post[o] - rpost).max() < 1e-6, (trial, o)
            assert (lab[o, 0], lab[o, 1], lab[o, 2]) == (rlab, rtop, rrolled), (trial, o, lab[o], (rlab, rtop, rrolled))
            assert abs(val[o, 0] - rname_p) < 1e-6 and abs(val[o, 1] - rtop_p) < 1e-6 and abs(val[o, 2] - rH) < 1e-5
