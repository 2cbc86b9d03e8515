"""Config 2 on the B200: tcgen05 association GEMM with the fused gate / top-1 epilogue (GPU).

1. Numerics: the raw tensor-core scores (fp32 accumulation of bf16 products) against a plain
   PyTorch fp32 matmul of the same bf16 values, within 2e-4 absolute (the K * 2^-23 bound of
   fp32 accumulation at K = 1152 is 1.4e-4), on aligned and ragged shapes.
2. Decisions: match indices identical to the CPU restatement (oracle/assoc_oracle.py: float32
   IoU gate > 0.1, fp64 index-order dot products, cosine >= 0.8, top-1, lowest index on ties)
   on full config-2 frames (256 detections x 16384 memories x 1152), scores within 1e-12.
3. Near-threshold and tie cases go through the exact recomputation and still match.
"""
import numpy as np
import pytest

from conftest import has_gpu

pytestmark = pytest.mark.gpu


def _dev(a, torch, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def _bf16_torch(u16, torch):
    return (torch.from_numpy(u16.astype(np.int32) << 16).view(torch.float32)).cuda()


@pytest.mark.parametrize("n_det,n_mem", [(256, 2048), (200, 1000), (37, 300)])
def test_scores_match_torch_fp32(n_det, n_mem):
    if not has_gpu():
        pytest.skip("no GPU")
    import torch
    from scenemap_b200.assoc import AssocGPU, to_bf16
    rng = np.random.default_rng(n_det + n_mem)
    D = 1152
    det = to_bf16(rng.standard_normal((n_det, D)).astype(np.float32) / np.sqrt(D))
    mem = to_bf16(rng.standard_normal((n_mem, D)).astype(np.float32) / np.sqrt(D))
    box = np.tile(np.array([0, 0, 0, 1, 1, 1], np.float32), (max(n_det, n_mem), 1))
    A = AssocGPU(n_det, n_mem, D)
    scores = torch.zeros((n_det, n_mem), dtype=torch.float32, device="cuda")
    m, s, c = A.match(_dev(det, torch, torch.int16), _dev(box[:n_det], torch), _dev(mem, torch, torch.int16),
                      _dev(box[:n_mem], torch), scores=scores)
    torch.cuda.synchronize()
    want = _bf16_torch(det, torch) @ _bf16_torch(mem, torch).T
    err = (scores - want).abs().max().item()
    assert err < 2e-4, err
    assert A.error() == 0


def test_decisions_match_restatement_full_frames():
    if not has_gpu():
        pytest.skip("no GPU")
    import torch
    from oracle import assoc_oracle as ao
    from scenemap_b200.assoc import AssocGPU, AssocWorkload
    W = AssocWorkload(seed=2)
    A = AssocGPU(W.n_det, W.n_mem, W.dim)
    mem = _dev(W.mem, torch, torch.int16)
    mbox = _dev(W.mem_box, torch)
    for k in range(3):
        z, box, _ = W.frame(k)
        m, s, c = A.match(_dev(z, torch, torch.int16), _dev(box, torch), mem, mbox)
        torch.cuda.synchronize()
        want_m, want_s, _ = ao.decide(z, box, W.mem, W.mem_box)
        m, s = m.cpu().numpy(), s.cpu().numpy()
        assert np.array_equal(m, want_m), f"frame {k}: {np.nonzero(m != want_m)[0][:10]}"
        assert np.allclose(s, want_s, rtol=0, atol=1e-12)
        assert (m >= 0).sum() > 50
    assert A.error() == 0


def test_near_threshold_and_ties_are_exact():
    if not has_gpu():
        pytest.skip("no GPU")
    import torch
    from oracle import assoc_oracle as ao
    from scenemap_b200.assoc import AssocGPU, to_bf16
    rng = np.random.default_rng(9)
    D, n_mem = 1152, 700
    mem = rng.standard_normal((n_mem, D)).astype(np.float32)
    mem /= np.linalg.norm(mem, axis=1, keepdims=True)
    mem[301] = mem[300]                      # exact duplicate: tie broken by the lower index
    mb = np.concatenate([rng.uniform(0, 5, (n_mem, 3)), np.zeros((n_mem, 3))], 1).astype(np.float32)
    mb[:, 3:] = mb[:, :3] + 0.5
    mb[301] = mb[300]
    memb = to_bf16(mem)
    dets, boxes = [], []
    for i in range(120):                     # cosines within ~1e-3 of the 0.8 threshold
        j = int(rng.integers(0, n_mem))
        u = rng.standard_normal(D).astype(np.float32)
        u -= u.dot(mem[j]) * mem[j]
        u /= np.linalg.norm(u)
        c = 0.8 + rng.uniform(-1.5e-3, 1.5e-3)
        dets.append(c * mem[j] + np.sqrt(1 - c * c) * u)
        boxes.append(mb[j])
    dets.append(mem[300] * 0.95 + 0.05 * rng.standard_normal(D).astype(np.float32) / np.sqrt(D))
    boxes.append(mb[300])
    dets = np.asarray(dets, np.float32)
    detb = to_bf16(dets)
    boxes = np.asarray(boxes, np.float32)
    A = AssocGPU(len(dets), n_mem, D)
    m, s, c = A.match(_dev(detb, torch, torch.int16), _dev(boxes, torch), _dev(memb, torch, torch.int16), _dev(mb, torch))
    torch.cuda.synchronize()
    want_m, want_s, _ = ao.decide(detb, boxes, memb, mb)
    m, s, c = m.cpu().numpy(), s.cpu().numpy(), c.cpu().numpy()
    assert np.array_equal(m, want_m)
    assert np.allclose(s, want_s, rtol=0, atol=1e-12)
    assert m[-1] == 300 and c[-1] == 0       # the duplicate tie was resolved exactly
    assert (c[:-1] == 0).sum() > 10          # near-threshold cases took the exact path
    assert A.error() == 0


@pytest.mark.parametrize("n_frames", [8, 3])
def test_frame_batches_match_restatement(n_frames):
    """Several frames against one bank in one call (their detections as consecutive rows): the
    persistent kernel's tile walk and double-buffered accumulators give every frame the
    decisions of the restatement."""
    if not has_gpu():
        pytest.skip("no GPU")
    import torch
    from oracle import assoc_oracle as ao
    from scenemap_b200.assoc import AssocGPU, AssocWorkload
    W = AssocWorkload(seed=5)
    fr = [W.frame(k) for k in range(n_frames)]
    z = np.concatenate([f[0] for f in fr])
    box = np.concatenate([f[1] for f in fr])
    A = AssocGPU(z.shape[0], W.n_mem, W.dim)
    m, s, c = A.match(_dev(z, torch, torch.int16), _dev(box, torch), _dev(W.mem, torch, torch.int16), _dev(W.mem_box, torch))
    torch.cuda.synchronize()
    m, s = m.cpu().numpy(), s.cpu().numpy()
    for k in range(n_frames):
        want_m, want_s, _ = ao.decide(fr[k][0], fr[k][1], W.mem, W.mem_box)
        sl = slice(k * W.n_det, (k + 1) * W.n_det)
        assert np.array_equal(m[sl], want_m), f"frame {k}: {np.nonzero(m[sl] != want_m)[0][:10]}"
        assert np.allclose(s[sl], want_s, rtol=0, atol=1e-12)
    assert A.error() == 0
