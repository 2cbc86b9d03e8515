"""CPU restatement of the config-2 association decision (TEST INFRASTRUCTURE ONLY).

The reference's association (scenemap objmap.cpp:774-810) gates object pairs by box geometry
and picks the best cosine above a threshold; BASELINE config 2 fixes the stress form: the 3D
AABB IoU gate > 0.1, cosine threshold 0.8, top-1.  This module restates that decision for bf16
embeddings:

- gate: IoU of the boxes > iou_min, in float32 with the operation order
  inter = (e_x * e_y) * e_z, vol = ((dx * dy) * dz), union = (vol_a + vol_b) - inter,
  accepted iff inter > iou_min * union;
- score: fp64 dot product of the bf16 values, summed in index order k = 0..D-1;
- decision: the gated memory with the largest score among scores >= cos_min (lowest memory
  index on ties), else -1.
"""
from __future__ import annotations

import numpy as np

F = np.float32


def bf16_to_f64(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def gate(det_box: np.ndarray, mem_box: np.ndarray, iou_min: float) -> np.ndarray:
    """(n_det, n_mem) bool gate matrix, float32 arithmetic."""
    a = np.asarray(det_box, F)[:, None, :]
    b = np.asarray(mem_box, F)[None, :, :]
    ok = np.ones((a.shape[0], b.shape[1]), bool)
    inter = np.ones(ok.shape, F)
    for k in range(3):
        lo = np.maximum(a[..., k], b[..., k])
        hi = np.minimum(a[..., 3 + k], b[..., 3 + k])
        e = (hi - lo).astype(F)
        ok &= e > F(0)
        inter = (inter * e).astype(F)
    avol = (((a[..., 3] - a[..., 0]) * (a[..., 4] - a[..., 1])).astype(F) * (a[..., 5] - a[..., 2])).astype(F)
    bvol = (((b[..., 3] - b[..., 0]) * (b[..., 4] - b[..., 1])).astype(F) * (b[..., 5] - b[..., 2])).astype(F)
    uni = ((avol + bvol).astype(F) - inter).astype(F)
    return ok & (inter > (F(iou_min) * uni).astype(F))


def dots_seq(det: np.ndarray, mem: np.ndarray, pairs: np.ndarray) -> np.ndarray:
    """fp64 dot products of the listed (d, j) pairs, summed in index order."""
    A = bf16_to_f64(det[pairs[:, 0]])
    B = bf16_to_f64(mem[pairs[:, 1]])
    s = np.zeros(len(pairs))
    for k in range(A.shape[1]):
        s = s + A[:, k] * B[:, k]
    return s


def decide(det, det_box, mem, mem_box, iou_min=0.1, cos_min=0.8):
    """(match (n_det,) int32, score (n_det,) float64, n_gated_pairs)."""
    G = gate(det_box, mem_box, iou_min)
    pairs = np.argwhere(G)
    s = dots_seq(det, mem, pairs) if len(pairs) else np.zeros(0)
    n_det = len(det_box)
    match = np.full(n_det, -1, np.int32)
    score = np.zeros(n_det)
    for (d, j), v in zip(pairs, s):   # pairs come in (d, j) order: the first maximum is the lowest j
        if v >= cos_min and (match[d] < 0 or v > score[d]):
            match[d], score[d] = j, v
    return match, score, len(pairs)
