"""The set-loss oracle (float64 torch autograd of the reference's loss code) against the closed
forms the CUDA kernel evaluates: the per-entry IA-BCE value and derivative, and the
hand-differentiated GIoU backward (ported here to NumPy, line for line with loss.cu).  CPU only."""

from __future__ import annotations

import numpy as np
import torch

from oracle import losses as OL
from oracle import matcher as OM


def _case(seed, batch=2, groups=2, per_group=12, classes=7, max_targets=5):
    rng = np.random.default_rng(seed)
    queries = groups * per_group
    logits = rng.standard_normal((batch, queries, classes)) * 2
    boxes = np.concatenate([rng.uniform(0.1, 0.9, (batch, queries, 2)), rng.uniform(-0.05, 0.4, (batch, queries, 2))], -1)
    sizes = np.array([max_targets, max(1, max_targets - 2)][:batch], np.int32)
    mask = np.arange(max_targets)[None] < sizes[:, None]
    labels = np.where(mask, rng.integers(0, classes, (batch, max_targets)), 0).astype(np.int32)
    tboxes = np.concatenate([rng.uniform(0.1, 0.9, (batch, max_targets, 2)), rng.uniform(0.05, 0.4, (batch, max_targets, 2))], -1)
    tboxes = np.where(mask[..., None], tboxes, 0.0)
    cost = OM.build_cost_matrix(logits.astype(np.float32), boxes.astype(np.float32), labels, tboxes.astype(np.float32), mask)
    rows, cols, valid = OM.hungarian_match(cost, sizes, groups)
    return logits, boxes, labels, tboxes, rows, cols, valid, float(valid.sum())


def _softplus(x):
    return np.maximum(x, 0) + np.log1p(np.exp(-np.abs(x)))


def _giou_loss_grad(s, t, scale):
    """NumPy port of giou_loss_grad in csrc/loss.cu."""
    wp, hp = max(s[2], 0.0), max(s[3], 0.0)
    a0, a1, a2, a3 = s[0] - 0.5 * wp, s[1] - 0.5 * hp, s[0] + 0.5 * wp, s[1] + 0.5 * hp
    tw, th = max(t[2], 0.0), max(t[3], 0.0)
    b0, b1, b2, b3 = t[0] - 0.5 * tw, t[1] - 0.5 * th, t[0] + 0.5 * tw, t[1] + 0.5 * th
    area1, area2 = (a2 - a0) * (a3 - a1), (b2 - b0) * (b3 - b1)
    iwr, ihr = min(a2, b2) - max(a0, b0), min(a3, b3) - max(a1, b1)
    iw, ih = max(iwr, 0.0), max(ihr, 0.0)
    inter = iw * ih
    uni = area1 + area2 - inter
    U = max(uni, 1e-7)
    iou = inter / U
    ewr, ehr = max(a2, b2) - min(a0, b0), max(a3, b3) - min(a1, b1)
    ew, eh = max(ewr, 0.0), max(ehr, 0.0)
    area = ew * eh
    A = max(area, 1e-7)
    loss = 1 - (iou - (area - uni) / A)
    d_giou = -scale
    d_uni = d_giou / A
    d_area = -d_giou / A + (d_giou * (area - uni) / (A * A) if area > 1e-7 else 0.0)
    d_inter = d_giou / U
    if uni > 1e-7:
        d_uni += -d_giou * inter / (U * U)
    d_area1 = d_uni
    d_inter -= d_uni
    d_iwr = d_inter * ih if iwr > 0 else 0.0
    d_ihr = d_inter * iw if ihr > 0 else 0.0
    d_ewr = d_area * eh if ewr > 0 else 0.0
    d_ehr = d_area * ew if ehr > 0 else 0.0
    d = [0.0, 0.0, 0.0, 0.0]
    if a2 < b2: d[2] += d_iwr
    if a0 > b0: d[0] -= d_iwr
    if a3 < b3: d[3] += d_ihr
    if a1 > b1: d[1] -= d_ihr
    if a2 > b2: d[2] += d_ewr
    if a0 < b0: d[0] -= d_ewr
    if a3 > b3: d[3] += d_ehr
    if a1 < b1: d[1] -= d_ehr
    d[2] += d_area1 * (a3 - a1); d[0] -= d_area1 * (a3 - a1)
    d[3] += d_area1 * (a2 - a0); d[1] -= d_area1 * (a2 - a0)
    g = [d[0] + d[2], d[1] + d[3], 0.5 * (d[2] - d[0]) if s[2] > 0 else 0.0, 0.5 * (d[3] - d[1]) if s[3] > 0 else 0.0]
    return loss, np.array(g)


def test_closed_forms_match_autograd():
    for seed in range(3):
        logits, boxes, labels, tboxes, rows, cols, valid, nb = _case(seed)
        ce, l1, giou, g_ce, g_l1, g_giou = OL.set_losses(logits, boxes, labels, tboxes, rows, cols, valid, nb)
        # IA-BCE closed forms (per entry), with the oracle's own weights.
        x = logits
        p = 1 / (1 + np.exp(-x))
        val = p * p * _softplus(x)
        grad = p ** 3 + 2 * p * p * (1 - p) * _softplus(x)
        for b in range(x.shape[0]):
            for s in np.flatnonzero(valid[b]):
                q, t = rows[b, s], cols[b, s]
                c = labels[b, t]
                tb, sb = tboxes[b, t], boxes[b, q]
                iou = _iou(sb, tb)
                w = max(p[b, q, c] ** 0.25 * iou ** 0.75, 0.01)
                val[b, q, c] = (1 - w) * x[b, q, c] + _softplus(-x[b, q, c])
                grad[b, q, c] = p[b, q, c] - w
        np.testing.assert_allclose(val.sum() / nb, ce, rtol=1e-12)
        np.testing.assert_allclose(grad / nb, g_ce, rtol=1e-10, atol=1e-14)
        # GIoU: the kernel's hand-derived backward.
        want = np.zeros_like(g_giou)
        total = 0.0
        for b in range(x.shape[0]):
            for s in np.flatnonzero(valid[b]):
                q, t = rows[b, s], cols[b, s]
                loss, g = _giou_loss_grad(boxes[b, q], tboxes[b, t], 1 / nb)
                total += loss / nb
                want[b, q] = g
        np.testing.assert_allclose(total, giou, rtol=1e-12)
        np.testing.assert_allclose(want, g_giou, rtol=1e-9, atol=1e-13)
        assert np.isfinite(l1) and np.abs(g_l1).max() <= 1 / nb + 1e-15


def _iou(s, t):
    def xyxy(b):
        w, h = max(b[2], 0.0), max(b[3], 0.0)
        return b[0] - 0.5 * w, b[1] - 0.5 * h, b[0] + 0.5 * w, b[1] + 0.5 * h
    a, b = xyxy(s), xyxy(t)
    area1, area2 = (a[2] - a[0]) * (a[3] - a[1]), (b[2] - b[0]) * (b[3] - b[1])
    inter = max(min(a[2], b[2]) - max(a[0], b[0]), 0.0) * max(min(a[3], b[3]) - max(a[1], b[1]), 0.0)
    return inter / max(area1 + area2 - inter, 1e-7)


def test_unmatched_layer_has_only_negative_terms():
    logits, boxes, labels, tboxes, rows, cols, valid, _ = _case(5)
    valid = np.zeros_like(valid)
    ce, l1, giou, g_ce, g_l1, g_giou = OL.set_losses(logits, boxes, labels, tboxes, rows, cols, valid, 1.0)
    p = 1 / (1 + np.exp(-logits))
    np.testing.assert_allclose(ce, (p * p * _softplus(logits)).sum(), rtol=1e-12)
    assert l1 == 0.0 and giou == 0.0 and not g_l1.any() and not g_giou.any()
    assert torch.is_tensor(torch.tensor(g_ce))


def test_focal_closed_forms_match_autograd():
    """ia_bce off: the sigmoid focal loss (gamma 2) closed forms the kernel evaluates, for a
    positive and a negative (disabled) alpha."""
    for alpha in (0.25, -1.0):
        logits, boxes, labels, tboxes, rows, cols, valid, nb = _case(11)
        ce, _, _, g_ce, _, _ = OL.set_losses(logits, boxes, labels, tboxes, rows, cols, valid, nb, alpha, ia_bce=False)
        a1, a0 = (alpha, 1 - alpha) if alpha >= 0 else (1.0, 1.0)
        x = logits
        p = 1 / (1 + np.exp(-x))
        val = a0 * p * p * _softplus(x)
        grad = a0 * (p ** 3 + 2 * p * p * (1 - p) * _softplus(x))
        for b in range(x.shape[0]):
            for s in np.flatnonzero(valid[b]):
                q, c = rows[b, s], labels[b, cols[b, s]]
                pm, sp = p[b, q, c], _softplus(-x[b, q, c])
                val[b, q, c] = a1 * (1 - pm) ** 2 * sp
                grad[b, q, c] = -a1 * (1 - pm) ** 2 * (2 * pm * sp + 1 - pm)
        np.testing.assert_allclose(val.sum() / nb, ce, rtol=1e-12)
        np.testing.assert_allclose(grad / nb, g_ce, rtol=1e-10, atol=1e-14)
