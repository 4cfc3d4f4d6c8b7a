"""Parity of the CUDA set losses (IA-BCE classification, L1 and GIoU over matched pairs) and
their gradients with the float64 oracle, at fp32 tolerance: 1e-5 relative + 1e-6 absolute on
every loss value and gradient entry."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import match_inputs
from oracle import losses as OL
from oracle import matcher as OM

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
RTOL, ATOL = 1e-5, 1e-6


def _layer(seed, batch, groups, per_group, classes, max_targets):
    logits, boxes, labels, tboxes, mask, sizes = match_inputs(seed, batch, groups * per_group, classes, max_targets)
    rng = np.random.default_rng(seed + 100)
    logits = (rng.standard_normal(logits.shape) * 2).astype(np.float32)
    boxes[..., 2:] = rng.uniform(-0.05, 0.5, boxes[..., 2:].shape).astype(np.float32)  # some clipped sizes
    cost = OM.build_cost_matrix(logits, boxes, labels, tboxes, mask)
    rows, cols, valid = OM.hungarian_match(cost, sizes, groups)
    return logits, boxes, labels, tboxes, rows, cols, valid


def _gpu(pkg, logits, boxes, labels, tboxes, rows, cols, valid, nb, ct=(1.0, 1.0, 1.0), alpha=0.25, ia_bce=True):
    t = lambda x: torch.tensor(x, device=DEV)  # noqa: E731
    x = t(logits).requires_grad_(True)
    b = t(boxes).requires_grad_(True)
    ce, l1, giou = pkg.set_losses(x, b, t(labels), t(tboxes), t(rows), t(cols), t(valid.astype(np.uint8)),
                                  torch.tensor(nb, device=DEV), alpha, ia_bce)
    (ce * ct[0] + l1 * ct[1] + giou * ct[2]).backward()
    return (float(ce.detach()), float(l1.detach()), float(giou.detach()), x.grad.cpu().numpy(), b.grad.cpu().numpy())


@pytest.mark.parametrize(("batch", "groups", "per_group", "classes", "max_targets"),
                         [(2, 2, 30, 7, 8), (3, 13, 20, 91, 12), (1, 1, 5, 3, 5)])
@pytest.mark.parametrize(("alpha", "ia_bce"), [(0.25, True), (0.25, False), (-1.0, False)])
def test_against_oracle(pkg, batch, groups, per_group, classes, max_targets, alpha, ia_bce):
    logits, boxes, labels, tboxes, rows, cols, valid = _layer(batch * 7 + groups, batch, groups, per_group, classes,
                                                             max_targets)
    nb = max(float(valid.sum()), 1.0)
    ct = (0.7, 1.3, -0.4)
    ce, l1, giou, gx, gb = _gpu(pkg, logits, boxes, labels, tboxes, rows, cols, valid, nb, ct, alpha, ia_bce)
    w = OL.set_losses(logits, boxes, labels, tboxes, rows, cols, valid, nb, alpha, ia_bce)
    np.testing.assert_allclose([ce, l1, giou], w[:3], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gx, ct[0] * w[3], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gb, ct[1] * w[4] + ct[2] * w[5], rtol=RTOL, atol=ATOL)


def test_config4_layer(pkg):
    """One layer at config-4 training shape (8 images, 13 x 300 queries, 91 classes, <= 100
    targets) with the device matcher's assignment."""
    logits, boxes, labels, tboxes, mask, sizes = match_inputs(41, 8, 3900, 91, 100)
    t = lambda x: torch.tensor(x, device=DEV)  # noqa: E731
    cost = pkg.build_cost_matrix(t(logits), t(boxes), t(labels), t(tboxes), t(mask), 2.0, 5.0, 2.0, 0.25)
    rows, cols, valid = (x.cpu().numpy() for x in pkg.hungarian_match(cost, t(sizes), 13))
    nb = float(valid.sum())
    ce, l1, giou, gx, gb = _gpu(pkg, logits, boxes, labels, tboxes, rows, cols, valid, nb)
    w = OL.set_losses(logits, boxes, labels, tboxes, rows, cols, valid, nb)
    np.testing.assert_allclose([ce, l1, giou], w[:3], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gx, w[3], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gb, w[4] + w[5], rtol=RTOL, atol=ATOL)


def test_no_matches_and_errors(pkg):
    logits, boxes, labels, tboxes, rows, cols, valid = _layer(3, 2, 2, 10, 5, 4)
    valid[:] = False
    ce, l1, giou, gx, gb = _gpu(pkg, logits, boxes, labels, tboxes, rows, cols, valid, 1.0)
    w = OL.set_losses(logits, boxes, labels, tboxes, rows, cols, valid, 1.0)
    np.testing.assert_allclose(ce, w[0], rtol=RTOL)
    assert l1 == 0.0 and giou == 0.0 and not gb.any()
    t = lambda x: torch.tensor(x, device=DEV)  # noqa: E731
    with pytest.raises(ValueError):
        pkg.set_losses(t(logits), t(boxes[:, :3]), t(labels), t(tboxes), t(rows), t(cols), t(valid.astype(np.uint8)),
                       1.0)


def test_stacked_layers(pkg):
    """Three layers in one launch (leading axis), each against the oracle; per-layer cotangents."""
    per = [_layer(60 + i, 2, 3, 20, 11, 6) for i in range(3)]
    labels, tboxes = per[0][2], per[0][3]
    logits = np.stack([p[0] for p in per])
    boxes = np.stack([p[1] for p in per])
    layer_match = []
    for lg, bx in zip(logits, boxes):
        mask = np.arange(tboxes.shape[1])[None] < (np.abs(tboxes).sum(-1) > 0).sum(1)[:, None]
        cost = OM.build_cost_matrix(lg, bx, labels, tboxes, mask)
        layer_match.append(OM.hungarian_match(cost, mask.sum(1).astype(np.int32), 3))
    rows, cols, valid = (np.stack([m[i] for m in layer_match]) for i in range(3))
    nb = 17.0
    t = lambda x: torch.tensor(x, device=DEV)  # noqa: E731
    x = t(logits).requires_grad_(True)
    b = t(boxes).requires_grad_(True)
    ce, l1, giou = pkg.set_losses(x, b, t(labels), t(tboxes), t(rows), t(cols), t(valid.astype(np.uint8)), nb)
    assert ce.shape == (3,)
    ct = torch.tensor([[0.5, 1.0, 2.0], [1.5, -1.0, 0.25], [1.0, 3.0, -0.5]], device=DEV)
    ((ce * ct[0]).sum() + (l1 * ct[1]).sum() + (giou * ct[2]).sum()).backward()
    ct = ct.cpu().numpy()
    for i in range(3):
        w = OL.set_losses(logits[i], boxes[i], labels, tboxes, rows[i], cols[i], valid[i], nb)
        got = [float(v[i].detach()) for v in (ce, l1, giou)]
        np.testing.assert_allclose(got, w[:3], rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(x.grad[i].cpu().numpy(), ct[0, i] * w[3], rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(b.grad[i].cpu().numpy(), ct[1, i] * w[4] + ct[2, i] * w[5], rtol=RTOL, atol=ATOL)


def test_unaligned_tiles(pkg):
    """Odd class count and query count: the tiles' logits are not 16-byte aligned (scalar path)."""
    logits, boxes, labels, tboxes, rows, cols, valid = _layer(77, 3, 1, 37, 13, 9)
    nb = max(float(valid.sum()), 1.0)
    ce, l1, giou, gx, gb = _gpu(pkg, logits, boxes, labels, tboxes, rows, cols, valid, nb)
    w = OL.set_losses(logits, boxes, labels, tboxes, rows, cols, valid, nb)
    np.testing.assert_allclose([ce, l1, giou], w[:3], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gx, w[3], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gb, w[4] + w[5], rtol=RTOL, atol=ATOL)
