"""Parity of the CUDA two-stage selection (class max + top-k) and select_rows: bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import load_golden
from oracle import topk as OT

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _select(pkg, logits, k):
    s, v, i = pkg.two_stage_topk(torch.tensor(logits, device=DEV), k)
    return s.cpu().numpy(), v.cpu().numpy(), i.cpu().numpy()


def test_golden(pkg):
    d = load_golden("topk_c4_small")
    s, v, i = _select(pkg, d["logits"], 300)
    np.testing.assert_array_equal(i, d["indices"])
    np.testing.assert_array_equal(v.view(np.uint32), d["values"].view(np.uint32))
    np.testing.assert_array_equal(s.view(np.uint32), d["scores"].view(np.uint32))
    s, v, i = _select(pkg, d["tie_logits"], 300)
    np.testing.assert_array_equal(i, d["tie_indices"])
    np.testing.assert_array_equal(v, d["tie_values"])


@pytest.mark.parametrize("path", ["cluster ranks", "bitonic sort"])
def test_config4_training_shape(pkg, tuning, path):
    """Config 4 at training shape: 13 groups x 8 images x 576 proposals x 91 classes, through
    both selection kernels (the cluster rank count serves rows of up to 2048 positions, the
    bitonic sort longer rows; the switch forces the sort here)."""
    if path == "bitonic sort":
        tuning("RFDETR_TOPK_SORT", "1")
    logits = np.random.default_rng(4).standard_normal((13, 8, 576, 91)).astype(np.float32)
    s, v, i = _select(pkg, logits, 300)
    ws, wv, wi = OT.two_stage_select(logits, 300)
    np.testing.assert_array_equal(i, wi)
    np.testing.assert_array_equal(v, wv)
    np.testing.assert_array_equal(s, ws)
    assert i.dtype == np.int32


def test_ties_keep_lower_index_first(pkg):
    """jax.lax.top_k order: equal scores come out in ascending index order."""
    scores = np.array([[5.0, 4.0, 4.0, 1.0, 0.5, 0.1, 4.0, 4.0]], np.float32)
    v, i = pkg.top_k(torch.tensor(scores, device=DEV), 5)
    np.testing.assert_array_equal(i.cpu().numpy(), [[0, 1, 2, 6, 7]])
    constant = np.zeros((3, 1000), np.float32)
    _, i = pkg.top_k(torch.tensor(constant, device=DEV), 300)
    np.testing.assert_array_equal(i.cpu().numpy(), np.tile(np.arange(300), (3, 1)))


@pytest.mark.parametrize("path", ["cluster ranks", "bitonic sort"])
def test_special_values(pkg, tuning, path):
    """NaN first, then +inf ... -inf; +0 above -0 (IEEE totalOrder)."""
    if path == "bitonic sort":
        tuning("RFDETR_TOPK_SORT", "1")
    row = np.array([1.0, -np.inf, np.nan, 0.0, -0.0, np.inf, -1.0, 2.0], np.float32)
    v, i = pkg.top_k(torch.tensor(row[None], device=DEV), 8)
    wv, wi = OT.top_k(row[None], 8)
    np.testing.assert_array_equal(i.cpu().numpy(), wi)
    np.testing.assert_array_equal(np.isnan(v.cpu().numpy()), np.isnan(wv))
    logits = np.random.default_rng(5).standard_normal((2, 40, 7)).astype(np.float32)
    logits[0, 3, 2] = np.nan
    logits[1, 5, :] = -np.inf
    s, _, i = _select(pkg, logits, 40)
    ws, _, wi = OT.two_stage_select(logits, 40)
    np.testing.assert_array_equal(i, wi)
    np.testing.assert_array_equal(np.isnan(s), np.isnan(ws))


@pytest.mark.parametrize(("positions", "classes", "k"), [(1, 1, 1), (7, 3, 7), (576, 91, 1), (1000, 1, 999),
                                                          (5000, 2, 300), (16384, 1, 16384), (2049, 1, 2049),
                                                          (4097, 1, 1), (20000, 1, 4096), (27300, 1, 300),
                                                          (60000, 1, 100)])
def test_sizes(pkg, positions, classes, k):
    logits = np.random.default_rng(positions).integers(-50, 50, (3, positions, classes)).astype(np.float32)
    s, v, i = _select(pkg, logits, k)
    ws, wv, wi = OT.two_stage_select(logits, k)
    np.testing.assert_array_equal(i, wi)
    np.testing.assert_array_equal(v, wv)


@pytest.mark.parametrize("unstaged", [False, True])
def test_radix_staging(pkg, tuning, unstaged):
    """The radix select with the row's keys staged in shared memory (rows up to ~48k) and without
    (RFDETR_TOPK_UNSTAGED, the path of longer rows) on the same tie-heavy rows."""
    if unstaged:
        tuning("RFDETR_TOPK_UNSTAGED", "1")
    logits = np.random.default_rng(11).integers(-20, 20, (4, 27300, 1)).astype(np.float32)
    s, v, i = _select(pkg, logits, 300)
    ws, wv, wi = OT.two_stage_select(logits, 300)
    np.testing.assert_array_equal(i, wi)
    np.testing.assert_array_equal(v, wv)


def test_select_rows(pkg):
    rng = np.random.default_rng(7)
    for dtype, width in ((torch.float32, 256), (torch.bfloat16, 256), (torch.float32, 5), (torch.bfloat16, 3)):
        values = torch.tensor(rng.standard_normal((13, 2, 576, width)), device=DEV).to(dtype)
        idx = torch.tensor(rng.integers(0, 576, (13, 2, 300)), device=DEV, dtype=torch.int32)
        got = pkg.select_rows(values, idx)
        want = torch.take_along_dim(values, idx.long()[..., None], dim=2)
        assert torch.equal(got, want)
    with pytest.raises(ValueError, match="out of bounds"):
        pkg.select_rows(values, torch.full((13, 2, 4), 576, device=DEV, dtype=torch.int32))


def test_errors(pkg):
    x = torch.zeros((2, 10), device=DEV)
    with pytest.raises(ValueError):
        pkg.top_k(x, 11)
    with pytest.raises(ValueError):
        pkg.top_k(x.double(), 3)


def test_inference_post_process_shape(pkg):
    """The post-process selection (postprocess.py:37-41): top-300 of Q*C = 300*91 flattened
    sigmoid scores per image, 8 images -- the radix-select path -- bit-exact, with saturated
    scores (many exact 1.0 ties), NaN, +-inf and -0 in the rows."""
    rng = np.random.default_rng(27)
    logits = rng.standard_normal((8, 300 * 91)).astype(np.float32) * 4
    scores = (1.0 / (1.0 + np.exp(-logits.astype(np.float64)))).astype(np.float32)
    scores[0, :500] = 1.0            # ties at the top: lower index first
    scores[1, 123] = np.nan
    scores[2, 7] = np.inf
    scores[3, 5:9] = [-0.0, 0.0, -np.inf, np.nan]
    v, i = pkg.top_k(torch.tensor(scores, device=DEV), 300)
    wv, wi = OT.top_k(scores, 300)
    np.testing.assert_array_equal(i.cpu().numpy(), wi)
    np.testing.assert_array_equal(v.cpu().numpy().view(np.uint32), wv.view(np.uint32))


def test_post_process(pkg):
    """``post_process`` (postprocess.py:19-51) at the inference shape: 8 images x 300 queries x 91
    classes, top 300.  The selection is checked bit-exact against the oracle on the same sigmoid
    scores (the sigmoid itself is an elementwise device op); labels exactly; boxes to float32."""
    rng = np.random.default_rng(31)
    logits = torch.tensor(rng.standard_normal((8, 300, 91)).astype(np.float32) * 3, device=DEV)
    boxes = np.concatenate([rng.uniform(0.05, 0.95, (8, 300, 2)), rng.uniform(-0.05, 0.5, (8, 300, 2))], -1)
    boxes = torch.tensor(boxes.astype(np.float32), device=DEV)
    sizes = torch.tensor(rng.integers(200, 1300, (8, 2)).astype(np.int32), device=DEV)
    scores, labels, xyxy = pkg.post_process(logits, boxes, sizes, 300)
    probs = torch.sigmoid(logits).reshape(8, -1).cpu().numpy()
    ws, wl, wb = OT.post_process(probs, boxes.cpu().numpy(), sizes.cpu().numpy(), 91, 300)
    np.testing.assert_array_equal(scores.cpu().numpy().view(np.uint32), ws.view(np.uint32))
    np.testing.assert_array_equal(labels.cpu().numpy(), wl)
    np.testing.assert_allclose(xyxy.cpu().numpy(), wb, rtol=1e-6, atol=1e-4)
    assert labels.dtype == torch.int32 and xyxy.shape == (8, 300, 4)
