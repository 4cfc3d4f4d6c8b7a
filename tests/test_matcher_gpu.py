"""Parity of the CUDA matching cost (fp32 tolerance) and batched assignment (bit-exact vs SciPy,
the reference's own solver, on the same float32 cost)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import load_golden, match_inputs
from oracle import matcher as OM

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
COST_RTOL = 1e-5  # fp32 cost vs the float64 oracle: |err| <= 1e-5 + 1e-5 |ref|
COST_ATOL = 1e-5


def _t(x, dtype=None):
    t = torch.tensor(x, device=DEV)
    return t.to(dtype) if dtype is not None else t


def _match(pkg, cost, sizes, groups):
    rows, cols, valid = pkg.hungarian_match(_t(cost), _t(sizes), groups)
    return rows.cpu().numpy(), cols.cpu().numpy(), valid.cpu().numpy()


def _assert_same(got, want):
    for g, w, n in zip(got, want, ("rows", "cols", "valid"), strict=True):
        np.testing.assert_array_equal(g, w, err_msg=n)


def test_golden(pkg):
    d = load_golden("match_c4_small")
    cost = pkg.build_cost_matrix(_t(d["pred_logits"]), _t(d["pred_boxes"]), _t(d["target_labels"]),
                                 _t(d["target_boxes"]), _t(d["target_mask"]), 2.0, 5.0, 2.0, 0.25)
    np.testing.assert_allclose(cost.cpu().numpy(), d["cost"], rtol=COST_RTOL, atol=COST_ATOL)
    _assert_same(_match(pkg, d["cost"], d["sizes"], int(d["groups"])), (d["rows"], d["cols"], d["valid"]))


def test_config4_full_step(pkg):
    """Config 4 at training shape: 3 stacked layers x 8 images x 13 groups x 300 queries, T=100."""
    groups, per_group, classes, max_targets, batch = 13, 300, 91, 100, 8
    layers = []
    for layer in range(3):
        logits, boxes, labels, tboxes, mask, sizes = match_inputs(
            10, batch, groups * per_group, classes, max_targets)
        logits = np.random.default_rng(100 + layer).standard_normal(logits.shape).astype(np.float32)
        layers.append((logits, boxes))
    costs_gpu = torch.stack([pkg.build_cost_matrix(_t(lg), _t(bx), _t(labels), _t(tboxes), _t(mask), 2.0, 5.0, 2.0,
                                                   0.25) for lg, bx in layers])
    costs_ref = np.stack([OM.build_cost_matrix(lg, bx, labels, tboxes, mask) for lg, bx in layers])
    np.testing.assert_allclose(costs_gpu.cpu().numpy(), costs_ref, rtol=COST_RTOL, atol=COST_ATOL)
    # Bit-exact assignment on the same cost bits (the kernel's own cost).
    cost_np = costs_gpu.cpu().numpy()
    got = _match(pkg, cost_np, sizes, groups)
    want = OM.hungarian_match(cost_np, sizes, groups)
    _assert_same(got, want)
    # And the end-to-end pipeline against the oracle's pipeline.
    want_e2e = OM.hungarian_match(costs_ref, sizes, groups)
    _assert_same(got, want_e2e)


@pytest.mark.parametrize("kind", ["normal", "integer", "constant", "columns", "rows"])
def test_tie_heavy(pkg, kind):
    rng = np.random.default_rng(["normal", "integer", "constant", "columns", "rows"].index(kind))
    n, groups, per_group, max_targets = 6, 3, 40, 12
    shape = (n, groups * per_group, max_targets)
    if kind == "normal":
        cost = rng.standard_normal(shape).astype(np.float32)
    elif kind == "integer":
        cost = rng.integers(0, 3, shape).astype(np.float32)
    elif kind == "constant":
        cost = np.ones(shape, np.float32)
    elif kind == "columns":
        cost = np.repeat(rng.standard_normal((n, groups * per_group, 1)), max_targets, -1).astype(np.float32)
    else:
        cost = np.repeat(rng.standard_normal((n, 1, max_targets)), groups * per_group, 1).astype(np.float32)
    sizes = rng.integers(0, max_targets + 1, n).astype(np.int32)
    sizes[0], sizes[1] = 0, max_targets
    _assert_same(_match(pkg, cost, sizes, groups), OM.hungarian_match(cost, sizes, groups))


def test_square_and_wide_blocks(pkg):
    """size == per_group (no transpose) and size > per_group (more targets than queries)."""
    rng = np.random.default_rng(11)
    for per_group, max_targets, size in ((10, 10, 10), (8, 12, 12), (8, 12, 9), (1, 3, 3), (5, 5, 1)):
        cost = rng.standard_normal((2, 2 * per_group, max_targets)).astype(np.float32)
        sizes = np.array([size, max(0, size - 1)], np.int32)
        _assert_same(_match(pkg, cost, sizes, 2), OM.hungarian_match(cost, sizes, 2))


def test_non_finite_costs(pkg):
    """NaN/inf entries are replaced by max(finite)+1 before solving (matcher.py:169-172)."""
    rng = np.random.default_rng(12)
    cost = rng.standard_normal((4, 60, 9)).astype(np.float32)
    cost[0, 3, 2] = np.nan
    cost[1, :, 0] = np.inf
    cost[2, 10, :] = -np.inf
    cost[3, :30, :] = np.nan  # a whole block non-finite -> sentinel 1
    sizes = np.array([9, 5, 9, 7], np.int32)
    _assert_same(_match(pkg, cost, sizes, 2), OM.hungarian_match(cost, sizes, 2))


def test_reference_matcher_cases(pkg):
    """Restated reference tests: hand-solved 3x2 (test_matcher.py:103-111), folded leading axes
    (:89-100), padded sentinel columns, groups independent and empty images
    (test_criterion.py:67-106)."""
    cost = np.array([[[[4.0, 1.0], [2.0, 3.0], [9.0, 9.0]]]], np.float32)
    rows, cols, valid = _match(pkg, cost, np.array([2], np.int32), 1)
    assert sorted(zip(rows[0, 0][valid[0, 0]].tolist(), cols[0, 0][valid[0, 0]].tolist())) == [(0, 1), (1, 0)]

    rng = np.random.default_rng(3)
    stacked = rng.standard_normal((3, 2, 30, 4)).astype(np.float32) * 3
    stacked[..., 3:] = 1e4
    sizes = np.array([3, 3], np.int32)
    folded = _match(pkg, stacked, sizes, 2)
    for layer in range(3):
        alone = _match(pkg, stacked[layer], sizes, 2)
        for f, a in zip(folded, alone, strict=True):
            np.testing.assert_array_equal(f[layer], a)

    logits, boxes, labels, tboxes, mask, sizes = match_inputs(1, 2, 20, 7, 4, sizes=[3, 1])
    cost = pkg.build_cost_matrix(_t(logits), _t(boxes), _t(labels), _t(tboxes), _t(mask), 2.0, 5.0, 2.0, 0.25)
    rows, cols, valid = (x.cpu().numpy() for x in pkg.hungarian_match(cost, _t(sizes), 4))
    assert valid.sum(1).tolist() == [3 * 4, 1 * 4]
    empty = np.zeros((1, 8, 3), np.float32)
    rows, cols, valid = _match(pkg, empty, np.array([0], np.int32), 1)
    assert not valid.any() and not rows.any() and not cols.any()


def test_cost_dtypes_and_errors(pkg):
    logits, boxes, labels, tboxes, mask, _ = match_inputs(2, 2, 50, 91, 10)
    ref = OM.build_cost_matrix(logits.astype(np.float32), boxes, labels, tboxes, mask)
    bl = torch.tensor(logits, device=DEV).bfloat16()
    got = pkg.build_cost_matrix(bl, _t(boxes), _t(labels), _t(tboxes), _t(mask), 2.0, 5.0, 2.0, 0.25)
    ref_bf = OM.build_cost_matrix(bl.float().cpu().numpy(), boxes, labels, tboxes, mask)
    np.testing.assert_allclose(got.cpu().numpy(), ref_bf, rtol=COST_RTOL, atol=COST_ATOL)
    assert np.abs(got.cpu().numpy() - ref).max() < 0.1
    with pytest.raises(NotImplementedError):
        pkg.build_cost_matrix(_t(logits), _t(boxes), _t(labels), _t(tboxes), _t(mask), 2.0, 5.0, 2.0, 0.25,
                              pred_masks=_t(logits))
    with pytest.raises(ValueError, match="divide"):
        pkg.hungarian_match(_t(np.zeros((1, 10, 3), np.float32)), _t(np.array([1], np.int32)), 3)
    cfg = pkg.CriterionConfig(matcher="auction")
    with pytest.raises(ValueError, match="unknown matcher"):
        cfg.solve(_t(np.zeros((1, 10, 3), np.float32)), _t(np.array([1], np.int32)), 1)


def _stacked_inputs(seed, layers, batch, groups, per_group, classes, max_targets, sizes=None):
    logits, boxes, labels, tboxes, mask, sizes = match_inputs(seed, batch, groups * per_group, classes, max_targets,
                                                              sizes)
    rng = np.random.default_rng(seed + 1)
    lg = np.stack([logits] + [rng.standard_normal(logits.shape).astype(np.float32) for _ in range(layers - 1)])
    bx = np.stack([boxes] + [np.concatenate([rng.uniform(0.05, 0.95, boxes.shape[:-1] + (2,)),
                                             rng.uniform(0.02, 0.5, boxes.shape[:-1] + (2,))], -1).astype(np.float32)
                             for _ in range(layers - 1)])
    return lg, bx, labels, tboxes, mask, sizes


def _stacked_vs_separate(pkg, lg, bx, labels, tboxes, mask, sizes, groups, dtype=None):
    args = [_t(lg, dtype), _t(bx, dtype), _t(labels), _t(tboxes), _t(mask)]
    cost, rows, cols, valid = pkg.match_stacked(*args, _t(sizes), groups, 2.0, 5.0, 2.0, 0.25)
    sep = torch.stack([pkg.build_cost_matrix(args[0][i], args[1][i], *args[2:], 2.0, 5.0, 2.0, 0.25)
                       for i in range(lg.shape[0])])
    np.testing.assert_array_equal(cost.cpu().numpy(), sep.cpu().numpy())  # NaN where the separate cost has NaN
    want = pkg.hungarian_match(sep, _t(sizes), groups)
    _assert_same([x.cpu().numpy() for x in (rows, cols, valid)], [x.cpu().numpy() for x in want])
    return cost.cpu().numpy(), [x.cpu().numpy() for x in (rows, cols, valid)]


def test_stacked_config4(pkg):
    """Cost + assignment of 3 stacked layers in one call at config-4 training shape: the separate
    calls' cost bits and assignment, and SciPy's assignment on that cost."""
    sizes = np.random.default_rng(21).integers(1, 101, 8)
    sizes[0], sizes[1] = 100, 1
    lg, bx, labels, tboxes, mask, sizes = _stacked_inputs(21, 3, 8, 13, 300, 91, 100, sizes=sizes)
    cost, got = _stacked_vs_separate(pkg, lg, bx, labels, tboxes, mask, sizes, 13)
    _assert_same(got, OM.hungarian_match(cost, sizes, 13))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_stacked_dtypes_and_edges(pkg, dtype):
    """bf16 predictions, an image with no targets, and non-finite logits (the solver's sentinel
    replacement, matcher.py:169-172) -- all as the separate calls."""
    lg, bx, labels, tboxes, mask, sizes = _stacked_inputs(33, 2, 4, 3, 40, 7, 9, sizes=[0, 9, 4, 1])
    lg[1, 2, 5, :] = np.nan
    lg[0, 1, 7, 3] = np.inf
    _stacked_vs_separate(pkg, lg, bx, labels, tboxes, mask, sizes, 3, dtype)


def test_stacked_single_layer_shape(pkg):
    """No leading layer axis: ``[B, Q, C]`` in, ``[B, G*T]`` out."""
    lg, bx, labels, tboxes, mask, sizes = _stacked_inputs(44, 1, 3, 2, 25, 5, 6)
    cost, rows, cols, valid = pkg.match_stacked(_t(lg[0]), _t(bx[0]), _t(labels), _t(tboxes), _t(mask), _t(sizes), 2,
                                                2.0, 5.0, 2.0, 0.25)
    assert cost.shape == (3, 50, 6) and rows.shape == (3, 12) and valid.dtype == torch.bool
    _assert_same([x.cpu().numpy() for x in (rows, cols, valid)], OM.hungarian_match(cost.cpu().numpy(), sizes, 2))


@pytest.mark.parametrize("budget_kb", ["0", "3", "100"])
def test_stage_budgets(pkg, tuning, budget_kb):
    """The solver with no shared-memory stage (costs read through L1, the path of rows past the
    stage), with a stage that holds only a block's first rows (3 KB), and with a smaller stage
    than the default, set through RFDETR_LSAP_STAGE_KB: SciPy's assignment every time."""
    tuning("RFDETR_LSAP_STAGE_KB", budget_kb)
    rng = np.random.default_rng(5)
    groups, per_group, max_targets = 4, 60, 30
    cost = rng.standard_normal((5, groups * per_group, max_targets)).astype(np.float32)
    cost[1, 3, 2] = np.nan
    sizes = np.array([30, 1, 17, 0, 29], np.int32)
    _assert_same(_match(pkg, cost, sizes, groups), OM.hungarian_match(cost, sizes, groups))


def test_config4_reference_order_flips(pkg):
    """The kernel pipeline (one ``match_stacked`` call: device cost, device solve) against SciPy
    -- the reference's solver -- on the cost evaluated in float32 in the reference's operation
    order (``oracle.matcher.build_cost_matrix_f32``), at config 4's training shape: 312
    assignments.  The two costs differ in the last bits (at most ~4e-6; asserted < 2e-5, the tie
    margin an assignment must fall inside to flip) and 0 of the 312 assignments differ."""
    groups, per_group, classes, max_targets, batch = 13, 300, 91, 100, 8
    lg, bx, labels, tboxes, mask, sizes = _stacked_inputs(10, 3, batch, groups, per_group, classes, max_targets)
    cost, rows, cols, valid = pkg.match_stacked(_t(lg), _t(bx), _t(labels), _t(tboxes), _t(mask), _t(sizes), groups,
                                                2.0, 5.0, 2.0, 0.25)
    ref_cost = np.stack([OM.build_cost_matrix_f32(lg[i], bx[i], labels, tboxes, mask) for i in range(3)])
    assert np.abs(cost.cpu().numpy().astype(np.float64) - ref_cost).max() < 2e-5
    want = OM.hungarian_match(ref_cost, sizes, groups)
    got = [x.cpu().numpy().reshape(3 * batch, groups, max_targets) for x in (rows, cols, valid)]
    want = [x.reshape(3 * batch, groups, max_targets) for x in want]
    flips = ((got[0] != want[0]) | (got[1] != want[1]) | (got[2] != want[2])).any(-1)
    assert int(flips.sum()) == 0, f"{int(flips.sum())} of {flips.size} assignments differ"


def test_nonfinite_logits_follow_the_onehot(pkg):
    """A non-finite logit poisons its row's class costs as the reference's one-hot contraction
    does (x * 0 = NaN at every other target), an infinite logit at the target's own class gives an
    infinite cost, and a label outside [0, C) reads logit 0; the assignment after the solver's
    sentinel replacement is SciPy's on the oracle's cost."""
    logits, boxes, labels, tboxes, mask, sizes = match_inputs(77, 3, 60, 11, 8, sizes=[8, 5, 3])
    logits[0, 4, 6] = np.nan
    logits[1, 10, :] = 0.5
    logits[1, 10, labels[1, 0]] = np.inf
    logits[2, 7, 3] = -np.inf
    labels[2, 1] = 11          # outside [0, C): an all-zero one-hot row
    labels[2, 2] = -1
    cost = pkg.build_cost_matrix(_t(logits), _t(boxes), _t(labels), _t(tboxes), _t(mask), 2.0, 5.0, 2.0, 0.25)
    got = cost.cpu().numpy()
    want = OM.build_cost_matrix_f32(logits, boxes, labels, tboxes, mask)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))
    np.testing.assert_array_equal(np.isinf(got), np.isinf(want))
    fin = np.isfinite(want)
    np.testing.assert_allclose(got[fin], want[fin], rtol=COST_RTOL, atol=COST_ATOL)
    assert np.isnan(got[0, 4, :sizes[0]]).all() and np.isinf(got[1, 10, 0])
    _assert_same(_match(pkg, got, sizes, 2), OM.hungarian_match(want, sizes, 2))


def test_step_cap_reports_and_leaves_no_stale_slots(pkg, tuning):
    """A solve that reaches its iteration cap (forced here by capping every augmenting path at one
    scan step: every target wants the same query -- the blocks are tall, so they are solved
    transposed with targets as rows -- and the second target's insertion needs two) reports
    RFDETR_ERR_LIMIT through the device status word, which the host raises, and leaves its slots
    cleared -- nothing stale from before the call survives.  The cap is a pure-compute loop
    bound: nothing waits."""
    tuning("RFDETR_LSAP_STEP_CAP", "1")
    n, groups, per_group, max_targets = 3, 2, 20, 6
    cost = np.ones((n, groups * per_group, max_targets), np.float32)
    cost[:, 3::per_group, :] = 0.0  # in each group, every target prefers the group's query 3
    sizes = np.array([6, 4, 2], np.int32)
    N = pkg._native
    dev_cost, dev_sizes = _t(cost), _t(sizes)
    rows = torch.full((n, groups * max_targets), -7, dtype=torch.int32, device=DEV)
    cols = torch.full_like(rows, -7)
    valid = torch.full((n, groups * max_targets), 0xAB, dtype=torch.uint8, device=DEV)
    status = torch.zeros((1,), dtype=torch.int32, device=DEV)
    st = N.lib().rfdetr_lsap_batched(torch.cuda.current_stream().cuda_stream, N.ptr(dev_cost), N.ptr(dev_sizes), n,
                                     groups * per_group, max_targets, groups, N.ptr(rows), N.ptr(cols), N.ptr(valid),
                                     N.ptr(status))
    assert st == N.OK
    assert int(status.item()) == N.ERR_LIMIT
    assert not rows.any() and not cols.any() and not valid.any()
    with pytest.raises(RuntimeError, match="iteration cap"):
        pkg.hungarian_match(dev_cost, dev_sizes, groups, check=True)
    # The python API collects the status in a caller's tensor without synchronising.
    word = torch.zeros((1,), dtype=torch.int32, device=DEV)
    pkg.hungarian_match(dev_cost, dev_sizes, groups, status=word)
    with pytest.raises(RuntimeError):
        pkg.check_device_status(word)
    # With the default cap the same problems solve, as SciPy does.
    tuning("RFDETR_LSAP_STEP_CAP", None)
    word.zero_()
    got = pkg.hungarian_match(dev_cost, dev_sizes, groups, status=word)
    pkg.check_device_status(word)
    _assert_same([x.cpu().numpy() for x in got], OM.hungarian_match(cost, sizes, groups))


@pytest.mark.parametrize("per_group,max_targets", [(100, 30), (200, 30), (384, 12), (385, 12), (450, 20)])
@pytest.mark.parametrize("kind", ["normal", "integer"])
def test_column_counts(pkg, per_group, max_targets, kind):
    """Blocks of 1, 2 and 3 columns per thread (the register-resident solver, up to 384 columns)
    and wider ones (the work-list solver), with random and tie-heavy costs: SciPy's
    assignment."""
    rng = np.random.default_rng(per_group + max_targets)
    groups, n = 2, 3
    shape = (n, groups * per_group, max_targets)
    if kind == "normal":
        cost = rng.standard_normal(shape).astype(np.float32)
    else:
        cost = rng.integers(0, 3, shape).astype(np.float32)
    sizes = np.array([max_targets, 1, max_targets // 2], np.int32)
    _assert_same(_match(pkg, cost, sizes, groups), OM.hungarian_match(cost, sizes, groups))
