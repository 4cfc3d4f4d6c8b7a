"""Generates the committed golden fixtures for the hot path (run from the repo root).

    python tests/golden/make_golden.py

The reference (JAX) is not installable in this environment, so the expected outputs come from
the CPU oracle (``oracle/``), which is itself pinned against the reference's known-answer tests,
``torch.nn.functional.grid_sample`` and SciPy (see ``oracle/__init__.py``).  Matcher fixtures use
SciPy's ``linear_sum_assignment`` -- the reference's own solver -- for the assignments.

Inputs follow the shapes and distributions of the benchmark configs (config 1 exactly; configs
2-4 at reduced batch/query counts so the files stay small), with the seeds listed below.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import matcher as OM  # noqa: E402
from oracle import msda as OS  # noqa: E402
from oracle import topk as OT  # noqa: E402


def softmax(x, axis=-1):
    x = x - x.max(axis=axis, keepdims=True)
    e = np.exp(x)
    return e / e.sum(axis=axis, keepdims=True)


def sampler_case(seed, batch, len_query, heads, shapes, points, dim, lo, hi, logit_sigma, bf16):
    rng = np.random.default_rng(seed)
    total = sum(h * w for h, w in shapes)
    levels = len(shapes)
    value = rng.standard_normal((batch * heads, total, dim)).astype(np.float32)
    loc = rng.uniform(lo, hi, (batch, len_query, heads, levels, points, 2)).astype(np.float32)
    attn = softmax(rng.normal(0.0, logit_sigma, (batch, len_query, heads, levels * points))).astype(np.float32)
    grad = rng.standard_normal((batch, len_query, heads * dim)).astype(np.float32)
    if bf16:
        value, attn, grad = OS.bf16_round(value), OS.bf16_round(attn), OS.bf16_round(grad)
    out = OS.ms_deform_attn_forward(value, shapes, loc, attn)
    gv, gl, ga = OS.ms_deform_attn_backward(value, shapes, loc, attn, grad)
    # Expected outputs are float64 results rounded to float32 (far below every tolerance);
    # bf16-valued inputs are stored as their 16-bit patterns.
    def pack(x):
        return (x.view(np.uint32) >> 16).astype(np.uint16) if bf16 else x

    return dict(value=pack(value), loc=loc, attn=pack(attn), grad=pack(grad), shapes=np.asarray(shapes, np.int64),
                out=out.astype(np.float32), grad_value=gv.astype(np.float32), grad_loc=gl.astype(np.float32),
                grad_attn=ga.astype(np.float32), bf16=np.asarray(bf16))


def main():
    cases = {
        # Config 1 exactly: B=2, 24x24, 16 heads x 16, Lq=300, P=2, fp32, seed 0.
        "msda_c1": sampler_case(0, 2, 300, 16, ((24, 24),), 2, 16, 0.0, 1.0, 1.0, False),
        # Config 2 distributions (bf16 value/weights, loc U(-0.05, 1.05)) at B=1, Lq=390.
        "msda_c2_small": sampler_case(1, 1, 390, 16, ((24, 24),), 2, 16, -0.05, 1.05, 1.0, True),
        # Config 3 geometry at B=1, 2 heads, Lq=60 (4 levels, head_dim 32, 4 points, logits N(0,2)).
        "msda_c3_small": sampler_case(2, 1, 60, 2, ((80, 80), (40, 40), (20, 20), (10, 10)), 4, 32, 0.0, 1.0,
                                      2.0, False),
        # Edge shapes: odd head_dim, 1-wide levels, far out-of-bounds samples.
        "msda_edge": sampler_case(5, 2, 17, 3, ((5, 1), (1, 7), (3, 3)), 3, 5, -0.6, 1.6, 1.0, False),
    }
    for name, arrays in cases.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)

    # Config 4 selection: logits N(0,1) [G=2, B=2, 576, 91] plus a tie-heavy row set.
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((2, 2, 576, 91)).astype(np.float32)
    ties = rng.integers(-3, 3, (2, 576, 91)).astype(np.float32)
    scores, values, indices = OT.two_stage_select(logits, 300)
    tscores, tvalues, tindices = OT.two_stage_select(ties, 300)
    np.savez_compressed(os.path.join(HERE, "topk_c4_small.npz"), logits=logits, scores=scores, values=values,
                        indices=indices, tie_logits=ties, tie_scores=tscores, tie_values=tvalues,
                        tie_indices=tindices)

    # Config 4 matching at B=2, 2 groups of 300 queries, T=100 padded targets.
    batch, groups, per_group, classes, max_targets = 2, 2, 300, 91, 100
    queries = groups * per_group
    sizes = np.array([37, 100], np.int32)
    labels = rng.integers(0, classes, (batch, max_targets)).astype(np.int32)
    cxcy = rng.uniform(0.05, 0.95, (batch, max_targets, 2))
    wh = rng.uniform(0.02, 0.5, (batch, max_targets, 2))
    tboxes = np.concatenate([cxcy, wh], -1).astype(np.float32)
    mask = np.arange(max_targets)[None, :] < sizes[:, None]
    labels = np.where(mask, labels, 0).astype(np.int32)
    tboxes = np.where(mask[..., None], tboxes, 0.0).astype(np.float32)
    plogits = rng.standard_normal((batch, queries, classes)).astype(np.float32)
    pcxcy = rng.uniform(0.05, 0.95, (batch, queries, 2))
    pwh = rng.uniform(0.02, 0.5, (batch, queries, 2))
    pboxes = np.concatenate([pcxcy, pwh], -1).astype(np.float32)
    cost = OM.build_cost_matrix(plogits, pboxes, labels, tboxes, mask, 2.0, 5.0, 2.0, 0.25)
    rows, cols, valid = OM.hungarian_match(cost, sizes, groups)
    np.savez_compressed(os.path.join(HERE, "match_c4_small.npz"), pred_logits=plogits, pred_boxes=pboxes,
                        target_labels=labels, target_boxes=tboxes, target_mask=mask, sizes=sizes, cost=cost,
                        rows=rows, cols=cols, valid=valid, groups=np.asarray(groups))
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
