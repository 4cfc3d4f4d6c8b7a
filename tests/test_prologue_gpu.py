"""Parity of the fused MSDA prologue (query -> sampling locations and attention weights,
``ops.py:381-404``) with the CPU oracle ``oracle/prologue.py``, which restates the reference's
arithmetic with its rounding steps: the projection rounded to the query dtype and the bias added
in it (``layers.py:276-279``), the softmax in float32, the point form's float32 division and the
box form's division by P in the query dtype.

Tolerances:

* bf16 queries: every location bit-identical to the oracle's, or to the oracle's other
  admissible rounding where the projection's rounding to bf16 is not determined by a float32
  sum (the oracle marks those; fewer than 10% of the entries); every attention weight
  bit-identical wherever the oracle's bf16 rounding is determined, and within the bf16 tolerance
  (2e-2 of scale and relative L2) everywhere.
* float32 queries: 1e-5 relative + 1e-6 absolute on every output.
* gradients against the oracle's float64 gradient: float32 within 1e-4 relative + 1e-5 absolute
  (float32 GEMM accumulation), bf16 within the bf16 tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, assert_fp32_close
from oracle import prologue as OP

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _params(seed, C, H, L, P, B, Lq, ref_dim):
    """Seeded float32 NumPy parameters (the Nano init's scales, offsets spread by x8)."""
    rng = np.random.default_rng(seed)
    hlp = H * L * P
    bound = 1.0 / np.sqrt(C)
    w_off = (rng.uniform(-1, 1, (hlp * 2, C)) * bound * 8).astype(np.float32)
    b_off = (rng.standard_normal(hlp * 2) * 2).astype(np.float32)
    w_att = (rng.uniform(-1, 1, (hlp, C)) * bound).astype(np.float32)
    b_att = (rng.standard_normal(hlp) * 0.1).astype(np.float32)
    query = rng.standard_normal((B, Lq, C)).astype(np.float32)
    ref = rng.uniform(0, 1, (B, Lq, L, 2)).astype(np.float32)
    if ref_dim == 4:
        ref = np.concatenate([ref, (rng.uniform(0, 1, (B, Lq, L, 2)) * 0.4 + 0.02).astype(np.float32)], -1)
    return query, ref, w_off, b_off, w_att, b_att


def _dev(args, dtype):
    query, ref, w_off, b_off, w_att, b_att = args
    q = torch.tensor(query, device=DEV).to(dtype)
    return [q] + [torch.tensor(a, device=DEV) for a in (ref, w_off, b_off, w_att, b_att)]


CASES = [  # (C, H, L, P, shapes, B, Lq)
    (256, 16, 1, 2, ((24, 24),), 2, 700),                          # the Nano decoder (config 2 layout)
    (256, 8, 4, 4, ((80, 80), (40, 40), (20, 20), (10, 10)), 2, 300),  # four levels (config 3 layout)
    (64, 4, 2, 1, ((7, 9), (3, 5)), 1, 37),                        # ragged row tail, odd level shapes
    (48, 6, 1, 4, ((9, 7),), 1, 29),                               # 6 heads: the per-row backward kernel
]


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("ref_dim", [2, 4])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_forward(pkg, dtype, ref_dim, case):
    C, H, L, P, shapes, B, Lq = CASES[case]
    args = _params(case * 10 + ref_dim, C, H, L, P, B, Lq, ref_dim)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    dev_args = _dev(args, tdt)
    loc, attn = pkg.msda_prologue(*dev_args[:2], shapes, *dev_args[2:], H, L, P)
    want = OP.prologue_forward(*args[:2], shapes, *args[2:], H, L, P, dtype)
    assert loc.dtype == torch.float32 and attn.dtype == tdt
    assert loc.shape == (B, Lq, H, L, P, 2) and attn.shape == (B, Lq, H, L * P)
    loc = loc.cpu().numpy()
    attn = attn.float().cpu().numpy()
    # The biased offsets the launch keeps for the box form's backward (``offsets_out``).
    from rfdetr_jax_b200 import ops as rops

    weight = torch.cat([dev_args[2], dev_args[4]], 0).to(tdt).contiguous()
    bias = torch.cat([dev_args[3], dev_args[5]], 0).float().contiguous()
    _, _, off = rops._prologue_launch(dev_args[0].contiguous(), dev_args[1].contiguous(), shapes, weight, bias, H, L,
                                      P, True)
    off = off.cpu().numpy().reshape(want["offsets"].shape)
    if dtype == "f32":
        assert_fp32_close(loc, want["loc"], "loc")
        assert_fp32_close(attn, want["attn"], "attn")
        # The raw projection: float32 accumulation over C products (the locations divide it by
        # the map size, so they meet the tighter bound).
        assert_fp32_close(off, want["offsets"], "offsets", rtol=1e-4, atol=1e-5)
        return
    ok_off = (off == want["offsets"]) | (off == want["offsets_alt"])
    assert ok_off.all(), f"offsets: {int((~ok_off).sum())} of {ok_off.size} differ from both admissible roundings"
    ok = (loc == want["loc"]) | (loc == want["loc_alt"])
    assert ok.all(), f"loc: {int((~ok).sum())} of {ok.size} differ from both admissible roundings"
    assert (want["loc"] != want["loc_alt"]).mean() < 0.1
    determined = np.broadcast_to(~(want["logits_ambiguous"].any(-1, keepdims=True) | want["attn_tie"]), attn.shape)
    assert determined.mean() > 0.3  # a head of 16 logits is undetermined if any of them is
    np.testing.assert_array_equal(attn[determined], want["attn"][determined], err_msg="attn (determined entries)")
    assert_bf16_close(attn, want["attn"], "attn")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("ref_dim", [2, 4])
@pytest.mark.parametrize("case", [0, 1, 3])
def test_backward(pkg, dtype, ref_dim, case):
    """Gradients with respect to the query, both projections and the reference points against
    the oracle's float64 gradient, at the config-2 and config-3 layouts."""
    C, H, L, P, shapes, B, _ = CASES[case]
    Lq = 64
    args = _params(7 + ref_dim + 10 * case, C, H, L, P, B, Lq, ref_dim)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    leaves = [t.requires_grad_(True) for t in _dev(args, tdt)]
    rng = np.random.default_rng(3 + case)
    g_loc = rng.standard_normal((B, Lq, H, L, P, 2)).astype(np.float32)
    g_attn = rng.standard_normal((B, Lq, H, L * P)).astype(np.float32)
    if dtype == "bf16":
        g_attn = OP.bf16_round(g_attn)
    loc, attn = pkg.msda_prologue(leaves[0], leaves[1], shapes, *leaves[2:], H, L, P)
    ((loc * torch.tensor(g_loc, device=DEV)).sum()
     + (attn.float() * torch.tensor(g_attn, device=DEV)).sum()).backward()
    want = OP.prologue_backward(*args[:2], shapes, *args[2:], H, L, P, g_loc, g_attn, dtype)
    for name, leaf, w in zip(("query", "ref", "w_off", "b_off", "w_att", "b_att"), leaves, want, strict=True):
        got = leaf.grad.float().cpu().numpy()
        if dtype == "f32":
            assert_fp32_close(got, w, name, rtol=1e-4, atol=1e-5)
        else:
            assert_bf16_close(got, w, name)


def test_feeds_the_sampler(pkg):
    """Prologue then sampler, bf16 end to end at the Nano layout: the sampler accepts the
    prologue's outputs as they are (layouts and dtypes)."""
    C, H, L, P, shapes, B, Lq = CASES[0]
    query, ref, w_off, b_off, w_att, b_att = _dev(_params(1, C, H, L, P, B, Lq, 4), torch.bfloat16)
    loc, attn = pkg.msda_prologue(query, ref, shapes, w_off, b_off, w_att, b_att, H, L, P)
    value = torch.randn(B * H, 24 * 24, C // H, device=DEV).to(torch.bfloat16)
    out = pkg.ms_deform_attn_core_rows(value, shapes, loc, attn, "cuda")
    assert out.shape == (B, Lq, C) and out.dtype == torch.bfloat16 and torch.isfinite(out.float()).all()


def test_rejects_bad_shapes(pkg):
    C, H, L, P, shapes, B, Lq = CASES[0]
    query, ref, w_off, b_off, w_att, b_att = _dev(_params(2, C, H, L, P, B, 8, 2), torch.bfloat16)
    with pytest.raises(ValueError):
        pkg.msda_prologue(query, ref[..., :1], shapes, w_off, b_off, w_att, b_att, H, L, P)
    with pytest.raises(ValueError):
        pkg.msda_prologue(query, ref, shapes, w_off[:-2], b_off, w_att, b_att, H, L, P)
