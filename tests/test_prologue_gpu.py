"""Parity of the fused MSDA prologue (query -> sampling locations and attention weights,
``ops.py:381-404``) with a torch restatement of the reference's arithmetic, rounding steps
included: the projection rounded to the query dtype and the bias added in it (``layers.py:276-279``),
the softmax in float32, the point form's float32 division and the box form's division by P in the
query dtype.

Tolerances: float32 queries 1e-5 relative + 1e-6 absolute on every output.  bf16 queries: the
projection's float32 accumulation order differs from cuBLAS's, which can move a rounding to bf16
by one unit, so each location is within one bf16 unit per rounding its offset passes through
(divided by the level size, or scaled as in the box form) of the restatement's, fewer than 1% of
them differ at all, and the attention weights are within the bf16 tolerance (2e-2 of scale and
relative L2)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, assert_fp32_close

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _params(seed, C, H, L, P, dtype, B, Lq, ref_dim):
    g = torch.Generator().manual_seed(seed)
    hlp = H * L * P
    bound = 1.0 / np.sqrt(C)
    w_off = (torch.rand(hlp * 2, C, generator=g) * 2 - 1) * bound * 8
    b_off = torch.randn(hlp * 2, generator=g) * 2
    w_att = (torch.rand(hlp, C, generator=g) * 2 - 1) * bound
    b_att = torch.randn(hlp, generator=g) * 0.1
    query = torch.randn(B, Lq, C, generator=g).to(dtype)
    if ref_dim == 2:
        ref = torch.rand(B, Lq, L, 2, generator=g)
    else:
        ref = torch.cat([torch.rand(B, Lq, L, 2, generator=g), torch.rand(B, Lq, L, 2, generator=g) * 0.4 + 0.02], -1)
    return [t.to(DEV) for t in (query, ref, w_off, b_off, w_att, b_att)]


def _restated(query, ref, shapes, w_off, b_off, w_att, b_att, H, L, P):
    """The reference's prologue in torch float32 with its rounding steps."""
    B, Lq, _ = query.shape
    dt = query.dtype

    def linear(w, b):
        y = torch.matmul(query.float(), w.to(dt).float().t()).to(dt)
        return (y.float() + b.to(dt).float()).to(dt), y.float()

    off, proj = linear(w_off, b_off)
    off = off.reshape(B, Lq, H, L, P, 2)
    proj = proj.reshape(B, Lq, H, L, P, 2)
    logits = linear(w_att, b_att)[0].reshape(B, Lq, H, L * P)
    if ref.shape[-1] == 2:
        norm = torch.tensor([[w, h] for h, w in shapes], dtype=torch.float32, device=query.device)
        loc = ref[:, :, None, :, None, :] + off.float() / norm[None, None, None, :, None, :]
        step = norm[None, None, None, :, None, :]
    else:
        t = (off.float() / P).to(dt).float()
        loc = ref[:, :, None, :, None, :2] + t * ref[:, :, None, :, None, 2:] * 0.5
        step = P / (0.5 * ref[:, :, None, :, None, 2:])
    attn = torch.softmax(logits.float(), -1).to(dt)
    return loc, attn, off.float(), proj, step


CASES = [  # (C, H, L, P, shapes, B, Lq)
    (256, 16, 1, 2, ((24, 24),), 2, 700),                          # the Nano decoder (config 2 layout)
    (256, 8, 4, 4, ((80, 80), (40, 40), (20, 20), (10, 10)), 2, 300),  # four levels (config 3 layout)
    (64, 4, 2, 1, ((7, 9), (3, 5)), 1, 37),                        # ragged row tail, odd level shapes
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("ref_dim", [2, 4])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_forward(pkg, dtype, ref_dim, case):
    C, H, L, P, shapes, B, Lq = CASES[case]
    query, ref, w_off, b_off, w_att, b_att = _params(case * 10 + ref_dim, C, H, L, P, dtype, B, Lq, ref_dim)
    loc, attn = pkg.msda_prologue(query, ref, shapes, w_off, b_off, w_att, b_att, H, L, P)
    want_loc, want_attn, off, proj, step = _restated(query, ref, shapes, w_off, b_off, w_att, b_att, H, L, P)
    assert loc.dtype == torch.float32 and attn.dtype == dtype
    assert loc.shape == (B, Lq, H, L, P, 2) and attn.shape == (B, Lq, H, L * P)
    if dtype == torch.float32:
        assert_fp32_close(loc.cpu().numpy(), want_loc.cpu().numpy(), "loc")
        assert_fp32_close(attn.cpu().numpy(), want_attn.cpu().numpy(), "attn")
    else:
        # One bf16 unit at each rounding the offset passes through: the projection (before the
        # bias, so a bias that cancels much of it cannot hide the unit), the sum with the bias,
        # and in the box form the division by P; then divided by the level size (points) or
        # scaled by the box (boxes).
        def unit(x):
            return torch.ldexp(torch.ones_like(x), torch.frexp(x.abs().clamp_min(1e-30))[1] - 8)

        slack = unit(proj) + unit(off)
        if ref_dim == 4:
            slack = slack + unit(off / P) * P
        bound = slack / step + 1e-6
        err = (loc - want_loc).abs()
        assert (err <= bound).all(), f"loc: {int((err > bound).sum())} entries beyond one bf16 unit"
        assert (err > 1e-6).float().mean() < 0.01, "more than 1% of the locations differ"
        assert_bf16_close(attn.float().cpu().numpy(), want_attn.float().cpu().numpy(), "attn")


@pytest.mark.parametrize("ref_dim", [2, 4])
def test_backward(pkg, ref_dim):
    """Gradients with respect to the query, both projections and the reference points (float32)
    against torch autograd of the restatement."""
    C, H, L, P, shapes, B, Lq = CASES[1]
    leaves = _params(7 + ref_dim, C, H, L, P, torch.float32, B, 50, ref_dim)
    mine = [t.clone().requires_grad_(True) for t in leaves]
    theirs = [t.clone().requires_grad_(True) for t in leaves]
    g = torch.Generator(device=DEV).manual_seed(3)
    loc, attn = pkg.msda_prologue(mine[0], mine[1], shapes, *mine[2:], H, L, P)
    g_loc = torch.randn(loc.shape, generator=g, device=DEV)
    g_attn = torch.randn(attn.shape, generator=g, device=DEV)
    ((loc * g_loc).sum() + (attn * g_attn).sum()).backward()
    want_loc, want_attn, _, _, _ = _restated(theirs[0], theirs[1], shapes, *theirs[2:], H, L, P)
    ((want_loc * g_loc).sum() + (want_attn * g_attn).sum()).backward()
    for name, a, b in zip(("query", "ref", "w_off", "b_off", "w_att", "b_att"), mine, theirs, strict=True):
        assert_fp32_close(a.grad.cpu().numpy(), b.grad.cpu().numpy(), name, rtol=1e-4, atol=1e-5)


def test_feeds_the_sampler(pkg):
    """Prologue then sampler, bf16 end to end at the Nano layout: the sampler accepts the
    prologue's outputs as they are (layouts and dtypes)."""
    C, H, L, P, shapes, B, Lq = CASES[0]
    query, ref, w_off, b_off, w_att, b_att = _params(1, C, H, L, P, torch.bfloat16, B, Lq, 4)
    loc, attn = pkg.msda_prologue(query, ref, shapes, w_off, b_off, w_att, b_att, H, L, P)
    value = torch.randn(B * H, 24 * 24, C // H, device=DEV).to(torch.bfloat16)
    out = pkg.ms_deform_attn_core_rows(value, shapes, loc, attn, "cuda")
    assert out.shape == (B, Lq, C) and out.dtype == torch.bfloat16 and torch.isfinite(out.float()).all()


def test_rejects_bad_shapes(pkg):
    C, H, L, P, shapes, B, Lq = CASES[0]
    query, ref, w_off, b_off, w_att, b_att = _params(2, C, H, L, P, torch.bfloat16, B, 8, 2)
    with pytest.raises(ValueError):
        pkg.msda_prologue(query, ref[..., :1], shapes, w_off, b_off, w_att, b_att, H, L, P)
    with pytest.raises(ValueError):
        pkg.msda_prologue(query, ref, shapes, w_off[:-2], b_off, w_att, b_att, H, L, P)


@pytest.mark.parametrize("ref_dim", [2, 4])
def test_backward_bf16(pkg, ref_dim):
    """bf16 queries: the same gradients as torch autograd of the restatement, within the bf16
    tolerance (the saved attention weights and the query gradient are bf16)."""
    C, H, L, P, shapes, B, Lq = CASES[0]
    leaves = _params(17 + ref_dim, C, H, L, P, torch.bfloat16, B, 64, ref_dim)
    mine = [t.clone().requires_grad_(True) for t in leaves]
    theirs = [t.clone().requires_grad_(True) for t in leaves]
    g = torch.Generator(device=DEV).manual_seed(4)
    loc, attn = pkg.msda_prologue(mine[0], mine[1], shapes, *mine[2:], H, L, P)
    g_loc = torch.randn(loc.shape, generator=g, device=DEV)
    g_attn = torch.randn(attn.shape, generator=g, device=DEV).to(torch.bfloat16)
    ((loc * g_loc).sum() + (attn.float() * g_attn.float()).sum()).backward()
    want_loc, want_attn, _, _, _ = _restated(theirs[0], theirs[1], shapes, *theirs[2:], H, L, P)
    ((want_loc * g_loc).sum() + (want_attn.float() * g_attn.float()).sum()).backward()
    for name, a, b in zip(("query", "ref", "w_off", "b_off", "w_att", "b_att"), mine, theirs, strict=True):
        assert_bf16_close(a.grad.float().cpu().numpy(), b.grad.float().cpu().numpy(), name)
