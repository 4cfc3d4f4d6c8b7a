"""Pins the CPU oracle of the MSDA prologue (``oracle/prologue.py``).

* ``precise_divide`` known answers of the reference (``tests/test_ops.py:264-279``): the point
  form's division is the IEEE float32 quotient, for an array divisor and for the int 24.
* An independent torch evaluation of ``ops.py:381-404`` in the query dtype (torch's CPU bf16
  matmul accumulates in float32 and rounds once, as XLA's does): its locations equal the
  oracle's, or the oracle's other admissible rounding where the oracle marks the projection's
  rounding as ambiguous, bit for bit; its float32 locations agree to float32 accuracy.
* The analytic float64 gradient against torch float64 autograd of the same expression.
* ``bf16_round`` against torch's float32 -> bfloat16 conversion.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import prologue as OP


def _params(seed, C, H, L, P, B, Lq, ref_dim):
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


CASES = [  # (C, H, L, P, shapes, B, Lq)
    (256, 16, 1, 2, ((24, 24),), 1, 96),                              # the Nano decoder layout
    (256, 8, 4, 4, ((80, 80), (40, 40), (20, 20), (10, 10)), 1, 40),  # four levels (config 3)
    (64, 4, 2, 1, ((7, 9), (3, 5)), 2, 13),                          # odd shapes
]


def test_precise_divide_known_answers():
    """``tests/test_ops.py:264-279``: the quotient rounds once, for an array and an int divisor,
    and the point form's location is ``ref + precise_divide(offset, W)``."""
    rng = np.random.default_rng(0)
    numerator = rng.uniform(0.0, 6.3, (512, 1)).astype(np.float32)
    frequencies = (10000.0 ** (2 * (np.arange(128) // 2) / 128)).astype(np.float32)
    np.testing.assert_array_equal(OP.precise_divide(numerator, frequencies[None]), numerator / frequencies[None])
    np.testing.assert_array_equal(OP.precise_divide(numerator, 24), numerator / np.float32(24))
    off = np.zeros((1, 512, 1, 1, 1, 2), np.float32)
    off[0, :, 0, 0, 0, 0] = numerator[:, 0]
    off[0, :, 0, 0, 0, 1] = numerator[:, 0]
    loc = OP._locations(off, np.zeros((1, 512, 1, 2), np.float32), ((7, 24),), 1, "f32")
    np.testing.assert_array_equal(loc[0, :, 0, 0, 0, 0], numerator[:, 0] / np.float32(24))
    np.testing.assert_array_equal(loc[0, :, 0, 0, 0, 1], numerator[:, 0] / np.float32(7))


def test_bf16_round_matches_torch():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(10000).astype(np.float32) * 10 ** rng.uniform(-5, 5, 10000),
                        np.array([0.0, -0.0, np.inf, -np.inf, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8], np.float32)])
    want = torch.from_numpy(x.astype(np.float32)).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(OP.bf16_round(x), want)


def _torch_forward(query, ref, shapes, w_off, b_off, w_att, b_att, H, L, P, dtype):
    """``ops.py:381-404`` evaluated by torch ops in the query dtype on the CPU."""
    B, Lq, _ = query.shape
    q = torch.from_numpy(query).to(dtype)
    w = torch.from_numpy(np.concatenate([w_off, w_att], 0)).to(dtype)
    b = torch.from_numpy(np.concatenate([b_off, b_att], 0)).to(dtype)
    y = torch.matmul(q, w.t()) + b  # rounded to the query dtype after the product and the sum
    hlp = H * L * P
    off = y[..., :2 * hlp].reshape(B, Lq, H, L, P, 2)
    logits = y[..., 2 * hlp:].reshape(B, Lq, H, L * P)
    r = torch.from_numpy(ref)
    if ref.shape[-1] == 2:
        norm = torch.tensor([[w_, h_] for h_, w_ in shapes], dtype=torch.float32)
        loc = r[:, :, None, :, None, :] + off.float() / norm[None, None, None, :, None, :]
    else:
        t = (off / P).float()  # the division in the query dtype
        loc = r[:, :, None, :, None, :2] + t * r[:, :, None, :, None, 2:] * 0.5
    attn = torch.softmax(logits.float(), -1).to(dtype)
    return loc.numpy(), attn.float().numpy()


@pytest.mark.parametrize("ref_dim", [2, 4])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_forward_against_torch(case, ref_dim):
    C, H, L, P, shapes, B, Lq = CASES[case]
    args = _params(case * 10 + ref_dim, C, H, L, P, B, Lq, ref_dim)
    for dtype, tdt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        o = OP.prologue_forward(*args[:2], shapes, *args[2:], H, L, P, dtype)
        loc, attn = _torch_forward(*args[:2], shapes, *args[2:], H, L, P, tdt)
        if dtype == "bf16":
            ok = (loc == o["loc"]) | (loc == o["loc_alt"])
            assert ok.all(), f"{int((~ok).sum())} bf16 locations differ from both admissible roundings"
            assert (o["loc"] != o["loc_alt"]).mean() < 0.1, "too many ambiguous roundings for a meaningful pin"
            determined = ~(o["logits_ambiguous"].any(-1, keepdims=True) | o["attn_tie"])
            np.testing.assert_array_equal(attn[np.broadcast_to(determined, attn.shape)],
                                          o["attn"][np.broadcast_to(determined, attn.shape)])
        else:
            np.testing.assert_allclose(loc, o["loc"], rtol=2e-6, atol=1e-6)
            np.testing.assert_allclose(attn, o["attn"], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("ref_dim", [2, 4])
def test_backward_against_autograd(ref_dim):
    C, H, L, P, shapes, B, Lq = CASES[1]
    args = _params(5 + ref_dim, C, H, L, P, B, 7, ref_dim)
    query, ref, w_off, b_off, w_att, b_att = args
    rng = np.random.default_rng(9)
    g_loc = rng.standard_normal((B, 7, H, L, P, 2))
    g_attn = rng.standard_normal((B, 7, H, L * P))
    got = OP.prologue_backward(*args[:2], shapes, *args[2:], H, L, P, g_loc, g_attn, "f32")
    leaves = [torch.tensor(np.asarray(a, np.float64), requires_grad=True) for a in args]
    q, r, wo, bo, wa, ba = leaves
    off = (q @ wo.t() + bo).reshape(B, 7, H, L, P, 2)
    logits = (q @ wa.t() + ba).reshape(B, 7, H, L * P)
    if ref_dim == 2:
        norm = torch.tensor([[w_, h_] for h_, w_ in shapes], dtype=torch.float64)
        loc = r[:, :, None, :, None, :] + off / norm[None, None, None, :, None, :]
    else:
        loc = r[:, :, None, :, None, :2] + off / P * r[:, :, None, :, None, 2:] * 0.5
    attn = torch.softmax(logits, -1)
    ((loc * torch.from_numpy(g_loc)).sum() + (attn * torch.from_numpy(g_attn)).sum()).backward()
    for name, g, leaf in zip(("query", "ref", "w_off", "b_off", "w_att", "b_att"), got, leaves, strict=True):
        np.testing.assert_allclose(g, leaf.grad.numpy(), rtol=1e-6, atol=1e-6, err_msg=name)
