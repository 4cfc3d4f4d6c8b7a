"""The workspace-free backward entry point, ``rfdetr_msda_backward_noalloc``, against the
regular one.

Some callers cannot hand the library a device workspace: a framework whose allocator owns all
device memory and gives its custom calls no scratch buffer, or code that must not allocate after
start-up.  For them the bf16 backward keeps its float32 accumulator in a static device array of
the library instead of a caller-provided workspace.  This test calls both entry points through
the C ABI on config-2 inputs and checks that two consecutive no-alloc calls each reproduce the
workspace call within the bf16 tolerance the other tests use (the array keeps the previous
call's contents, so the second call also checks that it is cleared) and the oracle, that a
problem needing more scratch than the array holds is refused without a launch, and that a large
problem the scratch-free kernels serve is not refused.  It lives in its own file, collected
last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, assert_fp32_close, sampler_inputs
from oracle import msda as O

pytestmark = pytest.mark.gpu

B, LQ, H, D, P = 8, 3900, 16, 16, 2
SHAPES = ((24, 24),)


def _buffers(dev):
    value, loc, attn, grad = sampler_inputs(21, B, LQ, H, SHAPES, P, D, lo=-0.05, hi=1.05)
    t = lambda x, dt: torch.tensor(x, device=dev).to(dt)  # noqa: E731
    return (t(value, torch.bfloat16), t(loc, torch.float32), t(attn, torch.bfloat16), t(grad, torch.bfloat16))


def _grads(dev, value, loc, attn):
    return torch.empty_like(value), torch.empty_like(loc), torch.empty_like(attn)


def test_noalloc_backward_matches_workspace_backward(pkg):
    N = pkg._native
    lib = N.lib()
    dev = torch.device("cuda:0")
    value, loc, attn, grad = _buffers(dev)
    shapes = N.int64_array([24, 24])
    stream = torch.cuda.current_stream(dev).cuda_stream

    gv, gl, ga = _grads(dev, value, loc, attn)
    ws_bytes = lib.rfdetr_msda_backward_workspace_size(N.BF16, B, H, D, 576)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    N.check(lib.rfdetr_msda_backward(stream, value.data_ptr(), N.BF16, shapes, None, loc.data_ptr(),
                                     attn.data_ptr(), N.BF16, grad.data_ptr(), N.BF16, gv.data_ptr(), gl.data_ptr(),
                                     ga.data_ptr(), ws.data_ptr(), ws_bytes, B, H, D, LQ, 1, P), "backward")
    torch.cuda.synchronize()
    want = [x.float().cpu().numpy() for x in (gv, gl, ga)]

    for call in range(2):
        nv, nl, na = _grads(dev, value, loc, attn)
        N.check(lib.rfdetr_msda_backward_noalloc(stream, value.data_ptr(), N.BF16, shapes, None, loc.data_ptr(),
                                                 attn.data_ptr(), N.BF16, grad.data_ptr(), N.BF16, nv.data_ptr(),
                                                 nl.data_ptr(), na.data_ptr(), B, H, D, LQ, 1, P),
                f"backward_noalloc call {call}")
        torch.cuda.synchronize()
        got = [x.float().cpu().numpy() for x in (nv, nl, na)]
        assert_bf16_close(got[0], want[0], f"call {call}: grad_value")
        assert_fp32_close(got[1], want[1], f"call {call}: grad_loc")
        assert_bf16_close(got[2], want[2], f"call {call}: grad_attn")

    # The no-alloc result agrees with the oracle too (the bf16 contract), on two of the images:
    # all three gradients.
    v = value.float().cpu().numpy()
    ref = O.ms_deform_attn_backward(v[: 2 * H], SHAPES, loc[:2].cpu().numpy(), attn[:2].float().cpu().numpy(),
                                    grad[:2].float().cpu().numpy())
    assert_bf16_close(got[0][: 2 * H], ref[0], "oracle: grad_value")
    assert_bf16_close(got[1][:2], ref[1], "oracle: grad_loc")
    assert_bf16_close(got[2][:2], ref[2], "oracle: grad_attn")


@pytest.mark.parametrize("weights_dtype", [torch.bfloat16, torch.float32])
def test_noalloc_uses_its_static_scratch(pkg, weights_dtype):
    """A shape served by the accumulate-in-scratch kernels (6 samples per head, 8 channels), so the
    static array is what holds the float32 accumulator; two calls in a row."""
    N = pkg._native
    lib = N.lib()
    dev = torch.device("cuda:0")
    shapes = ((8, 16), (4, 8))
    b, lq, h, p, d = 2, 70, 8, 3, 8
    value, loc, attn, grad = sampler_inputs(23, b, lq, h, shapes, p, d, lo=-0.1, hi=1.1)
    v = torch.tensor(value, device=dev).bfloat16()
    l = torch.tensor(loc, device=dev)
    a = torch.tensor(attn, device=dev).to(weights_dtype)
    out_dtype = torch.bfloat16 if weights_dtype == torch.bfloat16 else torch.float32
    g = torch.tensor(grad, device=dev).to(out_dtype)
    flat = N.int64_array([8, 16, 4, 8])
    stream = torch.cuda.current_stream(dev).cuda_stream
    lv = 8 * 16 + 4 * 8
    wd = N.dtype_code(weights_dtype)
    od = N.dtype_code(out_dtype)

    gv, gl, ga = torch.empty_like(v), torch.empty_like(l), torch.empty_like(a)
    ws_bytes = lib.rfdetr_msda_backward_workspace_size(N.BF16, b, h, d, lv)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    N.check(lib.rfdetr_msda_backward(stream, v.data_ptr(), N.BF16, flat, None, l.data_ptr(), a.data_ptr(), wd,
                                     g.data_ptr(), od, gv.data_ptr(), gl.data_ptr(), ga.data_ptr(), ws.data_ptr(),
                                     ws_bytes, b, h, d, lq, 2, p), "backward")
    torch.cuda.synchronize()
    want = [x.float().cpu().numpy() for x in (gv, gl, ga)]
    for call in range(2):
        nv, nl, na = torch.empty_like(v), torch.empty_like(l), torch.empty_like(a)
        N.check(lib.rfdetr_msda_backward_noalloc(stream, v.data_ptr(), N.BF16, flat, None, l.data_ptr(), a.data_ptr(),
                                                 wd, g.data_ptr(), od, nv.data_ptr(), nl.data_ptr(), na.data_ptr(), b,
                                                 h, d, lq, 2, p), f"backward_noalloc call {call}")
        torch.cuda.synchronize()
        got = [x.float().cpu().numpy() for x in (nv, nl, na)]
        assert_bf16_close(got[0], want[0], f"call {call}: grad_value")
        assert_bf16_close(got[1], want[1], f"call {call}: grad_loc")
        assert_bf16_close(got[2], want[2], f"call {call}: grad_attn")
    # And the oracle, on the same bf16-rounded inputs: all three gradients.
    f64 = lambda t: t.double().cpu().numpy()  # noqa: E731
    ref = O.ms_deform_attn_backward(f64(v), shapes, f64(l), f64(a), f64(g))
    for name, x, r in zip(("grad_value", "grad_loc", "grad_attn"), got, ref, strict=True):
        assert_bf16_close(x, r, f"oracle: {name}")


def _oversize(dev, b, h, shapes, p, d, lq):
    value, loc, attn, grad = sampler_inputs(29, b, lq, h, shapes, p, d, lo=-0.1, hi=1.1)
    t = lambda x, dt: torch.tensor(x, device=dev).to(dt)  # noqa: E731
    return t(value, torch.bfloat16), t(loc, torch.float32), t(attn, torch.bfloat16), t(grad, torch.bfloat16)


def test_noalloc_refuses_problems_beyond_its_scratch(pkg):
    """A shape that only the accumulate-in-scratch kernel serves, with more than 2,097,152 value
    elements (256 images x 8 heads x 160 positions x 8 channels): refused with
    RFDETR_ERR_CAPACITY, before any launch; the outputs stay untouched."""
    N = pkg._native
    lib = N.lib()
    dev = torch.device("cuda:0")
    b, h, d, p, lq = 256, 8, 8, 3, 2
    shapes = ((8, 16), (4, 8))
    v, l, a, g = _oversize(dev, b, h, shapes, p, d, lq)
    gv = torch.full_like(v, 7.0)
    gl, ga = torch.empty_like(l), torch.empty_like(a)
    status = lib.rfdetr_msda_backward_noalloc(torch.cuda.current_stream(dev).cuda_stream, v.data_ptr(), N.BF16,
                                              N.int64_array([8, 16, 4, 8]), None, l.data_ptr(), a.data_ptr(), N.BF16,
                                              g.data_ptr(), N.BF16, gv.data_ptr(), gl.data_ptr(), ga.data_ptr(), b, h,
                                              d, lq, 2, p)
    assert status == N.ERR_CAPACITY
    assert "static scratch" in N.status_text(status)
    torch.cuda.synchronize()
    assert bool((gv == 7.0).all())


def test_noalloc_serves_large_scratch_free_shapes(pkg):
    """The Nano decoder layout at 64 images (9.4M value elements, beyond the array) is served by
    the scratch-free owner kernel, so the no-alloc entry point takes it and matches the regular
    entry point."""
    N = pkg._native
    lib = N.lib()
    dev = torch.device("cuda:0")
    b, lq = 64, 300
    v, l, a, g = _oversize(dev, b, H, SHAPES, P, D, lq)
    stream = torch.cuda.current_stream(dev).cuda_stream
    shapes = N.int64_array([24, 24])
    out = []
    for noalloc in (False, True):
        gv, gl, ga = torch.empty_like(v), torch.empty_like(l), torch.empty_like(a)
        if noalloc:
            st = lib.rfdetr_msda_backward_noalloc(stream, v.data_ptr(), N.BF16, shapes, None, l.data_ptr(),
                                                  a.data_ptr(), N.BF16, g.data_ptr(), N.BF16, gv.data_ptr(),
                                                  gl.data_ptr(), ga.data_ptr(), b, H, D, lq, 1, P)
        else:
            ws_bytes = lib.rfdetr_msda_backward_workspace_size(N.BF16, b, H, D, 576)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
            st = lib.rfdetr_msda_backward(stream, v.data_ptr(), N.BF16, shapes, None, l.data_ptr(), a.data_ptr(),
                                          N.BF16, g.data_ptr(), N.BF16, gv.data_ptr(), gl.data_ptr(), ga.data_ptr(),
                                          ws.data_ptr(), ws_bytes, b, H, D, lq, 1, P)
        N.check(st, "noalloc" if noalloc else "backward")
        torch.cuda.synchronize()
        out.append([x.float().cpu().numpy() for x in (gv, gl, ga)])
    # The owner kernel's float32 accumulation order follows its shared-memory slot order, so two
    # runs can differ by one bf16 unit in grad_value: compare within the bf16 tolerance.
    for name, x, y in zip(("grad_value", "grad_loc", "grad_attn"), out[1], out[0], strict=True):
        assert_bf16_close(x, y, name)
