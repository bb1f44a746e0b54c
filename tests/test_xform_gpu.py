"""Input transforms of the _ex GEMVs (q3xk_xform): RMSNorm, DeltaNet gated
RMS and SwiGLU applied while the GEMV stages x.  Expected: the CPU oracle's
GEMV of the transformed vector, the transform computed in float64 by the
reference's formulas (engine.cpp:231-242, :374, :415-416), within the GEMV
bar (1e-5 of sum_k |w_rk x_k|).
"""
import ctypes

import numpy as np
import pytest

import oracle
from qwen3x_b200 import capi
from qwen3x_b200.capi import BF16, Q4_0, Q8_0, XForm, lib
from qwen3x_b200.linear import Linear
from qwen3x_b200.quant import gaussian, quantize, to_bf16_bits

pytestmark = pytest.mark.gpu

TOL = 1e-5
EPS = 1e-6


def silu(v):
    return v / (1.0 + np.exp(-v))


def rms_ref(x, w1):
    x = x.astype(np.float64)
    return x / np.sqrt(np.mean(x * x) + EPS) * w1


def gated_ref(o, norm, z, group):
    o = o.astype(np.float64).reshape(-1, group)
    scale = 1.0 / np.sqrt(np.mean(o * o, axis=1, keepdims=True) + EPS)
    return (o * scale * norm[None, :] * silu(z.astype(np.float64).reshape(-1, group))).reshape(-1)


def check(y, packed, mtype, rows, cols, xeff):
    xeff32 = xeff.astype(np.float32)
    ref = oracle.mv(packed, mtype, rows, cols, xeff32)
    mag = oracle.magnitude(packed, mtype, rows, cols, xeff32)
    err = float((np.abs(y.astype(np.float64) - ref) / np.maximum(mag, 1e-30)).max())
    assert err <= TOL, err


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda)


def packed_matrix(mtype, rows, cols, seed):
    w = gaussian((rows, cols), seed=seed, std=0.02)
    if mtype == BF16:
        return to_bf16_bits(w)
    return quantize(w, mtype)


@pytest.mark.parametrize("family", [0, 1], ids=["auto", "register"])
@pytest.mark.parametrize("mtype", [Q8_0, Q4_0, BF16])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (333, 512), (2048, 5120)])
def test_rms_xform(cuda, mtype, rows, cols, family):
    """RMSNorm applied while staging x, on the default kernel family (the ring
    GEMV for Q8_0 / Q4_0, statistics computed in its prologue) and on the
    register GEMV."""
    import torch

    assert lib().q3xk_gemv_set_family(family) == 0

    packed = packed_matrix(mtype, rows, cols, 3)
    lin = Linear.from_packed(packed, mtype, rows, cols, device=cuda)
    x = gaussian((cols,), seed=4, std=3.0)
    w1 = (1.0 + gaussian((cols,), seed=5, std=0.01)).astype(np.float32)
    xd, wd = dev(x, cuda), dev(w1, cuda)
    yd = torch.full((rows,), float("nan"), device=cuda)
    xf = XForm(kind=capi.XFORM_RMS, group=0, w=wd.data_ptr())
    try:
        capi.check(lib().q3xk_gemv_ex(ctypes.byref(lin.m), xd.data_ptr(), yd.data_ptr(), 0, ctypes.byref(xf),
                                      capi.stream_ptr()), "gemv_ex")
        torch.cuda.synchronize()
    finally:
        lib().q3xk_gemv_set_family(0)
    check(yd.cpu().numpy(), packed, mtype, rows, cols, rms_ref(x, w1))


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_gated_rms_xform_accumulate(cuda, mtype):
    import torch

    rows, cols, group = 1024, 4096, 128
    packed = packed_matrix(mtype, rows, cols, 6)
    lin = Linear.from_packed(packed, mtype, rows, cols, device=cuda)
    o = gaussian((cols,), seed=7, std=0.5)
    z = gaussian((cols,), seed=8, std=1.0)
    norm = (1.0 + gaussian((group,), seed=9, std=0.01)).astype(np.float32)
    y0 = gaussian((rows,), seed=10, std=1.0)
    yd = dev(y0, cuda)
    od, zd, nd = dev(o, cuda), dev(z, cuda), dev(norm, cuda)
    xf = XForm(kind=capi.XFORM_GATED_RMS, group=group, w=nd.data_ptr(), z=zd.data_ptr())
    capi.check(lib().q3xk_gemv_ex(ctypes.byref(lin.m), od.data_ptr(), yd.data_ptr(), 1, ctypes.byref(xf),
                                  capi.stream_ptr()), "gemv_ex")
    torch.cuda.synchronize()
    check(yd.cpu().numpy() - y0, packed, mtype, rows, cols, gated_ref(o, norm, z, group))


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_swiglu_xform(cuda, mtype):
    import torch

    rows, width = 512, 1024
    packed = packed_matrix(mtype, rows, width, 11)
    lin = Linear.from_packed(packed, mtype, rows, width, device=cuda)
    gu = gaussian((2 * width,), seed=12, std=2.0)
    gd = dev(gu, cuda)
    yd = torch.full((rows,), float("nan"), device=cuda)
    xf = XForm(kind=capi.XFORM_SWIGLU, group=width)
    capi.check(lib().q3xk_gemv_ex(ctypes.byref(lin.m), gd.data_ptr(), yd.data_ptr(), 0, ctypes.byref(xf),
                                  capi.stream_ptr()), "gemv_ex")
    torch.cuda.synchronize()
    g, u = gu[:width].astype(np.float64), gu[width:].astype(np.float64)
    check(yd.cpu().numpy(), packed, mtype, rows, width, silu(g) * u)


def test_moe_xforms_match_unfused_sequence(cuda):
    """rows_ex with RMS and segments_ex with weighted SwiGLU equal the unfused
    rms -> rows -> swiglu -> segments sequence (MoE decode, engine.cpp:406-430)."""
    import torch

    from qwen3x_b200.linear import expert_mv_rows, expert_mv_segments, swiglu

    E, S, H, I = 9, 5, 512, 256
    gup = Linear.from_packed(quantize(gaussian((E * 2 * I, H), seed=13, std=0.02), Q4_0), Q4_0, 2 * I, H,
                             experts=E, device=cuda)
    dnp = Linear.from_packed(quantize(gaussian((E * H, I), seed=14, std=0.02), Q4_0), Q4_0, H, I, experts=E,
                             device=cuda)
    x = gaussian((H,), seed=15, std=1.5)
    w1 = (1.0 + gaussian((H,), seed=16, std=0.01)).astype(np.float32)
    ids = torch.tensor([3, 0, 8, 5, 1], dtype=torch.int32, device=cuda)
    wts = dev(np.array([0.4, 0.3, 0.2, 0.1, 0.7], np.float32), cuda)
    xd, w1d = dev(x, cuda), dev(w1, cuda)
    stream = capi.stream_ptr()
    # fused
    gu = torch.empty(S * 2 * I, device=cuda)
    y = torch.zeros(H, device=cuda)
    xr = XForm(kind=capi.XFORM_RMS, w=w1d.data_ptr())
    capi.check(lib().q3xk_expert_gemv_rows_ex(ctypes.byref(gup.m), ids.data_ptr(), S, xd.data_ptr(),
                                              gu.data_ptr(), 0, ctypes.byref(xr), stream), "rows_ex")
    xs = XForm(kind=capi.XFORM_SWIGLU, group=I, seg_weights=wts.data_ptr())
    capi.check(lib().q3xk_expert_gemv_segments_ex(ctypes.byref(dnp.m), ids.data_ptr(), S, gu.data_ptr(),
                                                  y.data_ptr(), 1, ctypes.byref(xs), stream), "segments_ex")
    # unfused
    xn = dev(rms_ref(x, w1).astype(np.float32), cuda)
    gu2 = torch.empty(S * 2 * I, device=cuda)
    h = torch.empty(S * I, device=cuda)
    y2 = torch.zeros(H, device=cuda)
    expert_mv_rows(gup, ids, S, xn, gu2)
    swiglu(gu2, wts, S, I, h)
    expert_mv_segments(dnp, ids, S, h, y2, accumulate=True)
    torch.cuda.synchronize()
    scale = float(y2.abs().max())
    assert float((y - y2).abs().max()) <= 1e-5 * scale
    assert float((gu - gu2).abs().max()) <= 1e-5 * float(gu2.abs().max())


def test_xform_validation(cuda):
    import torch

    lin = Linear.from_packed(packed_matrix(Q8_0, 64, 256, 1), Q8_0, 64, 256, device=cuda)
    x = torch.zeros(512, device=cuda)
    y = torch.zeros(64, device=cuda)
    f = lib().q3xk_gemv_ex
    bad = [XForm(kind=capi.XFORM_RMS),  # no weights
           XForm(kind=capi.XFORM_GATED_RMS, group=100, w=x.data_ptr(), z=x.data_ptr()),  # not a divisor
           XForm(kind=capi.XFORM_SWIGLU, group=128),  # width != cols
           XForm(kind=9)]
    for xf in bad:
        assert f(ctypes.byref(lin.m), x.data_ptr(), y.data_ptr(), 0, ctypes.byref(xf), capi.stream_ptr()) != 0
    ok = XForm(kind=capi.XFORM_NONE)
    assert f(ctypes.byref(lin.m), x.data_ptr(), y.data_ptr(), 0, ctypes.byref(ok), capi.stream_ptr()) == 0
    assert f(ctypes.byref(lin.m), x.data_ptr(), y.data_ptr(), 0, None, capi.stream_ptr()) == 0
