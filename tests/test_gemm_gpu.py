"""Parity of the tcgen05 dequant-GEMM (q3xk_gemm / q3xk_gemm_ex) with the CPU oracle.

The reference CPU prefill is a per-token mv (engine.cpp:580-583), so the
oracle of Y[T, N] = X W^T is T independent matvecs.  Error measure:
max |Y - Y_ref| / sum_k |w_nk x_tk|.  Bars:
  split precision (q3xk_gemm's default): 1e-5, the CUDA-core GEMV's bar --
    both operands carry a residual FP16 plane, so the result is FP32-grade;
  FP16 precision (q3xk_gemm_ex, GEMM_FP16): 2e-3, the north-star bar for
    tensor-core prefill (measured ~1e-4).
"""
import numpy as np
import pytest

import oracle
from qwen3x_b200 import quant
from qwen3x_b200.capi import GEMM_FP16, GEMM_SPLIT, Q4_0, Q8_0
from qwen3x_b200.linear import Linear, batch_mv

pytestmark = pytest.mark.gpu

TOL = {GEMM_SPLIT: 1e-5, GEMM_FP16: 2e-3, None: 1e-5}
PRECISIONS = [None, GEMM_FP16]  # None = q3xk_gemm (split)


def run_gemm(cuda, packed, mtype, rows, cols, X, Y0=None, precision=None):
    import torch

    lin = Linear.from_packed(packed, mtype, rows, cols, device=cuda)
    Xd = torch.from_numpy(np.ascontiguousarray(X, np.float32)).to(cuda)
    if Y0 is None:
        Yd = torch.full((X.shape[0], rows), float("nan"), device=cuda)
    else:
        Yd = torch.from_numpy(np.ascontiguousarray(Y0, np.float32)).to(cuda)
    batch_mv(lin, Xd, Yd, add=Y0 is not None, precision=precision)
    torch.cuda.synchronize()
    return Yd.cpu().numpy()


def check(Y, packed, mtype, rows, cols, X, tokens=None, Y0=None):
    tokens = range(X.shape[0]) if tokens is None else tokens
    w = np.abs(quant.dequantize(packed, mtype, rows, cols).astype(np.float64))
    worst = 0.0
    for t in tokens:
        ref = oracle.mv(packed, mtype, rows, cols, X[t], threads=8).astype(np.float64)
        mag = w @ np.abs(X[t].astype(np.float64))
        if Y0 is not None:
            ref = ref + Y0[t]
            mag = mag + np.abs(Y0[t])
        worst = max(worst, float((np.abs(Y[t] - ref) / np.maximum(mag, 1e-30)).max()))
    return worst


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
@pytest.mark.parametrize("T,rows,cols", [(1, 128, 64), (8, 256, 512), (64, 333, 2176),
                                         (129, 1000, 1024), (300, 128, 4096)])
def test_gemm_shapes(cuda, mtype, T, rows, cols, precision):
    packed = quant.quantize(quant.gaussian((rows, cols), rows + cols + T, 0.02), mtype)
    X = quant.gaussian((T, cols), 7 + T)
    Y = run_gemm(cuda, packed, mtype, rows, cols, X, precision=precision)
    assert np.all(np.isfinite(Y))
    err = check(Y, packed, mtype, rows, cols, X)
    assert err <= TOL[precision], err


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_gemm_accumulate(cuda, mtype, precision):
    T, rows, cols = 40, 256, 1024
    packed = quant.quantize(quant.gaussian((rows, cols), 3, 0.02), mtype)
    X = quant.gaussian((T, cols), 4)
    Y0 = quant.gaussian((T, rows), 5)
    Y = run_gemm(cuda, packed, mtype, rows, cols, X, Y0, precision=precision)
    assert check(Y, packed, mtype, rows, cols, X, Y0=Y0) <= TOL[precision]


@pytest.mark.parametrize("precision", PRECISIONS)
def test_gemm_activation_range(cuda, precision):
    """Per-token scaling keeps FP16 in range for large and tiny activations."""
    T, rows, cols = 6, 256, 512
    packed = quant.quantize_q8_0(quant.gaussian((rows, cols), 8, 0.02))
    X = quant.gaussian((T, cols), 9)
    X[0] *= 1e6
    X[1] *= 1e-6
    X[2, ::3] = 0.0
    Y = run_gemm(cuda, packed, Q8_0, rows, cols, X, precision=precision)
    assert check(Y, packed, Q8_0, rows, cols, X) <= TOL[precision]


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
@pytest.mark.parametrize("T,rows,cols,add", [(2, 4096, 4096, False), (8, 4096, 4096, True), (16, 4096, 12288, False),
                                             (17, 4096, 4096, False), (64, 4096, 4096, True),
                                             (8, 12288, 4096, False), (5, 2048, 5120, True)])
def test_gemm_few_tokens_split_k(cuda, mtype, T, rows, cols, add, precision):
    """Few tokens: 16- and 64-token tiles with K split over CTAs (tiles < SMs;
    the last segment to finish adds the partials in segment order).  Two calls
    give bit-identical results (deterministic reduction, counters reset)."""
    import torch

    packed = quant.quantize(quant.gaussian((rows, cols), 40 + T, 0.02), mtype)
    X = quant.gaussian((T, cols), 41 + T)
    Y0 = quant.gaussian((T, rows), 42) if add else None
    Y = run_gemm(cuda, packed, mtype, rows, cols, X, Y0, precision=precision)
    assert np.all(np.isfinite(Y))
    assert check(Y, packed, mtype, rows, cols, X, Y0=Y0) <= TOL[precision]
    lin = Linear.from_packed(packed, mtype, rows, cols, device=cuda)
    Xd = torch.from_numpy(X).to(cuda)
    outs = []
    for _ in range(2):
        Yd = torch.zeros(T, rows, device=cuda)
        batch_mv(lin, Xd, Yd, precision=precision)
        outs.append(Yd)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_gemm_split_weight_residual_exact(cuda, mtype):
    """Split precision holds d*q exactly (w_hi + w_lo): with X = one-hot rows
    the GEMM returns single dequantised weights, which must equal the oracle's
    FP32 d*q bit for bit (including subnormal and large scales)."""
    rows, cols = 128, 256
    w = quant.gaussian((rows, cols), 11, 0.02)
    w[3] *= 1e-4   # tiny scales (FP16 subnormal products)
    w[7] *= 300.0  # large scales
    packed = quant.quantize(w, mtype)
    X = np.zeros((cols, cols), np.float32)
    X[np.arange(cols), np.arange(cols)] = 1.0
    Y = run_gemm(cuda, packed, mtype, rows, cols, X, precision=GEMM_SPLIT)
    ref = quant.dequantize(packed, mtype, rows, cols).astype(np.float32)
    assert np.array_equal(Y.T, ref)


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_gemm_cfg2_full_size(cuda, mtype, precision):
    """Benchmark config 2: T=4096, K=4096, N=12288; oracle on 12 sampled tokens."""
    T, rows, cols = 4096, 12288, 4096
    packed = quant.quantize(quant.gaussian((rows, cols), 1, 0.02), mtype)
    X = quant.gaussian((T, cols), 2)
    Y = run_gemm(cuda, packed, mtype, rows, cols, X, precision=precision)
    assert np.all(np.isfinite(Y))
    sample = [0, 1, 127, 128, 129, 1000, 2047, 2048, 3000, 4094, 4095, 511]
    assert check(Y, packed, mtype, rows, cols, X, tokens=sample) <= TOL[precision]


def test_gemm_no_device_timeouts(cuda):
    import ctypes

    from qwen3x_b200.capi import lib

    flags = ctypes.c_int(-1)
    assert lib().q3xk_gemm_device_error(ctypes.byref(flags)) == 0
    assert flags.value == 0
