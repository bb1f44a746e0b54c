"""Parity of the sm_100a decode GEMV (q3xk_gemv) with the CPU oracle.

Bar (north star): max_r |y_r - y_ref_r| / sum_k |w_rk x_k| <= 1e-5, the
magnitude-scaled form of tests/q8_cpu_test.cpp:65-68.  Expected values are
the reference's own outputs (tests/golden) or the C port pinned to them.
"""
import numpy as np
import pytest

import oracle
from qwen3x_b200 import quant
from qwen3x_b200.capi import BF16, Q4_0, Q8_0
from qwen3x_b200.linear import Linear, expert_mv, mv, mv_add

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(params=[0, 1, 2, 3], ids=["auto", "register", "ring16", "ring24"], autouse=True)
def gemv_family(request):
    """Every case runs on each plain-GEMV kernel family (q3xk_gemv_set_family):
    the automatic choice, register batches, and the shared-memory ring with
    16 and 24 warps."""
    from qwen3x_b200.capi import lib

    assert lib().q3xk_gemv_set_family(request.param) == 0
    yield request.param
    lib().q3xk_gemv_set_family(0)


def run_mv(cuda, packed, mtype, rows, cols, x, accumulate_into=None):
    import torch

    lin = Linear.from_packed(packed, mtype, rows, cols, device=cuda)
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(cuda)
    if accumulate_into is None:
        yd = torch.full((rows,), float("nan"), device=cuda)
        mv(lin, xd, yd)
    else:
        yd = torch.from_numpy(np.ascontiguousarray(accumulate_into, np.float32)).to(cuda)
        mv_add(lin, xd, yd)
    torch.cuda.synchronize()
    return yd.cpu().numpy()


def scaled_err(y, ref, packed, mtype, rows, cols, x):
    mag = oracle.magnitude(packed, mtype, rows, cols, x)
    return float((np.abs(y.astype(np.float64) - ref) / np.maximum(mag, 1e-30)).max())


@pytest.mark.parametrize("name,rows,cols,xkey", [
    ("ka_q8", 2, 64, "ka_x64"), ("ka_q4a", 1, 64, "ka_x64"),
    ("ka_q4b", 2, 64, "ka_x64"), ("ka_q4c", 2, 32, "ka_x32")])
def test_known_answers(cuda, golden, name, rows, cols, xkey):
    """q8_cpu_test.cpp:309-369, q4_cpu_test.cpp:138-178, q4_cuda_test.cu:31-60 (|d| < 1e-5)."""
    t = Q8_0 if name.startswith("ka_q8") else Q4_0
    y = run_mv(cuda, golden[f"{name}_w"], t, rows, cols, golden[xkey])
    assert np.abs(y - golden[f"{name}_y_v2"]).max() < 1e-5


@pytest.mark.parametrize("rows", [3, 1023, 1024, 1031])
def test_subnormal_and_odd_rows(cuda, golden, rows):
    w, x = golden[f"sub_w_{rows}"], golden["sub_x"]
    y = run_mv(cuda, w, Q8_0, rows, 96, x)
    assert scaled_err(y, golden[f"sub_y_{rows}_v2"], w, Q8_0, rows, 96, x) <= TOL


def test_random_reference_cases(cuda, golden, golden_meta):
    from tests.golden.make_golden import make_random

    for case in golden_meta["random_cases"]:
        packed, x = make_random(case["type"], case["rows"], case["cols"], case["seed_w"],
                                case["seed_x"], case["encoder"])
        y = run_mv(cuda, packed, case["type"], case["rows"], case["cols"], x)
        err = scaled_err(y, golden[f"rnd_{case['name']}_y_v2"], packed, case["type"],
                         case["rows"], case["cols"], x)
        assert err <= TOL, (case["name"], err)


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_cfg1_full_size(cuda, mtype):
    """Benchmark config 1: W 12288x4096, w ~ N(0, 0.02), x ~ N(0, 1)."""
    rows, cols = 12288, 4096
    w = quant.gaussian((rows, cols), 1, 0.02)
    packed = quant.quantize(w, mtype)
    x = quant.gaussian(cols, 2)
    ref = oracle.mv(packed, mtype, rows, cols, x, threads=8)
    y = run_mv(cuda, packed, mtype, rows, cols, x)
    assert scaled_err(y, ref, packed, mtype, rows, cols, x) <= TOL
    assert np.abs(y - ref).max() / np.abs(ref).max() <= TOL


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
@pytest.mark.parametrize("rows,cols", [(1, 32), (5, 4096), (333, 2176), (4096, 768),
                                       (2048, 512), (31, 17408), (248, 5120)])
def test_shapes(cuda, mtype, rows, cols):
    """Ragged rows, K not a multiple of the warp span, TP-8 shard widths."""
    w = quant.gaussian((rows, cols), rows + cols, 0.02)
    packed = quant.quantize(w, mtype)
    x = quant.gaussian(cols, 7)
    ref = oracle.mv(packed, mtype, rows, cols, x, threads=4)
    y = run_mv(cuda, packed, mtype, rows, cols, x)
    assert scaled_err(y, ref, packed, mtype, rows, cols, x) <= TOL


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_accumulate_is_mv_add(cuda, mtype):
    """engine.cu:584-612 mv_add_*: y += W x."""
    rows, cols = 1000, 1024
    packed = quant.quantize(quant.gaussian((rows, cols), 3, 0.02), mtype)
    x = quant.gaussian(cols, 4)
    y0 = quant.gaussian(rows, 5)
    ref = y0.astype(np.float64) + oracle.mv(packed, mtype, rows, cols, x)
    y = run_mv(cuda, packed, mtype, rows, cols, x, accumulate_into=y0)
    mag = oracle.magnitude(packed, mtype, rows, cols, x) + np.abs(y0)
    assert (np.abs(y - ref) / mag).max() <= TOL


def test_zero_scale_blocks_and_zero_input(cuda):
    """Zero-scale blocks every 7th (tests/metal_test.mm:18-73 pattern) and x = 0."""
    rows, cols = 64, 1024
    packed = quant.quantize_q8_0(quant.gaussian((rows, cols), 8, 0.02))
    blocks = packed.reshape(-1).view(quant.Q8_DTYPE)
    blocks["scale"][::7] = 0
    x = quant.gaussian(cols, 9)
    ref = oracle.mv(packed, Q8_0, rows, cols, x)
    y = run_mv(cuda, packed, Q8_0, rows, cols, x)
    assert scaled_err(y, ref, packed, Q8_0, rows, cols, x) <= TOL
    y = run_mv(cuda, packed, Q8_0, rows, cols, np.zeros(cols, np.float32))
    assert np.all(y == 0)


def test_bf16_router_shape(cuda):
    """BF16 GEMV (the MoE router, engine.cpp:408), 256 x 2048."""
    rows, cols = 256, 2048
    bits = quant.to_bf16_bits(quant.gaussian((rows, cols), 10, 0.02))
    x = quant.gaussian(cols, 11)
    ref = oracle.mv(bits, BF16, rows, cols, x)
    y = run_mv(cuda, bits, BF16, rows, cols, x)
    assert scaled_err(y, ref, bits, BF16, rows, cols, x) <= TOL


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_expert_gemv(cuda, mtype):
    """engine.cpp:214-224: one expert of a contiguous pool."""
    import torch

    experts, rows, cols = 6, 96, 512
    packed = quant.quantize(quant.gaussian((experts * rows, cols), 12, 0.02), mtype)
    x = quant.gaussian(cols, 13)
    lin = Linear.from_packed(packed, mtype, rows, cols, experts=experts, device=cuda)
    xd = torch.from_numpy(x).to(cuda)
    per = packed.reshape(experts, -1)
    for e in (0, 3, 5):
        yd = torch.empty(rows, device=cuda)
        expert_mv(lin, e, xd, yd)
        ref = oracle.mv(per[e], mtype, rows, cols, x)
        assert scaled_err(yd.cpu().numpy(), ref, per[e], mtype, rows, cols, x) <= TOL


def test_deterministic(cuda):
    import torch

    rows, cols = 4096, 4096
    packed = quant.quantize_q4_0(quant.gaussian((rows, cols), 14, 0.02))
    lin = Linear.from_packed(packed, Q4_0, rows, cols, device=cuda)
    xd = torch.from_numpy(quant.gaussian(cols, 15)).to(cuda)
    a = torch.empty(rows, device=cuda)
    b = torch.empty(rows, device=cuda)
    mv(lin, xd, a)
    mv(lin, xd, b)
    assert torch.equal(a, b)


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_huge_inputs_take_exact_fallback(cuda, mtype):
    """x entries >= 2^104 send their unit to the unscaled decode path."""
    rows, cols = 200, 2048
    packed = quant.quantize(quant.gaussian((rows, cols), 16, 0.02), mtype)
    x = quant.gaussian(cols, 17)
    x[::97] *= np.float32(3e32)
    ref = oracle.mv(packed, mtype, rows, cols, x)
    y = run_mv(cuda, packed, mtype, rows, cols, x)
    assert np.all(np.isfinite(y))
    assert scaled_err(y, ref, packed, mtype, rows, cols, x) <= TOL


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_non_finite_inputs_propagate_like_reference(cuda, mtype):
    """inf/nan in x give the reference's inf/nan pattern (q*inf, 0*inf = nan)."""
    rows, cols = 64, 512
    packed = quant.quantize(quant.gaussian((rows, cols), 18, 0.02), mtype)
    x = quant.gaussian(cols, 19)
    x[5] = np.inf
    x[300] = -np.inf if mtype == Q8_0 else np.nan
    ref = oracle.mv(packed, mtype, rows, cols, x)
    y = run_mv(cuda, packed, mtype, rows, cols, x)
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    fin = ~np.isnan(ref)
    assert np.array_equal(y[fin], ref[fin]) or np.array_equal(np.sign(y[fin]), np.sign(ref[fin]))


@pytest.mark.parametrize("cols", [4096, 6144])
def test_bf16_chunked(cuda, cols):
    rows = 100
    bits = quant.to_bf16_bits(quant.gaussian((rows, cols), 20, 0.02))
    x = quant.gaussian(cols, 21)
    ref = oracle.mv(bits, BF16, rows, cols, x)
    y = run_mv(cuda, bits, BF16, rows, cols, x)
    assert scaled_err(y, ref, bits, BF16, rows, cols, x) <= TOL


def test_device_error_word_is_the_gemm_word(cuda):
    """q3xk_device_error reports the dequant-GEMM's bounded-wait word (the
    GEMVs have no device-side waits): after a GEMM it is 0 and equal to
    q3xk_gemm_device_error, and clearing keeps it 0."""
    import ctypes

    import torch

    from qwen3x_b200.capi import lib
    from qwen3x_b200.linear import Linear, batch_mv

    rows, cols, T = 256, 512, 16
    lin = Linear.from_packed(quant.quantize_q8_0(quant.gaussian((rows, cols), 30, 0.02)), Q8_0, rows, cols,
                             device=cuda)
    X = torch.randn(T, cols, device=cuda)
    Y = torch.empty(T, rows, device=cuda)
    batch_mv(lin, X, Y)
    flags, gemm = ctypes.c_int(-1), ctypes.c_int(-1)
    assert lib().q3xk_device_error(ctypes.byref(flags)) == 0
    assert lib().q3xk_gemm_device_error(ctypes.byref(gemm)) == 0
    assert flags.value == gemm.value == 0
    assert lib().q3xk_clear_device_error() == 0
    assert lib().q3xk_device_error(ctypes.byref(flags)) == 0 and flags.value == 0
