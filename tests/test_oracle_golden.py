"""Pin the C restatement (oracle/q3x_oracle.c) to the reference's own outputs.

Expected values come from tests/golden/, produced by the unmodified
reference (its CPU engine compiled into oracle/_ref, its Python packer) by
tests/golden/make_golden.py.  The port keeps the reference's FP32 operation
order, so it must equal the no-FMA (x86-64-v2) reference build bit for bit;
the AVX-512 build contracts some multiply-adds, so it is matched within the
reference's own CPU tolerance (tests/q8_cpu_test.cpp:65-68).
"""
import hashlib

import numpy as np
import pytest

import oracle
from qwen3x_b200 import quant

Q8, Q4 = oracle.Q8_0, oracle.Q4_0


def port_mv(w, t, rows, cols, x, threads=1):
    return oracle.mv(w, t, rows, cols, x, threads=threads, impl="port")


def test_f16_decode_exhaustive():
    """arch/cpu.cpp:31-52 for all 65536 encodings (NaN payloads compared as NaN)."""
    lib = oracle.port()
    bits = np.arange(65536, dtype=np.uint16)
    ours = np.array([lib.q3xo_f16(int(b)) for b in bits], np.float32)
    ref = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(ours), nan)
    assert np.array_equal(ours[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_f32_to_f16_matches_numpy():
    lib = oracle.port()
    rng = np.random.default_rng(3)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 6, 20000),
        np.float32([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e9, 2.0 ** -24, 2.0 ** -25,
                    2.0 ** -25 * 1.0000001, 3 * 2.0 ** -26, 2.0 ** -14, 6.0975552e-05]),
    ]).astype(np.float32)
    ours = np.array([lib.q3xo_f32_to_f16(float(v)) for v in vals], np.uint16)
    with np.errstate(over="ignore"):
        expected = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, expected)


def test_quantized_bytes_rules():
    """tests/q8_cpu_test.cpp:17-43."""
    import ctypes

    lib = oracle.port()
    out = ctypes.c_size_t(123)
    assert not lib.q3xo_quantized_bytes(oracle.BF16, 3, 17, ctypes.byref(out)) and out.value == 123
    assert lib.q3xo_quantized_bytes(Q8, 3, 64, ctypes.byref(out)) and out.value == 204
    assert lib.q3xo_quantized_bytes(Q4, 3, 64, ctypes.byref(out)) and out.value == 108
    out.value = 123
    for t in (oracle.BF16, Q8, Q4):
        assert not lib.q3xo_quantized_bytes(t, 0, 32, ctypes.byref(out))
        assert not lib.q3xo_quantized_bytes(t, 1, -32, ctypes.byref(out))
    assert not lib.q3xo_quantized_bytes(Q8, 1, 33, ctypes.byref(out))
    assert not lib.q3xo_quantized_bytes(Q4, 1, 16, ctypes.byref(out))
    assert not lib.q3xo_quantized_bytes(999, 1, 32, ctypes.byref(out))
    assert out.value == 123
    large_cols = 2147483616
    assert lib.q3xo_quantized_bytes(Q8, 2147483647, large_cols, ctypes.byref(out))
    assert out.value == 2147483647 * (large_cols // 32) * 34


@pytest.mark.parametrize("name,rows,cols,xkey", [
    ("ka_q8", 2, 64, "ka_x64"), ("ka_q4a", 1, 64, "ka_x64"),
    ("ka_q4b", 2, 64, "ka_x64"), ("ka_q4c", 2, 32, "ka_x32")])
def test_known_answer_mv(golden, name, rows, cols, xkey):
    t = Q8 if name.startswith("ka_q8") else Q4
    y = port_mv(golden[f"{name}_w"], t, rows, cols, golden[xkey])
    assert np.array_equal(y, golden[f"{name}_y_v2"])
    if f"{name}_y_v4" in golden:
        assert np.allclose(y, golden[f"{name}_y_v4"], rtol=0, atol=1e-6)


def test_known_answer_closed_form(golden):
    """q8_cpu_test.cpp:324-334 / q4_cuda_test.cu:42-48 expected sums in FP32."""
    x64 = golden["ka_x64"]
    scales = [1.0, 0.5, 2.0, 0.25]
    expected = []
    for row in range(2):
        acc = np.float32(0)
        for b in range(2):
            inner = np.float32(0)
            for i in range(32):
                inner = np.float32(inner + np.float32(((i % 9) - 4 + row * 2 + b) * x64[b * 32 + i]))
            acc = np.float32(acc + np.float32(scales[row * 2 + b]) * inner)
        expected.append(acc)
    assert np.allclose(golden["ka_q8_y_v2"], expected, atol=1e-6)


def test_embed_rows(golden):
    lib = oracle.port()
    out = np.zeros(64, np.float32)
    w = golden["ka_q8_w"]
    assert lib.q3xo_embed(w.ctypes.data, Q8, 64, 1, out.ctypes.data) == 0
    assert np.array_equal(out, golden["ka_q8_embed_row1"])
    w = golden["ka_q4a_w"]
    assert lib.q3xo_embed(w.ctypes.data, Q4, 64, 0, out.ctypes.data) == 0
    assert np.array_equal(out, golden["ka_q4a_embed_row0"])


@pytest.mark.parametrize("rows", [3, 1023, 1024, 1031])
def test_subnormal_scales(golden, rows):
    """q8_cpu_test.cpp:108-134 scales incl. the smallest FP16 subnormal."""
    y = port_mv(golden[f"sub_w_{rows}"], Q8, rows, 96, golden["sub_x"])
    assert np.array_equal(y, golden[f"sub_y_{rows}_v2"])
    mag = oracle.magnitude(golden[f"sub_w_{rows}"], Q8, rows, 96, golden["sub_x"])
    assert np.all(np.abs(y - golden[f"sub_y_{rows}_v4"]) <= 2e-6 * (1 + mag))


def _random_case(case):
    from tests.golden.make_golden import make_random

    packed, x = make_random(case["type"], case["rows"], case["cols"], case["seed_w"],
                            case["seed_x"], case["encoder"])
    assert hashlib.sha256(packed.tobytes()).hexdigest() == case["sha256_w"]
    assert hashlib.sha256(x.tobytes()).hexdigest() == case["sha256_x"]
    return packed, x


def test_random_mv_bit_exact(golden, golden_meta):
    for case in golden_meta["random_cases"]:
        packed, x = _random_case(case)
        rows, cols = case["rows"], case["cols"]
        for threads in (1, 5):
            y = port_mv(packed, case["type"], rows, cols, x, threads)
            assert np.array_equal(y, golden[f"rnd_{case['name']}_y_v2"]), case["name"]
        mag = oracle.magnitude(packed, case["type"], rows, cols, x)
        err = np.abs(y - golden[f"rnd_{case['name']}_y_v4"]) / mag
        assert err.max() <= 1e-6, case["name"]


@pytest.mark.parametrize("name,k", [("small", 3), ("wide", 8), ("random", 8), ("ties", 8)])
def test_router_top_k(golden, name, k):
    """engine.cpp:377-405; q4_cpu_test.cpp:180-202 expects {3,1,5} and 255..248."""
    ids, probs = oracle.router_top_k(golden[f"router_{name}_logits"], k)
    assert np.array_equal(ids, golden[f"router_{name}_ids"])
    assert np.array_equal(probs, golden[f"router_{name}_probs"])
    if name == "small":
        assert ids.tolist() == [3, 1, 5]
    if name == "wide":
        assert ids.tolist() == list(range(255, 247, -1))
    assert abs(float(probs[ids].sum()) - 1.0) < 1e-6


def test_moe_closed_form(golden):
    """q4_cpu_test.cpp:217-276: constant 0x99 nibbles give a closed form."""
    g = golden
    y, ids, w = oracle.moe(g["moe_const_router"], g["moe_const_gate_up"], g["moe_const_down"],
                           g["moe_const_shared_gate"], g["moe_const_shared_gate"],
                           g["moe_const_shared_down"], g["moe_const_shared_scale"], Q4,
                           4, 2, 32, 32, 32, g["moe_const_x"])
    assert np.array_equal(y, g["moe_const_y_v2"])
    assert np.array_equal(ids, g["moe_const_ids_v2"]) and np.array_equal(w, g["moe_const_w_v2"])
    assert np.allclose(y, g["moe_const_y_v4"], rtol=1e-5)

    def silu(v):
        return v / (1 + np.exp(-v))

    H = I = 32
    p1 = np.exp(2.0 - 4.0)
    e1 = 0.5 * I * silu(0.5 * H) * (0.5 * H)
    e2 = 1.0 * I * silu(1.0 * H) * (1.0 * H)
    routed = (p1 * e1 + e2) / (p1 + 1.0)
    shared = 1 / (1 + np.exp(-1.0)) * 0.25 * I * silu(0.25 * H) * (0.25 * H)
    assert np.all(np.abs(y - (routed + shared)) < 1e-2)


def test_moe_random(golden, golden_meta):
    from tests.golden.make_golden import make_moe_random

    p = golden_meta["moe_random"]
    args = make_moe_random(p)
    assert hashlib.sha256(b"".join(a.tobytes() for a in args)).hexdigest() == p["sha256"]
    router, gate_up, down, sg, su, sd, ss, x = args
    y, ids, w = oracle.moe(router, gate_up, down, sg, su, sd, ss, Q4, p["experts"], p["top_k"],
                           p["H"], p["I"], p["shared_I"], x)
    assert np.array_equal(ids, golden["moe_rnd_ids_v2"])
    assert np.array_equal(w, golden["moe_rnd_w_v2"])
    assert np.array_equal(y, golden["moe_rnd_y_v2"])


@pytest.mark.parametrize("case", ["q8_boundary", "q8_random", "q4_layout", "big"])
def test_quantizers_match_packer(golden, case):
    """scripts/pack_weights.py:299-343 bytes, for the C port and for the
    product's numpy encoders (tests/test_pack_weights.py:204-236 inputs)."""
    bits = golden[f"pack_{case}_bf16"]
    n = bits.size
    lib = oracle.port()
    q8 = np.zeros(n // 32 * 34, np.uint8)
    q4 = np.zeros(n // 32 * 18, np.uint8)
    assert lib.q3xo_quantize_q8_0(bits.ctypes.data, n, q8.ctypes.data) == 0
    assert lib.q3xo_quantize_q4_0(bits.ctypes.data, n, q4.ctypes.data) == 0
    assert np.array_equal(q8, golden[f"pack_{case}_q8"])
    assert np.array_equal(q4, golden[f"pack_{case}_q4"])
    vals = quant.bf16_to_f32(bits)
    assert np.array_equal(quant.quantize_q8_0(vals).reshape(-1), golden[f"pack_{case}_q8"])
    assert np.array_equal(quant.quantize_q4_0_ggml(vals).reshape(-1), golden[f"pack_{case}_q4"])
    if case == "q8_boundary":
        assert bytes(q8[:34]) == bytes(34)
        assert q8[36:42].view(np.int8).tolist() == [127, -127, 127, -127, 1, -1]
    if case == "q4_layout":
        assert bytes(q4[:2]) == b"\0\x80" and bytes(q4[2:18]) == bytes([0x88] * 16)


def test_quantizers_reject_non_finite():
    lib = oracle.port()
    bits = quant.to_bf16_bits(np.float32([0] * 4 + [np.inf] + [0] * 27))
    out = np.zeros(34, np.uint8)
    assert lib.q3xo_quantize_q8_0(bits.ctypes.data, 32, out.ctypes.data) == -1
    assert lib.q3xo_quantize_q4_0(bits.ctypes.data, 32, out.ctypes.data) == -1
    with pytest.raises(ValueError):
        quant.quantize_q8_0(np.float32([np.nan] * 32))


def test_baseline_q4_encoder_decodes_within_half_step():
    """The benchmark configs' Q4_0 encoder (d = max|w|/8): |w - dequant| <= d/2,
    except near +max where q saturates at 15 (error <= d, plus the FP16
    rounding of d)."""
    w = quant.gaussian((64, 256), 9, 0.02)
    packed = quant.quantize_q4_0(w)
    deq = quant.dequantize(packed, Q4, 64, 256)
    d = (np.abs(w).reshape(-1, 32).max(axis=1) / 8).repeat(32).reshape(64, 256)
    err = np.abs(w - deq)
    assert np.all(err <= d * (1 + 2.0 ** -8))
    inner = w < (7.5 * d)  # no saturation: within half a step
    assert np.all(err[inner] <= 0.5 * d[inner] * (1 + 2.0 ** -8) + 8 * d[inner] * 2.0 ** -11)


def test_file_sizes_recorded(golden_meta):
    assert golden_meta["file_sizes"] == {"9000": 9514418816, "36035": 19528534784}
