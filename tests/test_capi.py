"""Host-side checks of the q3xk C ABI (no GPU needed, no kernel launched)."""
import ctypes
import re
from pathlib import Path

import pytest

from qwen3x_b200 import capi
from qwen3x_b200.capi import Matrix, lib

ROOT = Path(__file__).resolve().parents[1]


def declared(header: str, prefix: str = "q3xk"):
    text = (ROOT / "include" / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(" + prefix + r"\w*)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    names = declared("q3xk.h")
    assert "q3xk_gemv" in names and "q3xk_repack" in names
    handle = lib()
    missing = [n for n in names if not hasattr(handle, n)]
    assert not missing, missing
    # and the binding knows every one of them
    assert set(names) <= set(capi.declared_symbols())


def test_library_exports_the_backend_interface():
    """q3x_backend.h: the C mirror and the reference's C++ q3x_backend
    functions (internal.h:16-34), exported with their mangled C++ names."""
    names = declared("q3x_backend.h", "q3xb")
    assert "q3xb_state_forward" in names and len(names) >= 17
    handle = lib()
    assert not [n for n in names if not hasattr(handle, n)]
    assert set(names) <= set(capi.declared_symbols())
    import subprocess
    out = subprocess.run(["nm", "-DC", "--defined-only", str(capi.LIB_PATH)], capture_output=True,
                         text=True).stdout
    for fn in ["model_create(char const*, char*, unsigned long)", "model_destroy(", "state_create(",
               "state_destroy(", "state_reset(", "state_forward(", "state_checkpoint_save(",
               "state_checkpoint_restore(", "state_argmax(", "state_copy_logits(", "model_id(",
               "vocab_size()", "max_context()", "token_is_stop(int)"]:
        assert "q3x_backend::" + fn in out, fn


def test_backend_rejects_bad_model_files(tmp_path):
    """Model::load's checks and messages (engine.cpp:480-498), no GPU work:
    each file fails before any device memory is touched."""
    import struct
    err = ctypes.create_string_buffer(256)
    create = lib().q3xb_model_create

    def fails(data):
        p = tmp_path / "m.bin"
        p.write_bytes(data)
        assert not create(str(p).encode(), err, 256)
        return err.value.decode()

    from qwen3x_b200 import modelfile

    assert not create(str(tmp_path / "absent.bin").encode(), err, 256)
    assert err.value.decode() == "cannot open model.bin"
    assert fails(b"short") == "bad model.bin"
    assert fails(b"NOTMODEL" + bytes(64)) == "wrong model.bin magic"
    assert fails(b"Q3XMODL\0" + struct.pack("<16I", 1234, *([0] * 15))) == "unsupported Qwen model ID"
    assert fails(b"Q3XMODL\0" + struct.pack("<16I", 9000, *([0] * 15))) == "Qwen model.bin header mismatch"
    c = modelfile.CONFIGS[9091]
    assert fails(c.header() + bytes(1000)) == "truncated model.bin"
    assert fails(c.header() + bytes(modelfile.file_size(c) - 72 + 64)) == "model.bin size does not match schema"


def test_abi_version_and_status_strings():
    assert lib().q3xk_abi_version() == 1
    assert capi.status_string(capi.OK) == "ok"
    assert "align" in capi.status_string(capi.EALIGN)
    assert capi.status_string(99) == "unknown status"


def test_quantized_bytes_matches_reference_rules():
    """arch/cpu.cpp:161-179 via tests/q8_cpu_test.cpp:17-43."""
    f = lib().q3xk_quantized_bytes
    out = ctypes.c_size_t(123)
    assert f(capi.BF16, 3, 17, ctypes.byref(out)) == capi.EINVAL and out.value == 123
    assert f(capi.Q8_0, 3, 64, ctypes.byref(out)) == capi.OK and out.value == 204
    assert f(capi.Q4_0, 3, 64, ctypes.byref(out)) == capi.OK and out.value == 108
    out.value = 123
    for t in (capi.BF16, capi.Q8_0, capi.Q4_0):
        assert f(t, 0, 32, ctypes.byref(out)) == capi.EINVAL
        assert f(t, 1, -32, ctypes.byref(out)) == capi.EINVAL
    assert f(capi.Q8_0, 1, 33, ctypes.byref(out)) == capi.EINVAL
    assert f(capi.Q4_0, 1, 16, ctypes.byref(out)) == capi.EINVAL
    assert f(999, 1, 32, ctypes.byref(out)) == capi.EINVAL
    assert out.value == 123
    assert f(capi.Q8_0, 2147483647, 2147483616, ctypes.byref(out)) == capi.OK
    assert out.value == 2147483647 * (2147483616 // 32) * 34


@pytest.mark.parametrize("t,cols,stride", [
    (capi.Q8_0, 4096, 4096 + 256), (capi.Q4_0, 4096, 2048 + 256),
    (capi.Q8_0, 2176, 2176 + 144), (capi.Q4_0, 512, 256 + 32),
    (capi.Q8_0, 32, 32 + 16), (capi.BF16, 2048, 4096), (capi.BF16, 3, 16)])
def test_matrix_layout(t, cols, stride):
    m = Matrix()
    size = ctypes.c_size_t()
    assert lib().q3xk_matrix_layout(t, 7, cols, 3, ctypes.byref(m), ctypes.byref(size)) == capi.OK
    assert m.row_stride == stride and m.row_stride % 16 == 0
    assert m.expert_stride == 7 * stride and size.value == 21 * stride
    assert (m.type, m.rows, m.cols, m.experts) == (t, 7, cols, 3)


def test_layout_rejects_bad_shapes():
    m = Matrix()
    size = ctypes.c_size_t()
    f = lib().q3xk_matrix_layout
    assert f(capi.Q8_0, 4, 33, 1, ctypes.byref(m), ctypes.byref(size)) == capi.EINVAL
    assert f(capi.Q4_0, 0, 64, 1, ctypes.byref(m), ctypes.byref(size)) == capi.EINVAL
    assert f(7, 4, 64, 1, ctypes.byref(m), ctypes.byref(size)) == capi.EINVAL
    assert f(capi.Q8_0, 4, 64, 0, ctypes.byref(m), ctypes.byref(size)) == capi.EINVAL


def test_launchers_validate_before_launch():
    """Argument errors come back as status codes; nothing is launched."""
    L = lib()
    m = Matrix()
    size = ctypes.c_size_t()
    assert L.q3xk_matrix_layout(capi.Q8_0, 64, 128, 2, ctypes.byref(m), ctypes.byref(size)) == 0
    before = L.q3xk_launch_count()
    assert L.q3xk_gemv(None, 16, 16, 0, None) == capi.EINVAL
    assert L.q3xk_gemv(ctypes.byref(m), 16, 16, 0, None) == capi.EINVAL  # data is NULL
    m.data = 0x1008  # misaligned (not a real allocation: rejected before use)
    assert L.q3xk_gemv(ctypes.byref(m), 0x2000, 0x3000, 0, None) == capi.EALIGN
    m.data = 0x1000
    assert L.q3xk_gemv(ctypes.byref(m), 0x2004, 0x3000, 0, None) == capi.EALIGN
    assert L.q3xk_expert_gemv(ctypes.byref(m), 2, 0x2000, 0x3000, 0, None) == capi.EINVAL
    assert L.q3xk_expert_gemv(ctypes.byref(m), -1, 0x2000, 0x3000, 0, None) == capi.EINVAL
    bad = Matrix.from_buffer_copy(m)
    bad.row_stride += 16
    assert L.q3xk_gemv(ctypes.byref(bad), 0x2000, 0x3000, 0, None) == capi.EINVAL
    assert L.q3xk_repack(ctypes.byref(bad), 0x4000, None) == capi.EINVAL
    assert L.q3xk_launch_count() == before


def test_gemv_family_switch_validates():
    """q3xk_gemv_set_family takes 0 (automatic), 1 (register kernel), 2 and 3
    (ring kernel, 16 / 24 warps) and rejects anything else; host-side only."""
    handle = lib()
    try:
        for fam in (0, 1, 2, 3):
            assert handle.q3xk_gemv_set_family(fam) == capi.OK
        for bad in (-1, 4, 99):
            assert handle.q3xk_gemv_set_family(bad) == capi.EINVAL
    finally:
        handle.q3xk_gemv_set_family(0)


def test_linear_set_gemv_family_wrapper():
    from qwen3x_b200 import linear

    try:
        for fam in (linear.GEMV_AUTO, linear.GEMV_REGISTER, linear.GEMV_RING16, linear.GEMV_RING24):
            linear.set_gemv_family(fam)
        with pytest.raises(capi.Q3xkError):
            linear.set_gemv_family(7)
    finally:
        linear.set_gemv_family(linear.GEMV_AUTO)
