"""q3xk_try_mv_host_noalloc (fixed device scratch, no allocation) against
q3xk_try_mv_host (caller workspace), both through the C ABI, and both against
the reference CPU matvec (oracle.mv: arch/cpu.cpp's mv, compiled unmodified)
at the GEMV bar, max |y - y_ref| / sum_k |w x| <= 1e-5.

Collected last on purpose: it must pass after every other test has run in the
same process, and alone in a fresh one.
"""
import ctypes

import numpy as np
import pytest

import oracle
from qwen3x_b200 import capi
from qwen3x_b200.capi import Matrix, lib
from qwen3x_b200.quant import Q4_0, Q8_0, dequantize, gaussian, quantize

GEMV_TOL = 1e-5

SCRATCH_FLOATS = 1 << 20


def test_noalloc_rejects_sizes_beyond_the_scratch():
    """Checked before any CUDA call, so this runs without a GPU."""
    m = Matrix()
    assert lib().q3xk_matrix_layout(Q8_0, SCRATCH_FLOATS - 4096 + 1, 4096, 1, ctypes.byref(m), None) == 0
    m.data = 256  # never dereferenced: the size check comes first
    x = np.zeros(4096, np.float32)
    y = np.zeros(m.rows, np.float32)
    st = lib().q3xk_try_mv_host_noalloc(ctypes.byref(m), x.ctypes.data, y.ctypes.data, None)
    assert st == capi.EWORKSPACE
    assert lib().q3xk_try_mv_host_noalloc(None, x.ctypes.data, y.ctypes.data, None) == capi.EINVAL


@pytest.mark.gpu
@pytest.mark.parametrize("mtype,rows,cols", [(Q8_0, 12288, 4096), (Q4_0, 4096, 4096),
                                              (Q8_0, SCRATCH_FLOATS - 64, 64)])  # exactly full
def test_noalloc_matches_workspace_entry_point_twice(cuda, mtype, rows, cols):
    import torch

    from qwen3x_b200.linear import Linear

    w = gaussian((rows, cols), seed=71, std=0.02)
    packed = quantize(w, mtype)
    lin = Linear.from_packed(packed, mtype, rows, cols, device=cuda)
    wabs = np.abs(dequantize(packed, mtype, rows, cols))
    ws_bytes = ((cols * 4 + 15) & ~15) + rows * 4
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = gaussian((cols,), seed=100 + call, std=1.0)
        y_ref = np.empty(rows, np.float32)
        y = np.full(rows, np.nan, np.float32)
        capi.check(lib().q3xk_try_mv_host(ctypes.byref(lin.m), x.ctypes.data, y_ref.ctypes.data, ws.data_ptr(),
                                          ws_bytes, stream), "q3xk_try_mv_host")
        capi.check(lib().q3xk_try_mv_host_noalloc(ctypes.byref(lin.m), x.ctypes.data, y.ctypes.data, stream),
                   "q3xk_try_mv_host_noalloc")
        scale = np.abs(y_ref).max()
        assert np.abs(y - y_ref).max() <= 1e-6 * scale, call
        # the reference's own CPU matvec (the try_mv contract this replaces)
        ref = oracle.mv(packed, mtype, rows, cols, x, threads=8).astype(np.float64)
        mag = np.maximum(wabs @ np.abs(x), 1e-30)
        assert float((np.abs(y_ref - ref) / mag).max()) <= GEMV_TOL, call
        assert float((np.abs(y - ref) / mag).max()) <= GEMV_TOL, call
