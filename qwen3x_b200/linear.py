"""Host-side mirror of the reference's matrix entry points over the q3xk C ABI.

Names follow the reference:
  Linear            engine.cpp:31-35 / engine.cu `Linear` -- one device matrix
  mv, mv_add        engine.cu:1531-1561 (y = W x, y += W x)
  expert_mv         engine.cpp:214-224
  quantized_bytes   arch/cpu.cpp:161-179
Device memory comes from torch (plumbing only); every computation is a call
into libq3xk.so.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import capi
from .capi import BF16, Q4_0, Q8_0, Matrix, check, lib, ptr, stream_ptr


def quantized_bytes(mtype: int, rows: int, cols: int):
    """Packed model.bin size of a matrix, or None where the reference returns false."""
    out = ctypes.c_size_t(0)
    st = lib().q3xk_quantized_bytes(int(mtype), int(rows), int(cols), ctypes.byref(out))
    return out.value if st == capi.OK else None


class Linear:
    """A matrix (or an expert pool) in the row-record device layout."""

    def __init__(self, mtype: int, rows: int, cols: int, experts: int = 1, device="cuda"):
        import torch

        self.m = Matrix()
        size = ctypes.c_size_t(0)
        check(lib().q3xk_matrix_layout(int(mtype), int(rows), int(cols), int(experts),
                                       ctypes.byref(self.m), ctypes.byref(size)),
              "q3xk_matrix_layout")
        self.storage = torch.empty(size.value, dtype=torch.uint8, device=device)
        self.m.data = self.storage.data_ptr()
        self.type, self.rows, self.cols, self.experts = int(mtype), int(rows), int(cols), int(experts)

    @property
    def nbytes(self) -> int:
        return self.storage.numel()

    @property
    def packed_nbytes(self) -> int:
        if self.type == BF16:
            return self.rows * self.cols * 2 * self.experts
        return quantized_bytes(self.type, self.rows * self.experts, self.cols)

    @classmethod
    def from_packed(cls, packed, mtype: int, rows: int, cols: int, experts: int = 1,
                    device="cuda", stream=None) -> "Linear":
        """Upload model.bin-format bytes (numpy or torch) and repack on the device."""
        import torch

        lin = cls(mtype, rows, cols, experts, device)
        if isinstance(packed, np.ndarray):
            src = torch.from_numpy(np.ascontiguousarray(packed).reshape(-1).view(np.uint8))
        else:
            src = packed.reshape(-1).view(torch.uint8)
        if src.numel() != lin.packed_nbytes:
            raise ValueError(f"packed size {src.numel()} != {lin.packed_nbytes}")
        src = src.to(device, non_blocking=False)
        lin.repack_from(src, stream)
        torch.cuda.synchronize(device)  # `src` is freed on return
        return lin

    def repack_from(self, packed_device, stream=None) -> None:
        check(lib().q3xk_repack(ctypes.byref(self.m), ptr(packed_device), stream_ptr(stream)),
              "q3xk_repack")


GEMV_AUTO, GEMV_REGISTER, GEMV_RING16, GEMV_RING24 = range(4)


def set_gemv_family(family: int) -> None:
    """Kernel family of the plain GEMVs, process-wide (q3xk_gemv_set_family):
    GEMV_AUTO (default: the shared-memory ring kernel where it fits),
    GEMV_REGISTER, GEMV_RING16 or GEMV_RING24.  For comparisons and tests;
    every family meets the same parity bar."""
    check(lib().q3xk_gemv_set_family(int(family)), "q3xk_gemv_set_family")


def _gemv(linear: Linear, x, y, accumulate: int, stream) -> None:
    check(lib().q3xk_gemv(ctypes.byref(linear.m), ptr(x), ptr(y), accumulate, stream_ptr(stream)),
          "q3xk_gemv")


def mv(linear: Linear, x, y, stream=None) -> None:
    """y[rows] = W[rows, cols] x[cols] (engine.cu:1531 mv)."""
    _gemv(linear, x, y, 0, stream)


def mv_add(linear: Linear, x, y, stream=None) -> None:
    """y[rows] += W x (engine.cu:1547 mv_add)."""
    _gemv(linear, x, y, 1, stream)


def expert_mv(linear: Linear, expert: int, x, y, stream=None, accumulate: bool = False) -> None:
    """y = W[expert] x for a contiguous pool W[experts, rows, cols] (engine.cpp:214)."""
    check(lib().q3xk_expert_gemv(ctypes.byref(linear.m), int(expert), ptr(x), ptr(y),
                                 int(accumulate), stream_ptr(stream)), "q3xk_expert_gemv")


def expert_mv_rows(pool: Linear, ids, slots: int, x, y, accumulate=False, stream=None) -> None:
    """y[s*rows + r] (+)= W[ids[s]][r] . x for s < slots; ids on the device
    (an id < 0 skips its slot: those rows of y are left as they are)."""
    check(lib().q3xk_expert_gemv_rows(ctypes.byref(pool.m), ptr(ids), int(slots), ptr(x), ptr(y),
                                      int(accumulate), stream_ptr(stream)), "q3xk_expert_gemv_rows")


def expert_mv_segments(pool: Linear, ids, slots: int, x, y, accumulate=False, stream=None) -> None:
    """y[r] (+)= sum_s W[ids[s]][r] . x[s*cols:(s+1)*cols]; ids on the device
    (an id < 0 skips its segment)."""
    check(lib().q3xk_expert_gemv_segments(ctypes.byref(pool.m), ptr(ids), int(slots), ptr(x), ptr(y),
                                          int(accumulate), stream_ptr(stream)),
          "q3xk_expert_gemv_segments")


def router_top_k(logits, experts: int, top_k: int, ids, weights, with_shared=False,
                 stream=None) -> None:
    """engine.cpp:377-405 on the device (+ the shared-expert gate slot)."""
    check(lib().q3xk_router_topk(ptr(logits), int(experts), int(top_k), int(with_shared), ptr(ids),
                                 ptr(weights), stream_ptr(stream)), "q3xk_router_topk")


def swiglu(gate_up, weights, slots: int, width: int, out, stream=None) -> None:
    check(lib().q3xk_swiglu(ptr(gate_up), ptr(weights), int(slots), int(width), ptr(out),
                            stream_ptr(stream)), "q3xk_swiglu")


def argmax(values, n: int, out_index, workspace=None, stream=None) -> None:
    import torch

    if workspace is None:
        need = ctypes.c_size_t(0)
        check(lib().q3xk_argmax_workspace_bytes(ctypes.byref(need)), "q3xk_argmax_workspace_bytes")
        workspace = torch.empty(need.value, dtype=torch.uint8, device=values.device)
    check(lib().q3xk_argmax(ptr(values), int(n), ptr(out_index), ptr(workspace),
                            workspace.numel() * workspace.element_size(), stream_ptr(stream)),
          "q3xk_argmax")


def gemm_workspace_bytes(T: int, cols: int) -> int:
    out = ctypes.c_size_t(0)
    check(lib().q3xk_gemm_workspace_bytes(int(T), int(cols), ctypes.byref(out)),
          "q3xk_gemm_workspace_bytes")
    return out.value


def batch_mv(linear: Linear, X, Y, add: bool = False, workspace=None, stream=None,
             precision: int | None = None) -> None:
    """Y[T, rows] (+)= X[T, cols] W^T on tcgen05 (engine.cu:1568 batch_mv).

    precision None calls q3xk_gemm (split FP16 operands, FP32-grade);
    capi.GEMM_SPLIT / capi.GEMM_FP16 call q3xk_gemm_ex with that precision."""
    import torch

    T = int(X.shape[0])
    need = gemm_workspace_bytes(T, linear.cols)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=X.device)
    nbytes = workspace.numel() * workspace.element_size()
    if precision is None:
        check(lib().q3xk_gemm(ctypes.byref(linear.m), ptr(X), T, ptr(Y), int(add), ptr(workspace),
                              nbytes, stream_ptr(stream)), "q3xk_gemm")
    else:
        check(lib().q3xk_gemm_ex(ctypes.byref(linear.m), ptr(X), T, ptr(Y), int(add), int(precision),
                                 ptr(workspace), nbytes, stream_ptr(stream)), "q3xk_gemm_ex")


def try_mv(linear: Linear, x_host, y_host, workspace, stream=None) -> None:
    """Synchronous y_host = W x_host on host vectors (arch/cpu.cpp:192 try_mv
    contract); `workspace` is a device buffer of >= (cols + rows) floats."""
    nbytes = workspace.numel() * workspace.element_size()
    check(lib().q3xk_try_mv_host(ctypes.byref(linear.m), ptr(x_host), ptr(y_host), ptr(workspace),
                                 nbytes, stream_ptr(stream)), "q3xk_try_mv_host")


__all__ = ["Linear", "mv", "mv_add", "expert_mv", "try_mv", "batch_mv", "gemm_workspace_bytes",
           "expert_mv_rows", "expert_mv_segments", "router_top_k", "swiglu", "argmax",
           "quantized_bytes", "BF16", "Q8_0", "Q4_0"]
