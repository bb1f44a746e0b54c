"""ctypes binding of the q3xk C ABI (include/q3xk.h).

Loading fails loudly when libq3xk.so is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libq3xk.so"

# q3xk_status
OK, EINVAL, EUNSUPPORTED, ECUDA, EALIGN, ETIMEOUT, EWORKSPACE = range(7)
# q3xk_matrix_type == q3x_model::MatrixType (model_config.h:16-20)
BF16, Q8_0, Q4_0 = 0, 1, 2
TYPE_NAMES = {BF16: "BF16", Q8_0: "Q8_0", Q4_0: "Q4_0"}
# q3xk_gemm_ex precisions (include/q3xk.h)
GEMM_SPLIT, GEMM_FP16 = 0, 1


class Matrix(ctypes.Structure):
    """struct q3xk_matrix."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("row_stride", ctypes.c_int64),
        ("expert_stride", ctypes.c_int64),
        ("type", ctypes.c_int32),
        ("rows", ctypes.c_int32),
        ("cols", ctypes.c_int32),
        ("experts", ctypes.c_int32),
    ]


class XForm(ctypes.Structure):
    """struct q3xk_xform."""

    _fields_ = [
        ("kind", ctypes.c_int32),
        ("group", ctypes.c_int32),
        ("w", ctypes.c_void_p),
        ("z", ctypes.c_void_p),
        ("seg_weights", ctypes.c_void_p),
    ]


XFORM_NONE, XFORM_RMS, XFORM_GATED_RMS, XFORM_SWIGLU = range(4)


class Q3xkError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} ({status})")


_lib = None

# name -> (restype, argtypes)
_SIGNATURES = {
    "q3xk_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "q3xk_abi_version": (ctypes.c_int, []),
    "q3xk_quantized_bytes": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.POINTER(ctypes.c_size_t)]),
    "q3xk_matrix_layout": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.POINTER(Matrix), ctypes.POINTER(ctypes.c_size_t)]),
    "q3xk_repack": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p, ctypes.c_void_p]),
    "q3xk_gemv": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_int, ctypes.c_void_p]),
    "q3xk_gemv_ex": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_int, ctypes.POINTER(XForm), ctypes.c_void_p]),
    "q3xk_expert_gemv_rows_ex": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p, ctypes.c_int,
                                                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                ctypes.POINTER(XForm), ctypes.c_void_p]),
    "q3xk_expert_gemv_segments_ex": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p, ctypes.c_int,
                                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                    ctypes.POINTER(XForm), ctypes.c_void_p]),
    "q3xk_expert_gemv": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "q3xk_try_mv_host": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "q3xk_try_mv_host_noalloc": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p,
                                                ctypes.c_void_p, ctypes.c_void_p]),
    "q3xk_expert_gemv_rows": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p, ctypes.c_int,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                             ctypes.c_void_p]),
    "q3xk_expert_gemv_segments": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p, ctypes.c_int,
                                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                 ctypes.c_void_p]),
    "q3xk_router_topk": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "q3xk_swiglu": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_void_p, ctypes.c_void_p]),
    "q3xk_argmax_workspace_bytes": (ctypes.c_int, [ctypes.POINTER(ctypes.c_size_t)]),
    "q3xk_argmax": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_size_t, ctypes.c_void_p]),
    "q3xk_gemm_workspace_bytes": (ctypes.c_int, [ctypes.c_int, ctypes.c_int,
                                                 ctypes.POINTER(ctypes.c_size_t)]),
    "q3xk_gemm": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                 ctypes.c_void_p]),
    "q3xk_gemm_ex": (ctypes.c_int, [ctypes.POINTER(Matrix), ctypes.c_void_p, ctypes.c_int,
                                    ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                    ctypes.c_size_t, ctypes.c_void_p]),
    "q3xk_gemm_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "q3xk_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "q3xk_peer_buffer_bytes": (ctypes.c_size_t, [ctypes.c_int]),
    "q3xk_peer_allreduce_add": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                               ctypes.c_void_p, ctypes.c_double, ctypes.c_void_p]),
    "q3xk_clear_device_error": (ctypes.c_int, []),
    "q3xk_gemv_set_family": (ctypes.c_int, [ctypes.c_int]),
    "q3xk_launch_count": (ctypes.c_uint64, []),
    "q3xk_reset_launch_count": (None, []),
    # q3x_backend.h, C part
    "q3xb_model_create": (ctypes.c_void_p, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]),
    "q3xb_model_destroy": (None, [ctypes.c_void_p]),
    "q3xb_model_id": (ctypes.c_uint32, [ctypes.c_void_p]),
    "q3xb_model_config": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "q3xb_model_device_bytes": (ctypes.c_size_t, [ctypes.c_void_p]),
    "q3xb_state_create": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p,
                                            ctypes.c_size_t]),
    "q3xb_state_destroy": (None, [ctypes.c_void_p]),
    "q3xb_state_reset": (ctypes.c_int, [ctypes.c_void_p]),
    "q3xb_state_forward": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_int, ctypes.c_int]),
    "q3xb_state_forward_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_int]),
    "q3xb_state_checkpoint_save": (ctypes.c_int, [ctypes.c_void_p]),
    "q3xb_state_checkpoint_restore": (ctypes.c_int, [ctypes.c_void_p]),
    "q3xb_state_argmax": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]),
    "q3xb_state_copy_logits": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "q3xb_state_position": (ctypes.c_int, [ctypes.c_void_p]),
    "q3xb_state_synchronize": (ctypes.c_int, [ctypes.c_void_p]),
    "q3xb_state_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "q3xb_state_set_graphs": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "q3xb_state_set_exact_prefill": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "q3xb_state_set_prefill_chunk": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "q3xb_state_set_prefill_precision": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "q3xb_model_create_tp": (ctypes.c_void_p, [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_char_p,
                                               ctypes.c_size_t]),
    "q3xb_tp_unique_id": (ctypes.c_int, [ctypes.c_char_p]),
    "q3xb_state_create_tp": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p,
                                               ctypes.c_size_t]),
    "q3xb_model_shard": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "q3xb_state_ipc_handle": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p]),
    "q3xb_state_ipc_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p]),
    "q3xb_state_tp_error": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]),
    "q3xb_state_set_peer_timeout": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_double]),
    "q3xb_tp_plan": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                    ctypes.c_char_p, ctypes.c_size_t]),
}


def _nccl_hint():
    """Point the library's run-time NCCL loader at the copy torch ships
    (used only by tensor-parallel states)."""
    if os.environ.get("Q3XK_NCCL_LIBRARY"):
        return
    try:
        import nvidia.nccl

        cand = Path(list(nvidia.nccl.__path__)[0]) / "lib" / "libnccl.so.2"
        if cand.exists():
            os.environ["Q3XK_NCCL_LIBRARY"] = str(cand)
    except ImportError:
        pass


def lib():
    """The loaded libq3xk.so (raises if it was never built)."""
    global _lib
    if _lib is None:
        path = os.environ.get("Q3XK_LIBRARY", str(LIB_PATH))
        if not Path(path).exists():
            raise RuntimeError(
                f"{path} is missing: build it with `python -m qwen3x_b200.build` "
                "(the qwen3x_b200 kernels have no CPU fallback)")
        _nccl_hint()
        handle = ctypes.CDLL(path)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def declared_symbols():
    return list(_SIGNATURES)


def status_string(status: int) -> str:
    try:
        return lib().q3xk_status_string(status).decode()
    except Exception:  # pragma: no cover - only when the library is absent
        return "status"


def check(status: int, what: str) -> None:
    if status != OK:
        raise Q3xkError(status, what)


def ptr(t) -> int:
    """Device (or host) address of a torch tensor / numpy array / int."""
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    if hasattr(t, "ctypes"):
        return t.ctypes.data
    raise TypeError(type(t))


def stream_ptr(stream=None) -> int:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream
