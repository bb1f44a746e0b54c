"""Parity oracles for qwen3x's packed-weight matrix path -- TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may use
this package.  Two checkers live here:

  port()       libq3x_oracle.so: the C restatement in q3x_oracle.c (each
               function cites the reference routine it follows);
  reference()  _ref/libq3xref_v{4,2}.so: the reference's own engine.cpp and
               arch/cpu.cpp compiled unmodified (oracle/Makefile), with C
               entry points from ref_shim.cpp.

`make -C oracle` builds both (the _ref build needs the reference source tree;
elsewhere the prebuilt _ref libraries are used as they are).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "libq3x_oracle.so"
REF_DIR = HERE / "_ref"

BF16, Q8_0, Q4_0 = 0, 1, 2

_f = ctypes.c_float
_p = ctypes.c_void_p
_i = ctypes.c_int
_u32 = ctypes.c_uint32
_sz = ctypes.c_size_t

_PORT_SIGS = {
    "q3xo_f16": (_f, [ctypes.c_uint16]),
    "q3xo_f32_to_f16": (ctypes.c_uint16, [_f]),
    "q3xo_quantized_bytes": (_i, [_u32, _i, _i, ctypes.POINTER(_sz)]),
    "q3xo_mv": (_i, [_p, _u32, _i, _i, _p, _p, _i]),
    "q3xo_gemm": (_i, [_p, _u32, _i, _i, _p, _i, _p, _i]),
    "q3xo_embed": (_i, [_p, _u32, _i, _i, _p]),
    "q3xo_expert_mv": (_i, [_p, _u32, _i, _i, _i, _i, _p, _p]),
    "q3xo_router_top_k": (_i, [_p, _i, _i, _p, _p]),
    "q3xo_moe": (_i, [_p, _p, _p, _p, _p, _p, _p, _u32, _i, _i, _i, _i, _i, _p, _p, _p, _p]),
    "q3xo_argmax": (_i, [_p, _i]),
    "q3xo_quantize_q8_0": (_i, [_p, _sz, _p]),
    "q3xo_quantize_q4_0": (_i, [_p, _sz, _p]),
}

_REF_SIGS = {
    "q3xref_has_avx512": (_i, []),
    "q3xref_quantized_bytes": (_i, [_u32, _i, _i, ctypes.POINTER(_sz)]),
    "q3xref_try_mv": (_i, [_p, _u32, _i, _i, _p, _p]),
    "q3xref_try_embed": (_i, [_p, _u32, _i, _i, _p]),
    "q3xref_mv": (_i, [_p, _u32, _i, _i, _p, _p, _i]),
    "q3xref_router_top_k": (_i, [_p, _i, _i, _p, _p]),
    "q3xref_moe": (_i, [_p, _p, _p, _p, _p, _p, _p, _u32, _i, _i, _i, _i, _i, _p, _p, _p, _p]),
    "q3xref_model_create": (_p, [ctypes.c_char_p, ctypes.c_char_p, _sz]),
    "q3xref_model_destroy": (None, [_p]),
    "q3xref_state_create": (_p, [_p, _i]),
    "q3xref_state_destroy": (None, [_p]),
    "q3xref_state_reset": (None, [_p]),
    "q3xref_state_forward": (None, [_p, _p, _p, _i, _i]),
    "q3xref_state_argmax": (_i, [_p]),
    "q3xref_state_copy_logits": (None, [_p, _p]),
    "q3xref_state_checkpoint_save": (None, [_p]),
    "q3xref_state_checkpoint_restore": (None, [_p]),
    "q3xref_model_id": (_u32, [_p]),
    "q3xref_model_create_custom": (_p, [ctypes.c_char_p, _p, ctypes.c_char_p, _sz]),
}

_port = None
_ref = None


def _bind(handle, sigs):
    for name, (res, args) in sigs.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    return handle


def port():
    """The C restatement (libq3x_oracle.so); built on demand with make."""
    global _port
    if _port is None:
        if not PORT_LIB.exists():
            os.system(f"make -s -C {HERE} oracle >/dev/null")
        _port = _bind(ctypes.CDLL(str(PORT_LIB)), _PORT_SIGS)
    return _port


def _cpu_has_avx512() -> bool:
    try:
        flags = Path("/proc/cpuinfo").read_text()
    except OSError:
        return False
    return " avx512f " in flags and " avx512bw " in flags


def reference_path() -> Path | None:
    v4, v2 = REF_DIR / "libq3xref_v4.so", REF_DIR / "libq3xref_v2.so"
    if v4.exists() and _cpu_has_avx512():
        return v4
    if v2.exists():
        return v2
    return None


def reference():
    """The reference's own CPU engine (oracle/_ref), or None if it was never built."""
    global _ref
    if _ref is None:
        path = reference_path()
        if path is None:
            return None
        _ref = _bind(ctypes.CDLL(str(path)), _REF_SIGS)
    return _ref


class RefEngine:
    """The reference CPU forward (engine.cpp) on a model.bin, through oracle/_ref.

    `config` (a qwen3x_b200.modelfile.ModelConfig) is needed for model IDs the
    reference does not register; the tensor walk is then ref_shim.cpp's
    restatement of Model::load."""

    def __init__(self, path, config=None, context=512):
        self.lib = reference()
        if self.lib is None:
            raise RuntimeError("oracle/_ref was not built")
        err = ctypes.create_string_buffer(256)
        if config is None:
            self.model = self.lib.q3xref_model_create(str(path).encode(), err, 256)
            self.vocab = 248320
        else:
            c = config
            f = np.array([c.id, c.V, c.H, c.I, c.N, c.AI, c.AH, c.KVH, c.AD, c.RD, c.KH, c.VH, c.KD,
                          c.VD, c.CK, c.experts, c.top_k, c.shared_I, c.matrix_type, int(c.tied)],
                         np.int32)
            self.model = self.lib.q3xref_model_create_custom(str(path).encode(), f.ctypes.data, err, 256)
            self.vocab = c.V
        if not self.model:
            raise RuntimeError(err.value.decode())
        self.state = self.lib.q3xref_state_create(self.model, context)

    def forward(self, tokens, logits=True):
        t = np.ascontiguousarray(tokens, np.int32)
        self.lib.q3xref_state_forward(self.model, self.state, t.ctypes.data, t.size, int(logits))

    def logits(self):
        out = np.empty(self.vocab, np.float32)
        self.lib.q3xref_state_copy_logits(self.state, out.ctypes.data)
        return out

    def argmax(self):
        return self.lib.q3xref_state_argmax(self.state)

    def reset(self):
        self.lib.q3xref_state_reset(self.state)

    def checkpoint_save(self):
        self.lib.q3xref_state_checkpoint_save(self.state)

    def checkpoint_restore(self):
        self.lib.q3xref_state_checkpoint_restore(self.state)

    def close(self):
        if self.state:
            self.lib.q3xref_state_destroy(self.state)
            self.state = None
        if self.model:
            self.lib.q3xref_model_destroy(self.model)
            self.model = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _a(arr):
    return arr.ctypes.data if arr is not None else None


def mv(packed: np.ndarray, mtype: int, rows: int, cols: int, x: np.ndarray,
       threads: int = 1, impl: str = "port") -> np.ndarray:
    """y = W x on the CPU with the port or the reference library."""
    packed = np.ascontiguousarray(packed)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    if impl == "port":
        rc = port().q3xo_mv(_a(packed), mtype, rows, cols, _a(x), _a(y), threads)
    else:
        rc = reference().q3xref_mv(_a(packed), mtype, rows, cols, _a(x), _a(y), threads)
    if rc != 0:
        raise ValueError("oracle mv rejected the shape")
    return y


def gemm(packed, mtype, rows, cols, X, threads=1) -> np.ndarray:
    X = np.ascontiguousarray(X, dtype=np.float32)
    T = X.shape[0]
    Y = np.empty((T, rows), dtype=np.float32)
    if port().q3xo_gemm(_a(np.ascontiguousarray(packed)), mtype, rows, cols, _a(X), T, _a(Y), threads):
        raise ValueError("oracle gemm rejected the shape")
    return Y


def router_top_k(logits: np.ndarray, top_k: int, impl: str = "port"):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    ids = np.zeros(top_k, dtype=np.int32)
    probs = np.zeros(logits.size, dtype=np.float32)
    fn = port().q3xo_router_top_k if impl == "port" else reference().q3xref_router_top_k
    if fn(_a(logits), logits.size, top_k, _a(ids), _a(probs)):
        raise ValueError("router rejected the shape")
    return ids, probs


def moe(router, gate_up, down, shared_gate, shared_up, shared_down, shared_scale, mtype,
        experts, top_k, H, I, shared_I, x, impl: str = "port"):
    """One token through engine.cpp:406-430; returns (out[H], ids, weights)."""
    args = [np.ascontiguousarray(a) for a in (router, gate_up, down, shared_gate, shared_up,
                                               shared_down, shared_scale)]
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(H, dtype=np.float32)
    ids = np.zeros(top_k, dtype=np.int32)
    w = np.zeros(top_k, dtype=np.float32)
    fn = port().q3xo_moe if impl == "port" else reference().q3xref_moe
    rc = fn(*[_a(a) for a in args], mtype, experts, top_k, H, I, shared_I, _a(x), _a(out),
            _a(ids), _a(w))
    if rc:
        raise ValueError("moe rejected the shape")
    return out, ids, w


def magnitude(packed, mtype, rows, cols, x) -> np.ndarray:
    """sum_k |w_rk x_k| per row in float64 (the reference tests' error scale,
    tests/q8_cpu_test.cpp:65-68)."""
    from qwen3x_b200.quant import dequantize  # host-side decode of the block format

    w = dequantize(packed, mtype, rows, cols).astype(np.float64)
    return np.abs(w) @ np.abs(np.asarray(x, dtype=np.float64))
