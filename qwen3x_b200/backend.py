"""Python mirror of the qwen3x backend interface (internal.h:11-34) over the C ABI
of include/q3x_backend.h.

    model = Model("model.bin")            # q3x_backend::model_create
    state = State(model, context=4096)    # q3x_backend::state_create
    state.forward(prompt)                 # state_forward(..., compute_logits=True)
    token = state.argmax()                # state_argmax
    logits = state.logits()               # state_copy_logits

Errors raise (the reference aborts through Q3X_ASSERT); there is no CPU path.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import capi

FIELDS = ("id", "V", "H", "I", "N", "AI", "AH", "KVH", "AD", "RD", "KH", "VH", "KD", "VD", "CK",
          "context", "experts", "top_k", "shared_I", "matrix_type", "tied")
SHARD_FIELDS = ("rank", "world", "kh0", "vh0", "ah0", "kv0", "i0", "v0", "KH", "VH", "AH", "KVH", "I", "V",
                "e0", "experts")


def forward_batch(model: "Model", states, tokens) -> None:
    """One decode step of independent sequences: states[b] takes tokens[b]
    (q3xb_state_forward_batch; every matrix is read once for all of them)."""
    import ctypes

    n = len(states)
    handles = (ctypes.c_void_p * n)(*[s.handle for s in states])
    t = np.ascontiguousarray(tokens, np.int32)
    if t.size != n:
        raise ValueError("one token per state")
    capi.check(capi.lib().q3xb_state_forward_batch(model.handle, ctypes.cast(handles, ctypes.c_void_p),
                                                   t.ctypes.data, n), "state_forward_batch")


def tp_plan(model_id: int, rank: int, world: int) -> dict:
    """This rank's tensor-parallel share of a registered model (no loading)."""
    f = (ctypes.c_int * 16)()
    err = ctypes.create_string_buffer(256)
    st = capi.lib().q3xb_tp_plan(model_id, rank, world, f, err, 256)
    if st != capi.OK:
        raise ValueError(err.value.decode())
    return dict(zip(SHARD_FIELDS, list(f)))


def tp_unique_id() -> bytes:
    """A new NCCL communicator id (rank 0 makes it; every rank passes it to State)."""
    buf = ctypes.create_string_buffer(128)
    capi.check(capi.lib().q3xb_tp_unique_id(buf), "q3xb_tp_unique_id")
    return buf.raw


class Model:
    """q3x_backend::model_create; with world > 1 this rank's tensor-parallel share."""

    def __init__(self, path, rank: int = 0, world: int = 1):
        self.lib = capi.lib()
        err = ctypes.create_string_buffer(256)
        if world == 1:
            self.handle = self.lib.q3xb_model_create(str(path).encode(), err, 256)
        else:
            self.handle = self.lib.q3xb_model_create_tp(str(path).encode(), rank, world, err, 256)
        if not self.handle:
            raise RuntimeError(f"model_create: {err.value.decode()}")
        f = (ctypes.c_int * 21)()
        capi.check(self.lib.q3xb_model_config(self.handle, f), "q3xb_model_config")
        self.config = dict(zip(FIELDS, list(f)))
        sf = (ctypes.c_int * 16)()
        capi.check(self.lib.q3xb_model_shard(self.handle, sf), "q3xb_model_shard")
        self.shard = dict(zip(SHARD_FIELDS, list(sf)))

    @property
    def id(self) -> int:
        return self.lib.q3xb_model_id(self.handle)

    @property
    def vocab(self) -> int:
        return self.config["V"]

    @property
    def device_bytes(self) -> int:
        return self.lib.q3xb_model_device_bytes(self.handle)

    def close(self):
        if self.handle:
            self.lib.q3xb_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class State:
    """q3x_backend::state_create; tensor-parallel models need the communicator
    id from tp_unique_id() (the same bytes on every rank)."""

    def __init__(self, model: Model, context: int, nccl_id: bytes | None = None, exchange=None):
        self.model = model
        self.lib = model.lib
        err = ctypes.create_string_buffer(256)
        if model.shard["world"] == 1:
            self.handle = self.lib.q3xb_state_create(model.handle, int(context), err, 256)
        else:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("a tensor-parallel state needs the 128-byte communicator id")
            self.handle = self.lib.q3xb_state_create_tp(model.handle, int(context), nccl_id, err, 256)
        if not self.handle:
            raise RuntimeError(f"state_create: {err.value.decode()}")
        if model.shard["world"] > 1 and exchange is not None:
            # decode all-reduces over peer memory: exchange the IPC handles in rank order
            h = ctypes.create_string_buffer(64)
            capi.check(self.lib.q3xb_state_ipc_handle(self.handle, h), "q3xb_state_ipc_handle")
            handles = exchange(h.raw)
            capi.check(self.lib.q3xb_state_ipc_open(self.handle, b"".join(handles)), "q3xb_state_ipc_open")

    def tp_error(self) -> int:
        out = ctypes.c_int(0)
        capi.check(self.lib.q3xb_state_tp_error(self.handle, ctypes.byref(out)), "q3xb_state_tp_error")
        return out.value

    def forward(self, tokens, compute_logits: bool = True):
        t = np.ascontiguousarray(np.atleast_1d(tokens), dtype=np.int32)
        capi.check(self.lib.q3xb_state_forward(self.model.handle, self.handle, t.ctypes.data, t.size,
                                               int(compute_logits)), "state_forward")

    def argmax(self) -> int:
        out = ctypes.c_int(-1)
        capi.check(self.lib.q3xb_state_argmax(self.handle, ctypes.byref(out)), "state_argmax")
        return out.value

    def logits(self) -> np.ndarray:
        out = np.empty(self.model.vocab, np.float32)
        capi.check(self.lib.q3xb_state_copy_logits(self.handle, out.ctypes.data), "state_copy_logits")
        return out

    def reset(self):
        capi.check(self.lib.q3xb_state_reset(self.handle), "state_reset")

    def checkpoint_save(self):
        capi.check(self.lib.q3xb_state_checkpoint_save(self.handle), "state_checkpoint_save")

    def checkpoint_restore(self):
        capi.check(self.lib.q3xb_state_checkpoint_restore(self.handle), "state_checkpoint_restore")

    @property
    def position(self) -> int:
        return self.lib.q3xb_state_position(self.handle)

    @property
    def stream(self) -> int:
        return self.lib.q3xb_state_stream(self.handle) or 0

    def synchronize(self):
        capi.check(self.lib.q3xb_state_synchronize(self.handle), "state_synchronize")

    def set_graphs(self, enabled: bool):
        capi.check(self.lib.q3xb_state_set_graphs(self.handle, int(enabled)), "state_set_graphs")

    def set_exact_prefill(self, enabled: bool):
        capi.check(self.lib.q3xb_state_set_exact_prefill(self.handle, int(enabled)),
                   "state_set_exact_prefill")

    def set_peer_timeout(self, seconds: float):
        """Bound of the decode all-reduce's wait for a peer (before the first decode step)."""
        capi.check(self.lib.q3xb_state_set_peer_timeout(self.handle, float(seconds)), "state_set_peer_timeout")

    def set_prefill_precision(self, precision: int):
        """capi.GEMM_SPLIT (default) or capi.GEMM_FP16 for the prompt GEMMs."""
        capi.check(self.lib.q3xb_state_set_prefill_precision(self.handle, int(precision)),
                   "state_set_prefill_precision")

    def set_prefill_chunk(self, tokens: int):
        capi.check(self.lib.q3xb_state_set_prefill_chunk(self.handle, int(tokens)),
                   "state_set_prefill_chunk")

    def generate(self, prompt, steps: int):
        """Greedy decode: forward(prompt), then `steps` tokens fed back one at
        a time (runtime.cpp's greedy loop).  Returns the generated tokens."""
        self.forward(prompt)
        out = []
        for _ in range(steps):
            tok = self.argmax()
            out.append(tok)
            self.forward([tok])
        return out

    def close(self):
        if self.handle:
            self.lib.q3xb_state_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
