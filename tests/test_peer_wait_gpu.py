"""The peer-memory all-reduce of the multi-GPU decode step (q3xk_peer_allreduce_add)
on ONE GPU, with both ranks' buffers local.

No kernel ever waits for another kernel here: a "peer" that has published is
emulated by the host writing its flag and partial before the launch, and a
peer that never publishes is simply a flag nothing sets.  So the failure is
made on the host and the device wait runs out on its own bound (10 ms); the
kernel must report it through the error word and return, leaving the context
usable and y untouched.
"""
import ctypes

import numpy as np
import pytest

from qwen3x_b200 import capi
from qwen3x_b200.capi import lib

pytestmark = pytest.mark.gpu

N_MAX = 4096
MAX_RANKS = 8


def _buffers(cuda, world):
    import torch

    nbytes = lib().q3xk_peer_buffer_bytes(N_MAX)
    assert nbytes > 0
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda) for _ in range(world)]
    data_bytes = (2 * N_MAX * 4 + 255) // 256 * 256
    return bufs, data_bytes


def _flags(buf, data_bytes):
    import torch

    return buf[data_bytes:data_bytes + 2 * MAX_RANKS * 4].view(torch.int32).view(2, MAX_RANKS)


def _data(buf):
    import torch

    return buf[:2 * N_MAX * 4].view(torch.float32).view(2, N_MAX)


def _call(bases, world, seq, partial, y, n, err, timeout_s, stream):
    arr = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bases])
    return lib().q3xk_peer_allreduce_add(ctypes.cast(arr, ctypes.c_void_p), 0, world, N_MAX, seq.data_ptr(),
                                         partial.data_ptr(), y.data_ptr(), n, err.data_ptr(), float(timeout_s),
                                         stream)


def test_published_peer_is_summed_in_rank_order(cuda):
    import torch

    n = 4096
    bufs, data_bytes = _buffers(cuda, 2)
    seq = torch.zeros(1, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    g = torch.Generator(device="cpu").manual_seed(3)
    p0 = torch.randn(n, generator=g).to(cuda)
    p1 = torch.randn(n, generator=g).to(cuda)
    y0 = torch.randn(n, generator=g).to(cuda)
    y = y0.clone()
    # rank 1 has published call 1 (phase 1): its partial in its buffer, its flag in ours
    _data(bufs[1])[1, :n] = p1
    _flags(bufs[0], data_bytes)[1, 1] = 1
    stream = torch.cuda.current_stream().cuda_stream
    assert _call(bufs, 2, seq, p0, y, n, err, 1.0, stream) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert int(seq.item()) == 1
    expect = y0 + ((torch.zeros_like(p0) + p0) + p1)
    assert torch.equal(y, expect)
    # this rank published to both buffers
    assert int(_flags(bufs[0], data_bytes)[1, 0].item()) == 1
    assert int(_flags(bufs[1], data_bytes)[1, 0].item()) == 1


def test_silent_peer_times_out_and_reports(cuda):
    import time

    import torch

    n = 2048
    bufs, _ = _buffers(cuda, 2)
    seq = torch.zeros(1, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    partial = torch.ones(n, device=cuda)
    y0 = torch.arange(n, dtype=torch.float32, device=cuda)
    y = y0.clone()
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    assert _call(bufs, 2, seq, partial, y, n, err, 0.01, stream) == 0  # rank 1 never publishes
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(err.item()) == 1
    assert torch.equal(y, y0)  # nothing added
    assert int(seq.item()) == 0
    assert waited < 5.0
    # a later call on the failed state returns at once and changes nothing
    assert _call(bufs, 2, seq, partial, y, n, err, 10.0, stream) == 0
    t1 = time.perf_counter()
    torch.cuda.synchronize()
    assert time.perf_counter() - t1 < 5.0
    assert int(err.item()) == 1 and torch.equal(y, y0)
    # the context is still usable
    z = torch.ones(16, device=cuda) * 2
    assert float(z.sum().item()) == 32.0


def test_arguments_are_checked_on_the_host(cuda):
    import torch

    bufs, _ = _buffers(cuda, 2)
    seq = torch.zeros(1, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    v = torch.zeros(16, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    assert _call(bufs, 2, seq, v, v, 16, err, 0.0, stream) == capi.EINVAL      # no bound
    assert _call(bufs, 2, seq, v, v, 16, err, 100.0, stream) == capi.EINVAL    # bound too long
    assert _call(bufs, 2, seq, v, v, N_MAX + 1, err, 1.0, stream) == capi.EUNSUPPORTED
