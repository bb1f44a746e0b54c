"""Parity of the device MoE path (router, grouped expert GEMVs, SwiGLU) and
argmax with the CPU oracle (engine.cpp:377-430, :601-605)."""
import hashlib

import numpy as np
import pytest

import oracle
from qwen3x_b200 import quant
from qwen3x_b200.capi import BF16, Q4_0, Q8_0
from qwen3x_b200.linear import (Linear, argmax, expert_mv_rows, expert_mv_segments, mv,
                                router_top_k, swiglu)

pytestmark = pytest.mark.gpu


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("name,k", [("small", 3), ("wide", 8), ("random", 8), ("ties", 8)])
def test_router_matches_reference(cuda, golden, name, k):
    """q4_cpu_test.cpp:180-202 ({3,1,5}, 255..248), random and tied logits."""
    import torch

    logits = golden[f"router_{name}_logits"]
    ids = torch.zeros(k, dtype=torch.int32, device=cuda)
    w = torch.zeros(k, dtype=torch.float32, device=cuda)
    router_top_k(dev(logits, cuda), logits.size, k, ids, w)
    torch.cuda.synchronize()
    ref_ids = golden[f"router_{name}_ids"]
    assert ids.cpu().numpy().tolist() == ref_ids.tolist()
    ref_w = golden[f"router_{name}_probs"][ref_ids]
    assert np.allclose(w.cpu().numpy(), ref_w, rtol=2e-6, atol=1e-7)


def test_router_shared_slot(cuda):
    import torch

    logits = quant.gaussian(257, 5)
    ids = torch.zeros(9, dtype=torch.int32, device=cuda)
    w = torch.zeros(9, dtype=torch.float32, device=cuda)
    router_top_k(dev(logits, cuda), 256, 8, ids, w, with_shared=True)
    torch.cuda.synchronize()
    ref_ids, probs = oracle.router_top_k(logits[:256], 8)
    assert ids.cpu().numpy()[:8].tolist() == ref_ids.tolist()
    assert ids.cpu().numpy()[8] == 256
    assert abs(w.cpu().numpy()[8] - 1 / (1 + np.exp(-float(logits[256])))) < 1e-6


def test_swiglu(cuda):
    import torch

    S, I = 9, 512
    gu = quant.gaussian((S, 2 * I), 6) * 3
    wts = quant.gaussian(S, 7)
    out = torch.empty(S * I, device=cuda)
    swiglu(dev(gu, cuda), dev(wts, cuda), S, I, out)
    g, u = gu[:, :I].astype(np.float64), gu[:, I:].astype(np.float64)
    ref = wts[:, None] * (g / (1 + np.exp(-g))) * u
    assert np.allclose(out.cpu().numpy().reshape(S, I), ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("n", [1, 7, 248320])
def test_argmax(cuda, n):
    import torch

    v = quant.gaussian(n, 8 + n)
    if n > 10:
        v[1234] = v[99999] = v.max() + 1.0  # a tie: the first index wins
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    argmax(dev(v, cuda), n, out)
    torch.cuda.synchronize()
    assert int(out.item()) == oracle.port().q3xo_argmax(v.ctypes.data, n)


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_expert_rows_and_segments(cuda, mtype):
    import torch

    E, R, K, S = 10, 192, 512, 4
    packed = quant.quantize(quant.gaussian((E * R, K), 9, 0.02), mtype)
    pool = Linear.from_packed(packed, mtype, R, K, experts=E, device=cuda)
    per = packed.reshape(E, -1)
    ids = np.array([7, 2, 9, 2], np.int32)
    x = quant.gaussian(K, 10)
    y = torch.empty(S * R, device=cuda)
    expert_mv_rows(pool, dev(ids, cuda), S, dev(x, cuda), y)
    xs = quant.gaussian(S * K, 11)
    y2 = torch.from_numpy(quant.gaussian(R, 12)).to(cuda)
    y2_0 = y2.cpu().numpy().astype(np.float64)
    expert_mv_segments(pool, dev(ids, cuda), S, dev(xs, cuda), y2, accumulate=True)
    torch.cuda.synchronize()
    y = y.cpu().numpy().reshape(S, R)
    acc = y2_0.copy()
    mag = np.abs(y2_0)
    for s, e in enumerate(ids):
        ref = oracle.mv(per[e], mtype, R, K, x)
        m = oracle.magnitude(per[e], mtype, R, K, x)
        assert (np.abs(y[s] - ref) / m).max() <= 1e-5
        acc += oracle.mv(per[e], mtype, R, K, xs[s * K:(s + 1) * K])
        mag += oracle.magnitude(per[e], mtype, R, K, xs[s * K:(s + 1) * K])
    assert (np.abs(y2.cpu().numpy() - acc) / mag).max() <= 1e-5


@pytest.mark.parametrize("mtype", [Q8_0, Q4_0])
def test_expert_gathers_skip_negative_ids(cuda, mtype):
    """Expert parallelism marks the slots run on other GPUs with id -1: their
    rows are not written (row gather) and their segments add nothing, even
    when that segment of x holds NaN (segment gather)."""
    import torch

    E, R, K, S = 6, 128, 512, 5
    packed = quant.quantize(quant.gaussian((E * R, K), 19, 0.02), mtype)
    pool = Linear.from_packed(packed, mtype, R, K, experts=E, device=cuda)
    per = packed.reshape(E, -1)
    ids = np.array([4, -1, 0, -1, 5], np.int32)
    x = quant.gaussian(K, 20)
    y = torch.full((S * R,), 7.0, device=cuda)
    expert_mv_rows(pool, dev(ids, cuda), S, dev(x, cuda), y)
    xs = quant.gaussian(S * K, 21)
    xs[K:2 * K] = np.nan  # a skipped segment is never read as data
    y2 = torch.full((R,), 3.0, device=cuda)
    expert_mv_segments(pool, dev(ids, cuda), S, dev(xs, cuda), y2, accumulate=False)
    torch.cuda.synchronize()
    y = y.cpu().numpy().reshape(S, R)
    acc = np.zeros(R)
    mag = np.zeros(R)
    for s, e in enumerate(ids):
        if e < 0:
            assert (y[s] == 7.0).all()
            continue
        ref = oracle.mv(per[e], mtype, R, K, x)
        assert (np.abs(y[s] - ref) / oracle.magnitude(per[e], mtype, R, K, x)).max() <= 1e-5
        acc += oracle.mv(per[e], mtype, R, K, xs[s * K:(s + 1) * K])
        mag += oracle.magnitude(per[e], mtype, R, K, xs[s * K:(s + 1) * K])
    got = y2.cpu().numpy()
    assert np.isfinite(got).all()
    assert (np.abs(got - acc) / mag).max() <= 1e-5
    # every slot skipped: the output is written as zero
    none = np.full(S, -1, np.int32)
    expert_mv_segments(pool, dev(none, cuda), S, dev(xs, cuda), y2, accumulate=False)
    torch.cuda.synchronize()
    assert (y2.cpu().numpy() == 0).all()


def moe_layer_on_device(cuda, router, gate_up, down, sg, su, sd, ss, p, x):
    """engine.cpp:406-430 composed from the device kernels, shared expert as
    expert `experts` of each pool."""
    import torch

    E, k, H, I, SI = p["experts"], p["top_k"], p["H"], p["I"], p["shared_I"]
    assert SI == I
    r_all = np.concatenate([router.reshape(-1), ss.reshape(-1)]).view(np.uint8)
    gu_all = np.concatenate([gate_up.reshape(-1), sg.reshape(-1), su.reshape(-1)])
    dn_all = np.concatenate([down.reshape(-1), sd.reshape(-1)])
    rlin = Linear.from_packed(r_all, BF16, E + 1, H, device=cuda)
    gulin = Linear.from_packed(gu_all, Q4_0, 2 * I, H, experts=E + 1, device=cuda)
    dnlin = Linear.from_packed(dn_all, Q4_0, H, I, experts=E + 1, device=cuda)
    xd = dev(x, cuda)
    logits = torch.empty(E + 1, device=cuda)
    ids = torch.zeros(k + 1, dtype=torch.int32, device=cuda)
    w = torch.zeros(k + 1, device=cuda)
    gu = torch.empty((k + 1) * 2 * I, device=cuda)
    h = torch.empty((k + 1) * I, device=cuda)
    out = torch.zeros(H, device=cuda)
    mv(rlin, xd, logits)
    router_top_k(logits, E, k, ids, w, with_shared=True)
    expert_mv_rows(gulin, ids, k + 1, xd, gu)
    swiglu(gu, w, k + 1, I, h)
    expert_mv_segments(dnlin, ids, k + 1, h, out, accumulate=True)
    torch.cuda.synchronize()
    return out.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()


def test_moe_layer_matches_reference(cuda, golden, golden_meta):
    from tests.golden.make_golden import make_moe_random

    p = golden_meta["moe_random"]
    args = make_moe_random(p)
    assert hashlib.sha256(b"".join(a.tobytes() for a in args)).hexdigest() == p["sha256"]
    router, gate_up, down, sg, su, sd, ss, x = args
    out, ids, w = moe_layer_on_device(cuda, router, gate_up, down, sg, su, sd, ss, p, x)
    assert ids[:p["top_k"]].tolist() == golden["moe_rnd_ids_v2"].tolist()
    assert np.allclose(w[:p["top_k"]], golden["moe_rnd_w_v2"], rtol=1e-5)
    ref = golden["moe_rnd_y_v2"]
    assert np.abs(out - ref).max() <= 1e-4 * np.abs(ref).max() + 1e-6
