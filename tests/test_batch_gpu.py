"""Batched decode (q3xb_state_forward_batch): n independent sequences advanced
one token each per call, every matrix read once for all of them.

Checked against the same sequences stepped one at a time (state_forward with
one token: the GEMV path) and, for one sequence, against the reference CPU
forward (oracle/_ref): logits within 5e-4 of max(1, max|logit|) at every step
and identical greedy tokens.  The dense (9091) and MoE (35091) test models
cover the per-sequence DeltaNet and attention steps and the grouped expert
GEMMs over the batch.
"""
import numpy as np
import pytest

import oracle
from qwen3x_b200 import capi, modelfile

pytestmark = pytest.mark.gpu

TOL = 5e-4


def err(a, b):
    return float(np.abs(a - b).max() / max(1.0, np.abs(b).max()))


@pytest.fixture(scope="module")
def model_files(tmp_path_factory):
    d = tmp_path_factory.mktemp("batch_models")
    return {mid: modelfile.write_model(d / f"m{mid}.bin", modelfile.CONFIGS[mid], seed=mid + 11)
            for mid in (9091, 35091)}


@pytest.mark.parametrize("mid,n", [(9091, 8), (35091, 8), (9091, 3)])
def test_batch_matches_single_sequences_and_reference(cuda, model_files, mid, n):
    from qwen3x_b200.backend import Model, State, forward_batch

    c = modelfile.CONFIGS[mid]
    model = Model(model_files[mid])
    rng = np.random.default_rng(mid + n)
    prompts = [rng.integers(0, c.V, 5 + 3 * b).astype(np.int32) for b in range(n)]  # ragged positions
    batch = [State(model, 128) for _ in range(n)]
    single = [State(model, 128) for _ in range(n)]
    ref = oracle.RefEngine(model_files[mid], c, context=128)
    for b in range(n):
        batch[b].forward(prompts[b])
        single[b].forward(prompts[b])
    ref.forward(prompts[0])
    worst, worst_ref = 0.0, 0.0
    toks = [batch[b].argmax() for b in range(n)]
    for step in range(24):
        forward_batch(model, batch, toks)
        for b in range(n):
            single[b].forward([toks[b]])
        ref.forward([toks[0]])
        nxt = []
        for b in range(n):
            lb, ls = batch[b].logits(), single[b].logits()
            worst = max(worst, err(lb, ls))
            assert batch[b].argmax() == single[b].argmax(), (step, b)
            assert batch[b].position == single[b].position
            nxt.append(batch[b].argmax())
        worst_ref = max(worst_ref, err(batch[0].logits(), ref.logits()))
        assert nxt[0] == ref.argmax(), step
        toks = nxt
    assert worst <= TOL, worst
    assert worst_ref <= TOL, worst_ref
    for s in batch + single:
        s.close()
    model.close()


def test_batch_arguments_are_checked(cuda, model_files):
    import ctypes

    from qwen3x_b200.backend import Model, State, forward_batch

    mid = 9091
    model = Model(model_files[mid])
    s = [State(model, 8) for _ in range(2)]
    with pytest.raises(capi.Q3xkError):
        forward_batch(model, [s[0], s[0]], [1, 2])  # a sequence twice
    with pytest.raises(capi.Q3xkError):
        forward_batch(model, s, [1, modelfile.CONFIGS[mid].V])  # token out of range
    lib = capi.lib()
    handles = (ctypes.c_void_p * 17)(*([s[0].handle] * 17))
    toks = np.zeros(17, np.int32)
    assert lib.q3xb_state_forward_batch(model.handle, ctypes.cast(handles, ctypes.c_void_p), toks.ctypes.data,
                                        17) == capi.EINVAL
    for _ in range(8):
        forward_batch(model, s, [3, 4])
    with pytest.raises(capi.Q3xkError):
        forward_batch(model, s, [3, 4])  # beyond the context
    assert s[0].position == 8 and s[1].position == 8
    for x in s:
        x.close()
    model.close()


def test_batch_graph_replay_equals_eager(cuda, model_files):
    """The batched step replays a CUDA graph captured for its list of States;
    launched eagerly instead (set_graphs(False) on the lead State) it gives the
    same logits bit for bit, and a different list of States is captured anew."""
    from qwen3x_b200.backend import Model, State, forward_batch

    mid = 35091
    c = modelfile.CONFIGS[mid]
    model = Model(model_files[mid])
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, c.V, 6 + b).astype(np.int32) for b in range(4)]
    g = [State(model, 64) for _ in range(4)]
    e = [State(model, 64) for _ in range(4)]
    e[0].set_graphs(False)
    for b in range(4):
        g[b].forward(prompts[b])
        e[b].forward(prompts[b])
    for step in range(6):
        sub = 4 if step < 3 else 2  # the list changes: a new capture
        toks = [g[b].argmax() for b in range(sub)]
        forward_batch(model, g[:sub], toks)
        forward_batch(model, e[:sub], toks)
        for b in range(sub):
            np.testing.assert_array_equal(g[b].logits(), e[b].logits())
    for s in g + e:
        s.close()
    model.close()
