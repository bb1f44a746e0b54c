"""End-to-end parity of the B200 backend (q3x_backend.h) with the reference CPU
forward (engine.cpp, compiled unmodified into oracle/_ref) on seeded synthetic
model.bin files of the small test configurations (modelfile.CONFIGS 9091,
9092, 35091: real head sizes, few layers, 4096-token vocabulary).

Tolerances, as absolute logit error over max(1, max|logit|):
  5e-4, the reference's own cross-backend bar (tests/backend_smoke.py:28 of
  qwen3x), for every default path: decode (CUDA-core GEMV) and prompts
  through the tcgen05 dequant-GEMM in its default split precision (both
  operands as two FP16 planes, FP32-grade);
  5e-3 for the optional FP16-precision prompt GEMM (measured 6.7e-4 ..
  2.7e-3 on the dense models).  At that precision a MoE model's top-k
  routing can flip where two expert probabilities are closer than the
  rounding error (the 100-token prompt of model 35091 flips one route and
  misses by 4.2e-2), so the FP16-precision test covers the dense models and
  the MoE flip is pinned as an expected failure;
and greedy decoding must produce the same tokens as the reference.
"""
import numpy as np
import pytest

import oracle
from qwen3x_b200 import modelfile

pytestmark = pytest.mark.gpu

DECODE_TOL = 5e-4
PREFILL_TOL = 5e-4
FP16_PREFILL_TOL = 5e-3
IDS = [9091, 9092, 35091]


@pytest.fixture(scope="module")
def model_files(tmp_path_factory):
    d = tmp_path_factory.mktemp("models")
    return {mid: modelfile.write_model(d / f"m{mid}.bin", modelfile.CONFIGS[mid], seed=mid) for mid in IDS}


def err(a, b):
    return float(np.abs(a - b).max() / max(1.0, np.abs(b).max()))


def engines(path, mid, context):
    from qwen3x_b200.backend import Model, State

    model = Model(path)
    assert model.id == mid
    ref = oracle.RefEngine(path, modelfile.CONFIGS[mid], context=context)
    return model, State(model, context), ref


def prompt(mid, n, seed=0):
    return np.random.default_rng(seed + mid).integers(0, modelfile.CONFIGS[mid].V, n).astype(np.int32)


@pytest.mark.parametrize("mid", IDS)
def test_decode_path_matches_reference_token_by_token(cuda, model_files, mid):
    """Tokens fed one at a time: every step is a decode step (GEMV path,
    CUDA graph replay), compared with the reference after each token."""
    model, st, ref = engines(model_files[mid], mid, 256)
    worst = 0.0
    for tok in prompt(mid, 24):
        st.forward([tok])
        ref.forward([tok])
        worst = max(worst, err(st.logits(), ref.logits()))
        assert st.argmax() == ref.argmax()
    assert worst <= DECODE_TOL, worst
    assert st.position == 24


@pytest.mark.parametrize("mid,n", [(9091, 100), (9092, 100), (35091, 100), (35091, 33), (35091, 300)])
def test_prefill_matches_reference(cuda, model_files, mid, n):
    """A prompt in one call: the dequant-GEMM path (split precision) for T > 1.
    The 100-token MoE prompt is the one that flips a route at FP16 precision."""
    model, st, ref = engines(model_files[mid], mid, 512)
    p = prompt(mid, n, seed=1)
    st.forward(p)
    ref.forward(p)
    e = err(st.logits(), ref.logits())
    assert e <= PREFILL_TOL, e
    assert st.argmax() == ref.argmax()
    assert st.position == n


@pytest.mark.parametrize("mid,n", [(9091, 100), (9092, 100), (35091, 33)])
def test_fp16_prefill_matches_reference(cuda, model_files, mid, n):
    """The optional FP16-precision prompt GEMM, at its looser bar."""
    from qwen3x_b200.capi import GEMM_FP16

    model, st, ref = engines(model_files[mid], mid, 512)
    st.set_prefill_precision(GEMM_FP16)
    p = prompt(mid, n, seed=1)
    st.forward(p)
    ref.forward(p)
    e = err(st.logits(), ref.logits())
    assert e <= FP16_PREFILL_TOL, e


@pytest.mark.xfail(strict=True, reason="FP16 operands flip one top-8 route of this prompt (4.2e-2)")
def test_fp16_prefill_moe_route_flip(cuda, model_files):
    """Pins the known limit of FP16 precision on MoE models: this prompt
    misses the reference by far more than the FP16 bar once a route flips."""
    from qwen3x_b200.capi import GEMM_FP16

    mid = 35091
    model, st, ref = engines(model_files[mid], mid, 512)
    st.set_prefill_precision(GEMM_FP16)
    p = prompt(mid, 100, seed=1)
    st.forward(p)
    ref.forward(p)
    assert err(st.logits(), ref.logits()) <= FP16_PREFILL_TOL


@pytest.mark.parametrize("mid", IDS)
def test_exact_prefill_in_chunks_matches_reference(cuda, model_files, mid):
    """Exact mode (per-token GEMVs) with 7-token passes: checks the T > 1
    layer kernels (conv and DeltaNet over T tokens, causal attention inside a
    pass and across passes) at GEMV accuracy."""
    model, st, ref = engines(model_files[mid], mid, 512)
    st.set_exact_prefill(True)
    st.set_prefill_chunk(7)
    p = prompt(mid, 100, seed=1)
    st.forward(p[:61])
    st.forward(p[61:], compute_logits=True)
    ref.forward(p)
    e = err(st.logits(), ref.logits())
    assert e <= DECODE_TOL, e
    assert st.argmax() == ref.argmax()


@pytest.mark.parametrize("mid", [9092, 35091])
def test_gemm_prefill_in_chunks(cuda, model_files, mid):
    """The GEMM path over several passes matches the reference to the prefill
    tolerance."""
    model, st, ref = engines(model_files[mid], mid, 512)
    p = prompt(mid, 150, seed=6)
    st.set_prefill_chunk(64)  # 64 + 64 + 22
    st.forward(p)
    ref.forward(p)
    e = err(st.logits(), ref.logits())
    assert e <= PREFILL_TOL, e


@pytest.mark.parametrize("mid", [9091, 35091])
def test_greedy_256_steps_identical(cuda, model_files, mid):
    """The acceptance run: prompt, then 256 greedy decode steps; the token
    sequences must be identical and the decode logits within tolerance."""
    model, st, ref = engines(model_files[mid], mid, 512)
    p = prompt(mid, 16, seed=2)
    for tok in p:  # decode-path prompt so the comparison starts from matching states
        st.forward([tok])
        ref.forward([tok])
    ours, theirs, worst = [], [], 0.0
    for _ in range(256):
        a, b = st.argmax(), ref.argmax()
        ours.append(a)
        theirs.append(b)
        worst = max(worst, err(st.logits(), ref.logits()))
        st.forward([a])
        ref.forward([b])
    assert ours == theirs
    assert worst <= DECODE_TOL, worst


@pytest.mark.parametrize("mid", [9091, 35091])
def test_prefill_then_greedy_tokens_identical(cuda, model_files, mid):
    """GEMM-path prompt (the MoE model's route-sensitive 100-token one), then
    64 greedy steps: identical tokens, logits within the bar at every step."""
    model, st, ref = engines(model_files[mid], mid, 512)
    p = prompt(mid, 100, seed=1)
    st.forward(p)
    ref.forward(p)
    ours, theirs, worst = [], [], 0.0
    for _ in range(64):
        ours.append(st.argmax())
        theirs.append(ref.argmax())
        worst = max(worst, err(st.logits(), ref.logits()))
        st.forward([ours[-1]])
        ref.forward([theirs[-1]])
    assert ours == theirs
    assert worst <= PREFILL_TOL, worst


def test_checkpoint_restore_and_reset(cuda, model_files):
    """state_checkpoint_save/restore and state_reset (engine.cpp:584-600,
    :156-159): decoding after a restore repeats the same logits exactly."""
    mid = 9091
    model, st, ref = engines(model_files[mid], mid, 256)
    p = prompt(mid, 20, seed=4)
    st.forward(p)
    st.checkpoint_save()
    saved = st.logits()
    first = []
    for tok in [5, 6, 7]:
        st.forward([tok])
        first.append(st.logits())
    st.checkpoint_restore()
    assert st.position == 20
    np.testing.assert_array_equal(st.logits(), saved)
    for i, tok in enumerate([5, 6, 7]):
        st.forward([tok])
        np.testing.assert_array_equal(st.logits(), first[i])
    st.reset()
    assert st.position == 0
    st.forward(p)
    np.testing.assert_array_equal(st.logits(), saved)


def test_graph_replay_equals_eager(cuda, model_files):
    """The captured decode graph launches the same kernels as the eager path."""
    from qwen3x_b200.backend import State

    mid = 35091
    model, st, _ = engines(model_files[mid], mid, 128)
    eager = State(model, 128)
    eager.set_graphs(False)
    for tok in prompt(mid, 12, seed=5):
        st.forward([tok])
        eager.forward([tok])
        np.testing.assert_array_equal(st.logits(), eager.logits())


def test_forward_validates_arguments(cuda, model_files):
    from qwen3x_b200 import capi

    mid = 9092
    model, st, _ = engines(model_files[mid], mid, 8)
    with pytest.raises(capi.Q3xkError):
        st.forward([modelfile.CONFIGS[mid].V])  # token out of range
    with pytest.raises(capi.Q3xkError):
        st.forward(np.zeros(9, np.int32))  # beyond the context
    st.forward(np.zeros(8, np.int32))
    assert st.position == 8
