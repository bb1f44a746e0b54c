"""End-to-end parity at the BASELINE model shapes: the backend against golden
logits of the reference CPU forward (tests/golden/engine_<id>.npz, made by
tests/golden/make_engine_golden.py from oracle/_ref, the reference's own
engine.cpp + arch/cpu.cpp).

    9000   9B-shaped hybrid, Q8_0           (BASELINE config 3)
    36035  35B-A3B-shaped MoE, Q4_0         (BASELINE config 4)
    27008  27B-shaped hybrid, Q8_0          (BASELINE config 5)

The seeded model.bin is rebuilt here with the generator the golden run used
(weights on cuda:0) and checked against the stored fingerprint.  A 12-token
prompt goes through the prompt path (tcgen05 dequant-GEMM, split precision;
MoE through the grouped expert GEMMs), then 8 decode steps (GEMV path, CUDA
graph) are fed the reference's own greedy tokens.  Bars: logits within 5e-4
of max(1, max|logit|) at the stored vocabulary entries (2048 seeded ones plus
each step's top 16), identical argmax at every step.
"""
import os
from pathlib import Path

import numpy as np
import pytest

from qwen3x_b200 import modelfile

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = 5e-4
IDS = [9000, 36035, 27008]


def _golden(mid):
    f = GOLDEN / f"engine_{mid}.npz"
    if not f.exists():
        pytest.fail(f"{f.name} missing: run tests/golden/make_engine_golden.py on a GPU host")
    return np.load(f)


@pytest.mark.parametrize("mid", IDS)
def test_backend_matches_reference_golden_logits(cuda, mid):
    import torch

    from qwen3x_b200.backend import Model, State

    import importlib.util

    spec = importlib.util.spec_from_file_location("make_engine_golden", GOLDEN / "make_engine_golden.py")
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)

    g = _golden(mid)
    c = modelfile.CONFIGS[mid]
    free, _ = torch.cuda.mem_get_info(cuda)
    if free < modelfile.file_size(c) + (8 << 30):
        pytest.skip("not enough device memory for this model shape")
    path = gen.model_path(mid)
    try:
        modelfile.write_model(path, c, seed=int(g["seed"]), device=cuda)
        assert gen.fingerprint(path) == str(g["fingerprint"]), \
            "the seeded model.bin differs from the golden run's (generator changed): regenerate the goldens"
        model = Model(path)
        st = State(model, 64)
        st.forward(g["prompt"])
        worst = 0.0
        for step in range(len(g["greedy"])):
            logits = st.logits()
            idx = g["idx"][step]
            e = float(np.abs(logits[idx] - g["logits"][step]).max() / max(1.0, float(g["absmax"][step])))
            worst = max(worst, e)
            assert e <= TOL, (step, e)
            assert st.argmax() == int(g["greedy"][step]), step
            if step + 1 < len(g["greedy"]):
                st.forward([int(g["greedy"][step])])
        st.close()
        model.close()
        print(f"{mid}: worst logit error {worst:.2e}")
    finally:
        if os.path.exists(path):
            os.unlink(path)
