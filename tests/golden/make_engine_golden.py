"""Golden logits of the reference CPU forward at the BASELINE model shapes.

For each model ID (9000: 9B-shaped Q8_0, 36035: 35B-A3B-shaped MoE Q4_0,
27008: 27B-shaped Q8_0) this writes the seeded synthetic model.bin that the
GPU tests rebuild (qwen3x_b200.modelfile.write_model with the seed below and
the weights generated on cuda:0 -- the same generator the test uses, so the
files are byte-identical), runs the reference's own CPU engine on it
(oracle/_ref: engine.cpp + arch/cpu.cpp, compiled unmodified; engine.cpp:
431-459 forward), and stores, per step, the logits at a fixed seeded subset
of the vocabulary plus that step's top 16:

    step 0     after a PROMPT-token prompt in one forward call
    step 1..D  after each greedy token (teacher forcing: the reference's own
               argmax is fed back)

Run on a machine with a CUDA device (weights are generated there) and the
prebuilt oracle/_ref:

    python tests/golden/make_engine_golden.py [--ids 9000 36035 27008]

Output: tests/golden/engine_<id>.npz (a few hundred KB each) with the model
file's fingerprint, so a changed generator is detected instead of compared.
The reference CPU forward runs one token at a time on one core: the 27B
shape takes a few minutes.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from qwen3x_b200 import modelfile  # noqa: E402

SEED = 7            # model weights (the bench's engine legs use the same)
PROMPT = 12         # tokens of the prompt pass (T > 1: the dequant-GEMM path)
DECODE = 8          # greedy steps after it
SUBSET = 2048       # vocabulary entries kept per step (seeded), plus the top 16
TOP = 16
REGISTERED = {9000, 36035}  # IDs the reference's own loader knows (model_config.h:104-113)


def fingerprint(path: str) -> str:
    """sha256 over the file size and 1 MiB at the start, middle and end."""
    size = os.path.getsize(path)
    h = hashlib.sha256(str(size).encode())
    with open(path, "rb") as f:
        for off in (0, size // 2, max(0, size - (1 << 20))):
            f.seek(off)
            h.update(f.read(1 << 20))
    return h.hexdigest()


def prompt_tokens(mid: int, V: int) -> np.ndarray:
    return np.random.default_rng(1000 + mid).integers(0, V, PROMPT).astype(np.int32)


def subset_indices(mid: int, V: int) -> np.ndarray:
    return np.sort(np.random.default_rng(2000 + mid).choice(V, SUBSET, replace=False)).astype(np.int32)


def model_path(mid: int) -> str:
    d = "/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"
    return os.path.join(d, f"q3x_golden_{mid}_{os.getpid()}.bin")


def write(mid: int, path: str) -> str:
    import torch

    modelfile.write_model(path, modelfile.CONFIGS[mid], seed=SEED, device=torch.device("cuda", 0))
    return fingerprint(path)


def make(mid: int) -> dict:
    c = modelfile.CONFIGS[mid]
    path = model_path(mid)
    t0 = time.time()
    try:
        fp = write(mid, path)
        t1 = time.time()
        ref = oracle.RefEngine(path, None if mid in REGISTERED else c, context=PROMPT + DECODE + 8)
        sub = subset_indices(mid, c.V)
        p = prompt_tokens(mid, c.V)
        ref.forward(p)
        idx, val, greedy, vmax = [], [], [], []
        for step in range(DECODE + 1):
            logits = ref.logits()
            top = np.argsort(-logits, kind="stable")[:TOP].astype(np.int32)
            keep = np.concatenate([sub, top])
            idx.append(keep)
            val.append(logits[keep])
            vmax.append(float(np.abs(logits).max()))
            tok = ref.argmax()
            assert tok == int(top[0]) or logits[tok] == logits[top[0]]
            greedy.append(tok)
            if step < DECODE:
                ref.forward(np.array([tok], np.int32))
        t2 = time.time()
    finally:
        if os.path.exists(path):
            os.unlink(path)
    print(f"{mid}: model {t1 - t0:.0f} s, reference forward {t2 - t1:.0f} s, greedy {greedy}", flush=True)
    return {"id": np.int32(mid), "seed": np.int32(SEED), "fingerprint": np.array(fp), "prompt": p,
            "idx": np.stack(idx), "logits": np.stack(val).astype(np.float32),
            "absmax": np.array(vmax, np.float32), "greedy": np.array(greedy, np.int32)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ids", type=int, nargs="+", default=[9000, 36035, 27008])
    ap.add_argument("--out", default=str(HERE), help="output directory (default: tests/golden)")
    args = ap.parse_args(argv)
    for mid in args.ids:
        out = make(mid)
        np.savez_compressed(Path(args.out) / f"engine_{mid}.npz", **out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
