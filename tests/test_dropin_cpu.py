"""The reference's own program objects (main.cpp, runtime.cpp, log, parser,
render, spdlog; unmodified) linked against libq3xk.so in place of a reference
backend object (oracle/Makefile target `b200cli`): every q3x_backend symbol
the runtime calls resolves in this library, and the program starts.  Host
only: without a GPU the backend reports that no CUDA device is present."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
EXE = ROOT / "oracle" / "_ref" / "qwen3x-b200"

pytestmark = pytest.mark.skipif(not EXE.exists(), reason="qwen3x-b200 not built (make -C oracle b200cli REF=...)")


def test_links_this_library():
    out = subprocess.run(["ldd", str(EXE)], capture_output=True, text=True, check=True).stdout
    line = next(ln for ln in out.splitlines() if "libq3xk.so" in ln)
    assert str((ROOT / "qwen3x_b200" / "libq3xk.so").resolve()) in str(Path(line.split("=>")[1].split("(")[0].strip()).resolve())
    undefined = subprocess.run(["nm", "-D", "--undefined-only", str(EXE)], capture_output=True, text=True,
                               check=True).stdout
    assert "q3x_backend" in undefined  # the backend comes from the library, not from a reference object


def test_program_starts_and_parses_options():
    r = subprocess.run([str(EXE)], capture_output=True, text=True, timeout=60)
    assert "--bench PREFILL_TOKENS DECODE_TOKENS" in r.stderr


def test_backend_errors_reach_the_runtime(tmp_path):
    """model_create's error travels through the runtime to the program's log."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("host-only check")
    from qwen3x_b200 import modelfile

    path = modelfile.write_model(tmp_path / "m.bin", modelfile.CONFIGS[9092], seed=3)
    r = subprocess.run([str(EXE), "-m", str(path), "--bench", "4", "4"], capture_output=True, text=True, timeout=60)
    assert r.returncode != 0
    assert "no CUDA device" in (r.stdout + r.stderr)
