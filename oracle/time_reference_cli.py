"""Times the reference's own programs (oracle/_ref/qwen3x-cuda and
oracle/_ref/qwen3x, built by `make -C oracle cli` from the unmodified qwen3x
sources) with their `--bench PREFILL DECODE` mode (main.cpp:1310-1377 of
qwen3x) on the same seeded synthetic model.bin that bench.py's engine legs
use (modelfile.write_model, seed 7).  `--program b200` runs the same program
objects linked against this repository's libq3xk.so (`make -C oracle
b200cli`): the reference's CLI and Session runtime, unchanged, on this
backend.  Comparison measurement only; the product never calls it.

    python oracle/time_reference_cli.py --config 9000 --program cuda --bench 4096 256
    python oracle/time_reference_cli.py --config 9000 --program b200 --bench 4096 256
    python oracle/time_reference_cli.py --config 9000 --program cpu --bench 4 4

Prints one JSON line with the program's own prefill and decode rates (wall
clock around state_forward calls, as main.cpp measures them) and the host's
core count.  The reference CPU program runs one thread (arch/cpu.cpp:148-154).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
sys.path.insert(0, str(ROOT))

PROGRAMS = {"cuda": HERE / "_ref" / "qwen3x-cuda", "cpu": HERE / "_ref" / "qwen3x",
            "b200": HERE / "_ref" / "qwen3x-b200"}
LINE = re.compile(r"^(prefill|decode)\s+(\d+) tokens\s+([0-9.]+) s\s+([0-9.]+) tok/s")


def parse(text: str) -> dict:
    out = {}
    for line in text.splitlines():
        m = LINE.match(line.strip())
        if m:
            out[m.group(1)] = {"tokens": int(m.group(2)), "seconds": float(m.group(3)),
                               "tok_s": float(m.group(4))}
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, default=9000)
    ap.add_argument("--program", choices=sorted(PROGRAMS), default="cuda")
    ap.add_argument("--bench", type=int, nargs=2, metavar=("PREFILL", "DECODE"), default=(4096, 256))
    ap.add_argument("--model", default=None, help="existing model.bin (default: write the seeded one)")
    ap.add_argument("--timeout", type=float, default=1200.0)
    args = ap.parse_args(argv)

    from qwen3x_b200 import modelfile

    exe = PROGRAMS[args.program]
    if not exe.exists():
        print(json.dumps({"program": args.program, "unavailable": f"{exe.name} not built (make -C oracle cli)"}))
        return 0
    c = modelfile.CONFIGS[args.config]
    path = args.model
    written = False
    if path is None:
        d = "/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"
        path = os.path.join(d, f"q3x_refcli_{args.config}_{os.getpid()}.bin")
        t0 = time.time()
        dev = None
        try:
            import torch

            dev = torch.device("cuda", 0) if torch.cuda.is_available() else None
        except ImportError:
            pass
        modelfile.write_model(path, c, seed=7, device=dev)
        written = True
        print(f"model written in {time.time() - t0:.1f} s", file=sys.stderr)
    p, d = args.bench
    cmd = [str(exe), "--model", path, "--bench", str(p), str(d), "--session-context", str(p + d + 16)]
    try:
        t0 = time.time()
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=args.timeout)
        wall = time.time() - t0
    finally:
        if written and os.path.exists(path):
            os.unlink(path)
    res = {"program": args.program, "binary": f"oracle/_ref/{exe.name}", "config": f"{args.config} ({c.name})",
           "bench": [p, d], "rc": r.returncode, "wall_s": round(wall, 1), "host_cores": os.cpu_count(),
           "threads": 1 if args.program == "cpu" else None, **parse(r.stdout)}
    if r.returncode != 0:
        res["stderr"] = r.stderr[-800:]
    print(json.dumps(res))
    return 0 if r.returncode == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
