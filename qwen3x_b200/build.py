"""Build the sm_100a kernel library in-tree: qwen3x_b200/libq3xk.so.

Every .cu under qwen3x_b200/csrc is compiled by nvcc for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`) and linked into one shared library
that exports the C ABI of include/q3xk.h.  Objects go to qwen3x_b200/_build/.

    python -m qwen3x_b200.build            # incremental
    python -m qwen3x_b200.build --force    # rebuild everything
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libq3xk.so"
INCLUDE = ROOT / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
def _nccl_include():
    """nccl.h for the types and prototypes of tp.cu (NCCL itself is loaded at run time)."""
    try:
        import nvidia.nccl  # the copy torch ships

        inc = Path(list(nvidia.nccl.__path__)[0]) / "include"
        if (inc / "nccl.h").exists():
            return [f"-I{inc}"]
    except ImportError:
        pass
    return []


FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "-Xptxas", "-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}", *_nccl_include()]
LINK = ["-shared", "-lcuda", "-ldl"]


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps_newer(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, force: bool, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    if force or _deps_newer(obj, [src] + headers):
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(-4, "--resource-usage")
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        if verbose and (res.stdout or res.stderr):
            print(res.stdout + res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    if force or _deps_newer(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, *ARCH, *LINK, *map(str, objs), "-o", str(tmp)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
