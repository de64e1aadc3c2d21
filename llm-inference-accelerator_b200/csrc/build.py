"""Build libspecdecode_cuda.so for B200 (sm_100a) in-tree.

    python llm-inference-accelerator_b200/csrc/build.py [--force] [--verbose]

Compiles every .cu file beside this script with nvcc (cross-compiles without a
GPU) into _build/, then links the shared library into the Python package
directory (specdecode_b200/libspecdecode_cuda.so), where the ctypes loader
looks first.  The CUDA runtime is linked statically so the library needs only
the driver at run time.  Rebuilds only what changed unless --force is given.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PACKAGE_ROOT = CSRC.parent
REPO = PACKAGE_ROOT.parent
INCLUDE = REPO / "include"
BUILD = CSRC / "_build"
OUTPUT = PACKAGE_ROOT / "specdecode_b200" / "libspecdecode_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-Wall",
    "-I", str(INCLUDE), "-I", str(CSRC),
]


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path("/usr/local/cuda/bin/nvcc")
    if candidate.is_file():
        return str(candidate)
    raise FileNotFoundError("nvcc not found")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def build(force: bool = False, verbose: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    newest_header = max((p.stat().st_mtime for p in _headers()), default=0.0)
    objects = []
    for source in sources:
        obj = BUILD / (source.stem + ".o")
        objects.append(obj)
        stale = (force or not obj.exists() or obj.stat().st_mtime < source.stat().st_mtime
                 or obj.stat().st_mtime < newest_header)
        if not stale:
            continue
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(source), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    link_stale = force or not OUTPUT.exists() or any(
        OUTPUT.stat().st_mtime < o.stat().st_mtime for o in objects)
    if link_stale:
        tmp = OUTPUT.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        os.replace(tmp, OUTPUT)
    return OUTPUT


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
