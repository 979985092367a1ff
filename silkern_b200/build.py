"""Build ``_lib/libsilkern_b200.so`` in the source tree with nvcc for sm_100a.

    python -m silkern_b200.build [--force]

The library is a plain shared object (static CUDA runtime, C ABI from
``include/silkern_b200.h``); it has no dependency on torch.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PACKAGE_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PACKAGE_DIR)
CSRC = os.path.join(PACKAGE_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
SOURCES = [
    os.path.join(CSRC, "localize.cu"),
    os.path.join(CSRC, "topk_localize.cu"),
    os.path.join(CSRC, "atomic_baseline.cu"),
]
DEPENDS = SOURCES + [
    os.path.join(CSRC, "fastdiv.cuh"),
    os.path.join(CSRC, "ptx.cuh"),
    os.path.join(INCLUDE, "silkern_b200.h"),
]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(candidate):
        return candidate
    raise RuntimeError("nvcc not found")


def _stale(target: str) -> bool:
    if not os.path.exists(target):
        return True
    built = os.path.getmtime(target)
    return any(os.path.getmtime(src) > built for src in DEPENDS)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if it is missing or older than its sources; return its path."""
    from silkern_b200._native import LIB_DIR, LIB_PATH

    if not force and not _stale(LIB_PATH):
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [
        _nvcc(),
        "-O3",
        "-std=c++17",
        *ARCH_FLAGS,
        "-lineinfo",
        "-Xcompiler",
        "-fPIC",
        "-shared",
        "-I",
        INCLUDE,
        "-o",
        tmp,
        *SOURCES,
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
