"""The C ABI from a plain C program (no torch, no Python in the call path).

CPU: the header compiles as C11 and the program links against the library.
GPU: the program runs all three localization entry points and compares them
with the C oracle, then runs the fused top-k entry point on distinct scores
and checks it against a selection sorted in C, localized by the oracle.
"""

from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from silkern_b200.build import build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCE = os.path.join(REPO, "tests", "c_consumer", "localize_consumer.c")
ORACLE = os.path.join(REPO, "oracle", "localize_oracle.c")
LIB_DIR = os.path.join(REPO, "silkern_b200", "_lib")
CUDA = "/usr/local/cuda"


def _compile(out_path: str) -> None:
    build()
    if shutil.which("gcc") is None or not os.path.isdir(os.path.join(CUDA, "include")):
        pytest.skip("gcc or the CUDA toolkit headers are not available")
    subprocess.run(
        ["gcc", "-O2", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"),
         "-I", os.path.join(CUDA, "include"), SOURCE, ORACLE, "-o", out_path,
         "-L", LIB_DIR, "-lsilkern_b200", "-Wl,-rpath," + LIB_DIR,
         "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(CUDA, "lib64"),
         "-pthread"],
        check=True,
    )


def test_header_compiles_as_c_and_links(tmp_path) -> None:
    _compile(str(tmp_path / "consumer"))
    assert os.path.exists(tmp_path / "consumer")


@pytest.mark.gpu
def test_c_program_matches_oracle(tmp_path) -> None:
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("CUDA is required")
    exe = str(tmp_path / "consumer")
    _compile(exe)
    proc = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stderr + proc.stdout
    assert proc.stdout.startswith("ok")
