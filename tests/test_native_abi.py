"""The C-ABI library without a GPU: loads, exports every declared symbol, host checks.

No test here launches a kernel. Argument validation happens on the host
before any CUDA call, so rejected calls are checked with fake addresses that
are never dereferenced.
"""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from silkern_b200 import _native, workspace_shapes
from silkern_b200.build import build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "silkern_b200.h")


@pytest.fixture(scope="module")
def lib():
    build()
    return _native.load()


def declared_symbols() -> set[str]:
    text = open(HEADER).read()
    return set(re.findall(r"\b(silkern_\w+_v\d+)\s*\(", text))


def test_every_declared_symbol_is_exported(lib) -> None:
    symbols = declared_symbols()
    assert len(symbols) >= 8
    assert symbols == set(_native.SIGNATURES)
    for name in symbols:
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings(lib) -> None:
    assert lib.silkern_abi_version_v1() == _native.ABI_VERSION
    assert _native.status_string(0) == "ok"
    for code in range(1, 8):
        assert _native.status_string(code) != "unknown status"
    assert "dcp" in _native.status_string(3)


@pytest.mark.parametrize("width", [1, 129, 2048, 16384])
@pytest.mark.parametrize("tile", [64, 128, 256, 512, 1024])
def test_workspace_shapes_abi_matches_python(lib, width, tile) -> None:
    shapes = (ctypes.c_int64 * 8)()
    assert lib.silkern_workspace_shapes_v1(5, width, tile, shapes) == 0
    py = workspace_shapes(5, width, tile_size=tile)
    flat = [d for key in ("mapped", "local_positions", "tile_counts", "tile_offsets") for d in py[key]]
    assert list(shapes) == flat


def test_workspace_shapes_abi_rejects(lib) -> None:
    shapes = (ctypes.c_int64 * 8)()
    assert lib.silkern_workspace_shapes_v1(0, 8, 128, shapes) == 2
    assert lib.silkern_workspace_shapes_v1(1, 16385, 128, shapes) == 2
    assert lib.silkern_workspace_shapes_v1(1, 8, 96, shapes) == 5
    assert lib.silkern_workspace_shapes_v1(1, 8, 2048, shapes) == 5


@pytest.mark.parametrize("divisor", [1, 2, 3, 7, 48, 64, 1000, 65537, 2**31 - 1, 2**31])
def test_fastdiv_sampled_ranges(lib, divisor) -> None:
    for start in (0, 2**31 - 2**20, 123456789, 2**20):
        assert lib.silkern_fastdiv_selftest_v1(divisor, start, 2**20) == 0


@pytest.mark.parametrize("divisor", [3, 6, 641])
def test_fastdiv_exhaustive(lib, divisor) -> None:
    # every numerator the kernels can see (0 .. 2^31 - 1)
    assert lib.silkern_fastdiv_selftest_v1(divisor, 0, 2**31) == 0


def test_fastdiv_random_divisors(lib) -> None:
    rng = np.random.default_rng(11)
    for divisor in rng.integers(1, 2**31, size=300):
        start = int(rng.integers(0, 2**31 - 4096))
        assert lib.silkern_fastdiv_selftest_v1(int(divisor), start, 4096) == 0


# Fake, never-dereferenced device addresses for host-side validation.
REQ, TABLE, TOK, OUT, CNT = 0x10000, 0x20000, 0x40000, 0x80000, 0xC0000


def rowwise(lib, **over):
    args = dict(req=REQ, table=TABLE, rows=4, twidth=8, tok=TOK, out=OUT, cnt=CNT, batch=4, width=16,
                bs=64, dcp=2, rank=0, il=1, compact=1)
    args.update(over)
    return lib.silkern_localize_rowwise_v1(
        args["req"], args["table"], args["rows"], args["twidth"], args["tok"], args["out"],
        args["cnt"], args["batch"], args["width"], args["bs"], args["dcp"], args["rank"],
        args["il"], args["compact"], None, None,
    )


@pytest.mark.parametrize(
    ("override", "code"),
    [
        ({"req": None}, 1),
        ({"out": None}, 1),
        ({"batch": 0}, 2),
        ({"width": 0}, 2),
        ({"width": 16385}, 2),
        ({"rows": 0}, 2),
        ({"twidth": 0}, 2),
        ({"dcp": 0}, 3),
        ({"rank": 2}, 3),
        ({"rank": -1}, 3),
        ({"il": 0}, 3),
        ({"bs": 0}, 4),
        ({"il": 3}, 4),
        ({"out": TOK}, 6),
        ({"out": TOK + 60}, 6),
        ({"cnt": REQ}, 6),
        ({"cnt": OUT + 8}, 6),
    ],
)
def test_rowwise_rejects_before_launch(lib, override, code) -> None:
    assert rowwise(lib, **override) == code


def test_hierarchical_rejects_before_launch(lib) -> None:
    def call(tile, tc=0xD0000, to=0xE0000):
        return lib.silkern_localize_hierarchical_v1(
            REQ, TABLE, 4, 8, TOK, OUT, CNT, None, None, tc, to, 4, 16, 64, 2, 0, 1, 1, tile,
            None, None,
        )

    assert call(0) == 5
    assert call(96) == 5
    assert call(2048) == 5
    assert call(128, tc=None) == 1
    assert call(128, tc=OUT) == 6
    assert call(128, to=0xD0000) == 6


def test_noalloc_checks_arguments_in_the_workspace_entry_points_order(lib) -> None:
    """The allocation-free entry point rejects bad arguments with the same
    codes, in the same order, as the workspace entry point, and only then
    applies its own static-array limit (batch x tiles)."""
    far = 1 << 40  # fake buffers this far apart never overlap, whatever the shapes

    def call(req=REQ, out=3 * far, batch=4, width=16, dcp=2, tile=128):
        return lib.silkern_localize_hierarchical_noalloc_v1(
            req, far, 4, 8, 2 * far, out, 4 * far, batch, width, 64, dcp, 0, 1, 1, tile, None, None,
        )

    huge = 1 << 20  # batch x tiles far beyond the static array
    assert call(req=None, batch=huge) == 1
    assert call(out=None, batch=huge) == 1
    assert call(dcp=0, batch=huge) == 3
    assert call(tile=96, batch=huge) == 5
    assert call(out=2 * far, batch=4) == 6
    assert call(batch=huge, width=16384) == 8
    assert call(batch=40000, width=64, tile=64) == 8


def test_segment_mismatch_counter_rejects(lib) -> None:
    call = lib.silkern_count_segment_mismatches_v1
    assert call(None, TOK, 4, 16, CNT, None) == 1
    assert call(OUT, TOK, 4, 16, None, None) == 1
    assert call(OUT, TOK, 65536, 16, CNT, None) == 2
    assert call(OUT, TOK, -1, 16, CNT, None) == 2
    assert call(OUT, TOK, 0, 16, CNT, None) == 0  # nothing to compare: no launch


def test_copy_floor_rejects(lib) -> None:
    call = lib.silkern_copy_floor_v1
    assert call(None, OUT, 16, 8, 256, 0, None) == 1
    assert call(TOK, None, 16, 8, 256, 0, None) == 1
    assert call(TOK, OUT, -1, 8, 256, 0, None) == 2
    assert call(TOK, OUT, 16, 4, 256, 0, None) == 7
    assert call(TOK, OUT, 16, 8, 48, 0, None) == 7
    assert call(TOK, OUT, 16, 8, 2048, 0, None) == 7
    assert call(TOK, OUT, 16, 8, 256, -1, None) == 7
    assert call(TOK, OUT, 16, 8, 256, 9, None) == 7
    assert call(TOK, TOK + 32, 16, 8, 256, 0, None) == 6
    assert call(TOK, OUT, 0, 8, 256, 2, None) == 0  # nothing to copy: no launch


def test_explicit_rejects_bad_geometry(lib) -> None:
    def call(cluster, stage=-1, prefetch=-1, width=16, chunks=0):
        return lib.silkern_localize_explicit_v1(
            REQ, TABLE, 4, 8, TOK, OUT, CNT, None, None, 4, width, 64, 2, 0, 1, 1, 0, cluster,
            stage, prefetch, chunks, None, None,
        )

    assert call(0) == 7
    assert call(9) == 7
    assert call(1, stage=2) == 7
    assert call(1, prefetch=-2) == 7
    assert call(8, width=16) == 7  # 8 CTAs cannot each own 4-column slices of 16 columns
    assert call(1, chunks=3) == 7
    assert call(1, chunks=1, width=16384) == 7  # 4096 granules do not fit 512 threads x 1 chunk


LOGITS, LENS, POS = 0x100000, 0x200000, 0x300000


def topk(lib, explicit=None, **over):
    a = dict(logits=LOGITS, stride=4096, width=4096, lens=LENS, req=REQ, table=TABLE, rows=4, twidth=8,
             pos=POS, out=OUT, cnt=CNT, batch=4, k=64, bs=64, dcp=2, rank=0, il=1, compact=1)
    a.update(over)
    args = [a["logits"], a["stride"], a["width"], a["lens"], a["req"], a["table"], a["rows"], a["twidth"],
            a["pos"], a["out"], a["cnt"], a["batch"], a["k"], a["bs"], a["dcp"], a["rank"], a["il"],
            a["compact"]]
    if explicit is not None and len(explicit) == 3:
        return lib.silkern_topk_localize_explicit_v2(*args, *explicit, None, None)
    if explicit is not None:
        return lib.silkern_topk_localize_explicit_v1(*args, explicit[0], explicit[1], None, None)
    return lib.silkern_topk_localize_v1(*args, None, None)


@pytest.mark.parametrize(
    ("override", "code"),
    [
        ({"logits": None}, 1),
        ({"lens": None}, 1),
        ({"out": None}, 1),
        ({"batch": 0}, 2),
        ({"width": 0}, 2),
        ({"width": 262145, "stride": 262145}, 2),
        ({"stride": 4095}, 2),
        ({"k": 0}, 2),
        ({"k": 16385}, 2),
        ({"twidth": 0}, 2),
        ({"dcp": 0}, 3),
        ({"rank": 2}, 3),
        ({"bs": 0}, 4),
        ({"out": LOGITS + 64}, 6),  # out overlaps the logits
        ({"pos": OUT + 4}, 6),  # positions overlap out
        ({"cnt": LENS}, 6),
    ],
)
def test_topk_rejects_before_launch(lib, override, code) -> None:
    assert topk(lib, **override) == code


def test_topk_explicit_rejects_bad_geometry(lib) -> None:
    assert topk(lib, explicit=(63, -1)) == 7  # candidate list below top_k (64)
    assert topk(lib, explicit=(1 << 20, -1)) == 7  # candidate list beyond the shared-memory budget
    assert topk(lib, explicit=(-1, -1)) == 7
    assert topk(lib, explicit=(0, 2)) == 7  # stage_table not -1, 0 or 1
    assert topk(lib, explicit=(0, -2)) == 7
    assert topk(lib, explicit=(0, 1), twidth=4097, rows=1) == 7  # too wide to stage
    assert topk(lib, explicit=(63, -1, 0)) == 7  # the same checks through v2
    for threads in (-1, 1, 256, 513, 2048):  # CTA shape not 0, 512 or 1024
        assert topk(lib, explicit=(0, -1, threads)) == 7


def test_missing_library_fails_loudly(tmp_path) -> None:
    """No CPU or Triton fallback: without the library every launcher raises."""
    import subprocess
    import sys

    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "import silkern_b200._native as nat\n"
        "nat.LIB_PATH = %r\n"
        "from silkern_b200 import LocalizationError\n"
        "try:\n"
        "    nat.load()\n"
        "except LocalizationError as exc:\n"
        "    print('raised:', exc)\n"
        "else:\n"
        "    print('loaded')\n"
    ) % (REPO, str(tmp_path / "missing.so"))
    proc = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stderr
    assert proc.stdout.startswith("raised:") and "not built" in proc.stdout
