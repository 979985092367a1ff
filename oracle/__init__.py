"""CPU oracle of the localization converter -- TEST INFRASTRUCTURE ONLY.

``localize_oracle.c`` restates the reference's normative loop
(silkern/contract.py:67-158, ``localize_reference``) in plain C, and the
hierarchical tile decomposition (silkern/kernels.py:203-208, :240-247). Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package; the product (``silkern_b200``) never does.

The oracle is pinned against the reference itself: ``tests/golden/`` holds
digests and arrays produced by running the reference's ``localize_reference``
and its Triton kernels (CPU interpreter) on the same seeded inputs, and
``tests/test_oracle_golden.py`` checks the oracle against every one of them.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCE = os.path.join(HERE, "localize_oracle.c")
LIB = os.path.join(HERE, "_build", "liblocalize_oracle.so")

ORACLE_OK = 0
ORACLE_E_ARGS = 1
ORACLE_E_REQUEST = 2

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with gcc into oracle/_build/ (skipped when up to date)."""
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SOURCE):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    tmp = LIB + ".tmp"
    subprocess.run(
        ["gcc", "-O2", "-std=c11", "-shared", "-fPIC", "-pthread", "-o", tmp, SOURCE], check=True
    )
    os.replace(tmp, LIB)
    return LIB


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(LIB)
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        lib.oracle_localize.restype = ctypes.c_int
        lib.oracle_localize.argtypes = [p, p, i64, i64, p, p, p, i64, i64, i64, i64, i64, i64,
                                        ctypes.c_int, ctypes.c_int]
        lib.oracle_tiles.restype = ctypes.c_int
        lib.oracle_tiles.argtypes = [p, p, i64, i64, p, p, p, i64, i64, i64, i64, i64, i64, i64]
        _lib = lib
    return _lib


def _i32(array) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(array, dtype=np.int32))


def localize(req_ids, block_table, tokens, *, block_size, dcp_size, dcp_rank, dcp_interleave=1,
             compact_valid_to_front=True, threads=1):
    """Return ``(out, counts)`` as int32 numpy arrays; raises ValueError like the reference."""
    req = _i32(req_ids)
    table = _i32(block_table)
    tok = _i32(tokens)
    if tok.ndim != 2 or table.ndim != 2 or req.shape != (tok.shape[0],):
        raise ValueError("oracle: bad input shapes")
    out = np.empty_like(tok)
    counts = np.empty(tok.shape[0], dtype=np.int32)
    rc = _load().oracle_localize(
        req.ctypes.data, table.ctypes.data, table.shape[0], table.shape[1], tok.ctypes.data,
        out.ctypes.data, counts.ctypes.data, tok.shape[0], tok.shape[1], block_size, dcp_size,
        dcp_rank, dcp_interleave, 1 if compact_valid_to_front else 0, int(threads),
    )
    if rc == ORACLE_E_REQUEST:
        raise ValueError("oracle: request id is outside block_table")
    if rc != ORACLE_OK:
        raise ValueError("oracle: invalid configuration")
    return out, counts


def tiles(req_ids, block_table, tokens, *, block_size, dcp_size, dcp_rank, dcp_interleave=1,
          tile_size=128):
    """Return ``(tile_counts, tile_offsets)`` of the hierarchical decomposition."""
    req = _i32(req_ids)
    table = _i32(block_table)
    tok = _i32(tokens)
    ntiles = (tok.shape[1] + tile_size - 1) // tile_size
    counts = np.empty((tok.shape[0], ntiles), dtype=np.int32)
    offsets = np.empty_like(counts)
    rc = _load().oracle_tiles(
        req.ctypes.data, table.ctypes.data, table.shape[0], table.shape[1], tok.ctypes.data,
        counts.ctypes.data, offsets.ctypes.data, tok.shape[0], tok.shape[1], block_size,
        dcp_size, dcp_rank, dcp_interleave, tile_size,
    )
    if rc != ORACLE_OK:
        raise ValueError("oracle: invalid tile configuration")
    return counts, offsets
