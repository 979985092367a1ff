"""The CPU oracle of the fused top-k + localization, checked by brute force.

Selection is checked against a plain sort of every row by (order key
descending, position ascending), the order keys against the float order, and
the localization half against the pure-Python contract
(``silkern_b200.localize_reference``, a restatement of silkern/contract.py:67-158).
"""

from __future__ import annotations

import math
import struct

import numpy as np
import pytest

import oracle
from oracle.topk import order_keys, select_positions, topk_localize
from silkern_b200 import localize_reference


def _brute_select(row_values, length, top_k):
    if length <= top_k:
        return list(range(length))
    keys = order_keys(row_values[:length]).tolist()
    keyed = sorted(range(length), key=lambda p: (-keys[p], p))
    return sorted(keyed[:top_k])


def test_order_keys_follow_the_float_order() -> None:
    values = np.array([-math.inf, -3.0e38, -1.0, -1e-45, -0.0, 0.0, 1e-45, 1.0, 2.0, 3.4e38, math.inf],
                      dtype=np.float32)
    keys = order_keys(values)
    assert list(keys) == sorted(keys)
    assert len(set(keys.tolist())) == len(values)  # -0 and +0 differ: -0 < +0


def test_order_keys_place_nans_outside_the_infinities() -> None:
    pos_nan = np.frombuffer(struct.pack("<I", 0x7FC00000), dtype=np.float32)
    neg_nan = np.frombuffer(struct.pack("<I", 0xFFC00000), dtype=np.float32)
    inf = np.array([math.inf], dtype=np.float32)
    ninf = np.array([-math.inf], dtype=np.float32)
    assert order_keys(pos_nan)[0] > order_keys(inf)[0]
    assert order_keys(neg_nan)[0] < order_keys(ninf)[0]


def _values(rng, kind, shape):
    if kind == "normal":
        return rng.standard_normal(shape).astype(np.float32)
    if kind == "ties":
        return rng.integers(-3, 4, size=shape).astype(np.float32)
    if kind == "equal":
        return np.full(shape, 0.25, dtype=np.float32)
    if kind == "special":
        pool = np.array([math.inf, -math.inf, 0.0, -0.0, 1.0, -1.0, np.nan, 1e-40, -1e-40], dtype=np.float32)
        return pool[rng.integers(0, len(pool), size=shape)]
    raise ValueError(kind)


@pytest.mark.parametrize("kind", ["normal", "ties", "equal", "special"])
@pytest.mark.parametrize(("width", "top_k"), [(1, 1), (17, 5), (64, 64), (300, 17), (1000, 999)])
def test_selection_matches_brute_force(kind, width, top_k) -> None:
    rng = np.random.default_rng(7000 + width + top_k)
    batch = 6
    logits = _values(rng, kind, (batch, width))
    lens = np.array([0, 1, top_k, top_k + 1, width, width + 5][:batch], dtype=np.int32)
    lens = np.minimum(lens, width + 5)
    rows = select_positions(logits, lens, top_k)
    for b in range(batch):
        length = min(max(int(lens[b]), 0), width)
        want = _brute_select(logits[b], length, top_k)
        assert rows[b, : len(want)].tolist() == want
        assert (rows[b, len(want):] == -1).all()


def test_negative_and_oversized_lengths_are_clamped() -> None:
    logits = np.arange(12, dtype=np.float32).reshape(2, 6)
    rows = select_positions(logits, np.array([-4, 99], dtype=np.int32), 3)
    assert rows[0].tolist() == [-1, -1, -1]
    assert rows[1].tolist() == [3, 4, 5]


@pytest.mark.parametrize(("dcp", "rank", "il", "compact"),
                         [(1, 0, 1, True), (2, 1, 1, True), (4, 3, 1, False), (3, 2, 2, True)])
def test_localization_half_is_the_contract(dcp, rank, il, compact) -> None:
    rng = np.random.default_rng(7100 + dcp * 10 + rank)
    batch, width, top_k, block = 5, 900, 128, 32
    logits = rng.standard_normal((batch, width)).astype(np.float32)
    lens = rng.integers(0, width + 1, size=batch).astype(np.int32)
    table = rng.integers(-2, 5000, size=(7, 12)).astype(np.int32)
    req = np.array([3, 0, 6, 1, 3], dtype=np.int32)
    rows, out, counts = topk_localize(logits, lens, req, table, top_k=top_k, block_size=block,
                                      dcp_size=dcp, dcp_rank=rank, dcp_interleave=il,
                                      compact_valid_to_front=compact)
    want_out, want_counts = localize_reference(req.tolist(), table.tolist(), rows.tolist(),
                                               block_size=block, dcp_size=dcp, dcp_rank=rank,
                                               dcp_interleave=il, compact_valid_to_front=compact)
    assert out.tolist() == want_out
    assert counts.tolist() == want_counts
    direct_out, direct_counts = oracle.localize(req, table, rows, block_size=block, dcp_size=dcp,
                                                dcp_rank=rank, dcp_interleave=il,
                                                compact_valid_to_front=compact)
    assert np.array_equal(direct_out, out) and np.array_equal(direct_counts, counts)
