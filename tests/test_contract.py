"""Known-answer and validation tests of the contract (CPU).

The known answers are those of the reference's tests/test_contract.py:16-108;
each is checked against both the package's ``localize_reference`` and the C
oracle, so the oracle is pinned by the same facts the reference pins its own
oracle with.
"""

from __future__ import annotations

import random

import numpy as np
import pytest

import oracle
from silkern_b200 import (
    DEFAULT_TILE_SIZE,
    MAX_ROW_WIDTH,
    SUPPORTED_TILE_SIZES,
    LocalizationError,
    localize_reference,
    workspace_shapes,
)


def both(req_ids, table, rows, **kw):
    expected = localize_reference(req_ids, table, rows, **kw)
    out, counts = oracle.localize(req_ids, table, rows, **kw)
    assert out.tolist() == expected[0]
    assert counts.tolist() == expected[1]
    return expected


def test_routes_requests_and_nonidentity_blocks() -> None:
    rows = [[0, 1, 2, 3, 8, 9, -1, 99], [4, 5, 6, 7, 12, 13, 14, 15]]
    out, counts = both([1, 0], [[10, 30], [20, 40]], rows, block_size=4, dcp_size=2, dcp_rank=0)
    assert out == [[80, 81, 160, -1, -1, -1, -1, -1], [42, 43, 122, 123, -1, -1, -1, -1]]
    assert counts == [3, 4]


@pytest.mark.parametrize("rank", [0, 1])
def test_grouped_interleave(rank: int) -> None:
    out, counts = both([0], [[2, 3]], [list(range(8))], block_size=4, dcp_size=2, dcp_rank=rank,
                       dcp_interleave=2)
    assert out == [[8, 9, 10, 11, -1, -1, -1, -1]]
    assert counts == [4]


def test_dcp_size_one_keeps_columns() -> None:
    out, counts = both([0], [[7]], [[0, -1, 3, 4]], block_size=4, dcp_size=1, dcp_rank=0,
                       compact_valid_to_front=True)
    assert out == [[28, -1, 31, -1]]
    assert counts == [2]


def test_compaction_can_be_disabled() -> None:
    out, counts = both([0], [[5]], [[1, 0, 3, 2]], block_size=4, dcp_size=2, dcp_rank=0,
                       compact_valid_to_front=False)
    assert out == [[-1, 20, -1, 21]]
    assert counts == [2]


def test_owned_out_of_range_block_is_dropped() -> None:
    out, counts = both([0], [[0]], [[0, 2, 8]], block_size=4, dcp_size=2, dcp_rank=0)
    assert out == [[0, 1, -1]]
    assert counts == [2]


def test_negative_table_entry_used_verbatim() -> None:
    out, counts = both([0], [[-1]], [[0, 2]], block_size=4, dcp_size=2, dcp_rank=0)
    assert out == [[-4, -3]]
    assert counts == [2]


def test_valid_minus_one_counts_as_valid() -> None:
    # table entry -1, offset block_size-1: a valid slot whose value is -1.
    out, counts = both([0], [[-1]], [[6, 0]], block_size=4, dcp_size=2, dcp_rank=0)
    assert out == [[-1, -4]]
    assert counts == [2]


def _restated(req_ids, table, rows, *, block_size, dcp_size, rank, interleave):
    """Independent two-level divmod restatement (reference tests/test_contract.py:143-173)."""
    out_rows, counts = [], []
    for request, row in zip(req_ids, rows, strict=True):
        in_place, valid = [], []
        for token in row:
            value, keep = -1, False
            if token >= 0:
                group_index, lane = divmod(token, interleave)
                local_group, owner = divmod(group_index, dcp_size)
                if owner == rank:
                    block, offset = divmod(local_group * interleave + lane, block_size)
                    if block < len(table[request]):
                        value, keep = table[request][block] * block_size + offset, True
            in_place.append(value)
            if keep:
                valid.append(value)
        counts.append(len(valid))
        out_rows.append(in_place if dcp_size == 1 else valid + [-1] * (len(row) - len(valid)))
    return out_rows, counts


def test_randomized_contract_matrix() -> None:
    rng = random.Random(20260728)
    block_size = 8
    table = [[rng.randrange(0, 200) for _ in range(7)] for _ in range(3)]
    req_ids = [2, 0, 1, 2]
    for dcp_size in (1, 2, 3, 4):
        limit = block_size * len(table[0]) * dcp_size
        rows = [
            [rng.choice((-3, -1)) if rng.random() < 0.15 else rng.randrange(limit + block_size * dcp_size)
             for _ in range(37)]
            for _ in req_ids
        ]
        for interleave in (1, 2, 4):
            for rank in range(dcp_size):
                got = both(req_ids, table, rows, block_size=block_size, dcp_size=dcp_size,
                           dcp_rank=rank, dcp_interleave=interleave)
                want = _restated(req_ids, table, rows, block_size=block_size, dcp_size=dcp_size,
                                 rank=rank, interleave=interleave)
                assert got == want


def test_oracle_threads_agree() -> None:
    rng = np.random.default_rng(5)
    tokens = rng.integers(-5, 40000, size=(37, 300), dtype=np.int32)
    table = rng.integers(-2, 5000, size=(9, 70), dtype=np.int32)
    req = rng.integers(0, 9, size=37, dtype=np.int32)
    one = oracle.localize(req, table, tokens, block_size=32, dcp_size=4, dcp_rank=1, threads=1)
    many = oracle.localize(req, table, tokens, block_size=32, dcp_size=4, dcp_rank=1, threads=7)
    assert np.array_equal(one[0], many[0]) and np.array_equal(one[1], many[1])


def test_oracle_wraps_like_int32_lanes() -> None:
    # 2**26 * 64 + 5 = 2**32 + 5 does not fit in int32: stored mod 2**32 -> 5.
    out, counts = oracle.localize([0], [[2**26]], [[5]], block_size=64, dcp_size=1, dcp_rank=0)
    assert out.tolist() == [[5]]
    assert counts.tolist() == [1]
    # 2**25 * 64 = 2**31 wraps to INT32_MIN.
    out, _ = oracle.localize([0], [[2**25]], [[0]], block_size=64, dcp_size=1, dcp_rank=0)
    assert out.tolist() == [[-(2**31)]]


@pytest.mark.parametrize(
    "kwargs",
    [
        {"block_size": 0, "dcp_size": 2, "dcp_rank": 0},
        {"block_size": True, "dcp_size": 2, "dcp_rank": 0},
        {"block_size": 4, "dcp_size": 0, "dcp_rank": 0},
        {"block_size": 4, "dcp_size": 2.0, "dcp_rank": 0},
        {"block_size": 4, "dcp_size": 2, "dcp_rank": 2},
        {"block_size": 4, "dcp_size": 2, "dcp_rank": 0, "dcp_interleave": 3},
        {"block_size": 4, "dcp_size": 2, "dcp_rank": 0, "compact_valid_to_front": 1},
    ],
)
def test_rejects_invalid_configuration(kwargs: dict) -> None:
    with pytest.raises(LocalizationError):
        localize_reference([0], [[0]], [[0]], **kwargs)


def test_rejects_bad_request_routing() -> None:
    with pytest.raises(LocalizationError, match="request id"):
        localize_reference([1], [[0]], [[0]], block_size=4, dcp_size=2, dcp_rank=0)
    with pytest.raises(ValueError, match="request id"):
        oracle.localize([1], [[0]], [[0]], block_size=4, dcp_size=2, dcp_rank=0)


def test_rejects_row_count_mismatch() -> None:
    with pytest.raises(LocalizationError, match="one request id per row"):
        localize_reference([], [[0]], [[0]], block_size=4, dcp_size=2, dcp_rank=0)


@pytest.mark.parametrize(
    ("table", "rows", "message"),
    [
        ([[]], [[0]], "block_table"),
        ([[0], [1, 2]], [[0]], "block_table"),
        ([[0]], [], "rows"),
        ([[0]], [[]], "rows"),
        ([[0]], [[0], [0, 1]], "rows"),
    ],
)
def test_rejects_nonrectangular_inputs(table, rows, message) -> None:
    with pytest.raises(LocalizationError, match=message):
        localize_reference([0] * len(rows), table, rows, block_size=4, dcp_size=2, dcp_rank=0)


def test_workspace_shapes_cover_partial_tile() -> None:
    assert workspace_shapes(3, 129) == {
        "mapped": (3, 129),
        "local_positions": (3, 129),
        "tile_counts": (3, 2),
        "tile_offsets": (3, 2),
    }
    assert workspace_shapes(2, 257, tile_size=64)["tile_counts"] == (2, 5)
    assert workspace_shapes(32, 16384, tile_size=1024)["tile_offsets"] == (32, 16)
    assert DEFAULT_TILE_SIZE == 128
    assert SUPPORTED_TILE_SIZES == (64, 128, 256, 512, 1024)
    assert MAX_ROW_WIDTH == 16384


@pytest.mark.parametrize(
    ("batch", "width", "tile_size"),
    [
        (0, 1, 128),
        (1, 0, 128),
        (True, 1, 128),
        (1, 1.5, 128),
        (1, MAX_ROW_WIDTH + 1, 128),
        (1, 128, 32),
        (1, 128, 2048),
        (1, 128, 96),
    ],
)
def test_workspace_shapes_reject_invalid_configuration(batch, width, tile_size) -> None:
    with pytest.raises(LocalizationError):
        workspace_shapes(batch, width, tile_size=tile_size)
