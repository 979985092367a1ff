"""Property tests of the oracle on small random cases (hypothesis).

- The C oracle equals the pure-Python contract (``silkern_b200.localize_reference``,
  a restatement of silkern/contract.py:67-158) on every drawn case.
- The DCP ranks partition the tokens. Each token t >= 0 whose logical block
  is inside the table is valid on exactly one rank, so the counts over all
  ranks sum to the number of such tokens.
- Compaction is the in-place output with the invalid entries removed. For
  dcp_size > 1 the compacted row is the in-place row's valid entries, in
  order, followed by -1.
"""

from __future__ import annotations

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

import oracle
from silkern_b200 import localize_reference


@st.composite
def cases(draw):
    dcp = draw(st.integers(1, 5))
    il = draw(st.integers(1, 3))
    block = il * draw(st.integers(1, 4))
    rows = draw(st.integers(1, 3))
    twidth = draw(st.integers(1, 8))
    batch = draw(st.integers(1, 4))
    width = draw(st.integers(1, 64))
    span = twidth * block * dcp + 3
    table = draw(st.lists(st.lists(st.integers(-3, 5000), min_size=twidth, max_size=twidth),
                          min_size=rows, max_size=rows))
    req = draw(st.lists(st.integers(0, rows - 1), min_size=batch, max_size=batch))
    tokens = draw(st.lists(st.lists(st.integers(-4, span), min_size=width, max_size=width),
                           min_size=batch, max_size=batch))
    return req, table, tokens, block, dcp, il


@settings(max_examples=300, deadline=None)
@given(cases(), st.booleans())
def test_oracle_equals_contract(case, compact) -> None:
    req, table, tokens, block, dcp, il = case
    for rank in range(dcp):
        kw = dict(block_size=block, dcp_size=dcp, dcp_rank=rank, dcp_interleave=il,
                  compact_valid_to_front=compact)
        out, counts = oracle.localize(np.array(req), np.array(table), np.array(tokens), **kw)
        want_out, want_counts = localize_reference(req, table, tokens, **kw)
        assert out.tolist() == want_out
        assert counts.tolist() == want_counts


@settings(max_examples=300, deadline=None)
@given(cases())
def test_ranks_partition_the_tokens(case) -> None:
    req, table, tokens, block, dcp, il = case
    twidth = len(table[0])
    in_table = [sum(1 for t in row if t >= 0 and ((t // (dcp * il)) * il + t % il) // block < twidth)
                for row in tokens]
    total = np.zeros(len(tokens), dtype=np.int64)
    for rank in range(dcp):
        _, counts = oracle.localize(np.array(req), np.array(table), np.array(tokens), block_size=block,
                                    dcp_size=dcp, dcp_rank=rank, dcp_interleave=il)
        total += counts
    assert total.tolist() == in_table


@settings(max_examples=300, deadline=None)
@given(cases())
def test_compaction_is_the_in_place_row_filtered(case) -> None:
    req, table, tokens, block, dcp, il = case
    if dcp == 1:
        return  # compaction applies only across ranks
    for rank in range(dcp):
        kw = dict(block_size=block, dcp_size=dcp, dcp_rank=rank, dcp_interleave=il)
        packed, counts = oracle.localize(np.array(req), np.array(table), np.array(tokens),
                                         compact_valid_to_front=True, **kw)
        in_place, counts2 = oracle.localize(np.array(req), np.array(table), np.array(tokens),
                                            compact_valid_to_front=False, **kw)
        assert counts.tolist() == counts2.tolist()
        for r, row in enumerate(tokens):
            twidth = len(table[0])
            valid = [i for i, t in enumerate(row)
                     if t >= 0 and (t // il) % dcp == rank and ((t // (dcp * il)) * il + t % il) // block < twidth]
            assert len(valid) == counts[r]
            assert packed[r, :counts[r]].tolist() == [int(in_place[r, i]) for i in valid]
            assert (packed[r, counts[r]:] == -1).all()
