"""Pin the oracle to the reference: every golden case, CPU only.

``tests/golden/golden.json`` was produced by running the reference's own
``localize_reference`` and its Triton kernels (CPU interpreter) on these
inputs (``tests/golden/make_golden.py``). Here the C oracle, and the
package's pure-Python ``localize_reference`` on the smaller cases, must
reproduce every recorded digest; the hierarchical tile workspace digests pin
``oracle.tiles``.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN_DIR, golden_inputs, input_sha, load_golden
from silkern_b200 import localize_reference
from silkern_b200.workloads import digest

CASES = load_golden()["cases"]


def _geometry(entry):
    return {k: entry[k] for k in ("block_size", "dcp_size", "dcp_rank", "dcp_interleave")}


def test_golden_set_is_complete() -> None:
    ids = {c["id"] for c in CASES}
    assert len(ids) == len(CASES)
    kinds = {c["kind"] for c in CASES}
    assert kinds == {"random_case", "config"}
    assert {c["config"] for c in CASES if c["kind"] == "config"} == {1, 2, 3, 4, 5}
    # The reference's Triton kernels agreed with its oracle on every case they ran.
    for c in CASES:
        for key in ("triton_rowwise_sha256", "triton_hierarchical_sha256"):
            if key in c:
                assert c[key] == c["oracle_sha256"], (c["id"], key)


@pytest.mark.parametrize("entry", CASES, ids=[c["id"] for c in CASES])
def test_oracle_reproduces_reference(entry) -> None:
    req_ids, table, tokens = golden_inputs(entry)
    assert input_sha(req_ids, table, tokens) == entry["input_sha256"]
    compact = entry["compact_valid_to_front"]
    out, counts = oracle.localize(req_ids, table, tokens, compact_valid_to_front=compact,
                                  threads=4, **_geometry(entry))
    assert digest(out, counts) == entry["oracle_sha256"]
    if tokens.size <= 40_000:
        ref_out, ref_counts = localize_reference(req_ids.tolist(), table.tolist(), tokens.tolist(),
                                                 compact_valid_to_front=compact, **_geometry(entry))
        assert digest(np.asarray(ref_out, dtype=np.int32),
                      np.asarray(ref_counts, dtype=np.int32)) == entry["oracle_sha256"]
    if "triton_tiles_sha256" in entry:
        tc, to = oracle.tiles(req_ids, table, tokens, tile_size=entry["tile_size"], **_geometry(entry))
        assert digest(tc, to) == entry["triton_tiles_sha256"]


def test_config1_arrays() -> None:
    data = np.load(os.path.join(GOLDEN_DIR, "config1.npz"))
    for rank in (0, 1):
        out, counts = oracle.localize(data["req_ids"], data["block_table"], data["tokens"],
                                      block_size=64, dcp_size=2, dcp_rank=rank)
        assert np.array_equal(out, data[f"out_rank{rank}"])
        assert np.array_equal(counts, data[f"counts_rank{rank}"])
    # Every token is owned by exactly one rank, and here every owned block is in the table.
    assert int(data["counts_rank0"].sum() + data["counts_rank1"].sum()) == data["tokens"].size
