"""CPU tests of the conformance harness (behaviour of the reference's tests/test_verify.py).

The harness needs a GPU, but its report semantics, its independent order
derivation and its skip behaviour are checkable without one.
"""

from __future__ import annotations

import silkern_b200
from silkern_b200.verify import (
    CHECKS,
    DEFAULT_MATRIX,
    CellReport,
    ConformanceReport,
    ReplayGateReport,
    _expected_order,
    _random_case,
)


def test_conformance_skips_cleanly_without_a_device() -> None:
    report = silkern_b200.conformance()
    if report.skipped is not None:
        assert not report.ok
        assert not report
        assert report.skipped in {"torch is not installed", "no CUDA device is available"}
        assert "skipped" in report.summary()


def test_empty_report_is_not_ok() -> None:
    assert not ConformanceReport().ok


def test_cell_report_ok_requires_every_check() -> None:
    cell = CellReport(arm="row_stable", geometry={"width": 8})
    cell.checks = dict.fromkeys(CHECKS, True)
    assert cell.ok
    assert cell.failures() == []
    cell.checks["order"] = False
    assert not cell.ok
    assert cell.failures() == ["order"]
    cell.error = "boom"
    assert cell.failures() == ["error: boom"]


def test_failing_cell_summary_names_geometry_and_check() -> None:
    cell = CellReport(arm="row_stable", geometry={"width": 513, "dcp_size": 4})
    cell.checks = dict.fromkeys(CHECKS, True)
    cell.checks["determinism"] = False
    summary = ConformanceReport(cells=[cell], device="Test Device").summary()
    assert "FAIL" in summary and "row_stable" in summary
    assert "width=513" in summary and "determinism" in summary


def test_default_matrix_is_well_formed_and_crosses_boundaries() -> None:
    required = {"width", "block_size", "dcp_size", "dcp_rank", "dcp_interleave"}
    for geometry in DEFAULT_MATRIX:
        assert set(geometry) == required
        assert 0 <= geometry["dcp_rank"] < geometry["dcp_size"]
        assert geometry["width"] <= silkern_b200.MAX_ROW_WIDTH
        assert geometry["block_size"] % geometry["dcp_interleave"] == 0
    widths = {g["width"] for g in DEFAULT_MATRIX}
    assert {1, silkern_b200.MAX_ROW_WIDTH} <= widths
    assert any(w % 2 for w in widths)
    assert {g["dcp_size"] for g in DEFAULT_MATRIX} >= {1, 2, 4, 8}
    assert any(g["dcp_interleave"] > 1 for g in DEFAULT_MATRIX)
    assert any(g["dcp_rank"] == g["dcp_size"] - 1 for g in DEFAULT_MATRIX if g["dcp_size"] > 1)
    # a geometry off the power-of-two fast path
    assert any(g["dcp_size"] & (g["dcp_size"] - 1) for g in DEFAULT_MATRIX)


def test_independent_order_derivation_agrees_with_the_oracle() -> None:
    for seed in range(12):
        for dcp_size, dcp_rank, interleave in [(2, 0, 1), (2, 1, 2), (4, 3, 1), (4, 1, 4), (8, 7, 1),
                                               (3, 2, 2)]:
            req_ids, table, rows = _random_case(width=131, batch=3, block_size=64,
                                                dcp_size=dcp_size, seed=seed)
            out, counts = silkern_b200.localize_reference(
                req_ids, table, rows, block_size=64, dcp_size=dcp_size, dcp_rank=dcp_rank,
                dcp_interleave=interleave,
            )
            for index, row in enumerate(rows):
                want = _expected_order(row, table[req_ids[index]], block_size=64, dcp_size=dcp_size,
                                       dcp_rank=dcp_rank, dcp_interleave=interleave)
                assert want == out[index][: counts[index]]
                assert all(v == -1 for v in out[index][counts[index]:])


def test_random_case_actually_exercises_the_hard_paths() -> None:
    req_ids, table, rows = _random_case(width=256, batch=4, block_size=64, dcp_size=2, seed=7)
    flat = [v for row in rows for v in row]
    assert any(v < 0 for v in flat)
    assert any(v >= 64 * 17 * 2 for v in flat)
    assert len(set(req_ids)) > 1
    table_flat = [v for row in table for v in row]
    assert table_flat != sorted(table_flat)


def test_replay_gate_report_semantics() -> None:
    gate = ReplayGateReport(arm="row_stable", geometry={})
    assert not gate.ok
    gate.mismatches = 0
    gate.checkpoints = {0: {"pointers": True, "allocated": True}, 10: {"pointers": True, "allocated": True}}
    assert gate.ok
    gate.checkpoints[10]["allocated"] = False
    assert not gate.ok
