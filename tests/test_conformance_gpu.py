"""The conformance harness on a device: full matrix, both arms, and the 10,000-replay gate."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

import silkern_b200  # noqa: E402
from silkern_b200.verify import DEFAULT_MATRIX, GATE_CHECKPOINTS  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA is required", allow_module_level=True)


def test_conformance_default_matrix_passes() -> None:
    report = silkern_b200.conformance()
    assert report.skipped is None
    assert len(report.cells) == 2 * len(DEFAULT_MATRIX)
    assert report.ok, report.summary()


@pytest.mark.parametrize("tile_size", [64, 1024])
def test_conformance_other_tile_sizes(tile_size) -> None:
    report = silkern_b200.conformance(arms=("hierarchical_stable",), tile_size=tile_size)
    assert report.ok, report.summary()


@pytest.mark.parametrize("arm", ["row_stable", "hierarchical_stable"])
def test_ten_thousand_replays_fixed_pointers_no_growth_bit_exact(arm) -> None:
    gate = silkern_b200.replay_gate(DEFAULT_MATRIX[7], arm=arm, replays=10_000)
    assert gate.error is None, gate.error
    assert gate.replays == 10_000
    assert set(gate.checkpoints) == set(GATE_CHECKPOINTS)
    assert gate.mismatches == 0
    assert gate.ok, gate.checkpoints
