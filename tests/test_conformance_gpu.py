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


def _step_layers(dcp_rank: int, layers: int = 48, seed: int = 7000):
    from silkern_b200.workloads import config_case

    return [config_case(5, seed=seed + layer, dcp_rank=dcp_rank) for layer in range(layers)]


def _expected(layers):
    import oracle

    return [oracle.localize(c.req_ids, c.block_table, c.tokens, threads=4, **c.geometry()) for c in layers]


@pytest.mark.parametrize("dcp_rank", [0, 7])
def test_decode_step_gate_ten_thousand_replays(dcp_rank) -> None:
    """The 48-layer decode step (128 x 2048 per layer, dcp 8, each layer its
    own seeded selection) captured once and replayed 10,000 times; every
    layer of every replay is compared on the device."""
    from silkern_b200.verify import decode_step_gate

    layers = _step_layers(dcp_rank)
    gate = decode_step_gate(layers, expected=_expected(layers), replays=10_000)
    assert gate.error is None, gate.error
    assert gate.replays == 10_000 and gate.layers == 48
    assert gate.layer_mismatches == [0] * 48
    assert set(gate.checkpoints) == set(GATE_CHECKPOINTS)
    assert gate.ok, gate.checkpoints
    assert gate.step_us is not None and gate.step_us > 0


def test_decode_step_gate_counts_a_planted_mistake_in_its_layer() -> None:
    """A mistake planted in the expected result of one layer (on the CPU)
    shows up in that layer's counter on every replay, and only there."""
    from silkern_b200.verify import decode_step_gate

    layers = _step_layers(3, layers=6, seed=7100)
    expected = _expected(layers)
    out, counts = expected[4]
    out = out.copy()
    out[2, 0] ^= 1  # one element of layer 4
    expected[4] = (out, counts)
    gate = decode_step_gate(layers, expected=expected, replays=25, checkpoints=(0, 1, 25))
    assert gate.error is None, gate.error
    assert gate.layer_mismatches == [0, 0, 0, 0, 25, 0]
    assert not gate.ok
    assert gate.checkpoints[0]["exact"] and not gate.checkpoints[1]["exact"]


def test_segment_mismatch_counter() -> None:
    from silkern_b200.kernels import count_segment_mismatches

    gen = torch.Generator().manual_seed(5)
    a = torch.randint(-5, 5, (7, 3, 1000), generator=gen, dtype=torch.int32)
    b = a.clone()
    flip = torch.rand(a.shape, generator=gen) < 0.01
    b[flip] += 1
    counters = torch.zeros(7, dtype=torch.int32, device="cuda")
    count_segment_mismatches(a.cuda(), b.cuda(), counters)
    count_segment_mismatches(a.cuda(), b.cuda(), counters)
    want = 2 * flip.reshape(7, -1).sum(dim=1).to(torch.int32)
    assert torch.equal(counters.cpu(), want)
