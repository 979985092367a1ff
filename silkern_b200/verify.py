"""Conformance: try to prove the CUDA kernels wrong on the local device.

    >>> import silkern_b200
    >>> report = silkern_b200.conformance()     # doctest: +SKIP
    >>> report.ok                               # doctest: +SKIP
    True

Interface and checks of silkern/verify.py:389-447. Each (arm, geometry) cell
runs five checks:

``oracle``        output and counts equal :func:`localize_reference` elementwise;
``order``         the valid prefix equals the input row filtered by ownership and
                  table range, in input order (derived independently of the oracle);
``determinism``   repeated launches give a bytewise-identical output;
``replay``        the launch captured in a CUDA graph and replayed keeps every
                  pointer and ``torch.cuda.memory_allocated()`` unchanged and
                  still produces the oracle's output;
``immutability``  inputs are unchanged and the guard elements around every
                  output and workspace buffer are still zero.

:func:`replay_gate` adds the long-run check: a graph holding
(poison out, localize, device-side compare with the expected result) is
replayed 10,000 times; every replay is checked for bit-exactness through a
preallocated mismatch counter, and pointers plus the allocator are checked at
replay 0, 1, 10, 100, 1000 and 10000.

A failing cell is reported, not raised.
"""

from __future__ import annotations

import random
from collections.abc import Sequence
from dataclasses import dataclass, field

from silkern_b200.contract import DEFAULT_TILE_SIZE, MAX_ROW_WIDTH, localize_reference
from silkern_b200.errors import LocalizationError
from silkern_b200.kernels import count_mismatches, localize_hierarchical, localize_rowwise
from silkern_b200.workspace import workspace_shapes

CHECKS = ("oracle", "order", "determinism", "replay", "immutability")
ARMS = ("row_stable", "hierarchical_stable")

#: Geometry matrix of :func:`conformance` with no arguments: widths below, at
#: and above a tile, odd widths, both qualified page sizes, DCP degrees
#: 1/2/4/8, the last rank of each degree, grouped interleave and both width
#: extremes (1 and MAX_ROW_WIDTH).
DEFAULT_MATRIX: tuple[dict[str, int], ...] = (
    {"width": 1, "block_size": 64, "dcp_size": 1, "dcp_rank": 0, "dcp_interleave": 1},
    {"width": 63, "block_size": 32, "dcp_size": 2, "dcp_rank": 1, "dcp_interleave": 1},
    {"width": 128, "block_size": 64, "dcp_size": 2, "dcp_rank": 0, "dcp_interleave": 1},
    {"width": 129, "block_size": 64, "dcp_size": 4, "dcp_rank": 3, "dcp_interleave": 1},
    {"width": 513, "block_size": 32, "dcp_size": 4, "dcp_rank": 1, "dcp_interleave": 4},
    {"width": 1024, "block_size": 64, "dcp_size": 8, "dcp_rank": 7, "dcp_interleave": 1},
    {"width": 2048, "block_size": 64, "dcp_size": 2, "dcp_rank": 1, "dcp_interleave": 2},
    {"width": 2048, "block_size": 64, "dcp_size": 4, "dcp_rank": 2, "dcp_interleave": 1},
    {"width": 4096, "block_size": 64, "dcp_size": 2, "dcp_rank": 0, "dcp_interleave": 1},
    {"width": 6001, "block_size": 48, "dcp_size": 3, "dcp_rank": 2, "dcp_interleave": 3},
    {"width": MAX_ROW_WIDTH, "block_size": 64, "dcp_size": 8, "dcp_rank": 5, "dcp_interleave": 1},
)

GUARD_ELEMENTS = 64
REPLAY_COUNT = 32
DETERMINISM_REPEATS = 8
GATE_REPLAYS = 10_000
GATE_CHECKPOINTS = (0, 1, 10, 100, 1000, 10_000)
POISON = 0x5A5A5A5A


@dataclass
class CellReport:
    """Outcome of one (arm, geometry) cell."""

    arm: str
    geometry: dict[str, int]
    checks: dict[str, bool] = field(default_factory=dict)
    error: str | None = None

    @property
    def ok(self) -> bool:
        return self.error is None and all(self.checks.values())

    def failures(self) -> list[str]:
        if self.error is not None:
            return [f"error: {self.error}"]
        return [name for name, passed in self.checks.items() if not passed]


@dataclass
class ConformanceReport:
    """Aggregate outcome; truthy iff every cell passed every check."""

    cells: list[CellReport] = field(default_factory=list)
    device: str = "unknown"
    skipped: str | None = None

    @property
    def ok(self) -> bool:
        return self.skipped is None and bool(self.cells) and all(c.ok for c in self.cells)

    def __bool__(self) -> bool:
        return self.ok

    def summary(self) -> str:
        if self.skipped is not None:
            return f"conformance skipped: {self.skipped}"
        passed = sum(1 for c in self.cells if c.ok)
        head = (
            f"silkern_b200 conformance on {self.device}: "
            f"{passed}/{len(self.cells)} cells passed ({', '.join(CHECKS)})"
        )
        if passed == len(self.cells):
            return head
        lines = [head, ""]
        for cell in self.cells:
            if cell.ok:
                continue
            geometry = " ".join(f"{k}={v}" for k, v in cell.geometry.items())
            lines.append(f"  FAIL {cell.arm:22s} {geometry}")
            lines.extend(f"       - {failure}" for failure in cell.failures())
        return "\n".join(lines)

    def __str__(self) -> str:  # pragma: no cover - convenience
        return self.summary()


def _random_case(
    *,
    width: int,
    batch: int,
    block_size: int,
    dcp_size: int,
    seed: int,
) -> tuple[list[int], list[list[int]], list[list[int]]]:
    """One adversarial case (same mix as silkern/verify.py:132-170).

    About 12% negative tokens, 8% tokens just past the end of the page table,
    a fragmented page table with negative entries, four requests shared by the
    rows, and the extreme in-range positions in the first and last column.
    """
    rng = random.Random(seed)
    table_width = 17
    requests = 4
    req_ids = [(row * 3 + 1) % requests for row in range(batch)]
    block_table = [[rng.randrange(-2, 4096) for _ in range(table_width)] for _ in range(requests)]
    limit = block_size * table_width * dcp_size
    rows: list[list[int]] = []
    for _ in range(batch):
        row: list[int] = []
        for column in range(width):
            draw = rng.random()
            if draw < 0.12:
                row.append(rng.choice((-9, -3, -1)))
            elif draw < 0.20:
                row.append(limit + rng.randrange(block_size * dcp_size + 1))
            elif column == 0:
                row.append(0)
            elif column == width - 1:
                row.append(max(limit - 1, 0))
            else:
                row.append(rng.randrange(max(limit, 1)))
        rows.append(row)
    return req_ids, block_table, rows


def _expected_order(
    row: Sequence[int],
    table_row: Sequence[int],
    *,
    block_size: int,
    dcp_size: int,
    dcp_rank: int,
    dcp_interleave: int,
) -> list[int]:
    """The prefix a stable converter must produce, written as a filter.

    Deliberately not the oracle's control flow: ownership from a two-level
    divmod, so agreement with the oracle is evidence rather than a tautology.
    """
    kept: list[int] = []
    for raw in row:
        token = int(raw)
        if token < 0:
            continue
        group, lane = divmod(token, dcp_interleave)
        local_group, owner = divmod(group, dcp_size)
        if owner != dcp_rank:
            continue
        logical_block, offset = divmod(local_group * dcp_interleave + lane, block_size)
        if logical_block >= len(table_row):
            continue
        kept.append(int(table_row[logical_block]) * block_size + offset)
    return kept


def _guarded(torch, shape, device):
    """A zero-guarded int32 tensor: returns ``(view, backing storage)``."""
    total = 1
    for dim in shape:
        total *= dim
    storage = torch.zeros(total + 2 * GUARD_ELEMENTS, dtype=torch.int32, device=device)
    return storage[GUARD_ELEMENTS : GUARD_ELEMENTS + total].view(*shape), storage


def _guards_clean(storage) -> bool:
    return bool((storage[:GUARD_ELEMENTS] == 0).all() and (storage[-GUARD_ELEMENTS:] == 0).all())


def _launcher(arm, req, table, tokens, out, counts, workspace, geometry, tile_size):
    common = {
        "block_size": geometry["block_size"],
        "dcp_size": geometry["dcp_size"],
        "dcp_rank": geometry["dcp_rank"],
        "dcp_interleave": geometry["dcp_interleave"],
    }
    if arm == "row_stable":
        return lambda: localize_rowwise(req, table, tokens, out, counts, **common)
    return lambda: localize_hierarchical(
        req,
        table,
        tokens,
        out,
        counts,
        workspace["mapped"],
        workspace["local_positions"],
        workspace["tile_counts"],
        workspace["tile_offsets"],
        tile_size=tile_size,
        **common,
    )


def _run_cell(torch, arm, geometry, *, batch, seed, tile_size, device) -> CellReport:
    report = CellReport(arm=arm, geometry=dict(geometry))
    width = geometry["width"]
    req_ids, block_table, rows = _random_case(
        width=width,
        batch=batch,
        block_size=geometry["block_size"],
        dcp_size=geometry["dcp_size"],
        seed=seed,
    )
    req = torch.tensor(req_ids, dtype=torch.int32, device=device)
    table = torch.tensor(block_table, dtype=torch.int32, device=device)
    tokens = torch.tensor(rows, dtype=torch.int32, device=device)
    tokens_before = tokens.clone()
    table_before = table.clone()
    out, out_storage = _guarded(torch, (batch, width), device)
    counts, counts_storage = _guarded(torch, (batch,), device)
    guards = [out_storage, counts_storage]
    workspace: dict[str, object] = {}
    if arm == "hierarchical_stable":
        for name, shape in workspace_shapes(batch, width, tile_size=tile_size).items():
            view, storage = _guarded(torch, shape, device)
            workspace[name] = view
            guards.append(storage)
    launch = _launcher(arm, req, table, tokens, out, counts, workspace, geometry, tile_size)

    try:
        launch()
        torch.cuda.synchronize()
        observed_out = out.cpu().tolist()
        observed_counts = counts.cpu().tolist()
        expected_out, expected_counts = localize_reference(
            req_ids,
            block_table,
            rows,
            block_size=geometry["block_size"],
            dcp_size=geometry["dcp_size"],
            dcp_rank=geometry["dcp_rank"],
            dcp_interleave=geometry["dcp_interleave"],
        )
        report.checks["oracle"] = observed_out == expected_out and observed_counts == expected_counts

        if geometry["dcp_size"] == 1:
            report.checks["order"] = observed_out == expected_out
        else:
            order_ok = True
            for index, row in enumerate(rows):
                want = _expected_order(
                    row,
                    block_table[req_ids[index]],
                    block_size=geometry["block_size"],
                    dcp_size=geometry["dcp_size"],
                    dcp_rank=geometry["dcp_rank"],
                    dcp_interleave=geometry["dcp_interleave"],
                )
                count = observed_counts[index]
                if observed_out[index][:count] != want or any(
                    v != -1 for v in observed_out[index][count:]
                ):
                    order_ok = False
                    break
            report.checks["order"] = order_ok

        first = out.clone()
        stable = True
        for _ in range(DETERMINISM_REPEATS):
            launch()
            torch.cuda.synchronize()
            if not bool(torch.equal(out, first)):
                stable = False
                break
        report.checks["determinism"] = stable

        pointers = [t.data_ptr() for t in (req, table, tokens, out, counts)]
        pointers += [t.data_ptr() for t in workspace.values()]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                launch()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            launch()
        allocated_before = torch.cuda.memory_allocated()
        for _ in range(REPLAY_COUNT):
            graph.replay()
        torch.cuda.synchronize()
        after = [t.data_ptr() for t in (req, table, tokens, out, counts)]
        after += [t.data_ptr() for t in workspace.values()]
        report.checks["replay"] = (
            torch.cuda.memory_allocated() == allocated_before
            and after == pointers
            and out.cpu().tolist() == expected_out
        )
        del graph

        report.checks["immutability"] = (
            bool(torch.equal(tokens, tokens_before))
            and bool(torch.equal(table, table_before))
            and all(_guards_clean(storage) for storage in guards)
        )
    except Exception as exc:  # reported, not raised
        report.error = f"{type(exc).__name__}: {exc}"

    for name in CHECKS:
        report.checks.setdefault(name, False)
    return report


def _skip_reason(torch_module) -> str | None:
    if torch_module is None:
        return "torch is not installed"
    if not torch_module.cuda.is_available():
        return "no CUDA device is available"
    return None


def conformance(
    matrix: Sequence[dict[str, int]] | None = None,
    *,
    arms: Sequence[str] = ARMS,
    batch: int = 5,
    tile_size: int = DEFAULT_TILE_SIZE,
    seed: int = 20260803,
) -> ConformanceReport:
    """Run the conformance matrix on the local device.

    ``matrix`` holds geometry dicts with ``width``, ``block_size``,
    ``dcp_size``, ``dcp_rank`` and ``dcp_interleave`` (default
    :data:`DEFAULT_MATRIX`); every cell derives its own seed from ``seed``.
    Without torch or a CUDA device the report is skipped (falsy, with a
    reason) rather than raising, so it is safe to call in CI.
    """
    report = ConformanceReport()
    try:
        import torch
    except ModuleNotFoundError:
        torch = None
    reason = _skip_reason(torch)
    if reason is not None:
        report.skipped = reason
        return report
    report.device = torch.cuda.get_device_name(0)
    cells = tuple(DEFAULT_MATRIX if matrix is None else matrix)
    for arm in arms:
        if arm not in ARMS:
            raise LocalizationError(f"unknown arm: {arm}")
        for index, geometry in enumerate(cells):
            report.cells.append(
                _run_cell(torch, arm, geometry, batch=batch, seed=seed + index, tile_size=tile_size,
                          device="cuda")
            )
    return report


@dataclass
class ReplayGateReport:
    """Outcome of :func:`replay_gate`."""

    arm: str
    geometry: dict[str, int]
    replays: int = 0
    mismatches: int = -1
    checkpoints: dict[int, dict[str, bool]] = field(default_factory=dict)
    error: str | None = None

    @property
    def ok(self) -> bool:
        return (
            self.error is None
            and self.mismatches == 0
            and bool(self.checkpoints)
            and all(all(c.values()) for c in self.checkpoints.values())
        )


def replay_gate(
    geometry: dict[str, int],
    *,
    arm: str = "row_stable",
    batch: int = 8,
    replays: int = GATE_REPLAYS,
    checkpoints: Sequence[int] = GATE_CHECKPOINTS,
    tile_size: int = DEFAULT_TILE_SIZE,
    seed: int = 20261201,
) -> ReplayGateReport:
    """Replay one captured call ``replays`` times and check every replay.

    The graph holds: ``out`` and ``counts`` overwritten with a poison value,
    the localization call, and two device-side compares against the oracle's
    result that add into a preallocated mismatch counter. Pointers and
    ``torch.cuda.memory_allocated()`` are compared with their values before
    the first replay at every checkpoint (0 = right after capture).
    """
    import torch

    report = ReplayGateReport(arm=arm, geometry=dict(geometry))
    if arm not in ARMS:
        raise LocalizationError(f"unknown arm: {arm}")
    width = geometry["width"]
    req_ids, block_table, rows = _random_case(
        width=width,
        batch=batch,
        block_size=geometry["block_size"],
        dcp_size=geometry["dcp_size"],
        seed=seed,
    )
    expected_out, expected_counts = localize_reference(
        req_ids,
        block_table,
        rows,
        block_size=geometry["block_size"],
        dcp_size=geometry["dcp_size"],
        dcp_rank=geometry["dcp_rank"],
        dcp_interleave=geometry["dcp_interleave"],
    )
    device = "cuda"
    req = torch.tensor(req_ids, dtype=torch.int32, device=device)
    table = torch.tensor(block_table, dtype=torch.int32, device=device)
    tokens = torch.tensor(rows, dtype=torch.int32, device=device)
    want_out = torch.tensor(expected_out, dtype=torch.int32, device=device)
    want_counts = torch.tensor(expected_counts, dtype=torch.int32, device=device)
    out = torch.empty_like(tokens)
    counts = torch.empty(batch, dtype=torch.int32, device=device)
    mismatches = torch.zeros(1, dtype=torch.int32, device=device)
    workspace: dict[str, object] = {}
    if arm == "hierarchical_stable":
        workspace = {
            name: torch.empty(shape, dtype=torch.int32, device=device)
            for name, shape in workspace_shapes(batch, width, tile_size=tile_size).items()
        }
    launch = _launcher(arm, req, table, tokens, out, counts, workspace, geometry, tile_size)

    def step() -> None:
        out.fill_(POISON)
        counts.fill_(POISON)
        launch()
        count_mismatches(out, want_out, mismatches)
        count_mismatches(counts, want_counts, mismatches)

    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        torch.cuda.synchronize()
        mismatches.zero_()
        buffers = (req, table, tokens, out, counts, mismatches, *workspace.values())
        pointers = [t.data_ptr() for t in buffers]
        allocated = torch.cuda.memory_allocated()
        reserved = torch.cuda.memory_reserved()
        marks = sorted({c for c in checkpoints if 0 <= c <= replays})
        done = 0
        for mark in marks:
            while done < mark:
                graph.replay()
                done += 1
            torch.cuda.synchronize()
            report.checkpoints[mark] = {
                "pointers": [t.data_ptr() for t in buffers] == pointers,
                "allocated": torch.cuda.memory_allocated() == allocated,
                "reserved": torch.cuda.memory_reserved() == reserved,
                "exact": int(mismatches.item()) == 0,
            }
        while done < replays:
            graph.replay()
            done += 1
        torch.cuda.synchronize()
        report.replays = done
        report.mismatches = int(mismatches.item())
        del graph
    except Exception as exc:  # reported, not raised
        report.error = f"{type(exc).__name__}: {exc}"
    return report


def main(argv: Sequence[str] | None = None) -> int:  # pragma: no cover - CLI
    """``python -m silkern_b200``: exit non-zero if any cell fails."""
    import argparse

    parser = argparse.ArgumentParser(description="Run the silkern_b200 conformance matrix.")
    parser.add_argument("--batch", type=int, default=5)
    parser.add_argument("--tile-size", type=int, default=DEFAULT_TILE_SIZE)
    parser.add_argument("--seed", type=int, default=20260803)
    parser.add_argument("--arm", action="append", choices=list(ARMS))
    parser.add_argument("--replay-gate", type=int, default=0, metavar="N",
                        help="also run the N-replay CUDA-graph gate per arm")
    args = parser.parse_args(argv)
    arms = tuple(args.arm) if args.arm else ARMS
    report = conformance(arms=arms, batch=args.batch, tile_size=args.tile_size, seed=args.seed)
    print(report.summary())
    if report.skipped is not None:
        return 0
    ok = report.ok
    if args.replay_gate:
        for arm in arms:
            gate = replay_gate(DEFAULT_MATRIX[7], arm=arm, replays=args.replay_gate,
                               tile_size=args.tile_size)
            print(f"replay gate {arm}: {gate.replays} replays, {gate.mismatches} mismatches, "
                  f"ok={gate.ok}" + (f" ({gate.error})" if gate.error else ""))
            ok = ok and gate.ok
    return 0 if ok else 1


if __name__ == "__main__":  # pragma: no cover - CLI
    raise SystemExit(main())
