"""Seeded fuzzing of every CUDA entry point against the oracle, bit for bit.

Each test draws geometries the hand-written cases do not pin:
- any batch up to 300 and any width up to the 16384 limit;
- dcp_size 1..8 with every rank, and grouped interleave;
- block sizes that are not powers of two;
- narrow and wide tables with negative entries;
- every tile size, both compaction modes;
- views that start off a 16-byte boundary.

Each draw is checked against the C restatement of silkern/contract.py:67-158
(and, for the tile workspace, silkern/kernels.py:203-208, :240-247). The
fused top-k kernel is fuzzed the same way against its oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from oracle.topk import topk_localize as oracle_topk  # noqa: E402
from silkern_b200 import (  # noqa: E402
    localize_hierarchical,
    localize_rowwise,
    topk_localize,
    workspace_shapes,
)
from silkern_b200.contract import SUPPORTED_TILE_SIZES  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA is required", allow_module_level=True)

DEV = torch.device("cuda", 0)
WIDTHS = [1, 2, 3, 4, 5, 17, 64, 127, 128, 129, 511, 1000, 2047, 2048, 2049, 4096, 4099, 8191, 8192,
          8193, 12000, 16383, 16384]


def _draw(rng):
    batch = int(rng.choice([1, 2, 3, 7, 31, 64, 100, 148, 149, 257, 300]))
    width = int(rng.choice(WIDTHS)) if rng.random() < 0.7 else int(rng.integers(1, 16385))
    if batch * width > 2_000_000:  # keep each draw small
        batch = max(1, 2_000_000 // width)
    dcp = int(rng.integers(1, 9))
    rank = int(rng.integers(0, dcp))
    il = int(rng.choice([1, 1, 1, 2, 3, 4]))
    block = il * int(rng.integers(1, 33))
    rows = int(rng.integers(1, 20))
    twidth = int(rng.integers(1, 300))
    table = rng.integers(-5, 1 << 20, size=(rows, twidth)).astype(np.int32)
    req = rng.integers(0, rows, size=batch).astype(np.int32)
    span = max(1, int(1.2 * twidth * block * dcp))
    tokens = rng.integers(-8, span, size=(batch, width)).astype(np.int32)
    compact = bool(rng.random() < 0.8)
    geometry = dict(block_size=block, dcp_size=dcp, dcp_rank=rank, dcp_interleave=il,
                    compact_valid_to_front=compact)
    return req, table, tokens, geometry


def _dev(a, shift=0):
    """A device copy of `a`; with `shift` > 0 the view starts 4 * shift bytes
    past an allocation boundary (off the 16-byte grid)."""
    flat = torch.as_tensor(np.ascontiguousarray(a)).reshape(-1)
    base = torch.empty(flat.numel() + shift, dtype=torch.int32, device=DEV)
    view = base[shift:].view(a.shape)
    view.copy_(flat.view(a.shape).to(DEV))
    return view


@pytest.mark.parametrize("seed", range(40))
def test_converter_fuzz(seed) -> None:
    rng = np.random.default_rng(90000 + seed)
    for trial in range(5):
        req, table, tokens, geometry = _draw(rng)
        shift = int(rng.choice([0, 0, 1, 2, 3]))
        batch, width = tokens.shape
        want_out, want_counts = oracle.localize(req, table, tokens, threads=4, **geometry)
        d_req, d_table, d_tokens = _dev(req, shift), _dev(table, shift), _dev(tokens, shift)
        out = _dev(np.full((batch, width), 0x5A5A5A5A, dtype=np.int32), shift)
        counts = _dev(np.full((batch,), 0x5A5A5A5A, dtype=np.int32), shift)
        localize_rowwise(d_req, d_table, d_tokens, out, counts, **geometry)
        torch.cuda.synchronize()
        ctx = (seed, trial, batch, width, geometry, shift)
        assert np.array_equal(out.cpu().numpy(), want_out), ctx
        assert np.array_equal(counts.cpu().numpy(), want_counts), ctx

        tile = int(rng.choice(SUPPORTED_TILE_SIZES))
        ws = {name: torch.empty(shape, dtype=torch.int32, device=DEV)
              for name, shape in workspace_shapes(batch, width, tile_size=tile).items()}
        out_h = torch.full((batch, width), 0x5A5A5A5A, dtype=torch.int32, device=DEV)
        counts_h = torch.full((batch,), 0x5A5A5A5A, dtype=torch.int32, device=DEV)
        localize_hierarchical(d_req, d_table, d_tokens, out_h, counts_h, ws["mapped"], ws["local_positions"],
                              ws["tile_counts"], ws["tile_offsets"], tile_size=tile, **geometry)
        torch.cuda.synchronize()
        assert np.array_equal(out_h.cpu().numpy(), want_out), ctx + (tile,)
        assert np.array_equal(counts_h.cpu().numpy(), want_counts), ctx + (tile,)
        # the reference publishes the tile workspace in every mode
        want_tc, want_to = oracle.tiles(req, table, tokens, tile_size=tile,
                                        **{k: v for k, v in geometry.items() if k != "compact_valid_to_front"})
        assert np.array_equal(ws["tile_counts"].cpu().numpy(), want_tc), ctx + (tile,)
        assert np.array_equal(ws["tile_offsets"].cpu().numpy(), want_to), ctx + (tile,)


KINDS = ("normal", "ties", "equal", "special", "sorted", "reversed")


def _scores(rng, kind, shape):
    if kind == "normal":
        return rng.standard_normal(shape).astype(np.float32)
    if kind == "ties":
        return rng.integers(-2, 3, size=shape).astype(np.float32)
    if kind == "equal":
        return np.full(shape, -1.5, dtype=np.float32)
    if kind == "special":
        pool = np.array([np.inf, -np.inf, 0.0, -0.0, np.nan, 1e-45, -1e-45, 7.0], dtype=np.float32)
        return pool[rng.integers(0, len(pool), size=shape)]
    ramp = np.broadcast_to(np.arange(shape[1], dtype=np.float32), shape).copy()
    return ramp if kind == "sorted" else -ramp  # the top scores at one end of the row


@pytest.mark.parametrize("seed", range(12))
def test_topk_fuzz(seed) -> None:
    rng = np.random.default_rng(91000 + seed)
    for trial in range(3):
        batch = int(rng.integers(1, 40))
        width = int(rng.choice([1, 100, 2048, 3000, 20000, 65536, 70001]))
        top_k = int(min(16384, rng.choice([1, 7, 64, 512, 2048, 4096])))
        kind = str(rng.choice(KINDS))
        logits = _scores(rng, kind, (batch, width))
        lens = rng.integers(-3, width + 4, size=batch).astype(np.int32)
        rows, twidth = int(rng.integers(1, 8)), int(rng.integers(1, 2000))
        table = rng.integers(-5, 1 << 20, size=(rows, twidth)).astype(np.int32)
        req = rng.integers(0, rows, size=batch).astype(np.int32)
        dcp = int(rng.integers(1, 9))
        il = int(rng.choice([1, 1, 2]))
        geometry = dict(block_size=il * int(rng.integers(1, 65)), dcp_size=dcp, dcp_rank=int(rng.integers(0, dcp)),
                        dcp_interleave=il, compact_valid_to_front=bool(rng.random() < 0.8))
        out = torch.empty((batch, top_k), dtype=torch.int32, device=DEV)
        counts = torch.empty(batch, dtype=torch.int32, device=DEV)
        pos = torch.empty((batch, top_k), dtype=torch.int32, device=DEV)
        threads = int(rng.choice([0, 512, 1024]))
        topk_localize(torch.as_tensor(logits).to(DEV), torch.as_tensor(lens).to(DEV), torch.as_tensor(req).to(DEV),
                      torch.as_tensor(table).to(DEV), out, counts, positions=pos, cta_threads=threads, **geometry)
        torch.cuda.synchronize()
        want_pos, want_out, want_counts = oracle_topk(logits, lens, req, table, top_k=top_k, threads=4, **geometry)
        ctx = (seed, trial, batch, width, top_k, kind, geometry, threads)
        assert np.array_equal(pos.cpu().numpy(), want_pos), ctx
        assert np.array_equal(out.cpu().numpy(), want_out), ctx
        assert np.array_equal(counts.cpu().numpy(), want_counts), ctx
