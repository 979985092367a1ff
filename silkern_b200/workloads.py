"""Seeded synthetic selection batches with the shapes of the benchmark configs.

Each generator returns a :class:`Case` of numpy int32 arrays plus its
geometry. Positions are unique per row, drawn uniformly without replacement
from the request's context and emitted in random (selector) order; block
tables are disjoint slices of one random permutation of a physical block
pool. ``numpy.random.default_rng(seed)`` drives everything, so a seed names a
case exactly.

=========  =======================================================================
config     shape
=========  =======================================================================
1          B=4, W=2048, seq 8192, bs 64, dcp 2 (ranks 0 and 1), table (4, 64)
           from a 4096-block pool; the CPU-runnable oracle case
2          B=64, W=2048, seq 32768, bs 64, dcp 2 rank 0, table (64, 256), pool 16384
3          B=256, W=2048, seq ~ U[1024, 65536] per request, rows shorter than W
           padded with -1, bs 64, dcp 4, table (256, 256), pool 65536 (headline)
4          B=32, W=16384, seq 131072, hierarchical tile 1024, bs 64, dcp 8,
           table (32, 256), pool 8192
5          one layer of a 48-layer decode step: B=128, W=2048, seq 32768, bs 64,
           dcp 8, table (128, 64); layer l uses seed + l
=========  =======================================================================
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Case:
    name: str
    req_ids: np.ndarray  # (B,) int32
    block_table: np.ndarray  # (R, Wt) int32
    tokens: np.ndarray  # (B, W) int32
    block_size: int
    dcp_size: int
    dcp_rank: int
    dcp_interleave: int = 1
    arm: str = "row_stable"
    tile_size: int = 128

    @property
    def batch(self) -> int:
        return int(self.tokens.shape[0])

    @property
    def width(self) -> int:
        return int(self.tokens.shape[1])

    def geometry(self) -> dict[str, int]:
        return {
            "block_size": self.block_size,
            "dcp_size": self.dcp_size,
            "dcp_rank": self.dcp_rank,
            "dcp_interleave": self.dcp_interleave,
        }

    def algorithmic_bytes(self) -> int:
        """Bytes one compacting call must move: tokens in, out, req_ids, counts,
        and the block-table rows of the routed requests (upper bound: each
        distinct routed row read once)."""
        batch, width = self.tokens.shape
        routed = len(np.unique(self.req_ids[(self.req_ids >= 0) & (self.req_ids < self.block_table.shape[0])]))
        return 8 * batch * width + 8 * batch + 4 * routed * int(self.block_table.shape[1])


def _rows_unique(rng: np.random.Generator, batch: int, width: int, seq_lens) -> np.ndarray:
    tokens = np.full((batch, width), -1, dtype=np.int32)
    for row in range(batch):
        seq = int(seq_lens[row])
        take = min(width, seq)
        tokens[row, :take] = rng.choice(seq, size=take, replace=False).astype(np.int32)
    return tokens


def _table(rng: np.random.Generator, rows: int, width: int, pool: int) -> np.ndarray:
    perm = rng.permutation(pool).astype(np.int32)
    return np.ascontiguousarray(perm[: rows * width].reshape(rows, width))


def config_case(config: int, *, seed: int = 0, dcp_rank: int = 0, batch: int | None = None) -> Case:
    """The synthetic case of benchmark config ``config`` (1-5).

    ``batch`` keeps the first rows only (same distribution, smaller case);
    the block table keeps its full shape.
    """
    rng = np.random.default_rng(seed)
    if config == 1:
        b, w, seq, pool, tw = 4, 2048, 8192, 4096, 64
        table = _table(rng, b, tw, pool)
        tokens = _rows_unique(rng, b, w, [seq] * b)
        case = Case("config1", np.arange(b, dtype=np.int32), table, tokens, 64, 2, dcp_rank)
    elif config == 2:
        b, w, seq, pool, tw = 64, 2048, 32768, 16384, 256
        table = _table(rng, b, tw, pool)
        tokens = _rows_unique(rng, b, w, [seq] * b)
        case = Case("config2", np.arange(b, dtype=np.int32), table, tokens, 64, 2, dcp_rank)
    elif config == 3:
        b, w, pool, tw = 256, 2048, 65536, 256
        table = _table(rng, b, tw, pool)
        seq_lens = rng.integers(1024, 65536, size=b, endpoint=True)
        tokens = _rows_unique(rng, b, w, seq_lens)
        case = Case("config3", np.arange(b, dtype=np.int32), table, tokens, 64, 4, dcp_rank)
    elif config == 4:
        b, w, seq, pool, tw = 32, 16384, 131072, 8192, 256
        table = _table(rng, b, tw, pool)
        tokens = _rows_unique(rng, b, w, [seq] * b)
        case = Case("config4", np.arange(b, dtype=np.int32), table, tokens, 64, 8, dcp_rank,
                    arm="hierarchical_stable", tile_size=1024)
    elif config == 5:
        b, w, seq, pool, tw = 128, 2048, 32768, 8192, 64
        table = _table(rng, b, tw, pool)
        tokens = _rows_unique(rng, b, w, [seq] * b)
        case = Case("config5", np.arange(b, dtype=np.int32), table, tokens, 64, 8, dcp_rank)
    else:
        raise ValueError(f"unknown config {config}")
    if batch is not None:
        case.tokens = np.ascontiguousarray(case.tokens[:batch])
        case.req_ids = np.ascontiguousarray(case.req_ids[:batch])
    return case


def digest(out: np.ndarray, counts: np.ndarray) -> str:
    """sha256 of the little-endian int32 bytes of ``out`` then ``counts``."""
    import hashlib

    h = hashlib.sha256()
    h.update(np.ascontiguousarray(out, dtype="<i4").tobytes())
    h.update(np.ascontiguousarray(counts, dtype="<i4").tobytes())
    return h.hexdigest()


def input_digest(case: Case) -> str:
    """sha256 of req_ids, block_table and tokens (little-endian int32)."""
    import hashlib

    h = hashlib.sha256()
    for array in (case.req_ids, case.block_table, case.tokens):
        h.update(np.ascontiguousarray(array, dtype="<i4").tobytes())
    return h.hexdigest()
