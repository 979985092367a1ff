"""CPU oracle of the fused top-k + localization -- TEST INFRASTRUCTURE ONLY.

Selection (numpy): row r scores positions [0, L), L = seq_lens[r] clamped to
[0, width]; every position when L <= top_k, otherwise the top_k positions
with the largest order keys (float bit patterns ordered totally: negative
patterns with every bit flipped, non-negative ones with the sign bit
flipped), ties to the lower position. The selected positions in ascending
order, padded with -1 to top_k, form the selection row, which is localized by
the C oracle of the converter (``oracle.localize``, a restatement of
silkern/contract.py:67-158). Only ``tests/`` and ``bench.py`` use this module.
"""

from __future__ import annotations

import numpy as np

from oracle import localize


def order_keys(values) -> np.ndarray:
    """uint32 keys whose unsigned order is the total order of the float32 bit patterns."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    flip = np.where(bits >> np.uint32(31), np.uint32(0xFFFFFFFF), np.uint32(0x80000000))
    return bits ^ flip


def select_positions(logits, seq_lens, top_k: int) -> np.ndarray:
    """(batch, top_k) int32 selection rows: ascending selected positions, -1 padded."""
    logits = np.asarray(logits, dtype=np.float32)
    batch, width = logits.shape
    rows = np.full((batch, top_k), -1, dtype=np.int32)
    for b in range(batch):
        length = int(min(max(int(seq_lens[b]), 0), width))
        if length <= top_k:
            rows[b, :length] = np.arange(length, dtype=np.int32)
            continue
        # unique 64-bit sort keys: descending order key, then ascending position
        inv = (~order_keys(logits[b, :length])).astype(np.uint64)
        combined = (inv << np.uint64(32)) | np.arange(length, dtype=np.uint64)
        best = np.argpartition(combined, top_k - 1)[:top_k]
        rows[b] = np.sort(best).astype(np.int32)
    return rows


def topk_localize(logits, seq_lens, req_ids, block_table, *, top_k: int, block_size: int,
                  dcp_size: int, dcp_rank: int, dcp_interleave: int = 1,
                  compact_valid_to_front: bool = True, threads: int = 1):
    """Return ``(positions, out, counts)`` for the fused operation."""
    rows = select_positions(logits, seq_lens, top_k)
    out, counts = localize(req_ids, block_table, rows, block_size=block_size, dcp_size=dcp_size,
                           dcp_rank=dcp_rank, dcp_interleave=dcp_interleave,
                           compact_valid_to_front=compact_valid_to_front, threads=threads)
    return rows, out, counts
