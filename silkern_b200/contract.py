"""The localization contract: geometry validation and its normative Python form.

Pure Python with no GPU dependency, importable anywhere. The CUDA kernels in
``silkern_b200/csrc`` must reproduce :func:`localize_reference` element for
element, and :func:`silkern_b200.conformance` checks that on a device.

Per selection row the contract does, in order (silkern/contract.py:8-36):

1. request routing: ``req_ids[row]`` picks the block-table row;
2. ownership: ``owner = (token // interleave) % dcp_size``; other ranks'
   tokens are dropped, as are negative tokens;
3. deinterleave: ``local = (token // (dcp_size * interleave)) * interleave
   + token % interleave``;
4. paged translation: ``logical_block, offset = divmod(local, block_size)``;
   a block past the end of the table row drops the token, otherwise
   ``physical = table_row[logical_block] * block_size + offset`` (a negative
   table entry is used as it is);
5. stable front compaction: the surviving values keep their input order and
   fill the front of the row; the tail is ``-1``.

``dcp_size == 1`` skips step 5: every column keeps its own value (``-1`` when
dropped), as does ``compact_valid_to_front=False``. ``counts[row]`` is the
number of survivors in both modes.
"""

from __future__ import annotations

from collections.abc import Sequence
from numbers import Integral

from silkern_b200.errors import LocalizationError

#: Widest selection row accepted by both GPU entry points and by
#: :func:`silkern_b200.workspace_shapes`.
MAX_ROW_WIDTH = 16384
DEFAULT_TILE_SIZE = 128
SUPPORTED_TILE_SIZES = (64, 128, 256, 512, 1024)


def _is_int(value: object) -> bool:
    return isinstance(value, Integral) and not isinstance(value, bool)


def _validate_dcp_config(dcp_size: int, dcp_rank: int, dcp_interleave: int) -> None:
    """silkern/contract.py:50-59."""
    if not all(_is_int(v) for v in (dcp_size, dcp_rank, dcp_interleave)):
        raise LocalizationError("DCP size, rank, and interleave must be integers")
    if dcp_size < 1 or not 0 <= dcp_rank < dcp_size:
        raise LocalizationError("invalid dcp configuration")
    if dcp_interleave < 1:
        raise LocalizationError("dcp_interleave must be positive")


def _validate_compact_flag(compact_valid_to_front: bool) -> None:
    """silkern/contract.py:62-64."""
    if not isinstance(compact_valid_to_front, bool):
        raise LocalizationError("compact_valid_to_front must be a bool")


def _validate_block_size(block_size: int, dcp_interleave: int) -> None:
    """silkern/contract.py:105-110."""
    if not _is_int(block_size):
        raise LocalizationError("block_size must be an integer")
    if block_size < 1:
        raise LocalizationError("block_size must be positive")
    if block_size % dcp_interleave:
        raise LocalizationError("block_size must be divisible by dcp_interleave")


def localize_reference(
    req_ids: Sequence[int],
    block_table: Sequence[Sequence[int]],
    rows: Sequence[Sequence[int]],
    *,
    block_size: int,
    dcp_size: int,
    dcp_rank: int,
    dcp_interleave: int = 1,
    compact_valid_to_front: bool = True,
) -> tuple[list[list[int]], list[int]]:
    """The contract as a plain per-element loop; the normative definition.

    Same signature, errors and results as silkern/contract.py:67-158. Values
    are Python integers, so nothing wraps; the GPU kernels compute in int32
    lanes and agree whenever ``table_entry * block_size + offset`` fits in
    int32.
    """
    _validate_dcp_config(dcp_size, dcp_rank, dcp_interleave)
    _validate_compact_flag(compact_valid_to_front)
    _validate_block_size(block_size, dcp_interleave)
    if len(req_ids) != len(rows):
        raise LocalizationError("req_ids must contain one request id per row")
    if len(block_table) == 0:
        raise LocalizationError("block_table must contain at least one request row")
    if len(rows) == 0:
        raise LocalizationError("rows must contain at least one nonempty row")
    table_width = len(block_table[0])
    if table_width == 0 or any(len(entry) != table_width for entry in block_table):
        raise LocalizationError("block_table must be nonempty and rectangular")
    width = len(rows[0])
    if width == 0 or any(len(row) != width for row in rows):
        raise LocalizationError("rows must be nonempty and rectangular")

    group = dcp_size * dcp_interleave
    compact = compact_valid_to_front and dcp_size > 1
    out_rows: list[list[int]] = []
    counts: list[int] = []
    for index, row in enumerate(rows):
        request = int(req_ids[index])
        if request < 0 or request >= len(block_table):
            raise LocalizationError(f"request id {request} is outside block_table")
        entries = block_table[request]
        in_place: list[int] = []
        kept: list[int] = []
        for raw in row:
            token = int(raw)
            value = -1
            if token >= 0 and (token // dcp_interleave) % dcp_size == dcp_rank:
                local = (token // group) * dcp_interleave + token % dcp_interleave
                logical_block, offset = divmod(local, block_size)
                if logical_block < table_width:
                    value = int(entries[logical_block]) * block_size + offset
                    kept.append(value)
            in_place.append(value)
        counts.append(len(kept))
        out_rows.append(kept + [-1] * (width - len(kept)) if compact else in_place)
    return out_rows, counts
