"""Caller-owned workspace sizing for :func:`localize_hierarchical`.

The hierarchical launcher takes its scratch from the caller so that every
address is fixed before CUDA-graph capture. This module only computes shapes:
it allocates nothing and imports no GPU library.

Interface of silkern/workspace.py:22-53 (``workspace_shapes``), with the tile
geometry of this implementation: tiles of 64 to 1024 columns (powers of two)
and rows up to :data:`MAX_ROW_WIDTH` = 16384 columns.
"""

from __future__ import annotations

from numbers import Integral

from silkern_b200.contract import DEFAULT_TILE_SIZE, MAX_ROW_WIDTH, SUPPORTED_TILE_SIZES
from silkern_b200.errors import LocalizationError


def workspace_shapes(
    batch: int,
    width: int,
    *,
    tile_size: int = DEFAULT_TILE_SIZE,
) -> dict[str, tuple[int, ...]]:
    """Exact int32 workspace shapes, as plain tuples, for one geometry.

    ``tile_counts`` and ``tile_offsets`` receive the per-tile valid counts and
    their exclusive row prefix; ``mapped`` and ``local_positions`` are kept
    for interface compatibility and are not touched by the kernels.
    """
    if any(
        not isinstance(value, Integral) or isinstance(value, bool)
        for value in (batch, width, tile_size)
    ):
        raise LocalizationError("batch, width, and tile_size must be integers")
    if batch < 1 or width < 1:
        raise LocalizationError("batch and width must be positive")
    if width > MAX_ROW_WIDTH:
        raise LocalizationError(
            f"exact row width exceeds the current {MAX_ROW_WIDTH}-element limit"
        )
    if tile_size not in SUPPORTED_TILE_SIZES:
        supported = ", ".join(str(value) for value in SUPPORTED_TILE_SIZES)
        raise LocalizationError(f"tile_size must be one of {supported}")
    tiles = (width + tile_size - 1) // tile_size
    return {
        "mapped": (batch, width),
        "local_positions": (batch, width),
        "tile_counts": (batch, tiles),
        "tile_offsets": (batch, tiles),
    }
