"""Alias of :mod:`silkern_b200.contract`."""

from silkern_b200.contract import (  # noqa: F401
    DEFAULT_TILE_SIZE,
    MAX_ROW_WIDTH,
    SUPPORTED_TILE_SIZES,
    _validate_compact_flag,
    _validate_dcp_config,
    localize_reference,
)
