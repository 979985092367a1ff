"""silkern_b200 -- deterministic sparse-index localization for context-parallel decode on B200.

A top-k selector returns global logical token positions; a decode
context-parallel (DCP) rank needs the physical KV slots it owns, compacted to
the front of each row in the selector's order, with an exact count. This
package does that with hand-written sm_100a CUDA kernels behind a C ABI
(``include/silkern_b200.h``), called from the same Python surface as the
reference silkern package:

    import silkern_b200 as silkern

    out, counts = silkern.localize_reference(req_ids, block_table, rows,
                                             block_size=64, dcp_size=2, dcp_rank=0)
    silkern.localize_rowwise(req, table, tokens, out, counts,
                             block_size=64, dcp_size=2, dcp_rank=0)
    report = silkern.conformance()

The GPU entry points allocate nothing and never synchronise, so a whole decode
step captures and replays as a CUDA graph. ``import silkern_b200`` needs
neither torch nor a GPU; the launchers load the CUDA library on first use and
raise :class:`LocalizationError` if it is missing.
"""

from __future__ import annotations

from silkern_b200.contract import (
    DEFAULT_TILE_SIZE,
    MAX_ROW_WIDTH,
    SUPPORTED_TILE_SIZES,
    localize_reference,
)
from silkern_b200.errors import LocalizationError
from silkern_b200.kernels import localize_hierarchical, localize_rowwise
from silkern_b200.topk import topk_localize
from silkern_b200.verify import (
    CellReport,
    ConformanceReport,
    ReplayGateReport,
    conformance,
    replay_gate,
)
from silkern_b200.workspace import workspace_shapes

__version__ = "0.1.0"

#: Name used by the reference's adapter test for the oracle.
exact_stable_compact_reference = localize_reference

__all__ = [
    "DEFAULT_TILE_SIZE",
    "MAX_ROW_WIDTH",
    "SUPPORTED_TILE_SIZES",
    "CellReport",
    "ConformanceReport",
    "LocalizationError",
    "ReplayGateReport",
    "conformance",
    "exact_stable_compact_reference",
    "localize_hierarchical",
    "localize_reference",
    "localize_rowwise",
    "topk_localize",
    "replay_gate",
    "workspace_shapes",
]
