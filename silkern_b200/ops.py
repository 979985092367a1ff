"""``torch.library`` custom ops over the C ABI.

    torch.ops.silkern_b200.localize_rowwise(req_ids, block_table, tokens, out, counts,
                                            block_size, dcp_size, dcp_rank, dcp_interleave,
                                            compact_valid_to_front, num_warps, status)
    torch.ops.silkern_b200.localize_hierarchical(req_ids, block_table, tokens, out, counts,
                                                 mapped, local_positions, tile_counts, tile_offsets,
                                                 block_size, dcp_size, dcp_rank, dcp_interleave,
                                                 compact_valid_to_front, tile_size, num_warps, status)

Each op declares the buffers the kernel writes as mutated (``out``, ``counts``,
the tile workspace and ``status``; the hierarchical op's ``mapped`` and
``local_positions`` are only read for their shapes) and has a fake
implementation, so ``torch.compile`` traces a call as one opaque node, with no
graph break, where the ctypes call of the eager launchers would break the
graph. At run time an op does exactly what the eager launcher does: the
reference's checks, then one C ABI call on the current stream.

The public launchers in :mod:`silkern_b200.kernels` route through these ops
while ``torch.compile`` traces them and call the C ABI directly otherwise: a
trip through the dispatcher costs tens of microseconds of host time per call,
which an eager caller would pay for nothing.

:func:`register` is idempotent. It runs when :mod:`silkern_b200.kernels` is
imported after torch, and on the first eager launch otherwise; a program that
compiles a call before either should call it first.
"""

# No ``from __future__ import annotations``: torch.library reads the
# annotations below as types to build the op schemas.
from typing import Optional

_REGISTERED = False


def registered() -> bool:
    return _REGISTERED


def register() -> None:
    """Define the ``silkern_b200`` ops (once per process)."""
    global _REGISTERED
    if _REGISTERED:
        return
    import torch

    from silkern_b200 import kernels

    @torch.library.custom_op("silkern_b200::localize_rowwise", mutates_args=("out", "counts", "status"))
    def localize_rowwise(
        req_ids: torch.Tensor,
        block_table: torch.Tensor,
        tokens: torch.Tensor,
        out: torch.Tensor,
        counts: torch.Tensor,
        block_size: int,
        dcp_size: int,
        dcp_rank: int,
        dcp_interleave: int,
        compact_valid_to_front: bool,
        num_warps: int,
        status: Optional[torch.Tensor],
    ) -> None:
        kernels._rowwise_eager(req_ids, block_table, tokens, out, counts, block_size=block_size,
                               dcp_size=dcp_size, dcp_rank=dcp_rank, dcp_interleave=dcp_interleave,
                               compact_valid_to_front=compact_valid_to_front, num_warps=num_warps,
                               status=status)

    @localize_rowwise.register_fake
    def _(req_ids, block_table, tokens, out, counts, block_size, dcp_size, dcp_rank, dcp_interleave,
          compact_valid_to_front, num_warps, status) -> None:
        return None

    @torch.library.custom_op(
        "silkern_b200::localize_hierarchical",
        mutates_args=("out", "counts", "tile_counts", "tile_offsets", "status"),
    )
    def localize_hierarchical(
        req_ids: torch.Tensor,
        block_table: torch.Tensor,
        tokens: torch.Tensor,
        out: torch.Tensor,
        counts: torch.Tensor,
        mapped: torch.Tensor,
        local_positions: torch.Tensor,
        tile_counts: torch.Tensor,
        tile_offsets: torch.Tensor,
        block_size: int,
        dcp_size: int,
        dcp_rank: int,
        dcp_interleave: int,
        compact_valid_to_front: bool,
        tile_size: int,
        num_warps: int,
        status: Optional[torch.Tensor],
    ) -> None:
        kernels._hierarchical_eager(req_ids, block_table, tokens, out, counts, mapped, local_positions,
                                    tile_counts, tile_offsets, block_size=block_size, dcp_size=dcp_size,
                                    dcp_rank=dcp_rank, dcp_interleave=dcp_interleave,
                                    compact_valid_to_front=compact_valid_to_front, tile_size=tile_size,
                                    num_warps=num_warps, status=status)

    @localize_hierarchical.register_fake
    def _(req_ids, block_table, tokens, out, counts, mapped, local_positions, tile_counts, tile_offsets,
          block_size, dcp_size, dcp_rank, dcp_interleave, compact_valid_to_front, tile_size, num_warps,
          status) -> None:
        return None

    _REGISTERED = True
