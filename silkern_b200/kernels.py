"""Allocation-free launchers for the sm_100a localization kernels.

Both launchers keep the signatures, validation order and error messages of
the reference launchers (silkern/kernels.py:318-434 and :436-633), then call
the C ABI of ``libsilkern_b200.so`` on the caller's current CUDA stream.
Nothing is allocated and nothing synchronises, so a call can be captured in a
CUDA graph and replayed at fixed addresses.

``localize_rowwise``
    One launch; each row is scanned by one CTA, or by a thread-block cluster
    when rows are long and few.
``localize_hierarchical``
    One launch; each row is split into tiles, the CTAs of a row form a
    cluster, compose their tile prefixes deterministically and publish the
    per-tile counts and offsets into the caller's ``tile_counts`` and
    ``tile_offsets`` workspace.

``torch`` is imported inside the launchers, so ``import silkern_b200`` works on
a machine without it.
"""

from __future__ import annotations

import contextlib
import sys
from numbers import Integral

from silkern_b200 import _native
from silkern_b200.contract import (
    DEFAULT_TILE_SIZE,
    MAX_ROW_WIDTH,
    _validate_compact_flag,
    _validate_dcp_config,
)
from silkern_b200.errors import LocalizationError
from silkern_b200.workspace import workspace_shapes


def _is_int(value: object) -> bool:
    return isinstance(value, Integral) and not isinstance(value, bool)


def _check_buffers(torch, tensors, prefix: str, contiguous_message: str) -> None:
    if any(not isinstance(t, torch.Tensor) for t in tensors):
        raise LocalizationError(f"all {prefix} buffers must be torch tensors")
    if any(not t.is_cuda for t in tensors):
        raise LocalizationError(f"all {prefix} buffers must be CUDA tensors")
    device = tensors[2].device
    if any(t.device != device for t in tensors):
        raise LocalizationError(f"all {prefix} buffers must be on the same device")
    if any(t.dtype != torch.int32 for t in tensors):
        raise LocalizationError(f"all {prefix} buffers must use int32")
    if any(not t.is_contiguous() for t in tensors):
        raise LocalizationError(contiguous_message)


def _check_geometry(req_ids, block_table, tokens, out, counts) -> tuple[int, int]:
    if tokens.ndim != 2 or out.shape != tokens.shape:
        raise LocalizationError("tokens and out must have the same 2D shape")
    if block_table.ndim != 2:
        raise LocalizationError("block_table must be 2D")
    batch, width = tokens.shape
    if req_ids.shape != (batch,) or counts.shape != (batch,):
        raise LocalizationError("req_ids and counts must contain one element per row")
    if batch < 1 or width < 1 or block_table.shape[0] < 1 or block_table.shape[1] < 1:
        raise LocalizationError("batch, width, and both block-table dimensions must be positive")
    return int(batch), int(width)


def _check_scalars(block_size, dcp_size, dcp_rank, dcp_interleave, compact, num_warps) -> None:
    _validate_dcp_config(dcp_size, dcp_rank, dcp_interleave)
    _validate_compact_flag(compact)
    if not _is_int(block_size) or block_size < 1 or block_size % dcp_interleave:
        raise LocalizationError("block_size must be a positive integer divisible by dcp_interleave")
    if not _is_int(num_warps) or num_warps not in (4, 8):
        raise LocalizationError("num_warps must be 4 or 8")


def _check_status(torch, status, device):
    if status is None:
        return None
    if (
        not isinstance(status, torch.Tensor)
        or not status.is_cuda
        or status.device != device
        or status.dtype != torch.int32
        or status.numel() < 1
    ):
        raise LocalizationError("status must be an int32 CUDA tensor on the buffers' device")
    return status.data_ptr()


def _ensure_ops() -> None:
    """Register the torch.library ops on the first eager launch, so a later
    torch.compile of the caller finds them."""
    from silkern_b200 import ops

    if not ops.registered():
        ops.register()


def _device_scope(torch, device):
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _compiling(torch) -> bool:
    """True while torch.compile traces the caller."""
    compiler = getattr(torch, "compiler", None)
    return bool(compiler is not None and compiler.is_compiling())


def _traced_op(torch, name: str):
    from silkern_b200 import ops

    if not ops.registered():
        raise LocalizationError(
            "silkern_b200 ops are not registered: call silkern_b200.ops.register() (or launch once "
            "eagerly) before compiling"
        )
    return getattr(torch.ops.silkern_b200, name)


def localize_rowwise(
    req_ids,
    block_table,
    tokens,
    out,
    counts,
    *,
    block_size: int,
    dcp_size: int,
    dcp_rank: int,
    dcp_interleave: int = 1,
    compact_valid_to_front: bool = True,
    num_warps: int = 8,
    status=None,
) -> None:
    """Row-wise stable localization: one launch over the whole batch.

    Every buffer is a caller-owned contiguous int32 CUDA tensor; ``out`` is
    shaped like ``tokens`` and ``counts`` has one element per row; outputs
    must not share storage with inputs. ``num_warps`` is validated for
    interface compatibility (4 or 8); the launch geometry is chosen by the
    library. ``status`` (optional, one int32 element) receives
    ``SILKERN_STATUS_BAD_REQUEST`` if a request id is outside the block table;
    such a row is emitted as all ``-1`` with count 0. A row split over a
    thread-block cluster (rows wider than 8192 columns, few rows) whose count
    exchange runs out of its wait bound ORs in
    ``SILKERN_STATUS_EXCHANGE_TIMEOUT`` (4); the CTAs that gave up store
    nothing for it.

    Under ``torch.compile`` the call is the custom op
    ``torch.ops.silkern_b200.localize_rowwise`` (one opaque node, checked and
    launched when the compiled code runs); otherwise the C ABI is called
    directly.

    Raises :class:`LocalizationError` on any unsupported geometry or binding.
    """
    import torch

    if _compiling(torch):
        _traced_op(torch, "localize_rowwise")(
            req_ids, block_table, tokens, out, counts, block_size, dcp_size, dcp_rank, dcp_interleave,
            compact_valid_to_front, num_warps, status)
        return
    _ensure_ops()
    _rowwise_eager(req_ids, block_table, tokens, out, counts, block_size=block_size, dcp_size=dcp_size,
                   dcp_rank=dcp_rank, dcp_interleave=dcp_interleave,
                   compact_valid_to_front=compact_valid_to_front, num_warps=num_warps, status=status)


def _rowwise_eager(
    req_ids,
    block_table,
    tokens,
    out,
    counts,
    *,
    block_size: int,
    dcp_size: int,
    dcp_rank: int,
    dcp_interleave: int = 1,
    compact_valid_to_front: bool = True,
    num_warps: int = 8,
    status=None,
) -> None:
    """The reference's checks for localize_rowwise (kernels.py:351-409), then
    one C ABI call on the current stream."""
    import torch

    tensors = (req_ids, block_table, tokens, out, counts)
    _check_buffers(torch, tensors, "localization", "stable localization requires contiguous tensors")
    batch, width = _check_geometry(req_ids, block_table, tokens, out, counts)
    if width > MAX_ROW_WIDTH:
        raise LocalizationError(
            f"exact row width exceeds the current {MAX_ROW_WIDTH}-element limit"
        )
    inputs = {
        req_ids.untyped_storage().data_ptr(),
        block_table.untyped_storage().data_ptr(),
        tokens.untyped_storage().data_ptr(),
    }
    out_storage = out.untyped_storage().data_ptr()
    if out_storage in inputs:
        raise LocalizationError("out must not share storage with an input")
    if counts.untyped_storage().data_ptr() in inputs | {out_storage}:
        raise LocalizationError("counts must not share storage with another buffer")
    _check_scalars(block_size, dcp_size, dcp_rank, dcp_interleave, compact_valid_to_front, num_warps)
    status_ptr = _check_status(torch, status, tokens.device)

    lib = _native.load()
    with _device_scope(torch, tokens.device):
        stream = torch.cuda.current_stream(tokens.device).cuda_stream
        code = lib.silkern_localize_rowwise_v1(
            req_ids.data_ptr(),
            block_table.data_ptr(),
            block_table.shape[0],
            block_table.shape[1],
            tokens.data_ptr(),
            out.data_ptr(),
            counts.data_ptr(),
            batch,
            width,
            int(block_size),
            int(dcp_size),
            int(dcp_rank),
            int(dcp_interleave),
            1 if compact_valid_to_front else 0,
            status_ptr,
            stream,
        )
    _native.check(code, "localize_rowwise")


def localize_hierarchical(
    req_ids,
    block_table,
    tokens,
    out,
    counts,
    mapped_workspace,
    local_positions_workspace,
    tile_counts_workspace,
    tile_offsets_workspace,
    *,
    block_size: int,
    dcp_size: int,
    dcp_rank: int,
    dcp_interleave: int = 1,
    compact_valid_to_front: bool = True,
    tile_size: int = DEFAULT_TILE_SIZE,
    num_warps: int = 4,
    status=None,
) -> None:
    """Hierarchical stable localization for wide rows, in one launch.

    The four workspace tensors must have the shapes
    :func:`silkern_b200.workspace_shapes` returns; all nine buffers are
    contiguous int32 CUDA tensors on one device with distinct storage. After
    the call ``tile_counts_workspace[r, k]`` holds the number of valid
    elements in tile ``k`` of row ``r`` and ``tile_offsets_workspace[r, k]``
    their exclusive prefix; ``mapped_workspace`` and
    ``local_positions_workspace`` are validated but not touched.

    Under ``torch.compile`` the call is the custom op
    ``torch.ops.silkern_b200.localize_hierarchical``; otherwise the C ABI is
    called directly.
    """
    import torch

    if _compiling(torch):
        _traced_op(torch, "localize_hierarchical")(
            req_ids, block_table, tokens, out, counts, mapped_workspace, local_positions_workspace,
            tile_counts_workspace, tile_offsets_workspace, block_size, dcp_size, dcp_rank, dcp_interleave,
            compact_valid_to_front, tile_size, num_warps, status)
        return
    _ensure_ops()
    _hierarchical_eager(req_ids, block_table, tokens, out, counts, mapped_workspace,
                        local_positions_workspace, tile_counts_workspace, tile_offsets_workspace,
                        block_size=block_size, dcp_size=dcp_size, dcp_rank=dcp_rank,
                        dcp_interleave=dcp_interleave, compact_valid_to_front=compact_valid_to_front,
                        tile_size=tile_size, num_warps=num_warps, status=status)


def _hierarchical_eager(
    req_ids,
    block_table,
    tokens,
    out,
    counts,
    mapped_workspace,
    local_positions_workspace,
    tile_counts_workspace,
    tile_offsets_workspace,
    *,
    block_size: int,
    dcp_size: int,
    dcp_rank: int,
    dcp_interleave: int = 1,
    compact_valid_to_front: bool = True,
    tile_size: int = DEFAULT_TILE_SIZE,
    num_warps: int = 4,
    status=None,
) -> None:
    """The reference's checks for localize_hierarchical (kernels.py:467-558),
    then one C ABI call on the current stream."""
    import torch

    tensors = (
        req_ids,
        block_table,
        tokens,
        out,
        counts,
        mapped_workspace,
        local_positions_workspace,
        tile_counts_workspace,
        tile_offsets_workspace,
    )
    _check_buffers(
        torch,
        tensors,
        "hierarchical localization",
        "hierarchical stable localization requires contiguous tensors",
    )
    batch, width = _check_geometry(req_ids, block_table, tokens, out, counts)
    shapes = workspace_shapes(batch, width, tile_size=tile_size)
    observed = {
        "mapped": tuple(mapped_workspace.shape),
        "local_positions": tuple(local_positions_workspace.shape),
        "tile_counts": tuple(tile_counts_workspace.shape),
        "tile_offsets": tuple(tile_offsets_workspace.shape),
    }
    for name, expected in shapes.items():
        if observed[name] != expected:
            raise LocalizationError(
                f"{name} workspace shape mismatch: expected {expected}, observed {observed[name]}"
            )
    storages = [t.untyped_storage().data_ptr() for t in tensors]
    if len(set(storages)) != len(storages):
        raise LocalizationError("hierarchical localization buffers must use distinct storage")
    _check_scalars(block_size, dcp_size, dcp_rank, dcp_interleave, compact_valid_to_front, num_warps)
    status_ptr = _check_status(torch, status, tokens.device)

    lib = _native.load()
    with _device_scope(torch, tokens.device):
        stream = torch.cuda.current_stream(tokens.device).cuda_stream
        code = lib.silkern_localize_hierarchical_v1(
            req_ids.data_ptr(),
            block_table.data_ptr(),
            block_table.shape[0],
            block_table.shape[1],
            tokens.data_ptr(),
            out.data_ptr(),
            counts.data_ptr(),
            mapped_workspace.data_ptr(),
            local_positions_workspace.data_ptr(),
            tile_counts_workspace.data_ptr(),
            tile_offsets_workspace.data_ptr(),
            batch,
            width,
            int(block_size),
            int(dcp_size),
            int(dcp_rank),
            int(dcp_interleave),
            1 if compact_valid_to_front else 0,
            int(tile_size),
            status_ptr,
            stream,
        )
    _native.check(code, "localize_hierarchical")


def localize_explicit(
    req_ids,
    block_table,
    tokens,
    out,
    counts,
    *,
    block_size: int,
    dcp_size: int,
    dcp_rank: int,
    dcp_interleave: int = 1,
    compact_valid_to_front: bool = True,
    cluster_size: int = 1,
    stage_table: int = -1,
    prefetch_table: int = -1,
    chunks_per_thread: int = 0,
    tile_size: int = 0,
    tile_counts=None,
    tile_offsets=None,
    status=None,
) -> None:
    """Localization with an explicit launch geometry (conformance sweeps, tuning).

    Same outputs as the two public launchers; ``cluster_size`` CTAs per row,
    ``stage_table``/``prefetch_table`` 1, 0 or -1 (library choice),
    ``chunks_per_thread`` 1, 2, 4, 8 or 0 (library choice): each thread maps
    a run of 4 x chunks_per_thread consecutive columns. With
    ``tile_size`` > 0 the hierarchical tile workspace is published. Buffers
    are checked by the C ABI only.
    """
    import torch

    lib = _native.load()
    ptr = (lambda t: None if t is None else t.data_ptr())
    with _device_scope(torch, tokens.device):
        stream = torch.cuda.current_stream(tokens.device).cuda_stream
        code = lib.silkern_localize_explicit_v1(
            req_ids.data_ptr(),
            block_table.data_ptr(),
            block_table.shape[0],
            block_table.shape[1],
            tokens.data_ptr(),
            out.data_ptr(),
            counts.data_ptr(),
            ptr(tile_counts),
            ptr(tile_offsets),
            tokens.shape[0],
            tokens.shape[1],
            int(block_size),
            int(dcp_size),
            int(dcp_rank),
            int(dcp_interleave),
            1 if compact_valid_to_front else 0,
            int(tile_size),
            int(cluster_size),
            int(stage_table),
            int(prefetch_table),
            int(chunks_per_thread),
            ptr(status),
            stream,
        )
    _native.check(code, "localize_explicit")


def count_mismatches(a, b, mismatches) -> None:
    """Add the number of differing int32 elements of ``a`` and ``b`` to ``mismatches[0]``.

    Device-side check used by the replay gate; capturable in a CUDA graph.
    """
    import torch

    if a.shape != b.shape or a.dtype != torch.int32 or b.dtype != torch.int32:
        raise LocalizationError("count_mismatches needs two int32 tensors of one shape")
    lib = _native.load()
    with _device_scope(torch, a.device):
        stream = torch.cuda.current_stream(a.device).cuda_stream
        code = lib.silkern_count_mismatches_v1(
            a.data_ptr(), b.data_ptr(), a.numel(), mismatches.data_ptr(), stream
        )
    _native.check(code, "count_mismatches")


def count_segment_mismatches(a, b, counters) -> None:
    """``counters[s] +=`` the number of differing elements in segment ``s``,
    where segment ``s`` is ``a[s]`` against ``b[s]`` (int32 tensors of one
    shape, first dimension = segments). One launch; capturable in a CUDA graph.
    """
    import torch

    if a.shape != b.shape or a.dtype != torch.int32 or b.dtype != torch.int32 or a.dim() < 1:
        raise LocalizationError("count_segment_mismatches needs two int32 tensors of one shape")
    if not (a.is_contiguous() and b.is_contiguous()) or counters.numel() < a.shape[0]:
        raise LocalizationError("count_segment_mismatches needs contiguous inputs and one counter per segment")
    lib = _native.load()
    segments = a.shape[0]
    with _device_scope(torch, a.device):
        stream = torch.cuda.current_stream(a.device).cuda_stream
        code = lib.silkern_count_segment_mismatches_v1(
            a.data_ptr(), b.data_ptr(), segments, a.numel() // max(segments, 1), counters.data_ptr(), stream
        )
    _native.check(code, "count_segment_mismatches")


def copy_floor(src, dst, *, run: int = 8, threads: int = 256, ctas_per_sm: int = 0) -> None:
    """``dst.copy_(src)`` (int32, contiguous, same number of elements) with the
    converter's data movement and launch mode and none of its work: the floor
    a converter call over the same bytes is measured against. CTAs of
    ``threads`` threads, each thread a run of ``run`` (8 or 16) elements; with
    ``ctas_per_sm`` (1-8) at most that many CTAs share an SM (0: no limit).
    Capturable in a CUDA graph.
    """
    import torch

    if src.dtype != torch.int32 or dst.dtype != torch.int32 or src.numel() != dst.numel():
        raise LocalizationError("copy_floor needs two int32 tensors with the same number of elements")
    if not (src.is_contiguous() and dst.is_contiguous()):
        raise LocalizationError("copy_floor needs contiguous tensors")
    lib = _native.load()
    with _device_scope(torch, src.device):
        stream = torch.cuda.current_stream(src.device).cuda_stream
        code = lib.silkern_copy_floor_v1(src.data_ptr(), dst.data_ptr(), src.numel(), int(run), int(threads),
                                         int(ctas_per_sm), stream)
    _native.check(code, "copy_floor")


if "torch" in sys.modules:  # torch is already loaded: define the ops now (see silkern_b200.ops)
    from silkern_b200 import ops as _ops

    _ops.register()

