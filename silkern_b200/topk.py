"""Fused indexer top-k + localization launcher (one sm_100a kernel).

A sparse decode step scores every context position of a request (the
indexer's logits), selects the ``top_k`` best, and localizes the selection
for this DCP rank. ``topk_localize`` does both in one launch, so the
(batch, top_k) selection never makes a round trip through HBM. Its
localization half is the converter's contract (silkern/contract.py:67-158)
applied to the selection row; the selection is defined here:

* row ``r`` scores positions ``[0, L)``, ``L = seq_lens[r]`` (clamped to
  ``[0, logits.shape[1]]``; out-of-range lengths are flagged in ``status``);
  columns at and beyond ``L`` are never read;
* ``L <= top_k``: every position is selected; otherwise the ``top_k``
  positions with the largest order keys (the float order extended to a total
  order on bit patterns: -NaN < -inf < ... < -0 < +0 < ... < +inf < +NaN),
  ties to the lower position;
* the selection row is the selected positions in ascending order, padded
  with -1 to ``top_k``; ``out``/``counts`` are that row localized exactly as
  :func:`silkern_b200.localize_rowwise` would localize it, and ``positions``
  (optional) receives the row itself.

Nothing is allocated and nothing synchronises: the call can be captured in a
CUDA graph.
"""

from __future__ import annotations

from silkern_b200 import _native
from silkern_b200.contract import MAX_ROW_WIDTH, _validate_compact_flag, _validate_dcp_config
from silkern_b200.errors import LocalizationError
from silkern_b200.kernels import _check_status, _device_scope, _is_int

#: Widest logits row the kernel accepts (SILKERN_TOPK_MAX_WIDTH).
MAX_LOGITS_WIDTH = 262144
#: Status bit (OR-ed into ``status``) besides SILKERN_STATUS_BAD_REQUEST (1):
#: a seq_len outside [0, logits width], clamped.
STATUS_BAD_LENGTH = 2


def topk_localize(
    logits,
    seq_lens,
    req_ids,
    block_table,
    out,
    counts,
    *,
    block_size: int,
    dcp_size: int,
    dcp_rank: int,
    dcp_interleave: int = 1,
    compact_valid_to_front: bool = True,
    positions=None,
    status=None,
    candidate_capacity: int = 0,
    stage_table: int = -1,
    cta_threads: int = 0,
) -> None:
    """Select the top ``out.shape[1]`` positions of every logits row and localize them.

    ``logits`` is float32 (batch, width) on a CUDA device with unit column
    stride (rows may be padded); ``seq_lens`` and ``req_ids`` are int32
    (batch,); ``block_table`` int32 (rows, table_width); ``out`` int32
    (batch, top_k); ``counts`` int32 (batch,); ``positions`` optional int32
    (batch, top_k). Outputs must not share storage with inputs or with each
    other. ``candidate_capacity`` (0 = library choice), ``stage_table``
    (-1 = library choice, 0 or 1) and ``cta_threads`` (0 = library choice,
    512 or 1024) pin internals for tests and tuning; a capacity of ``top_k``
    forces the whole-row selection path. Raises
    :class:`LocalizationError` before launch on any unsupported binding or
    geometry.
    """
    import torch

    ints = [seq_lens, req_ids, block_table, out, counts] + ([positions] if positions is not None else [])
    if not isinstance(logits, torch.Tensor) or any(not isinstance(t, torch.Tensor) for t in ints):
        raise LocalizationError("all top-k localization buffers must be torch tensors")
    if not logits.is_cuda or any(not t.is_cuda for t in ints):
        raise LocalizationError("all top-k localization buffers must be CUDA tensors")
    device = logits.device
    if any(t.device != device for t in ints):
        raise LocalizationError("all top-k localization buffers must be on the same device")
    if logits.dtype != torch.float32:
        raise LocalizationError("logits must be float32")
    if any(t.dtype != torch.int32 for t in ints):
        raise LocalizationError("seq_lens, req_ids, block_table and the outputs must use int32")
    if any(not t.is_contiguous() for t in ints):
        raise LocalizationError("top-k localization requires contiguous int32 tensors")
    if logits.ndim != 2 or logits.stride(1) != 1 or logits.stride(0) < logits.shape[1]:
        raise LocalizationError("logits must be 2D with unit column stride")
    batch, width = (int(d) for d in logits.shape)
    if out.ndim != 2 or out.shape[0] != batch:
        raise LocalizationError("out must be (batch, top_k)")
    top_k = int(out.shape[1])
    if positions is not None and tuple(positions.shape) != (batch, top_k):
        raise LocalizationError("positions must have the shape of out")
    if seq_lens.shape != (batch,) or req_ids.shape != (batch,) or counts.shape != (batch,):
        raise LocalizationError("seq_lens, req_ids and counts must contain one element per row")
    if block_table.ndim != 2 or block_table.shape[0] < 1 or block_table.shape[1] < 1:
        raise LocalizationError("block_table must be 2D and non-empty")
    if batch < 1 or width < 1 or top_k < 1:
        raise LocalizationError("batch, logits width and top_k must be positive")
    if top_k > MAX_ROW_WIDTH:
        raise LocalizationError(f"top_k exceeds the current {MAX_ROW_WIDTH}-element limit")
    if width > MAX_LOGITS_WIDTH:
        raise LocalizationError(f"logits width exceeds the current {MAX_LOGITS_WIDTH}-column limit")
    inputs = {t.untyped_storage().data_ptr() for t in (logits, seq_lens, req_ids, block_table)}
    outputs = [t.untyped_storage().data_ptr() for t in (out, counts, positions) if t is not None]
    if inputs & set(outputs) or len(set(outputs)) != len(outputs):
        raise LocalizationError("outputs must not share storage with inputs or with each other")
    _validate_dcp_config(dcp_size, dcp_rank, dcp_interleave)
    _validate_compact_flag(compact_valid_to_front)
    if not _is_int(block_size) or block_size < 1 or block_size % dcp_interleave:
        raise LocalizationError("block_size must be a positive integer divisible by dcp_interleave")
    if not _is_int(candidate_capacity) or candidate_capacity < 0:
        raise LocalizationError("candidate_capacity must be a non-negative integer")
    if not _is_int(stage_table) or stage_table not in (-1, 0, 1):
        raise LocalizationError("stage_table must be -1, 0 or 1")
    if not _is_int(cta_threads) or cta_threads not in (0, 512, 1024):
        raise LocalizationError("cta_threads must be 0, 512 or 1024")
    status_ptr = _check_status(torch, status, device)

    lib = _native.load()
    args = [
        logits.data_ptr(),
        logits.stride(0),
        width,
        seq_lens.data_ptr(),
        req_ids.data_ptr(),
        block_table.data_ptr(),
        block_table.shape[0],
        block_table.shape[1],
        None if positions is None else positions.data_ptr(),
        out.data_ptr(),
        counts.data_ptr(),
        batch,
        top_k,
        int(block_size),
        int(dcp_size),
        int(dcp_rank),
        int(dcp_interleave),
        1 if compact_valid_to_front else 0,
    ]
    with _device_scope(torch, device):
        stream = torch.cuda.current_stream(device).cuda_stream
        if candidate_capacity or stage_table != -1 or cta_threads:
            code = lib.silkern_topk_localize_explicit_v2(
                *args, int(candidate_capacity), int(stage_table), int(cta_threads), status_ptr, stream)
        else:
            code = lib.silkern_topk_localize_v1(*args, status_ptr, stream)
    _native.check(code, "topk_localize")
