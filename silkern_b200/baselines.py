"""The atomic-reservation converter, as a comparison baseline.

Same interface and checks as the reference's bench/atomic_baseline.py:313-385
(``launch_atomic_baseline``), on the CUDA restatement in
``csrc/atomic_baseline.cu``. It returns the right set and count in an order
that depends on which tile's atomicAdd lands first; it is here to be timed
beside the stable converter and to show that instability, not to be used.
"""

from __future__ import annotations

from silkern_b200 import _native
from silkern_b200.contract import _validate_dcp_config
from silkern_b200.errors import LocalizationError


def launch_atomic_baseline(
    req_ids,
    block_table,
    tokens,
    out,
    counts,
    scratch,
    *,
    block_size: int,
    dcp_size: int,
    dcp_rank: int,
    dcp_interleave: int = 1,
) -> None:
    """Run the atomic baseline: correct set and count, unspecified order.

    ``scratch`` is an int32 ``(batch,)`` buffer for the per-row reservation
    counters; ``counts`` receives their final values.
    """
    import torch

    tensors = (req_ids, block_table, tokens, out, counts, scratch)
    if any(not isinstance(t, torch.Tensor) for t in tensors):
        raise LocalizationError("all baseline buffers must be torch tensors")
    if any(not t.is_cuda for t in tensors):
        raise LocalizationError("all baseline buffers must be CUDA tensors")
    if any(t.dtype != torch.int32 for t in tensors):
        raise LocalizationError("all baseline buffers must use int32")
    if any(not t.is_contiguous() for t in tensors):
        raise LocalizationError("the baseline requires contiguous tensors")
    if tokens.ndim != 2 or out.shape != tokens.shape:
        raise LocalizationError("tokens and out must have the same 2D shape")
    _validate_dcp_config(dcp_size, dcp_rank, dcp_interleave)
    batch, width = tokens.shape
    if counts.shape != (batch,) or scratch.shape != (batch,):
        raise LocalizationError("counts and scratch must hold one element per row")
    lib = _native.load()
    code = lib.silkern_atomic_baseline_v1(
        req_ids.data_ptr(), block_table.data_ptr(), block_table.shape[0], block_table.shape[1],
        tokens.data_ptr(), out.data_ptr(), counts.data_ptr(), scratch.data_ptr(), batch, width,
        int(block_size), int(dcp_size), int(dcp_rank), int(dcp_interleave),
        torch.cuda.current_stream(tokens.device).cuda_stream,
    )
    _native.check(code, "atomic baseline")
