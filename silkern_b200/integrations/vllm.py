"""Fixed-address stand-in for vLLM's sparse-DCP index converter.

vLLM's sparse-MLA path calls ``triton_filter_and_convert_dcp_index`` and gets
freshly allocated tensors back, which cannot live inside a captured CUDA
graph. :class:`WorkspaceAdapter` offers the same call surface with every
output and scratch buffer allocated once, up front:

1. :meth:`WorkspaceAdapter.prepare` (before warm-up and capture) allocates the
   output, the counts and, for the hierarchical arm, the workspace, and
   records the address/shape/stride/dtype/device of each input;
2. :meth:`WorkspaceAdapter.__call__` (every step, also during replay)
   allocates nothing and raises :class:`AdapterError` if the geometry or any
   input binding differs from the registered one.

:func:`install_converter` swaps the module attribute for the duration of a
``with`` block. Interface of silkern/integrations/vllm.py (adapter
:171-407, validation :71-145, installation :410-428).
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import contextmanager
from dataclasses import dataclass
from numbers import Integral
from typing import Any, Literal

from silkern_b200.contract import DEFAULT_TILE_SIZE
from silkern_b200.errors import LocalizationError
from silkern_b200.kernels import localize_hierarchical, localize_rowwise
from silkern_b200.workspace import workspace_shapes

Arm = Literal["row_stable", "hierarchical_stable"]

#: Upstream revision and file digests the call signature and geometry were
#: checked against (the values pinned by silkern/integrations/vllm.py:43-52).
UPSTREAM_COMMIT = "67f9046e4a12d939ffad0abc917585a00ef5b42d"
UPSTREAM_SPARSE_UTILS_SHA256 = "a15a5767a6afe1427dccc395d7125d3f8f2b701b859c31eec91918d04d5761b4"
UPSTREAM_WRAPPER_SHA256 = "550079022e858952c37bfa1198dbb1c77884571af30eb4c2f1a8055cd6ca7b07"
UPSTREAM_INDEXER_SHA256 = "e9bc6fbe3bd83f2116e7ba48f3a581e0699fbcce602a816724261a13ba64f1a5"

QUALIFIED_DCP_SIZES = (2, 4)
QUALIFIED_INTERLEAVES = (1,)
QUALIFIED_BLOCK_SIZES = (32, 64)
QUALIFIED_TOPK_WIDTHS = (2048,)
QUALIFIED_BLOCK_N = 128

_ATTRIBUTE = "triton_filter_and_convert_dcp_index"


class AdapterError(LocalizationError):
    """The call geometry or fixed-address binding is unsupported."""


def _positive_int(name: str, value: Any) -> int:
    if not isinstance(value, Integral) or isinstance(value, bool) or value < 1:
        raise AdapterError(f"{name} must be a positive integer")
    return int(value)


def validate_production_call(
    *,
    dcp_size: int,
    dcp_rank: int,
    cp_kv_cache_interleave_size: int,
    block_size: int,
    num_topk_tokens: int,
    block_n: int,
    return_valid_counts: bool,
    compact_valid_to_front: bool,
) -> None:
    """Reject any call outside the surface the integration is qualified on.

    Narrower than what the kernels accept on purpose: DCP 2 or 4 (the
    upstream indexer refuses interleave > 1), page sizes 32 and 64, top-k
    2048, ``BLOCK_N`` 128, valid counts returned and a compacted prefix.
    """
    size = _positive_int("dcp_size", dcp_size)
    if not isinstance(dcp_rank, Integral) or isinstance(dcp_rank, bool) or dcp_rank < 0:
        raise AdapterError("dcp_rank must be a nonnegative integer")
    rank = int(dcp_rank)
    interleave = _positive_int("cp_kv_cache_interleave_size", cp_kv_cache_interleave_size)
    block = _positive_int("block_size", block_size)
    width = _positive_int("num_topk_tokens", num_topk_tokens)
    tile = _positive_int("block_n", block_n)
    if size not in QUALIFIED_DCP_SIZES:
        raise AdapterError(
            f"dcp_size={size} is outside the integrated qualification {QUALIFIED_DCP_SIZES}"
        )
    if not 0 <= rank < size:
        raise AdapterError(f"dcp_rank={rank} is outside [0, {size})")
    if interleave not in QUALIFIED_INTERLEAVES:
        raise AdapterError("the upstream sparse indexer fails closed for DCP interleave > 1")
    if block not in QUALIFIED_BLOCK_SIZES:
        raise AdapterError(
            f"block_size={block} is outside the qualified backend surface {QUALIFIED_BLOCK_SIZES}"
        )
    if width not in QUALIFIED_TOPK_WIDTHS:
        raise AdapterError(
            f"top-k width={width} is outside the compatible sparse-MLA surface "
            f"{QUALIFIED_TOPK_WIDTHS}"
        )
    if tile != QUALIFIED_BLOCK_N:
        raise AdapterError(f"BLOCK_N={tile} differs from the qualified wrapper value {QUALIFIED_BLOCK_N}")
    if return_valid_counts is not True:
        raise AdapterError("the production sparse-attention call requires valid counts")
    if compact_valid_to_front is not True:
        raise AdapterError("the production sparse-attention call requires a contiguous valid prefix")


def _signature(tensor: Any) -> tuple[Any, ...]:
    """Address/shape/stride/dtype/device of a tensor, without importing torch."""
    return (
        int(tensor.data_ptr()),
        tuple(tensor.shape),
        tuple(tensor.stride()),
        str(tensor.dtype),
        str(tensor.device),
    )


@dataclass
class _Binding:
    call: tuple[int, ...]
    inputs: tuple[tuple[Any, ...], ...]
    out: Any
    counts: Any
    workspace: dict[str, Any]


class WorkspaceAdapter:
    """Pre-registered, allocation-free replacement for the upstream converter."""

    def __init__(self, arm: Arm, *, hierarchical_tile_size: int = DEFAULT_TILE_SIZE) -> None:
        if arm not in ("row_stable", "hierarchical_stable"):
            raise AdapterError(f"unknown arm: {arm}")
        self.arm = arm
        self.hierarchical_tile_size = _positive_int("hierarchical_tile_size", hierarchical_tile_size)
        self._binding: _Binding | None = None
        self.calls = 0

    @staticmethod
    def _call_key(dcp_size, dcp_rank, interleave, block_size, num_topk_tokens, block_n):
        return (int(dcp_size), int(dcp_rank), int(interleave), int(block_size),
                int(num_topk_tokens), int(block_n))

    def prepare(
        self,
        req_id: Any,
        block_table: Any,
        token_indices: Any,
        *,
        dcp_size: int,
        dcp_rank: int,
        cp_kv_cache_interleave_size: int = 1,
        block_size: int = 64,
        num_topk_tokens: int = 2048,
        block_n: int = QUALIFIED_BLOCK_N,
    ) -> None:
        """Allocate and bind the fixed buffers; call before warm-up or capture."""
        validate_production_call(
            dcp_size=dcp_size,
            dcp_rank=dcp_rank,
            cp_kv_cache_interleave_size=cp_kv_cache_interleave_size,
            block_size=block_size,
            num_topk_tokens=num_topk_tokens,
            block_n=block_n,
            return_valid_counts=True,
            compact_valid_to_front=True,
        )
        try:
            import torch
        except ModuleNotFoundError as exc:  # pragma: no cover - GPU-only branch
            raise AdapterError("torch is required to prepare CUDA buffers") from exc
        if not all(isinstance(t, torch.Tensor) for t in (req_id, block_table, token_indices)):
            raise AdapterError("all production inputs must be torch tensors")
        if token_indices.ndim != 2:
            raise AdapterError("token_indices must be two-dimensional")
        if token_indices.shape[1] != num_topk_tokens:
            raise AdapterError("token_indices width does not match NUM_TOPK_TOKENS")
        if req_id.shape != (token_indices.shape[0],):
            raise AdapterError("req_id must contain one id per token row")

        rows = token_indices.shape[0]
        device = token_indices.device
        out = torch.empty_like(token_indices)
        counts = torch.empty(rows, dtype=torch.int32, device=device)
        workspace: dict[str, Any] = {}
        if self.arm == "hierarchical_stable":
            shapes = workspace_shapes(rows, token_indices.shape[1], tile_size=self.hierarchical_tile_size)
            workspace = {
                name: torch.empty(shape, dtype=torch.int32, device=device)
                for name, shape in shapes.items()
            }
        self._binding = _Binding(
            call=self._call_key(dcp_size, dcp_rank, cp_kv_cache_interleave_size, block_size,
                                num_topk_tokens, block_n),
            inputs=(_signature(req_id), _signature(block_table), _signature(token_indices)),
            out=out,
            counts=counts,
            workspace=workspace,
        )

    @property
    def prepared(self) -> bool:
        return self._binding is not None

    def _bound(self) -> _Binding:
        if self._binding is None:
            raise AdapterError("adapter has not been prepared")
        return self._binding

    @property
    def output(self) -> Any:
        return self._bound().out

    @property
    def counts(self) -> Any:
        return self._bound().counts

    @property
    def fixed_buffer_signatures(self) -> dict[str, tuple[Any, ...]]:
        binding = self._bound()
        signatures = {"out": _signature(binding.out), "counts": _signature(binding.counts)}
        signatures.update({name: _signature(t) for name, t in binding.workspace.items()})
        return signatures

    def __call__(
        self,
        req_id: Any,
        block_table: Any,
        token_indices: Any,
        dcp_size: int,
        dcp_rank: int,
        cp_kv_cache_interleave_size: int = 1,
        BLOCK_SIZE: int = 64,
        NUM_TOPK_TOKENS: int = 2048,
        BLOCK_N: int = QUALIFIED_BLOCK_N,
        return_valid_counts: bool = False,
        compact_valid_to_front: bool = True,
    ) -> tuple[Any, Any]:
        validate_production_call(
            dcp_size=dcp_size,
            dcp_rank=dcp_rank,
            cp_kv_cache_interleave_size=cp_kv_cache_interleave_size,
            block_size=BLOCK_SIZE,
            num_topk_tokens=NUM_TOPK_TOKENS,
            block_n=BLOCK_N,
            return_valid_counts=return_valid_counts,
            compact_valid_to_front=compact_valid_to_front,
        )
        if self._binding is None:
            raise AdapterError("graph bucket is unregistered; call prepare before wrapper execution")
        binding = self._binding
        call = self._call_key(dcp_size, dcp_rank, cp_kv_cache_interleave_size, BLOCK_SIZE,
                              NUM_TOPK_TOKENS, BLOCK_N)
        if call != binding.call:
            raise AdapterError(f"call geometry {call} differs from registered {binding.call}")
        observed = (_signature(req_id), _signature(block_table), _signature(token_indices))
        if observed != binding.inputs:
            raise AdapterError("production input tensor address/shape/stride binding changed")

        if self.arm == "row_stable":
            localize_rowwise(
                req_id,
                block_table,
                token_indices,
                binding.out,
                binding.counts,
                block_size=BLOCK_SIZE,
                dcp_size=dcp_size,
                dcp_rank=dcp_rank,
                dcp_interleave=cp_kv_cache_interleave_size,
                compact_valid_to_front=True,
            )
        else:
            ws = binding.workspace
            localize_hierarchical(
                req_id,
                block_table,
                token_indices,
                binding.out,
                binding.counts,
                ws["mapped"],
                ws["local_positions"],
                ws["tile_counts"],
                ws["tile_offsets"],
                block_size=BLOCK_SIZE,
                dcp_size=dcp_size,
                dcp_rank=dcp_rank,
                dcp_interleave=cp_kv_cache_interleave_size,
                compact_valid_to_front=True,
                tile_size=self.hierarchical_tile_size,
            )
        self.calls += 1
        return binding.out, binding.counts


@contextmanager
def install_converter(module: Any, adapter: WorkspaceAdapter) -> Iterator[None]:
    """Put ``adapter`` at the module's call site for the duration of the block.

    The original callable is restored on exit, exceptions included; no
    upstream file is modified.
    """
    if not hasattr(module, _ATTRIBUTE):
        raise AdapterError(f"module has no {_ATTRIBUTE}; this is not the expected call site")
    original = getattr(module, _ATTRIBUTE)
    setattr(module, _ATTRIBUTE, adapter)
    try:
        yield
    finally:
        setattr(module, _ATTRIBUTE, original)
