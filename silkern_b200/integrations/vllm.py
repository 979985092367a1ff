"""Fixed-address stand-in for vLLM's sparse-DCP index converter.

vLLM's sparse-MLA path calls ``triton_filter_and_convert_dcp_index`` and gets
freshly allocated tensors back, which cannot live inside a captured CUDA
graph. :class:`WorkspaceAdapter` answers the same call with buffers it
allocated once, up front:

1. :meth:`WorkspaceAdapter.prepare` (before warm-up and capture) allocates the
   output, the counts and, for the hierarchical arm, the workspace, and
   freezes a *binding key*: the call geometry plus the address, shape,
   stride, dtype and device of each input tensor;
2. :meth:`WorkspaceAdapter.__call__` (every step, also during replay)
   recomputes that key from its arguments, raises :class:`AdapterError` if it
   differs, and otherwise runs the launch chosen at ``prepare`` time. It
   allocates nothing.

Calls outside the qualified surface are refused by one table of rules,
:data:`_QUALIFICATION`, checked in order. :func:`install_converter` swaps the
module attribute for the duration of a ``with`` block. Interface (names,
constants, messages) of silkern/integrations/vllm.py (adapter :171-407,
qualification :71-145, installation :410-428).
"""

from __future__ import annotations

from collections.abc import Callable, Iterator
from contextlib import contextmanager
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
_ARMS = ("row_stable", "hierarchical_stable")


class AdapterError(LocalizationError):
    """The call geometry or fixed-address binding is unsupported."""


def _is_count(value: Any, minimum: int) -> bool:
    return isinstance(value, Integral) and not isinstance(value, bool) and value >= minimum


#: Integer fields of a production call: (name, smallest accepted value, message).
_INTEGER_FIELDS = (
    ("dcp_size", 1, "dcp_size must be a positive integer"),
    ("dcp_rank", 0, "dcp_rank must be a nonnegative integer"),
    ("cp_kv_cache_interleave_size", 1, "cp_kv_cache_interleave_size must be a positive integer"),
    ("block_size", 1, "block_size must be a positive integer"),
    ("num_topk_tokens", 1, "num_topk_tokens must be a positive integer"),
    ("block_n", 1, "block_n must be a positive integer"),
)

#: The qualified surface, checked in order once the integers are well formed:
#: (predicate over the call, message for a call that fails it). Narrower than
#: what the kernels accept on purpose: DCP 2 or 4 (the upstream indexer
#: refuses interleave > 1), page sizes 32 and 64, top-k 2048, BLOCK_N 128,
#: valid counts returned and a compacted prefix.
_QUALIFICATION: tuple[tuple[Callable[[dict], bool], Callable[[dict], str]], ...] = (
    (lambda c: c["dcp_size"] in QUALIFIED_DCP_SIZES,
     lambda c: f"dcp_size={c['dcp_size']} is outside the integrated qualification {QUALIFIED_DCP_SIZES}"),
    (lambda c: c["dcp_rank"] < c["dcp_size"],
     lambda c: f"dcp_rank={c['dcp_rank']} is outside [0, {c['dcp_size']})"),
    (lambda c: c["cp_kv_cache_interleave_size"] in QUALIFIED_INTERLEAVES,
     lambda c: "the upstream sparse indexer fails closed for DCP interleave > 1"),
    (lambda c: c["block_size"] in QUALIFIED_BLOCK_SIZES,
     lambda c: f"block_size={c['block_size']} is outside the qualified backend surface {QUALIFIED_BLOCK_SIZES}"),
    (lambda c: c["num_topk_tokens"] in QUALIFIED_TOPK_WIDTHS,
     lambda c: f"top-k width={c['num_topk_tokens']} is outside the compatible sparse-MLA surface "
               f"{QUALIFIED_TOPK_WIDTHS}"),
    (lambda c: c["block_n"] == QUALIFIED_BLOCK_N,
     lambda c: f"BLOCK_N={c['block_n']} differs from the qualified wrapper value {QUALIFIED_BLOCK_N}"),
    (lambda c: c["return_valid_counts"] is True,
     lambda c: "the production sparse-attention call requires valid counts"),
    (lambda c: c["compact_valid_to_front"] is True,
     lambda c: "the production sparse-attention call requires a contiguous valid prefix"),
)


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
    """Reject any call outside the surface the integration is qualified on."""
    call = dict(dcp_size=dcp_size, dcp_rank=dcp_rank, cp_kv_cache_interleave_size=cp_kv_cache_interleave_size,
                block_size=block_size, num_topk_tokens=num_topk_tokens, block_n=block_n,
                return_valid_counts=return_valid_counts, compact_valid_to_front=compact_valid_to_front)
    for name, minimum, message in _INTEGER_FIELDS:
        if not _is_count(call[name], minimum):
            raise AdapterError(message)
        call[name] = int(call[name])
    for holds, message in _QUALIFICATION:
        if not holds(call):
            raise AdapterError(message(call))


def _tensor_key(tensor: Any) -> tuple[Any, ...]:
    """Address, shape, stride, dtype and device of a tensor (no torch import)."""
    return (int(tensor.data_ptr()), tuple(tensor.shape), tuple(tensor.stride()), str(tensor.dtype),
            str(tensor.device))


def _binding_key(geometry: tuple[int, ...], *tensors: Any) -> tuple[Any, ...]:
    """The whole binding as one comparable value: geometry, then each input."""
    return (geometry, *(_tensor_key(t) for t in tensors))


class WorkspaceAdapter:
    """Pre-registered, allocation-free replacement for the upstream converter."""

    def __init__(self, arm: Arm, *, hierarchical_tile_size: int = DEFAULT_TILE_SIZE) -> None:
        if arm not in _ARMS:
            raise AdapterError(f"unknown arm: {arm}")
        if not _is_count(hierarchical_tile_size, 1):
            raise AdapterError("hierarchical_tile_size must be a positive integer")
        self.arm = arm
        self.hierarchical_tile_size = int(hierarchical_tile_size)
        self.calls = 0
        self._key: tuple[Any, ...] | None = None
        self._buffers: dict[str, Any] = {}
        self._launch: Callable[..., None] | None = None

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
            dcp_size=dcp_size, dcp_rank=dcp_rank, cp_kv_cache_interleave_size=cp_kv_cache_interleave_size,
            block_size=block_size, num_topk_tokens=num_topk_tokens, block_n=block_n,
            return_valid_counts=True, compact_valid_to_front=True)
        try:
            import torch
        except ModuleNotFoundError as exc:  # pragma: no cover - GPU-only branch
            raise AdapterError("torch is required to prepare CUDA buffers") from exc
        if not all(isinstance(t, torch.Tensor) for t in (req_id, block_table, token_indices)):
            raise AdapterError("all production inputs must be torch tensors")
        if token_indices.ndim != 2:
            raise AdapterError("token_indices must be two-dimensional")
        rows, width = token_indices.shape
        if width != num_topk_tokens:
            raise AdapterError("token_indices width does not match NUM_TOPK_TOKENS")
        if req_id.shape != (rows,):
            raise AdapterError("req_id must contain one id per token row")

        device = token_indices.device
        buffers = {"out": torch.empty_like(token_indices),
                   "counts": torch.empty(rows, dtype=torch.int32, device=device)}
        if self.arm == "hierarchical_stable":
            for name, shape in workspace_shapes(rows, width, tile_size=self.hierarchical_tile_size).items():
                buffers[name] = torch.empty(shape, dtype=torch.int32, device=device)
        geometry = (int(dcp_size), int(dcp_rank), int(cp_kv_cache_interleave_size), int(block_size),
                    int(num_topk_tokens), int(block_n))
        self._buffers = buffers
        self._key = _binding_key(geometry, req_id, block_table, token_indices)
        self._launch = self._bind_launch(geometry)

    def _bind_launch(self, geometry: tuple[int, ...]) -> Callable[..., None]:
        """The converter call for this arm and geometry, on the fixed buffers."""
        dcp_size, dcp_rank, interleave, block_size = geometry[:4]
        kw = dict(block_size=block_size, dcp_size=dcp_size, dcp_rank=dcp_rank, dcp_interleave=interleave,
                  compact_valid_to_front=True)
        b = self._buffers
        if self.arm == "row_stable":
            return lambda req, table, tokens: localize_rowwise(req, table, tokens, b["out"], b["counts"], **kw)
        tile = self.hierarchical_tile_size
        return lambda req, table, tokens: localize_hierarchical(
            req, table, tokens, b["out"], b["counts"], b["mapped"], b["local_positions"], b["tile_counts"],
            b["tile_offsets"], tile_size=tile, **kw)

    @property
    def prepared(self) -> bool:
        return self._key is not None

    def _buffer(self, name: str) -> Any:
        if self._key is None:
            raise AdapterError("adapter has not been prepared")
        return self._buffers[name]

    @property
    def output(self) -> Any:
        return self._buffer("out")

    @property
    def counts(self) -> Any:
        return self._buffer("counts")

    @property
    def fixed_buffer_signatures(self) -> dict[str, tuple[Any, ...]]:
        self._buffer("out")  # raises when unprepared
        return {name: _tensor_key(t) for name, t in self._buffers.items()}

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
            dcp_size=dcp_size, dcp_rank=dcp_rank, cp_kv_cache_interleave_size=cp_kv_cache_interleave_size,
            block_size=BLOCK_SIZE, num_topk_tokens=NUM_TOPK_TOKENS, block_n=BLOCK_N,
            return_valid_counts=return_valid_counts, compact_valid_to_front=compact_valid_to_front)
        if self._key is None or self._launch is None:
            raise AdapterError("graph bucket is unregistered; call prepare before wrapper execution")
        geometry = (int(dcp_size), int(dcp_rank), int(cp_kv_cache_interleave_size), int(BLOCK_SIZE),
                    int(NUM_TOPK_TOKENS), int(BLOCK_N))
        key = _binding_key(geometry, req_id, block_table, token_indices)
        if key != self._key:
            if key[0] != self._key[0]:
                raise AdapterError(f"call geometry {key[0]} differs from registered {self._key[0]}")
            raise AdapterError("production input tensor address/shape/stride binding changed")
        self._launch(req_id, block_table, token_indices)
        self.calls += 1
        return self._buffers["out"], self._buffers["counts"]


@contextmanager
def install_converter(module: Any, adapter: WorkspaceAdapter) -> Iterator[None]:
    """Put ``adapter`` at the module's call site for the duration of the block.

    The original callable is restored on exit, exceptions included; no
    upstream file is modified.
    """
    original = getattr(module, _ATTRIBUTE, _ABSENT)
    if original is _ABSENT:
        raise AdapterError(f"module has no {_ATTRIBUTE}; this is not the expected call site")
    setattr(module, _ATTRIBUTE, adapter)
    try:
        yield
    finally:
        setattr(module, _ATTRIBUTE, original)


_ABSENT = object()
