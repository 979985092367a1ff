"""Alias of :mod:`silkern_b200.integrations.vllm`."""

from silkern_b200.integrations.vllm import (  # noqa: F401
    QUALIFIED_BLOCK_N,
    QUALIFIED_BLOCK_SIZES,
    QUALIFIED_DCP_SIZES,
    QUALIFIED_INTERLEAVES,
    QUALIFIED_TOPK_WIDTHS,
    UPSTREAM_COMMIT,
    UPSTREAM_INDEXER_SHA256,
    UPSTREAM_SPARSE_UTILS_SHA256,
    UPSTREAM_WRAPPER_SHA256,
    AdapterError,
    WorkspaceAdapter,
    install_converter,
    validate_production_call,
)
