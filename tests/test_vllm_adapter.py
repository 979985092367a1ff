"""CPU tests of the vLLM call-site adapter (reference tests/test_vllm_adapter.py)."""

from __future__ import annotations

from types import SimpleNamespace

import pytest

from silkern_b200.integrations.vllm import (
    AdapterError,
    WorkspaceAdapter,
    install_converter,
    validate_production_call,
)


def _valid_call() -> dict:
    return {
        "dcp_size": 2,
        "dcp_rank": 0,
        "cp_kv_cache_interleave_size": 1,
        "block_size": 64,
        "num_topk_tokens": 2048,
        "block_n": 128,
        "return_valid_counts": True,
        "compact_valid_to_front": True,
    }


@pytest.mark.parametrize("dcp_size", [2, 4])
@pytest.mark.parametrize("block_size", [32, 64])
def test_accepts_qualified_geometry(dcp_size: int, block_size: int) -> None:
    values = _valid_call()
    values.update(dcp_size=dcp_size, dcp_rank=dcp_size - 1, block_size=block_size)
    validate_production_call(**values)


@pytest.mark.parametrize(
    ("field", "value"),
    [
        ("dcp_size", 1),
        ("dcp_size", 8),
        ("dcp_rank", -1),
        ("dcp_rank", 2),
        ("dcp_rank", True),
        ("cp_kv_cache_interleave_size", 2),
        ("block_size", 16),
        ("block_size", 128),
        ("num_topk_tokens", 1024),
        ("block_n", 64),
        ("return_valid_counts", False),
        ("compact_valid_to_front", False),
    ],
)
def test_fails_closed(field: str, value: object) -> None:
    values = _valid_call()
    values[field] = value
    with pytest.raises(AdapterError):
        validate_production_call(**values)


def test_requires_known_arm() -> None:
    with pytest.raises(AdapterError):
        WorkspaceAdapter("atomic")  # type: ignore[arg-type]


def test_unprepared_adapter_refuses_calls() -> None:
    adapter = WorkspaceAdapter("row_stable")
    assert not adapter.prepared
    with pytest.raises(AdapterError, match="unregistered"):
        adapter(None, None, None, 2, 0, return_valid_counts=True)
    with pytest.raises(AdapterError, match="not been prepared"):
        _ = adapter.output


def test_installation_is_scoped_and_restored() -> None:
    native = object()
    module = SimpleNamespace(triton_filter_and_convert_dcp_index=native)
    adapter = WorkspaceAdapter("row_stable")
    with install_converter(module, adapter):
        assert module.triton_filter_and_convert_dcp_index is adapter
    assert module.triton_filter_and_convert_dcp_index is native


def test_installation_restores_on_exception() -> None:
    native = object()
    module = SimpleNamespace(triton_filter_and_convert_dcp_index=native)
    with pytest.raises(RuntimeError):
        with install_converter(module, WorkspaceAdapter("hierarchical_stable")):
            raise RuntimeError("boom")
    assert module.triton_filter_and_convert_dcp_index is native


def test_installation_rejects_unknown_source_surface() -> None:
    with pytest.raises(AdapterError):
        with install_converter(SimpleNamespace(), WorkspaceAdapter("row_stable")):
            pass


def test_drop_in_alias_package() -> None:
    import silkern
    import silkern.integrations.vllm as alias
    import silkern_b200

    assert silkern.localize_rowwise is silkern_b200.localize_rowwise
    assert silkern.exact_stable_compact_reference is silkern_b200.localize_reference
    assert alias.WorkspaceAdapter is WorkspaceAdapter
