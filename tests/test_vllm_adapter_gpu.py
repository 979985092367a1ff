"""The vLLM adapter on a device (reference tests/test_vllm_adapter_gpu.py)."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from silkern import exact_stable_compact_reference  # noqa: E402  (drop-in alias package)
from silkern_b200.integrations.vllm import AdapterError, WorkspaceAdapter  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA is required", allow_module_level=True)


def _case():
    batch, width, table_width = 3, 2048, 32
    req_ids = [2, 0, 1]
    block_table = [[request * table_width + (column * 7) % table_width for column in range(table_width)]
                   for request in range(3)]
    rows = [[-1 if column % 19 == 0 else (column * 13 + row * 17) % 4096 for column in range(width)]
            for row in range(batch)]
    return req_ids, block_table, rows


@pytest.mark.parametrize("arm", ["row_stable", "hierarchical_stable"])
def test_adapter_matches_exact_oracle_and_replays_at_fixed_addresses(arm: str) -> None:
    case = _case()
    expected = exact_stable_compact_reference(*case, block_size=64, dcp_size=2, dcp_rank=1,
                                              dcp_interleave=1)
    req_ids, block_table, tokens = (torch.tensor(v, dtype=torch.int32, device="cuda") for v in case)
    adapter = WorkspaceAdapter(arm)  # type: ignore[arg-type]
    adapter.prepare(req_ids, block_table, tokens, dcp_size=2, dcp_rank=1, block_size=64)
    signatures = adapter.fixed_buffer_signatures

    def op() -> None:
        output, counts = adapter(req_ids, block_table, tokens, 2, 1, BLOCK_SIZE=64,
                                 NUM_TOPK_TOKENS=2048, BLOCK_N=128, return_valid_counts=True)
        assert output.data_ptr() == adapter.output.data_ptr()
        assert counts.data_ptr() == adapter.counts.data_ptr()

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            op()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        op()
    allocated = torch.cuda.memory_allocated()
    adapter.output.fill_(0)
    for _ in range(100):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == allocated
    assert adapter.fixed_buffer_signatures == signatures
    assert adapter.output.cpu().tolist() == expected[0]
    assert adapter.counts.cpu().tolist() == expected[1]
    assert adapter.calls == 4


def test_adapter_rejects_a_different_fixed_address_binding() -> None:
    req_ids, block_table, tokens = (torch.tensor(v, dtype=torch.int32, device="cuda") for v in _case())
    adapter = WorkspaceAdapter("row_stable")
    adapter.prepare(req_ids, block_table, tokens, dcp_size=2, dcp_rank=0, block_size=64)
    with pytest.raises(AdapterError, match="binding changed"):
        adapter(req_ids.clone(), block_table, tokens, 2, 0, BLOCK_SIZE=64, NUM_TOPK_TOKENS=2048,
                return_valid_counts=True)
    with pytest.raises(AdapterError, match="differs from registered"):
        adapter(req_ids, block_table, tokens, 2, 1, BLOCK_SIZE=64, NUM_TOPK_TOKENS=2048,
                return_valid_counts=True)


def test_installed_adapter_inside_a_captured_stand_in_decode_step() -> None:
    """The adapter installed at a stand-in module's converter attribute and
    called from a stand-in sparse-attention step (converter, then a gather of
    a fake KV cache at the returned slots, masked by the counts). The whole
    step is captured once; every replay gets a fresh selection written into
    the bound token buffer, as the upstream top-k would, and its result is
    checked against the contract on the host."""
    from types import SimpleNamespace

    import numpy as np

    from silkern_b200.integrations.vllm import install_converter

    def upstream(*args, **kwargs):
        raise AssertionError("the upstream converter must not run while the adapter is installed")

    module = SimpleNamespace(triton_filter_and_convert_dcp_index=upstream)
    req_list, table_list, _ = _case()
    req_ids = torch.tensor(req_list, dtype=torch.int32, device="cuda")
    block_table = torch.tensor(table_list, dtype=torch.int32, device="cuda")
    tokens = torch.zeros((3, 2048), dtype=torch.int32, device="cuda")
    kv = torch.arange(8192, dtype=torch.int64, device="cuda") * 3 + 1
    result = torch.zeros(3, dtype=torch.int64, device="cuda")
    columns = torch.arange(2048, device="cuda")
    adapter = WorkspaceAdapter("row_stable")
    adapter.prepare(req_ids, block_table, tokens, dcp_size=2, dcp_rank=1, block_size=64)

    def sparse_attention_step() -> None:
        out, counts = module.triton_filter_and_convert_dcp_index(
            req_ids, block_table, tokens, 2, 1, 1, BLOCK_SIZE=64, NUM_TOPK_TOKENS=2048, BLOCK_N=128,
            return_valid_counts=True)
        valid = columns[None, :] < counts[:, None]
        result.copy_((kv[out.clamp_min(0).long()] * valid).sum(dim=1))

    kv_host = kv.cpu().numpy()
    rng = np.random.default_rng(31)
    with install_converter(module, adapter):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                sparse_attention_step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            sparse_attention_step()
        for _ in range(30):
            selection = rng.integers(-2, 4096, size=(3, 2048), dtype=np.int32)
            tokens.copy_(torch.as_tensor(selection))
            graph.replay()
            torch.cuda.synchronize()
            want_out, want_counts = exact_stable_compact_reference(
                req_list, table_list, selection.tolist(), block_size=64, dcp_size=2, dcp_rank=1,
                dcp_interleave=1)
            assert adapter.output.cpu().tolist() == want_out
            want = [int(kv_host[row[:n]].sum()) for row, n in zip(want_out, want_counts, strict=True)]
            assert result.cpu().tolist() == want
        del graph
    assert module.triton_filter_and_convert_dcp_index is upstream
