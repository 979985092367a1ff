"""The torch.library ops: schemas, fake implementations and a full-graph trace (CPU)."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from silkern_b200 import localize_hierarchical, localize_rowwise, ops, workspace_shapes  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def _registered():
    ops.register()


def _written(op) -> set[str]:
    return {a.name for a in op.default._schema.arguments if a.alias_info is not None and a.alias_info.is_write}


def test_schemas_mark_exactly_the_written_buffers() -> None:
    assert _written(torch.ops.silkern_b200.localize_rowwise) == {"out", "counts", "status"}
    assert _written(torch.ops.silkern_b200.localize_hierarchical) == {
        "out", "counts", "tile_counts", "tile_offsets", "status"}


def test_register_is_idempotent() -> None:
    ops.register()
    ops.register()
    assert ops.registered()


def test_fake_implementations_launch_nothing() -> None:
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        i32 = dict(dtype=torch.int32)
        req, table = torch.empty(4, **i32), torch.empty(4, 8, **i32)
        tokens, out, counts = torch.empty(4, 16, **i32), torch.empty(4, 16, **i32), torch.empty(4, **i32)
        assert torch.ops.silkern_b200.localize_rowwise(req, table, tokens, out, counts, 64, 2, 0, 1, True, 8,
                                                       None) is None
        ws = [torch.empty(s, **i32) for s in workspace_shapes(4, 16, tile_size=64).values()]
        assert torch.ops.silkern_b200.localize_hierarchical(req, table, tokens, out, counts, *ws, 64, 2, 0, 1,
                                                            True, 64, 4, None) is None


def test_public_launchers_trace_as_two_op_nodes_without_a_graph_break() -> None:
    """torch.compile(fullgraph=True) of a function that calls both public
    launchers: the trace holds one node per op and no break. The backend only
    inspects the graph (nothing runs; there is no GPU here)."""
    graphs = []

    def inspect(gm, example_inputs):
        graphs.append(gm)
        return lambda *args: None

    def step(req, table, tokens, out, counts, mapped, positions, tile_counts, tile_offsets, out2, counts2):
        localize_rowwise(req, table, tokens, out, counts, block_size=64, dcp_size=4, dcp_rank=1)
        localize_hierarchical(req, table, tokens, out2, counts2, mapped, positions, tile_counts, tile_offsets,
                              block_size=64, dcp_size=4, dcp_rank=1, tile_size=64)

    i32 = dict(dtype=torch.int32)
    args = [torch.zeros(4, **i32), torch.zeros(4, 8, **i32), torch.zeros(4, 128, **i32),
            torch.zeros(4, 128, **i32), torch.zeros(4, **i32)]
    args += [torch.zeros(s, **i32) for s in workspace_shapes(4, 128, tile_size=64).values()]
    args += [torch.zeros(4, 128, **i32), torch.zeros(4, **i32)]
    torch._dynamo.reset()
    torch.compile(step, backend=inspect, fullgraph=True)(*args)
    assert len(graphs) == 1
    targets = [str(node.target) for node in graphs[0].graph.nodes if node.op == "call_function"]
    assert sum("silkern_b200.localize_rowwise" in t for t in targets) == 1
    assert sum("silkern_b200.localize_hierarchical" in t for t in targets) == 1
