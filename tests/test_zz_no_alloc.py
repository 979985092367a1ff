"""The allocation-free hierarchical entry point, through the C ABI, on a GPU.

Some callers cannot allocate device memory on their call path: plugin hosts
and serving runtimes whose enqueue step forbids cudaMalloc, or code that runs
while another framework records a CUDA graph. For them
``silkern_localize_hierarchical_noalloc_v1`` keeps its tile workspace in a
fixed array inside the library instead of taking workspace buffers. This file
checks that it returns exactly what ``silkern_localize_hierarchical_v1``
returns, on two calls in a row with different inputs (the second call
must not be helped by anything the first left in the shared array), and that
a geometry larger than the array is refused before launch.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one; it also passes alone in a fresh process.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from silkern_b200 import _native  # noqa: E402
from silkern_b200.workloads import config_case  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA is required", allow_module_level=True)

MAX_TILES = 32768  # SILKERN_NOALLOC_MAX_TILES
E_SCRATCH = 8  # SILKERN_E_SCRATCH
POISON = 0x5A5A5A5A


def _inputs(case, dev):
    return tuple(torch.as_tensor(np.ascontiguousarray(a)).to(dev)
                 for a in (case.req_ids, case.block_table, case.tokens))


def _with_workspace(lib, req, table, tokens, kw, tile_size, stream):
    batch, width = tokens.shape
    tiles = (width + tile_size - 1) // tile_size
    out = torch.full_like(tokens, POISON)
    counts = torch.full((batch,), POISON, dtype=torch.int32, device=tokens.device)
    tile_counts = torch.empty((batch, tiles), dtype=torch.int32, device=tokens.device)
    tile_offsets = torch.empty_like(tile_counts)
    rc = lib.silkern_localize_hierarchical_v1(
        req.data_ptr(), table.data_ptr(), table.shape[0], table.shape[1], tokens.data_ptr(),
        out.data_ptr(), counts.data_ptr(), None, None, tile_counts.data_ptr(),
        tile_offsets.data_ptr(), batch, width, kw["block_size"], kw["dcp_size"], kw["dcp_rank"],
        kw["dcp_interleave"], 1, tile_size, None, stream,
    )
    assert rc == 0, _native.status_string(rc)
    return out, counts


def _no_alloc(lib, req, table, tokens, kw, tile_size, stream):
    batch, width = tokens.shape
    out = torch.full_like(tokens, POISON)
    counts = torch.full((batch,), POISON, dtype=torch.int32, device=tokens.device)
    rc = lib.silkern_localize_hierarchical_noalloc_v1(
        req.data_ptr(), table.data_ptr(), table.shape[0], table.shape[1], tokens.data_ptr(),
        out.data_ptr(), counts.data_ptr(), batch, width, kw["block_size"], kw["dcp_size"],
        kw["dcp_rank"], kw["dcp_interleave"], 1, tile_size, None, stream,
    )
    assert rc == 0, _native.status_string(rc)
    return out, counts


def test_no_alloc_entry_point_matches_workspace_entry_point_twice() -> None:
    lib = _native.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev).cuda_stream
    # Two different wide-row calls in a row: config 4 shapes (32 x 16384,
    # tile 1024) at two DCP ranks and seeds, then a narrow row with tile 64.
    calls = [
        (config_case(4, seed=41, dcp_rank=3), 1024),
        (config_case(4, seed=42, dcp_rank=6), 1024),
        (config_case(3, seed=43, dcp_rank=1, batch=64), 64),
    ]
    for case, tile_size in calls:
        req, table, tokens = _inputs(case, dev)
        kw = case.geometry()
        want = _with_workspace(lib, req, table, tokens, kw, tile_size, stream)
        got = _no_alloc(lib, req, table, tokens, kw, tile_size, stream)
        torch.cuda.synchronize()
        assert torch.equal(got[0], want[0])
        assert torch.equal(got[1], want[1])
        assert int(got[1].sum()) > 0


def test_no_alloc_entry_point_refuses_geometry_beyond_its_array() -> None:
    lib = _native.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    tokens = torch.zeros((MAX_TILES // 16 + 1, 16 * 64), dtype=torch.int32, device=dev)
    out = torch.empty_like(tokens)
    counts = torch.empty(tokens.shape[0], dtype=torch.int32, device=dev)
    req = torch.zeros(tokens.shape[0], dtype=torch.int32, device=dev)
    table = torch.zeros((1, 4), dtype=torch.int32, device=dev)
    rc = lib.silkern_localize_hierarchical_noalloc_v1(
        req.data_ptr(), table.data_ptr(), 1, 4, tokens.data_ptr(), out.data_ptr(),
        counts.data_ptr(), tokens.shape[0], tokens.shape[1], 64, 2, 0, 1, 1, 64, None,
        torch.cuda.current_stream(dev).cuda_stream,
    )
    assert rc == E_SCRATCH
    assert "static workspace" in _native.status_string(rc)
