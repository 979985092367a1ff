"""Buffers on a device other than the current one (needs two GPUs).

The launchers switch to the buffers' device for the call, and the library's
CUDA runtime then launches on that device's context and stream.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from silkern_b200 import localize_hierarchical, localize_rowwise, workspace_shapes  # noqa: E402
from silkern_b200.workloads import config_case  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("two CUDA devices are required", allow_module_level=True)


@pytest.mark.parametrize("device_index", [1, 0])
def test_buffers_on_a_non_current_device(device_index) -> None:
    case = config_case(2, seed=21, dcp_rank=1, batch=16)
    dev = torch.device("cuda", device_index)
    other = 1 - device_index
    req, table, tokens = (torch.as_tensor(a).to(dev) for a in (case.req_ids, case.block_table, case.tokens))
    out = torch.empty_like(tokens)
    counts = torch.empty(case.batch, dtype=torch.int32, device=dev)
    want = oracle.localize(case.req_ids, case.block_table, case.tokens, **case.geometry())
    with torch.cuda.device(other):
        localize_rowwise(req, table, tokens, out, counts, **case.geometry())
        ws = {name: torch.empty(shape, dtype=torch.int32, device=dev)
              for name, shape in workspace_shapes(case.batch, case.width).items()}
        out_h = torch.empty_like(tokens)
        counts_h = torch.empty_like(counts)
        localize_hierarchical(req, table, tokens, out_h, counts_h, ws["mapped"], ws["local_positions"],
                              ws["tile_counts"], ws["tile_offsets"], **case.geometry())
    torch.cuda.synchronize(dev)
    for got_out, got_counts in ((out, counts), (out_h, counts_h)):
        assert np.array_equal(got_out.cpu().numpy(), want[0])
        assert np.array_equal(got_counts.cpu().numpy(), want[1])


@pytest.mark.parametrize("device_index", [1, 0])
def test_fused_topk_on_a_non_current_device(device_index) -> None:
    """The fused launcher's per-device state (SM count, shared-memory opt-in)
    follows the buffers' device; both CTA shapes run there."""
    from oracle.topk import topk_localize as oracle_topk
    from silkern_b200 import topk_localize

    rng = np.random.default_rng(31 + device_index)
    dev = torch.device("cuda", device_index)
    other = 1 - device_index
    batch, width, top_k = 6, 20000, 1024
    logits = rng.standard_normal((batch, width)).astype(np.float32)
    lens = rng.integers(0, width + 1, size=batch).astype(np.int32)
    table = rng.integers(-5, 1 << 20, size=(4, 400)).astype(np.int32)
    req = rng.integers(0, 4, size=batch).astype(np.int32)
    kw = dict(block_size=32, dcp_size=2, dcp_rank=1)
    want = oracle_topk(logits, lens, req, table, top_k=top_k, **kw)
    for threads in (0, 512):
        out = torch.empty((batch, top_k), dtype=torch.int32, device=dev)
        counts = torch.empty(batch, dtype=torch.int32, device=dev)
        with torch.cuda.device(other):
            topk_localize(torch.as_tensor(logits).to(dev), torch.as_tensor(lens).to(dev),
                          torch.as_tensor(req).to(dev), torch.as_tensor(table).to(dev), out, counts,
                          cta_threads=threads, **kw)
        torch.cuda.synchronize(dev)
        assert np.array_equal(out.cpu().numpy(), want[1]), threads
        assert np.array_equal(counts.cpu().numpy(), want[2]), threads
