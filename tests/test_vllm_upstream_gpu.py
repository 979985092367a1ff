"""The CUDA converter against vLLM's own converter, both on the GPU, at ``dcp_size == 1``.

At ``dcp_size == 1`` the reference contract (silkern/contract.py:67-158) and
vLLM's ``triton_convert_req_index_to_global_index``
(vllm/v1/attention/backends/mla/sparse_utils.py, ``return_valid_counts=True``)
are the same function; the fixtures recorded from vLLM and, where vLLM is
installed, vLLM's kernel run natively beside ours on full-size inputs, must
agree bit for bit with both entry points.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from conftest import GOLDEN_DIR, golden_inputs  # noqa: E402
from silkern_b200 import localize_hierarchical, localize_rowwise, workspace_shapes  # noqa: E402
from silkern_b200.verify import _random_case  # noqa: E402
from silkern_b200.workloads import config_case, digest  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA is required", allow_module_level=True)

with open(os.path.join(GOLDEN_DIR, "vllm_golden.json")) as _fh:
    CASES = json.load(_fh)["cases"]


def _dev(array):
    return torch.as_tensor(np.ascontiguousarray(array, dtype=np.int32)).cuda()


def _ours(req, table, tokens, *, block_size, arm, tile_size=128):
    batch, width = tokens.shape
    out = torch.empty_like(tokens)
    counts = torch.empty(batch, dtype=torch.int32, device=tokens.device)
    kw = dict(block_size=block_size, dcp_size=1, dcp_rank=0)
    if arm == "rowwise":
        localize_rowwise(req, table, tokens, out, counts, **kw)
    else:
        ws = {name: torch.empty(shape, dtype=torch.int32, device=tokens.device)
              for name, shape in workspace_shapes(batch, width, tile_size=tile_size).items()}
        localize_hierarchical(req, table, tokens, out, counts, ws["mapped"], ws["local_positions"],
                              ws["tile_counts"], ws["tile_offsets"], tile_size=tile_size, **kw)
    return out, counts


@pytest.mark.parametrize("arm", ["rowwise", "hierarchical"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"config{c['config']}" if c["kind"] == "config"
                         else f"w{c['width']}-bs{c['block_size']}-g{c['gen_dcp_size']}")
def test_matches_recorded_vllm_outputs(case, arm) -> None:
    req, table, tokens = (_dev(a) for a in golden_inputs(case))
    out, counts = _ours(req, table, tokens, block_size=case["block_size"], arm=arm)
    torch.cuda.synchronize()
    assert digest(out.cpu().numpy(), counts.cpu().numpy()) == case["vllm_sha256"]


def _live_inputs(name):
    if name.startswith("config"):
        case = config_case(int(name[-1]), seed=11, dcp_rank=0)
        return case.req_ids, case.block_table, case.tokens, 64
    if name == "dense":
        # every position of a 16384-token sequence is mapped; 5% padding
        rng = np.random.default_rng(661002)
        table = rng.permutation(65536)[: 256 * 256].reshape(256, 256)
        tokens = np.stack([rng.permutation(16384)[:2048] for _ in range(256)])
        tokens[rng.random(tokens.shape) < 0.05] = -1
        return np.arange(256), table, tokens, 64
    req, table, rows = _random_case(width=2048, batch=64, block_size=32, dcp_size=1, seed=661001)
    return np.asarray(req), np.asarray(table), np.asarray(rows), 32


@pytest.mark.parametrize("name", ["config3", "config4", "config5", "dense", "adversarial"])
def test_matches_vllm_kernel_on_device(name) -> None:
    sparse_utils = pytest.importorskip("vllm.v1.attention.backends.mla.sparse_utils")
    req_np, table_np, tokens_np, block_size = _live_inputs(name)
    req, table, tokens = _dev(req_np), _dev(table_np), _dev(tokens_np)
    want_out, want_counts = sparse_utils.triton_convert_req_index_to_global_index(
        req, table, tokens, BLOCK_SIZE=block_size, NUM_TOPK_TOKENS=tokens.shape[1],
        return_valid_counts=True)
    tile = 1024 if tokens.shape[1] > 4096 else 128
    for arm in ("rowwise", "hierarchical"):
        out, counts = _ours(req, table, tokens, block_size=block_size, arm=arm, tile_size=tile)
        assert torch.equal(out, want_out), (name, arm)
        assert torch.equal(counts, want_counts), (name, arm)
    assert int(want_counts.sum()) > 0
