"""The atomic-reservation baseline (comparison only) against the oracle and the stable kernel.

Restates the reference's bench/order_instability.py check: on byte-identical
input the stable converter returns one output order every time; the atomic
baseline returns the same set and count, in an order that is free to change.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from silkern_b200 import localize_rowwise  # noqa: E402
from silkern_b200.baselines import launch_atomic_baseline  # noqa: E402
from silkern_b200.workloads import config_case  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA is required", allow_module_level=True)


def _buffers(case):
    dev = torch.device("cuda")
    req, table, tokens = (torch.as_tensor(a).to(dev) for a in (case.req_ids, case.block_table, case.tokens))
    return (req, table, tokens, torch.empty_like(tokens),
            torch.empty(case.batch, dtype=torch.int32, device=dev),
            torch.empty(case.batch, dtype=torch.int32, device=dev))


def _sorted_prefixes(out, counts):
    return [sorted(row[:c]) for row, c in zip(out.tolist(), counts.tolist(), strict=True)]


@pytest.mark.parametrize("config", [1, 2, 3])
def test_atomic_baseline_has_the_oracle_set_and_count(config) -> None:
    case = config_case(config, seed=7, dcp_rank=1)
    req, table, tokens, out, counts, scratch = _buffers(case)
    launch_atomic_baseline(req, table, tokens, out, counts, scratch, **case.geometry())
    torch.cuda.synchronize()
    want_out, want_counts = oracle.localize(case.req_ids, case.block_table, case.tokens, threads=4,
                                            **case.geometry())
    got_out, got_counts = out.cpu().numpy(), counts.cpu().numpy()
    assert np.array_equal(got_counts, want_counts)
    assert _sorted_prefixes(got_out, got_counts) == _sorted_prefixes(want_out, want_counts)
    for row, count in zip(got_out, got_counts, strict=True):
        assert np.all(row[count:] == -1)


def test_order_instability_stable_vs_atomic() -> None:
    case = config_case(3, seed=11, dcp_rank=0, batch=8)
    req, table, tokens, out, counts, scratch = _buffers(case)
    stable, atomic_orders, atomic_sets = set(), set(), set()
    for _ in range(20):
        localize_rowwise(req, table, tokens, out, counts, **case.geometry())
        torch.cuda.synchronize()
        stable.add(hashlib.sha256(out.cpu().numpy().tobytes()).hexdigest())
        launch_atomic_baseline(req, table, tokens, out, counts, scratch, **case.geometry())
        torch.cuda.synchronize()
        atomic_orders.add(hashlib.sha256(out.cpu().numpy().tobytes()).hexdigest())
        atomic_sets.add(repr(_sorted_prefixes(out.cpu().numpy(), counts.cpu().numpy())))
    assert len(stable) == 1
    assert len(atomic_sets) == 1
    print(f"distinct output orders over 20 runs: stable {len(stable)}, atomic {len(atomic_orders)}")
