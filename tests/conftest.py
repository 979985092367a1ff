"""Shared test setup: repository root on sys.path, the ``gpu`` marker, fixtures."""

from __future__ import annotations

import json
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN_DIR = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (B200) and the built library (deselect with -m 'not gpu')"
    )


def load_golden() -> dict:
    with open(os.path.join(GOLDEN_DIR, "golden.json")) as fh:
        return json.load(fh)


def golden_inputs(entry: dict):
    """Regenerate the inputs of one golden case (numpy int32 arrays)."""
    import numpy as np

    from silkern_b200.verify import _random_case
    from silkern_b200.workloads import config_case

    if entry["kind"] == "random_case":
        req_ids, table, rows = _random_case(
            width=entry["width"],
            batch=entry["batch"],
            block_size=entry["block_size"],
            dcp_size=entry["gen_dcp_size"],
            seed=entry["seed"],
        )
        return (np.asarray(req_ids, dtype=np.int32), np.asarray(table, dtype=np.int32),
                np.asarray(rows, dtype=np.int32))
    case = config_case(entry["config"], seed=entry["seed"], dcp_rank=entry["dcp_rank"],
                       batch=entry["batch_limit"])
    return case.req_ids, case.block_table, case.tokens


def input_sha(req_ids, table, tokens) -> str:
    import hashlib

    import numpy as np

    h = hashlib.sha256()
    for array in (req_ids, table, tokens):
        h.update(np.ascontiguousarray(array, dtype="<i4").tobytes())
    return h.hexdigest()


@pytest.fixture(scope="session")
def golden() -> dict:
    return load_golden()
