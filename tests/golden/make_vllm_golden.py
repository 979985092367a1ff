"""Record the outputs of vLLM's own sparse index converter as fixtures.

    python tests/golden/make_vllm_golden.py [--out PATH]

vLLM ships ``triton_convert_req_index_to_global_index``
(vllm/v1/attention/backends/mla/sparse_utils.py), the converter that the
DCP-aware ``triton_filter_and_convert_dcp_index`` targeted by the reference's
adapter (silkern/integrations/vllm.py:1-25) grew out of. The installed
revision has no DCP variant, but at ``dcp_size == 1`` the two contracts are the
same function: every token is owned, ``local = t``, ``lb, off = divmod(t,
block_size)``, an element is valid iff ``t >= 0`` and ``lb < table_width``,
``phys = table[req][lb] * block_size + off`` in int32 (negative table entries
pass through verbatim), invalid elements are ``-1`` in place (no compaction at
``dcp_size == 1``, silkern/contract.py:126), and the count is the number of
valid elements (``return_valid_counts=True``).

This script runs that vLLM function through the Triton CPU interpreter
(``TRITON_INTERPRET=1``) on seeded inputs from this repository's generators and
records, per case, the sha256 of the inputs and of vLLM's ``out`` then
``counts`` (``silkern_b200.workloads.digest``). It needs vLLM and triton, not a
GPU. Output: tests/golden/vllm_golden.json.
"""

from __future__ import annotations

import argparse
import hashlib
import inspect
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

# Seeded cases: (kind, parameters). Widths are multiples of vLLM's BLOCK_N=128.
RANDOM_CASES = [
    {"width": width, "block_size": block_size, "gen_dcp_size": gen_dcp, "batch": 4,
     "seed": 660000 + 100 * i + 10 * j + k}
    for i, width in enumerate((128, 256, 1024, 2048))
    for j, block_size in enumerate((32, 64))
    for k, gen_dcp in enumerate((1, 2))
]
CONFIG_CASES = [
    {"config": 1, "seed": 0, "batch_limit": None},
    {"config": 2, "seed": 2, "batch_limit": 8},
    {"config": 3, "seed": 3, "batch_limit": 8},
    {"config": 5, "seed": 5, "batch_limit": 8},
]


def _inputs(entry):
    sys.path.insert(0, REPO)
    from tests.conftest import golden_inputs

    return golden_inputs(entry)


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--out", default=os.path.join(HERE, "vllm_golden.json"))
    args = parser.parse_args(argv)
    os.environ["TRITON_INTERPRET"] = "1"
    sys.dont_write_bytecode = True
    sys.path.insert(0, REPO)
    import numpy as np
    import torch
    import vllm
    from vllm.v1.attention.backends.mla import sparse_utils

    from silkern_b200.workloads import digest
    from tests.conftest import input_sha

    source = inspect.getsource(sparse_utils).encode()
    entries = []
    for params in RANDOM_CASES:
        entries.append({"kind": "random_case", "dcp_rank": 0, **params})
    for params in CONFIG_CASES:
        entries.append({"kind": "config", "dcp_rank": 0, **params})

    cases = []
    start = time.time()
    for entry in entries:
        req_ids, table, tokens = _inputs(entry)
        block_size = entry.get("block_size", 64)
        out, counts = sparse_utils.triton_convert_req_index_to_global_index(
            torch.from_numpy(np.ascontiguousarray(req_ids)),
            torch.from_numpy(np.ascontiguousarray(table)),
            torch.from_numpy(np.ascontiguousarray(tokens)),
            BLOCK_SIZE=block_size,
            NUM_TOPK_TOKENS=tokens.shape[1],
            return_valid_counts=True,
        )
        case = dict(entry)
        case.update(
            block_size=block_size,
            shape=[int(tokens.shape[0]), int(tokens.shape[1])],
            input_sha256=input_sha(req_ids, table, tokens),
            vllm_sha256=digest(out.numpy(), counts.numpy()),
            valid=int(counts.sum()),
        )
        cases.append(case)
        print(f"{entry.get('config', 'random')} {tokens.shape} valid={case['valid']} "
              f"{time.time() - start:.1f}s", flush=True)

    payload = {
        "function": "vllm.v1.attention.backends.mla.sparse_utils."
                    "triton_convert_req_index_to_global_index",
        "vllm_version": vllm.__version__,
        "sparse_utils_source_sha256": hashlib.sha256(source).hexdigest(),
        "block_n": 128,
        "cases": cases,
    }
    with open(args.out, "w") as fh:
        json.dump(payload, fh, indent=1)
        fh.write("\n")
    print(args.out)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
