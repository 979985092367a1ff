"""The oracle against vLLM's own sparse index converter at ``dcp_size == 1``.

vLLM's ``triton_convert_req_index_to_global_index``
(vllm/v1/attention/backends/mla/sparse_utils.py) is the non-DCP ancestor of
the converter the reference's adapter replaces (silkern/integrations/vllm.py).
At ``dcp_size == 1`` it computes the reference contract exactly
(silkern/contract.py:67-158 with every token owned and no compaction), so its
recorded outputs in ``tests/golden/vllm_golden.json`` pin the oracle and the
pure-Python ``localize_reference`` to upstream code, and a live run through the
Triton interpreter shows the fixtures still match the installed vLLM.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from conftest import GOLDEN_DIR, REPO, golden_inputs, input_sha

np = pytest.importorskip("numpy")


def _load():
    with open(os.path.join(GOLDEN_DIR, "vllm_golden.json")) as fh:
        return json.load(fh)


CASES = _load()["cases"]


def _case_id(case) -> str:
    if case["kind"] == "config":
        return f"config{case['config']}"
    return f"w{case['width']}-bs{case['block_size']}-g{case['gen_dcp_size']}"


@pytest.mark.parametrize("case", CASES, ids=_case_id)
@pytest.mark.parametrize("compact", [True, False])
def test_oracle_matches_vllm_converter(case, compact: bool) -> None:
    import oracle
    from silkern_b200.workloads import digest

    req_ids, table, tokens = golden_inputs(case)
    assert input_sha(req_ids, table, tokens) == case["input_sha256"]
    out, counts = oracle.localize(req_ids, table, tokens, block_size=case["block_size"], dcp_size=1,
                                  dcp_rank=0, compact_valid_to_front=compact)
    assert int(counts.sum()) == case["valid"]
    assert digest(out, counts) == case["vllm_sha256"]


@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "random_case"
                                  and c["width"] <= 256], ids=_case_id)
def test_localize_reference_matches_vllm_converter(case) -> None:
    from silkern_b200.contract import localize_reference
    from silkern_b200.workloads import digest

    req_ids, table, tokens = golden_inputs(case)
    out, counts = localize_reference(req_ids.tolist(), table.tolist(), tokens.tolist(),
                                     block_size=case["block_size"], dcp_size=1, dcp_rank=0)
    assert digest(np.asarray(out, dtype=np.int32), np.asarray(counts, dtype=np.int32)) \
        == case["vllm_sha256"]


def test_fixtures_reproduce_with_installed_vllm(tmp_path) -> None:
    """Re-run the fixture script against the installed vLLM (Triton interpreter)."""
    pytest.importorskip("vllm")
    pytest.importorskip("triton")
    recorded = _load()
    target = tmp_path / "vllm_golden.json"
    script = os.path.join(GOLDEN_DIR, "make_vllm_golden.py")
    env = dict(os.environ, TRITON_INTERPRET="1", CUDA_VISIBLE_DEVICES="")
    subprocess.run([sys.executable, script, "--out", str(target)], cwd=REPO, env=env, check=True,
                   capture_output=True, timeout=600)
    fresh = json.loads(target.read_text())
    if fresh["sparse_utils_source_sha256"] != recorded["sparse_utils_source_sha256"]:
        pytest.skip(f"installed vLLM {fresh['vllm_version']} differs from the recorded "
                    f"{recorded['vllm_version']}")
    assert [c["vllm_sha256"] for c in fresh["cases"]] == [c["vllm_sha256"] for c in recorded["cases"]]
