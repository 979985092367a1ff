"""Host-side logic of the multi-GPU bench, on CPU: gloo ranks, no GPU.

Each rank of ``bench.py`` converts its own DCP rank independently; the only
cross-process steps are barriers and reductions of the timed durations and
the checks. Here two gloo processes run exactly those steps.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest

import bench

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shard_plan_assigns_every_dcp_rank_and_distinct_seeds() -> None:
    plans = [bench.shard_plan(r, 8) for r in range(8)]
    assert [p["dcp_rank"] for p in plans] == [0, 1, 2, 3, 0, 1, 2, 3]
    assert len({p["base_seed"] for p in plans}) == 8
    with pytest.raises(ValueError):
        bench.shard_plan(2, 2)


def test_reduce_max_without_dist() -> None:
    assert bench.reduce_max(None, 1.5) == 1.5


def _worker(rank: int, world: int, port: int, out_path: str) -> None:
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        plan = bench.shard_plan(rank, world)
        dist.barrier()
        value = bench.reduce_max(dist, 10.0 * (rank + 1))
        # the same collective steps, in the same order, on every rank
        fewest = bench._min_over_ranks(dist, 10_000 - rank)
        all_ok = bench._all_ranks(dist, rank != 1)
        all_true = bench._all_ranks(dist, True)
        with open(f"{out_path}.{rank}", "w") as fh:
            json.dump({"plan": plan, "max": value, "fewest": fewest, "all_ok": all_ok,
                       "all_true": all_true}, fh)
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_barrier_and_max(tmp_path) -> None:
    import torch.multiprocessing as mp

    port = _free_port()
    out = str(tmp_path / "rank")
    mp.start_processes(_worker, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    results = [json.load(open(f"{out}.{r}")) for r in range(2)]
    assert [r["plan"]["dcp_rank"] for r in results] == [0, 1]
    assert all(r["max"] == 20.0 for r in results)
    assert all(r["fewest"] == 9_999 for r in results)
    assert all(r["all_ok"] is False and r["all_true"] is True for r in results)


def test_traffic_is_used_only_for_the_kernel_source_it_was_captured_from(tmp_path, monkeypatch) -> None:
    data = {"kernel_sha256": bench.kernel_digest(), "configs": {"3": {"read": 100, "write": 20}}}
    path = tmp_path / "traffic.json"
    path.write_text(json.dumps(data))
    monkeypatch.setattr(bench, "TRAFFIC_FILE", str(path))
    assert bench._traffic(3)["bytes"] == 120
    assert bench._traffic(4)["bytes"] is None
    data["kernel_sha256"] = "0" * 64
    path.write_text(json.dumps(data))
    stale = bench._traffic(3)
    assert stale["bytes"] is None and "predates" in stale["source"]
    monkeypatch.setattr(bench, "TRAFFIC_FILE", str(tmp_path / "missing.json"))
    assert bench._traffic(3)["bytes"] is None


def test_reference_arm_line_on_cpu() -> None:
    proc = subprocess.run(
        [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "2",
         "--warmup", "1"],
        capture_output=True, text=True, timeout=300, check=True,
    )
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["unit"] == "Gindices/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def test_reference_arm_steps_are_calibrated_samples(monkeypatch) -> None:
    """A reference step is R whole calls, R sized so the K steps take about
    REFERENCE_SECONDS; the line's rate, per-step and per-call times agree."""
    import argparse
    import re

    monkeypatch.setattr(bench, "REFERENCE_SECONDS", 0.5)
    args = argparse.Namespace(config=3, steps=4, warmup=1)
    line = bench.run_reference(args, 0, 1)
    reps = int(re.search(r"of (\d+) full workload steps", line["cpu_baseline"]["sample"]).group(1))
    assert reps >= 1 and line["steps"] == 4
    indices = 256 * 2048
    assert line["value"] == pytest.approx(reps * indices / (line["ms_per_step"] * 1e-3) / 1e9, rel=1e-9)
    assert line["us_per_call"] == pytest.approx(line["ms_per_step"] * 1e3 / reps, rel=1e-9)
    assert line["e2e"]["value"] == line["value"] == line["cpu_baseline"]["value"]


def test_reference_arm_other_ranks_print_nothing() -> None:
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    proc = subprocess.run(
        [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "0"],
        capture_output=True, text=True, timeout=300, check=True, env=env,
    )
    assert proc.stdout.strip() == ""


def test_stacked_rows_repeat_the_case_in_order() -> None:
    """`--rows R`: a call of R rows is the config's rows repeated, with the
    requests repeated alongside and the block table unchanged."""
    import numpy as np

    from silkern_b200.workloads import config_case

    case = config_case(2, seed=3)
    stacked = bench._stack_rows(case, 150)
    assert stacked.tokens.shape == (150, case.width)
    assert stacked.req_ids.shape == (150,)
    assert np.array_equal(stacked.tokens[:64], case.tokens)
    assert np.array_equal(stacked.tokens[64:128], case.tokens)
    assert np.array_equal(stacked.tokens[128:], case.tokens[:22])
    assert np.array_equal(stacked.req_ids[64:128], case.req_ids)
    assert stacked.block_table is case.block_table
    assert stacked.geometry() == case.geometry()
    assert stacked.tokens.flags.c_contiguous and stacked.req_ids.flags.c_contiguous


def test_cli_accepts_the_sizing_and_lane_options() -> None:
    """The options that size the work parse, with the defaults the bench
    documents (the run itself needs a GPU)."""
    import argparse

    seen = {}

    def fake_parse(self, argv=None, namespace=None):
        args = original(self, argv, namespace)
        seen.update(vars(args))
        raise SystemExit(0)

    original = argparse.ArgumentParser.parse_args
    argparse.ArgumentParser.parse_args = fake_parse
    try:
        with pytest.raises(SystemExit):
            bench.main(["--impl", "link", "--rows", "4096", "--e2e-lanes", "8", "--batch", "16"])
    finally:
        argparse.ArgumentParser.parse_args = original
    assert seen["impl"] == "link" and seen["rows"] == 4096 and seen["e2e_lanes"] == 8 and seen["batch"] == 16
    seen.clear()
    argparse.ArgumentParser.parse_args = fake_parse
    try:
        with pytest.raises(SystemExit):
            bench.main([])
    finally:
        argparse.ArgumentParser.parse_args = original
    assert seen["impl"] == "ours" and seen["rows"] == 0 and seen["e2e_lanes"] == 8 and seen["config"] == 3
