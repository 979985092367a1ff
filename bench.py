"""Benchmark of the localization converter on B200: the headline selection batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1)

Workload (one step = one converter call): a selection batch of 256 requests x
top_k 2048 int32 positions, per-request context U[1024, 65536] (shorter rows
padded with -1), block_size 64, dcp_size 4, block table (256, 256) over a
65536-block pool; seeded synthetic data. Each GPU runs the DCP rank
``gpu_index % 4`` on its own inputs, with no collective on the data path, so
the per-GPU work is fixed as N grows (weak scaling); rank processes meet only
on a host barrier and a max-reduction of the timed duration.

Timed region (our arm): K row-wise calls captured in CUDA graphs and replayed
on one stream, bracketed by CUDA events; inputs rotate over 64 resident
buffer sets (about 275 MB, more than twice the 126 MB L2), so every call
reads cold data. ``value`` is localized indices per second over all GPUs;
``e2e`` is the same metric through the public Python API with the inputs
copied from pinned host memory and the results copied back every step.
After timing, every buffer set's output is compared with the oracle.

``--impl reference`` times the reference algorithm on the host instead: the C
restatement of the reference's ``localize_reference`` (oracle/) with every
host thread, on the same workload (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

CONFIG = 3
DCP_SIZE = 4
BUFFER_SETS = 64
DISTINCT_CASES = 8
CHUNK = 256  # calls per captured graph
METRIC = "Gindices/s per B200 at 256x2048 (localized selection indices per second)"
UNIT = "Gindices/s"


def _peaks() -> dict:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            data = json.load(fh)
        return {"hbm_gbs": float(data["hbm_gbs"]), "source": "measured (MEASURED_PEAKS.json)"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "source": "fallback"}


def _workload_config(rank: int, world: int) -> dict:
    return {
        "workload": "config3: batch 256 x top_k 2048 int32, seq U[1024,65536] with -1 padding, "
                    "block_size 64, dcp_size 4, table (256,256)",
        "batch": 256,
        "top_k": 2048,
        "dcp_size": DCP_SIZE,
        "dcp_rank": "gpu_index % 4",
        "block_size": 64,
        "arm": "row_stable (localize_rowwise)",
        "l2": f"inputs larger than L2: {BUFFER_SETS} rotating buffer sets",
        "parallelism": f"{world} independent DCP-rank shards, no data-path collective",
    }


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle",
        0x2: "applications_clocks_setting",
        0x4: "sw_power_cap",
        0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.period = period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report no clocks
            self._nvml = None

    def _sample(self):
        n = self._nvml
        sm = n.nvmlDeviceGetClockInfo(self._handle, n.NVML_CLOCK_SM)
        reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
        self.samples.append((sm, reasons))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._sample()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
            self._sample()

    def summary(self) -> dict | None:
        if not self.samples:
            return None
        mask = 0
        for _, reasons in self.samples:
            mask |= reasons
        names = sorted(name for bit, name in self.REASONS.items() if mask & bit and name != "gpu_idle")
        return {
            "sm_mhz": statistics.median(s for s, _ in self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": names,
            "samples": len(self.samples),
        }


def _cpu_baseline(threads: int, seconds: float = 2.0) -> dict:
    """The C oracle (restatement of the reference's localize_reference) on host cores."""
    import oracle
    from silkern_b200.workloads import config_case

    case = config_case(CONFIG, seed=0, dcp_rank=0)
    kw = case.geometry()
    oracle.localize(case.req_ids, case.block_table, case.tokens, threads=threads, **kw)
    calls = 0
    start = time.perf_counter()
    while True:
        oracle.localize(case.req_ids, case.block_table, case.tokens, threads=threads, **kw)
        calls += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds and calls >= 3:
            break
    rate = calls * case.batch * case.width / elapsed / 1e9
    return {
        "value": rate,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{calls} full calls of the 256x2048 dcp-4 rank-0 batch in {elapsed:.2f} s "
                  f"({threads} threads, oracle/localize_oracle.c)",
    }


def shard_plan(rank: int, world: int) -> dict:
    """What one rank converts: its DCP rank and the seed of its own inputs.

    Ranks are independent shards (no data is exchanged); rank r converts the
    DCP rank r % 4 on inputs seeded by its global rank.
    """
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return {"dcp_rank": rank % DCP_SIZE, "base_seed": 1000 * (rank + 1)}


def reduce_max(dist, value: float) -> float:
    """Max of a host float over all ranks (gloo), or the value itself without dist."""
    if dist is None:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def run_reference(args, rank: int, world: int) -> dict | None:
    if rank != 0:
        return None
    import oracle
    from silkern_b200.workloads import config_case

    threads = _host_threads()
    case = config_case(CONFIG, seed=0, dcp_rank=0)
    kw = case.geometry()
    for _ in range(args.warmup):
        oracle.localize(case.req_ids, case.block_table, case.tokens, threads=threads, **kw)
    start = time.perf_counter()
    for _ in range(args.steps):
        oracle.localize(case.req_ids, case.block_table, case.tokens, threads=threads, **kw)
    elapsed = time.perf_counter() - start
    per_step = elapsed / args.steps
    value = case.batch * case.width / per_step / 1e9
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_step * 1e3,
        "us_per_call": per_step * 1e6,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int32",
        "data": "synthetic (seeded)",
        "config": _workload_config(0, 1),
        "cpu_baseline": {
            "value": value,
            "unit": UNIT,
            "cores": threads,
            "kind": "port",
            "sample": f"{args.steps} full calls of the 256x2048 dcp-4 rank-0 batch, {threads} threads "
                      "(C restatement of silkern/contract.py:67-158 in oracle/localize_oracle.c)",
        },
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_ours(args, rank: int, world: int, local_rank: int, dist) -> dict | None:
    import numpy as np
    import torch

    import oracle
    import silkern_b200 as silkern
    from silkern_b200.kernels import localize_rowwise
    from silkern_b200.workloads import config_case

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    plan = shard_plan(rank, world)
    dcp_rank = plan["dcp_rank"]
    base_seed = plan["base_seed"]

    # Distinct seeded cases, laid out in BUFFER_SETS separate resident buffer sets.
    cases = [config_case(CONFIG, seed=base_seed + i, dcp_rank=dcp_rank) for i in range(DISTINCT_CASES)]
    sets = []
    for i in range(BUFFER_SETS):
        case = cases[i % DISTINCT_CASES]
        req, table, tokens = (torch.as_tensor(a).to(dev) for a in (case.req_ids, case.block_table, case.tokens))
        out = torch.empty_like(tokens)
        counts = torch.empty(case.batch, dtype=torch.int32, device=dev)
        sets.append((req, table, tokens, out, counts))
    geometry = cases[0].geometry()
    algorithmic = cases[0].algorithmic_bytes()
    indices_per_call = cases[0].batch * cases[0].width

    def call(i: int) -> None:
        req, table, tokens, out, counts = sets[i % BUFFER_SETS]
        localize_rowwise(req, table, tokens, out, counts, **geometry)

    # Eager warm-up (also loads the library and its kernels) on a side stream.
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for i in range(max(3, BUFFER_SETS)):
            call(i)
    torch.cuda.synchronize(dev)

    def capture(first: int, count: int):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(first, first + count):
                call(i)
        return graph

    def plan(steps: int):
        graphs = []
        done = 0
        while done < steps:
            count = min(CHUNK, steps - done)
            graphs.append(capture(done, count))
            done += count
        return graphs

    warm_graphs = plan(args.warmup)
    main_graphs = plan(args.steps)
    torch.cuda.synchronize(dev)

    with torch.cuda.stream(stream):
        for g in warm_graphs:
            g.replay()
    torch.cuda.synchronize(dev)

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local_rank)
    with sampler:
        with torch.cuda.stream(stream):
            torch.cuda._sleep(200_000)  # keep the GPU busy while the replays are queued
            start.record(stream)
            for g in main_graphs:
                g.replay()
            end.record(stream)
        torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    elapsed_ms = reduce_max(dist, start.elapsed_time(end))
    per_call_s = elapsed_ms / 1e3 / args.steps

    # The timed outputs must be the reference's: check every buffer set.
    expected = [oracle.localize(c.req_ids, c.block_table, c.tokens, threads=4, **c.geometry())
                for c in cases]
    bit_exact = True
    last_use = {}
    for i in range(args.steps):
        last_use[i % BUFFER_SETS] = True
    for index, (_, _, _, out, counts) in enumerate(sets):
        if index not in last_use:
            continue
        want_out, want_counts = expected[index % DISTINCT_CASES]
        if not (np.array_equal(out.cpu().numpy(), want_out)
                and np.array_equal(counts.cpu().numpy(), want_counts)):
            bit_exact = False
    del warm_graphs, main_graphs

    e2e = run_e2e(args, cases[0], dev, geometry, dist)

    value = world * indices_per_call / per_call_s / 1e9
    peaks = _peaks()
    achieved = algorithmic / per_call_s / 1e9
    result = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_call_s * 1e3,
        "us_per_call": per_call_s * 1e6,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int32",
        "data": "synthetic (seeded; config 3 shapes)",
        "config": _workload_config(rank, world),
        "bit_exact": bit_exact,
        "hbm_gbs": achieved,
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"],
            "traffic": None,
            "algorithmic_bytes_per_call": algorithmic,
            "peak_source": peaks["source"],
            "timing": "CUDA events around the graph replays of the timed calls, per call",
        },
        "gpu_launches": args.steps,
        "e2e": e2e,
        "clocks": sampler.summary(),
        "library": silkern._native.LIB_PATH if hasattr(silkern, "_native") else None,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = _cpu_baseline(_host_threads())
    return result if rank == 0 else None


def run_e2e(args, case, dev, geometry, dist) -> dict:
    """Same metric through the public API, host inputs in and results out every step."""
    import torch

    from silkern_b200.kernels import localize_rowwise

    steps = args.e2e_steps if args.e2e_steps > 0 else args.steps
    batch, width = case.tokens.shape
    n_req, n_table = case.req_ids.size, case.block_table.size
    n_in = n_req + n_table + case.tokens.size
    host_in = torch.empty(n_in, dtype=torch.int32).pin_memory()
    host_in[:n_req] = torch.as_tensor(case.req_ids)
    host_in[n_req:n_req + n_table] = torch.as_tensor(case.block_table.ravel())
    host_in[n_req + n_table:] = torch.as_tensor(case.tokens.ravel())
    lanes = []
    for _ in range(2):
        # Inputs share one device buffer (one H2D copy); the two outputs must
        # not share storage, so they come back in two D2H copies.
        dev_in = torch.empty(n_in, dtype=torch.int32, device=dev)
        out = torch.empty((batch, width), dtype=torch.int32, device=dev)
        counts = torch.empty(batch, dtype=torch.int32, device=dev)
        host_out = torch.empty((batch, width), dtype=torch.int32).pin_memory()
        host_counts = torch.empty(batch, dtype=torch.int32).pin_memory()
        req = dev_in[:n_req]
        table = dev_in[n_req:n_req + n_table].view(case.block_table.shape)
        tokens = dev_in[n_req + n_table:].view(batch, width)
        lanes.append((torch.cuda.Stream(device=dev), dev_in, req, table, tokens, out, counts,
                      host_out, host_counts))

    def step(i: int) -> None:
        stream, dev_in, req, table, tokens, out, counts, host_out, host_counts = lanes[i % 2]
        with torch.cuda.stream(stream):
            dev_in.copy_(host_in, non_blocking=True)
            localize_rowwise(req, table, tokens, out, counts, **geometry)
            host_out.copy_(out, non_blocking=True)
            host_counts.copy_(counts, non_blocking=True)

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    current = torch.cuda.current_stream(dev)
    current.synchronize()
    start.record(current)
    for lane in lanes:
        lane[0].wait_event(start)
    for i in range(steps):
        step(i)
    for lane in lanes:
        current.wait_stream(lane[0])
    end.record(current)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    elapsed_ms = reduce_max(dist, start.elapsed_time(end))
    world = dist.get_world_size() if dist is not None else 1
    per_step = elapsed_ms / 1e3 / steps
    return {
        "value": world * batch * width / per_step / 1e9,
        "unit": UNIT,
        "h2d_bytes_per_step": 4 * n_in,
        "d2h_bytes_per_step": 4 * (batch * width + batch),
        "steps": steps,
        "us_per_step": per_step * 1e6,
        "path": "silkern_b200.localize_rowwise on 2 streams, pinned host buffers",
    }


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=2000)
    parser.add_argument("--warmup", type=int, default=64)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--e2e-steps", type=int, default=0, help="end-to-end steps (default: --steps)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    args = parser.parse_args(argv)
    if args.steps < 1 or args.warmup < 0:
        parser.error("--steps must be >= 1 and --warmup >= 0")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        result = run_reference(args, rank, world)
        if result is not None:
            print(json.dumps(result), flush=True)
        return 0

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as torch_dist

        torch_dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        dist = torch_dist
    try:
        result = run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
