"""Benchmark of the localization converter on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--impl ours|reference|triton|vllm|fused|atomic|link] [--config C] [--batch B]
                    [--rows R] [--e2e-steps S] [--e2e-lanes L] [--no-cpu-baseline]
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1)

Default workload (config 3, one step = one converter call): a selection batch
of 256 requests x top_k 2048 int32 positions, per-request context
U[1024, 65536] (shorter rows padded with -1), block_size 64, dcp_size 4, block
table (256, 256) over a 65536-block pool; seeded synthetic data. Other
configs: 2 (64 x 2048, dcp 2), 4 (32 x 16384 through the hierarchical entry
point, tile 1024, dcp 8) and 5 (one step = a 48-layer decode step, 48 calls of
128 x 2048, dcp 8).

Each GPU runs the DCP rank ``gpu_index % dcp_size`` on its own inputs, with no
collective on the data path, so the per-GPU work is fixed as N grows (weak
scaling); rank processes meet only on a host barrier and a max-reduction of
the timed duration.

Timed region (our arm): W warm-up steps, then exactly K steps, all captured in
CUDA graphs and replayed on one stream, bracketed by CUDA events. Inputs
rotate over enough resident buffer sets to exceed twice the 126 MB L2, so
every call reads data that is not already in L2. ``value`` is localized
indices per second over all GPUs; ``e2e`` is the same metric through the
public Python API with the inputs copied from pinned host memory and the
results copied back every step. After timing, every buffer set's output is
compared with the oracle (``bit_exact``).

``--impl reference`` times the reference algorithm on the host instead: the C
restatement of the reference's ``localize_reference`` (oracle/) with every
host thread, on the same workload (rank 0 only). ``--impl triton`` times the
reference's own Triton launchers on this GPU when the reference package is
present under baseline/_ref (a comparison arm; not part of the product).
``--impl vllm`` times vLLM's own non-DCP converter beside ours on the
workload's shapes at dcp_size 1, where the two compute the same function.
``--impl fused`` times the fused indexer top-k + localization kernel on
256 x 65536 logits (top_k 2048, dcp 4; ``--batch`` sets the rows) beside
vLLM's top-k followed by the converter. ``--impl link`` times the end-to-end
step's host copies alone, the host link's ceiling for ``e2e``.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

L2_BYTES = 126 * 1024 * 1024
DISTINCT_CASES = 8
CHUNK = 256  # launches per captured graph
UNIT = "Gindices/s"
METRIC = "Gindices/s per B200 at 256x2048 (localized selection indices per second)"

WORKLOADS = {
    2: {"desc": "config2: batch 64 x top_k 2048 int32, seq 32768, block_size 64, dcp_size 2, "
                "table (64,256)", "dcp_size": 2, "calls": 1, "arm": "row_stable"},
    3: {"desc": "config3: batch 256 x top_k 2048 int32, seq U[1024,65536] with -1 padding, "
                "block_size 64, dcp_size 4, table (256,256)", "dcp_size": 4, "calls": 1,
        "arm": "row_stable"},
    4: {"desc": "config4: batch 32 x top_k 16384 int32, seq 131072, hierarchical tile 1024, "
                "block_size 64, dcp_size 8, table (32,256)", "dcp_size": 8, "calls": 1,
        "arm": "hierarchical_stable"},
    5: {"desc": "config5: 48-layer decode step, each layer batch 128 x top_k 2048 int32, "
                "seq 32768, block_size 64, dcp_size 8, table (128,64)", "dcp_size": 8, "calls": 48,
        "arm": "row_stable"},
}


def _peaks() -> dict:
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as fh:
            data = json.load(fh)
        return {"hbm_gbs": float(data["hbm_gbs"]), "source": "measured (MEASURED_PEAKS.json)"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "source": "fallback"}


TRAFFIC_FILE = os.path.join(REPO, "profiles", "dram_traffic.json")
KERNEL_SOURCE = os.path.join(REPO, "silkern_b200", "csrc", "localize.cu")


def kernel_digest() -> str:
    """sha256 of the converter kernel's code (its source without comments or
    whitespace, so an edited comment keeps a capture current), which a
    traffic capture is tied to."""
    import hashlib

    with open(KERNEL_SOURCE) as fh:
        code = re.sub(r"//[^\n]*", "", fh.read())
    return hashlib.sha256("".join(code.split()).encode()).hexdigest()


def _traffic(config: int) -> dict:
    """DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)
    for this workload from the capture data file, when that capture was taken
    of the current kernel source; otherwise bytes None and the reason."""
    try:
        with open(TRAFFIC_FILE) as fh:
            data = json.load(fh)
    except (OSError, ValueError):
        return {"bytes": None, "source": "no capture data"}
    entry = data.get("configs", {}).get(str(config))
    if entry is None:
        return {"bytes": None, "source": f"no capture of config {config}"}
    if data.get("kernel_sha256") != kernel_digest():
        return {"bytes": None, "source": "capture predates the current kernel source"}
    return {"bytes": int(entry["read"]) + int(entry["write"]), "read": int(entry["read"]),
            "write": int(entry["write"]), "source": os.path.relpath(TRAFFIC_FILE, REPO)}


def _case(config: int, *, seed: int, dcp_rank: int):
    from silkern_b200.workloads import config_case

    return config_case(config, seed=seed, dcp_rank=dcp_rank)


def _workload_config(config: int, world: int, n_sets: int) -> dict:
    w = WORKLOADS[config]
    case = _case(config, seed=0, dcp_rank=0)
    return {
        "workload": w["desc"],
        "batch": case.batch,
        "top_k": case.width,
        "dcp_size": w["dcp_size"],
        "dcp_rank": f"gpu_index % {w['dcp_size']}",
        "block_size": case.block_size,
        "calls_per_step": w["calls"],
        "arm": w["arm"],
        "l2": f"inputs larger than L2: {n_sets} rotating buffer sets",
        "parallelism": f"{world} independent DCP-rank shards, no data-path collective",
    }


def shard_plan(rank: int, world: int, config: int = 3) -> dict:
    """What one rank converts: its DCP rank and the seed of its own inputs.

    Ranks are independent shards (no data is exchanged); rank r converts the
    DCP rank r % dcp_size on inputs seeded by its global rank.
    """
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return {"dcp_rank": rank % WORKLOADS[config]["dcp_size"], "base_seed": 1000 * (rank + 1)}


def reduce_max(dist, value: float) -> float:
    """Max of a host float over all ranks (gloo), or the value itself without dist."""
    if dist is None:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


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


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def _oracle_step(cases, threads: int) -> None:
    import oracle

    for case in cases:
        oracle.localize(case.req_ids, case.block_table, case.tokens, threads=threads, **case.geometry())


def _cpu_baseline(config: int, threads: int, seconds: float = 10.0) -> dict:
    """The C oracle (restatement of the reference's localize_reference) on host cores."""
    calls = WORKLOADS[config]["calls"]
    cases = [_case(config, seed=layer, dcp_rank=0) for layer in range(calls)]
    _oracle_step(cases[:1], threads)
    steps = 0
    start = time.perf_counter()
    while True:
        _oracle_step(cases, threads)
        steps += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds and steps >= 3:
            break
    indices = calls * cases[0].batch * cases[0].width
    return {
        "value": steps * indices / elapsed / 1e9,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{steps} full steps ({calls} call(s) of {cases[0].batch}x{cases[0].width}) in "
                  f"{elapsed:.2f} s, {threads} threads, oracle/localize_oracle.c",
    }


# Seconds the reference arm's timed steps take in all, whatever --steps is.
REFERENCE_SECONDS = 10.0


def run_reference(args, rank: int, world: int) -> dict | None:
    if rank != 0:
        return None
    config = args.config
    threads = _host_threads()
    calls = WORKLOADS[config]["calls"]
    cases = [_case(config, seed=layer, dcp_rank=0) for layer in range(calls)]
    for _ in range(max(1, args.warmup)):
        _oracle_step(cases, threads)
    # A step is `reps` full workload steps, sized so that the K timed steps
    # take about REFERENCE_SECONDS in all: a window of a few milliseconds
    # (20 single calls) measured host noise, not the port.
    t0 = time.perf_counter()
    _oracle_step(cases, threads)
    one = time.perf_counter() - t0
    reps = max(1, math.ceil(REFERENCE_SECONDS / (args.steps * max(one, 1e-6))))
    start = time.perf_counter()
    for _ in range(args.steps * reps):
        _oracle_step(cases, threads)
    elapsed = time.perf_counter() - start
    per_step = elapsed / args.steps
    indices = reps * calls * cases[0].batch * cases[0].width
    value = indices / per_step / 1e9
    return {
        "impl": "reference",
        "metric": METRIC if config == 3 else f"Gindices/s per B200, config {config}",
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_step * 1e3,
        "us_per_call": per_step * 1e6 / (reps * calls),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int32",
        "data": "synthetic (seeded)",
        "config": _workload_config(config, 1, 0),
        "cpu_baseline": {
            "value": value,
            "unit": UNIT,
            "cores": threads,
            "kind": "port",
            "sample": f"{args.steps} steps of {reps} full workload steps ({reps * calls} call(s) of "
                      f"{cases[0].batch}x{cases[0].width}) in {elapsed:.2f} s, {threads} threads (C "
                      "restatement of silkern/contract.py:67-158 in oracle/localize_oracle.c)",
        },
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def _reference_hierarchical_direct(ref_silkern, b: dict, g: dict, tile_size: int) -> None:
    """The reference's hierarchical Triton kernels, launched as its launcher does.

    Launch parameters of the reference's silkern/kernels.py:560-633, for widths
    and tile sizes its workspace checks reject.
    """
    import triton

    k = ref_silkern.kernels
    tokens, out = b["tokens"], b["out"]
    batch, width = tokens.shape
    tiles = b["tile_counts"].shape[1]
    compact = g["dcp_size"] > 1
    k._map_tiles_kernel[(batch, tiles)](
        b["req"], b["table"], tokens, out, b["mapped"], b["local_positions"], b["tile_counts"],
        b["table"].stride(0), b["table"].stride(1), tokens.stride(0), tokens.stride(1),
        out.stride(0), out.stride(1), b["mapped"].stride(0), b["mapped"].stride(1),
        b["local_positions"].stride(0), b["local_positions"].stride(1),
        b["tile_counts"].stride(0), b["tile_counts"].stride(1),
        WIDTH=width, BLOCK_TABLE_WIDTH=b["table"].shape[1], BLOCK_SIZE=g["block_size"],
        DCP_SIZE=g["dcp_size"], DCP_RANK=g["dcp_rank"], DCP_INTERLEAVE=g["dcp_interleave"],
        TILE_SIZE=tile_size, DIRECT_OUTPUT=not compact, num_warps=4)
    k._tile_prefix_kernel[(batch,)](
        b["tile_counts"], b["tile_offsets"], b["counts"], b["tile_counts"].stride(0),
        b["tile_counts"].stride(1), b["tile_offsets"].stride(0), b["tile_offsets"].stride(1),
        NUM_TILES=tiles, PADDED_TILES=triton.next_power_of_2(tiles), num_warps=1)
    if compact:
        elements = batch * width
        k._fill_output_kernel[(triton.cdiv(elements, 256),)](out, elements, BLOCK=256, num_warps=4)
        k._scatter_tiles_kernel[(batch, tiles)](
            out, b["mapped"], b["local_positions"], b["tile_counts"], b["tile_offsets"],
            out.stride(0), out.stride(1), b["mapped"].stride(0), b["mapped"].stride(1),
            b["local_positions"].stride(0), b["local_positions"].stride(1),
            b["tile_counts"].stride(0), b["tile_counts"].stride(1), b["tile_offsets"].stride(0),
            b["tile_offsets"].stride(1), WIDTH=width, TILE_SIZE=tile_size, num_warps=4)


def _replay_seconds(launch, warm_launches: int, timed_launches: int, stream, dev) -> float:
    """Device seconds taken by ``timed_launches`` calls replayed from CUDA graphs.

    ``launch(i)`` issues call ``i``. Calls ``0 .. warm_launches-1`` are the
    warm-up and the timed calls follow them in the same captured sequence (up
    to CHUNK calls per graph). The two CUDA events are recorded inside the
    graphs (external event nodes): the start event on a branch that forks
    off after the last warm-up call, so it stamps that call's completion
    without standing between it and the first timed call (which keeps its
    programmatic dependent launch), and the end event after the last timed
    call. The timed region therefore holds exactly the timed calls' work in
    steady state; the latency of launching the first graph is not in it. A
    ~1 ms device sleep ahead of the replays lets the host queue every graph
    first.
    """
    import torch

    start = torch.cuda.Event(enable_timing=True, external=True)
    end = torch.cuda.Event(enable_timing=True, external=True)
    total = warm_launches + timed_launches
    graphs = []
    first = 0
    side = torch.cuda.Stream(device=dev)
    while first < total:
        n = min(CHUNK, total - first)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            forked = False
            for i in range(first, first + n):
                if i == warm_launches:
                    if i > first:  # fork the start stamp off the last warm-up call
                        side.wait_stream(stream)
                        start.record(side)
                        forked = True
                    else:
                        start.record(stream)
                launch(i)
            if forked:
                stream.wait_stream(side)
            if first + n == total:
                end.record(stream)
        graphs.append(graph)
        first += n
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(2_000_000)
        for graph in graphs:
            graph.replay()
    torch.cuda.synchronize(dev)
    seconds = start.elapsed_time(end) / 1e3
    del graphs
    return seconds


def run_triton(args, rank: int, world: int) -> dict | None:
    """The reference's own Triton launchers on this GPU, timed like our arm.

    Needs the reference package under baseline/_ref (not part of this
    repository); prints an ``unavailable`` line otherwise. Same workload,
    buffer rotation and graph-replay timing as ``run_ours``; outputs are
    checked against the oracle.
    """
    ref_silkern = _reference_package()
    if ref_silkern is None:
        return {"impl": "triton-reference", "unavailable": "reference package not present in baseline/_ref"}
    if rank != 0:
        return None
    import torch

    config = args.config
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    sets = ConverterSets(config, shard_plan(0, 1, config), dev, impl="triton", ref_silkern=ref_silkern)
    t = measure_converter(sets, args.steps, args.warmup, dev)
    peaks = _peaks()
    achieved = sets.bytes_per_call / t["per_call_s"] / 1e9
    return {
        "impl": "triton-reference",
        "metric": METRIC if config == 3 else f"Gindices/s per B200, config {config}",
        "value": sets.calls * sets.indices_per_call / t["per_step_s"] / 1e9,
        "unit": UNIT,
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "us_per_call": t["per_call_s"] * 1e6,
        "bit_exact": t["bit_exact"],
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"]},
        "config": _workload_config(config, 1, sets.n_sets),
        "source": "reference silkern.localize_rowwise / localize_hierarchical (Triton) from baseline/_ref",
    }


def run_vllm(args, rank: int, world: int) -> dict | None:
    """vLLM's own sparse index converter beside ours, both at ``dcp_size`` 1.

    ``vllm.v1.attention.backends.mla.sparse_utils.triton_convert_req_index_to_global_index``
    has no DCP split. At ``dcp_size`` 1 it computes the same function as the
    localizer (every token owned, invalid elements -1 in place, no compaction),
    so both run on the workload's shapes with ``dcp_size`` set to 1: vLLM's
    call as its attention backends make it (output and zeroed counts allocated
    per call, ``return_valid_counts=True``), and ours through the public
    launcher on caller-owned buffers. Same buffer rotation and graph-replay
    timing as the other arms; every buffer set's eager output of both is
    compared with the oracle. A comparison arm, rank 0 only.
    """
    if rank != 0:
        return None
    try:
        import vllm
        from vllm.v1.attention.backends.mla import sparse_utils
    except Exception as exc:  # noqa: BLE001  (any import failure means no comparison)
        return {"impl": "vllm-upstream", "unavailable": f"vLLM converter not importable: {exc!r}"[:300]}
    import dataclasses

    import numpy as np
    import torch

    import oracle
    from silkern_b200.workspace import workspace_shapes

    config = args.config
    spec = WORKLOADS[config]
    calls = spec["calls"]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    distinct = calls if calls > 1 else DISTINCT_CASES
    cases = [dataclasses.replace(_case(config, seed=1000 + i, dcp_rank=0), dcp_size=1, dcp_rank=0)
             for i in range(distinct)]
    bytes_per_call = cases[0].algorithmic_bytes()
    n_sets = max(64, math.ceil(2.05 * L2_BYTES / bytes_per_call))
    n_sets = math.ceil(n_sets / distinct) * distinct
    sets = []
    for i in range(n_sets):
        case = cases[i % distinct]
        bufs = {name: torch.as_tensor(a).to(dev) for name, a in
                (("req", case.req_ids), ("table", case.block_table), ("tokens", case.tokens))}
        bufs["out"] = torch.empty_like(bufs["tokens"])
        bufs["counts"] = torch.empty(case.batch, dtype=torch.int32, device=dev)
        if spec["arm"] == "hierarchical_stable":
            for name, shape in workspace_shapes(case.batch, case.width, tile_size=case.tile_size).items():
                bufs[name] = torch.empty(shape, dtype=torch.int32, device=dev)
        sets.append(bufs)
    geometry = cases[0].geometry()
    block_size, width = cases[0].block_size, cases[0].width

    def vllm_call(b):
        return sparse_utils.triton_convert_req_index_to_global_index(
            b["req"], b["table"], b["tokens"], BLOCK_SIZE=block_size, NUM_TOPK_TOKENS=width,
            return_valid_counts=True)

    ours = [_make_call(spec["arm"], b, geometry, cases[0].tile_size) for b in sets]
    expected = [oracle.localize(c.req_ids, c.block_table, c.tokens, threads=4, **c.geometry()) for c in cases]
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    exact = {"vllm": True, "ours": True}
    with torch.cuda.stream(stream):
        for i, b in enumerate(sets):
            want_out, want_counts = expected[i % distinct]
            got_out, got_counts = vllm_call(b)
            ours[i]()
            torch.cuda.synchronize(dev)
            exact["vllm"] &= (np.array_equal(got_out.cpu().numpy(), want_out)
                              and np.array_equal(got_counts.cpu().numpy(), want_counts))
            exact["ours"] &= (np.array_equal(b["out"].cpu().numpy(), want_out)
                              and np.array_equal(b["counts"].cpu().numpy(), want_counts))
    warm, timed = args.warmup * calls, args.steps * calls
    vllm_s = _replay_seconds(lambda i: vllm_call(sets[i % n_sets]), warm, timed, stream, dev)
    ours_s = _replay_seconds(lambda i: ours[i % n_sets](), warm, timed, stream, dev)
    indices = cases[0].batch * width
    return {
        "impl": "vllm-upstream",
        "metric": f"Gindices/s per B200, config {config} shapes at dcp_size 1",
        "value": indices * timed / vllm_s / 1e9,
        "unit": UNIT,
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "us_per_call": vllm_s / timed * 1e6,
        "ours_us_per_call": ours_s / timed * 1e6,
        "ours_value": indices * timed / ours_s / 1e9,
        "bit_exact": exact,
        "vllm_version": vllm.__version__,
        "config": {**_workload_config(config, 1, n_sets), "dcp_size": 1, "dcp_rank": 0},
        "source": "vllm.v1.attention.backends.mla.sparse_utils.triton_convert_req_index_to_global_index"
                  " (per-call allocation included) vs silkern_b200 "
                  + ("localize_rowwise" if spec["arm"] == "row_stable" else "localize_hierarchical"),
    }


FUSED = {
    "desc": "indexer top-k + localize: batch 256 x logits 65536 float32 (row lengths U[1024, 65536], "
            "config 3's context lengths), top_k 2048, block_size 64, dcp_size 4, table (256,256)",
    "batch": 256, "width": 65536, "top_k": 2048,
}


def _fused_sets(n_sets: int, batch: int, dev):
    """Seeded logits rows (normal scores, the row's context length per request)."""
    import numpy as np
    import torch

    case = _case(3, seed=1000, dcp_rank=0)
    rng = np.random.default_rng(2026)
    lens = rng.integers(1024, FUSED["width"], size=batch, endpoint=True).astype(np.int32)
    req = np.resize(case.req_ids, batch).astype(np.int32)  # the workload's requests, repeated
    gen = torch.Generator(device=dev).manual_seed(2026)
    sets = []
    for _ in range(n_sets):
        sets.append({
            "logits": torch.randn(batch, FUSED["width"], device=dev, generator=gen),
            "lens": torch.as_tensor(lens).to(dev),
            "req": torch.as_tensor(req).to(dev),
            "table": torch.as_tensor(case.block_table).to(dev),
            "out": torch.empty(batch, FUSED["top_k"], dtype=torch.int32, device=dev),
            "counts": torch.empty(batch, dtype=torch.int32, device=dev),
            "sel": torch.empty(batch, FUSED["top_k"], dtype=torch.int32, device=dev),
        })
    return sets, case, lens, req


def run_fused(args, rank: int, world: int) -> dict | None:
    """The fused indexer top-k + localization kernel, beside the two-kernel pipeline.

    One call selects the top 2048 of every logits row and localizes the
    selection for one DCP rank (``silkern_b200.topk_localize``). Beside it,
    when vLLM is importable, the production pipeline it replaces: vLLM's
    decode top-k (``torch.ops._C.persistent_topk``) then this library's
    converter on its selection. Same graph-replay timing as the other arms,
    with the logits rotating over at least 4 sets and 256 MB (twice L2; 4 sets
    of 64 MB at the default 256 rows, ``--batch`` sets the rows); the fused
    output of one set is compared with the oracle. A comparison arm, rank 0
    only.
    """
    if rank != 0:
        return None
    import numpy as np
    import torch

    from oracle.topk import topk_localize as oracle_topk
    from silkern_b200 import localize_rowwise, topk_localize

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    batch = args.batch if args.batch > 0 else FUSED["batch"]
    # at least 4 sets and about 256 MB of logits rotating (over twice L2)
    n_sets = max(4, -(-1024 // batch))
    sets, case, lens, req = _fused_sets(n_sets, batch, dev)
    geometry = dict(block_size=case.block_size, dcp_size=case.dcp_size, dcp_rank=0)

    def fused(i):
        d = sets[i % n_sets]
        topk_localize(d["logits"], d["lens"], d["req"], d["table"], d["out"], d["counts"], **geometry)

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        fused(0)
    torch.cuda.synchronize(dev)
    _, want_out, want_counts = oracle_topk(sets[0]["logits"].cpu().numpy(), lens, req, case.block_table,
                                           top_k=FUSED["top_k"], threads=_host_threads(), **geometry)
    bit_exact = (np.array_equal(sets[0]["out"].cpu().numpy(), want_out)
                 and np.array_equal(sets[0]["counts"].cpu().numpy(), want_counts))
    warm, timed = args.warmup, args.steps
    fused_s = _replay_seconds(fused, warm, timed, stream, dev) / timed
    pipeline_s = None
    try:
        import vllm._custom_ops  # noqa: F401  (registers torch.ops._C)

        workspace = torch.zeros(1024 * 1024, dtype=torch.uint8, device=dev)
        max_len = int(lens.max())

        def pipeline(i):
            d = sets[i % n_sets]
            torch.ops._C.persistent_topk(d["logits"], d["lens"], d["sel"], workspace, FUSED["top_k"], max_len)
            localize_rowwise(d["req"], d["table"], d["sel"], d["out"], d["counts"], **geometry)

        pipeline_s = _replay_seconds(pipeline, warm, timed, stream, dev) / timed
    except Exception:  # noqa: BLE001  (vLLM absent or its op unavailable: no comparison)
        pipeline_s = None
    logit_bytes = int(lens.sum()) * 4
    out_bytes = batch * FUSED["top_k"] * 4 + batch * 4
    bytes_per_call = logit_bytes + out_bytes + int(case.block_table.nbytes) + batch * 8
    peaks = _peaks()
    achieved = bytes_per_call / fused_s / 1e9
    return {
        "impl": "fused-topk-localize",
        "metric": "us per call, indexer top-k + localization (lower is better)",
        "value": fused_s * 1e6,
        "unit": "us/call",
        "higher_is_better": False,
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "bit_exact": bit_exact,
        "vllm_topk_then_converter_us": None if pipeline_s is None else pipeline_s * 1e6,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "algorithmic_bytes_per_call": bytes_per_call,
                     "peak_source": peaks["source"]},
        "gpu_launches": timed,
        "config": {"workload": FUSED["desc"] if batch == FUSED["batch"] else
                   FUSED["desc"].replace("batch 256", f"batch {batch}"),
                   "batch": batch, "l2": f"inputs larger than L2: {n_sets} rotating logits sets"},
        "data": "synthetic (seeded normal scores)",
    }


def run_link(args, rank: int, world: int) -> dict | None:
    """The host link's ceiling for the end-to-end line: its copies alone.

    Per step, the end-to-end arm moves the workload's inputs to the device
    (one H2D copy per call: req_ids, table and tokens) and its results back
    (two D2H copies per call: out and counts) from pinned host buffers, the
    steps alternating over ``--e2e-lanes`` streams. This arm times the same
    copies on the same lanes with no kernel: H2D alone, D2H alone, and both
    (the end-to-end step without its kernel). A comparison arm, rank 0 only;
    no localization runs.
    """
    if rank != 0:
        return None
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    calls = WORKLOADS[args.config]["calls"]
    case = _case(args.config, seed=0, dcp_rank=0)
    n_in = case.req_ids.size + case.block_table.size + case.tokens.size
    n_out = case.tokens.size
    n_lanes = max(1, args.e2e_lanes)
    lanes = []  # per lane: its stream and one buffer set per call, as in the end-to-end arm
    for _ in range(n_lanes):
        sets = []
        for _ in range(calls):
            sets.append((torch.empty(n_in, dtype=torch.int32).pin_memory(),
                         torch.empty(n_in, dtype=torch.int32, device=dev),
                         torch.empty(n_out, dtype=torch.int32, device=dev),
                         torch.empty(n_out, dtype=torch.int32).pin_memory(),
                         torch.empty(case.batch, dtype=torch.int32, device=dev),
                         torch.empty(case.batch, dtype=torch.int32).pin_memory()))
        lanes.append((torch.cuda.Stream(device=dev), sets))
    steps = max(1, min(args.steps, 200))

    def step(i: int, inbound: bool, outbound: bool) -> None:
        stream, sets = lanes[i % n_lanes]
        with torch.cuda.stream(stream):
            for host_in, dev_in, dev_out, host_out, dev_counts, host_counts in sets:
                if inbound:
                    dev_in.copy_(host_in, non_blocking=True)
                if outbound:
                    host_out.copy_(dev_out, non_blocking=True)
                    host_counts.copy_(dev_counts, non_blocking=True)

    def timed(inbound: bool, outbound: bool) -> float:
        """Seconds per step, the best of three runs after a warm-up."""
        current = torch.cuda.current_stream(dev)
        for i in range(max(3, args.warmup)):
            step(i, inbound, outbound)
        torch.cuda.synchronize(dev)
        best = math.inf
        for _ in range(3):
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(current)
            for stream, _ in lanes:
                stream.wait_event(start)
            for i in range(steps):
                step(i, inbound, outbound)
            for stream, _ in lanes:
                current.wait_stream(stream)
            end.record(current)
            torch.cuda.synchronize(dev)
            best = min(best, start.elapsed_time(end) / 1e3 / steps)
        return best

    h2d_bytes = 4 * n_in * calls
    d2h_bytes = 4 * (n_out + case.batch) * calls
    t_in = timed(True, False)
    t_out = timed(False, True)
    t_both = timed(True, True)
    return {
        "impl": "host-link",
        "metric": "us per step, the end-to-end step's host copies alone (no kernel)",
        "unit": "us/step",
        "higher_is_better": False,
        "steps": steps,
        "h2d_bytes_per_step": h2d_bytes,
        "d2h_bytes_per_step": d2h_bytes,
        "h2d_us_per_step": t_in * 1e6,
        "d2h_us_per_step": t_out * 1e6,
        "both_us_per_step": t_both * 1e6,
        "value": t_both * 1e6,
        "h2d_gbs": h2d_bytes / t_in / 1e9,
        "d2h_gbs": d2h_bytes / t_out / 1e9,
        "both_gbs": (h2d_bytes + d2h_bytes) / t_both / 1e9,
        "config": {"workload": WORKLOADS[args.config]["desc"],
                   "buffers": f"pinned host, {n_lanes} streams alternating, each with its own buffers"},
        "data": "synthetic",
    }


def _make_call(arm: str, bufs: dict, geometry: dict, tile_size: int):
    from silkern_b200.baselines import launch_atomic_baseline
    from silkern_b200.kernels import localize_hierarchical, localize_rowwise

    if arm == "atomic":
        return lambda: launch_atomic_baseline(bufs["req"], bufs["table"], bufs["tokens"], bufs["out"],
                                              bufs["counts"], bufs["scratch"], **geometry)
    if arm == "row_stable":
        return lambda: localize_rowwise(bufs["req"], bufs["table"], bufs["tokens"], bufs["out"],
                                        bufs["counts"], **geometry)
    return lambda: localize_hierarchical(
        bufs["req"], bufs["table"], bufs["tokens"], bufs["out"], bufs["counts"], bufs["mapped"],
        bufs["local_positions"], bufs["tile_counts"], bufs["tile_offsets"], tile_size=tile_size,
        **geometry)


def _reference_package():
    """The reference's own silkern package from baseline/_ref, or None."""
    ref_dir = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref_dir, "silkern", "kernels.py")):
        return None
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    for name in [m for m in sys.modules if m == "silkern" or m.startswith("silkern.")]:
        del sys.modules[name]
    import silkern as ref_silkern  # the reference implementation

    if not os.path.abspath(ref_silkern.__file__).startswith(ref_dir):
        return None
    return ref_silkern


def _reference_call(ref_silkern, arm: str, bufs: dict, case):
    """The reference's own launcher (Triton) for one buffer set."""
    g = case.geometry()
    if arm == "row_stable":
        return lambda: ref_silkern.localize_rowwise(bufs["req"], bufs["table"], bufs["tokens"], bufs["out"],
                                                    bufs["counts"], **g)
    if case.width > ref_silkern.MAX_ROW_WIDTH or case.tile_size not in ref_silkern.SUPPORTED_TILE_SIZES:
        # The reference launcher rejects this width/tile (its workspace
        # limits), so its four Triton kernels are launched directly with the
        # launcher's own parameters.
        return lambda: _reference_hierarchical_direct(ref_silkern, bufs, g, case.tile_size)
    return lambda: ref_silkern.localize_hierarchical(
        bufs["req"], bufs["table"], bufs["tokens"], bufs["out"], bufs["counts"], bufs["mapped"],
        bufs["local_positions"], bufs["tile_counts"], bufs["tile_offsets"], tile_size=case.tile_size, **g)


class ConverterSets:
    """Resident buffer sets for one workload, each with its converter call.

    Inputs rotate over enough sets to exceed 2.05 x L2 (126 MB), so every
    timed call reads data that is not already in L2. ``impl`` is "ours" (the
    public launchers), "atomic" (the comparison baseline) or "triton" (the
    reference's own launchers, ``ref_silkern``).
    """

    def __init__(self, config: int, plan: dict, dev, *, impl: str = "ours", rows: int = 0,
                 ref_silkern=None, min_sets: int = 64):
        import torch

        from silkern_b200.workspace import workspace_shapes

        spec = WORKLOADS[config]
        self.config = config
        self.arm = spec["arm"]
        self.calls = spec["calls"]
        distinct = self.calls if self.calls > 1 else DISTINCT_CASES
        if rows > 0:  # fewer, larger cases: every call's rows repeat a config case's
            distinct = self.calls if self.calls > 1 else 2
        cases = [_case(config, seed=plan["base_seed"] + i, dcp_rank=plan["dcp_rank"]) for i in range(distinct)]
        if rows > 0:
            cases = [_stack_rows(c, rows) for c in cases]
        self.cases = cases
        self.distinct = distinct
        self.bytes_per_call = cases[0].algorithmic_bytes()
        self.indices_per_call = cases[0].batch * cases[0].width
        n_sets = max(min_sets if rows == 0 else 2, math.ceil(2.05 * L2_BYTES / self.bytes_per_call))
        self.n_sets = math.ceil(n_sets / distinct) * distinct
        self.impl = impl
        self.sets = []
        for i in range(self.n_sets):
            case = cases[i % distinct]
            bufs = {name: torch.as_tensor(a).to(dev) for name, a in
                    (("req", case.req_ids), ("table", case.block_table), ("tokens", case.tokens))}
            bufs["out"] = torch.empty_like(bufs["tokens"])
            bufs["counts"] = torch.empty(case.batch, dtype=torch.int32, device=dev)
            if self.arm == "hierarchical_stable":
                for name, shape in workspace_shapes(case.batch, case.width, tile_size=case.tile_size).items():
                    bufs[name] = torch.empty(shape, dtype=torch.int32, device=dev)
            if impl == "atomic":
                bufs["scratch"] = torch.empty(case.batch, dtype=torch.int32, device=dev)
            if impl == "triton":
                call = _reference_call(ref_silkern, self.arm, bufs, case)
            else:
                call = _make_call("atomic" if impl == "atomic" else self.arm, bufs, case.geometry(),
                                  case.tile_size)
            self.sets.append((bufs, call))

    def launch(self, i: int) -> None:
        self.sets[i % self.n_sets][1]()

    def bit_exact(self, used) -> bool:
        """Every used set's out and counts equal the oracle's (for the atomic
        baseline: the same set and counts, in any order)."""
        import numpy as np

        import oracle

        expected = [oracle.localize(c.req_ids, c.block_table, c.tokens, threads=4, **c.geometry())
                    for c in self.cases]
        ok = True
        for index in sorted(used):
            bufs = self.sets[index][0]
            want_out, want_counts = expected[index % self.distinct]
            got_out = bufs["out"].cpu().numpy()
            if self.impl == "atomic":
                big = np.iinfo(np.int32).max
                got_out = np.sort(np.where(got_out < 0, big, got_out), axis=1)
                want_out = np.sort(np.where(want_out < 0, big, want_out), axis=1)
            if not (np.array_equal(got_out, want_out)
                    and np.array_equal(bufs["counts"].cpu().numpy(), want_counts)):
                ok = False
        return ok


def _min_over_ranks(dist, value: int) -> int:
    """The smallest ``value`` over all ranks."""
    return int(-reduce_max(dist, -float(value)))


def _all_ranks(dist, ok: bool) -> bool:
    """True when ``ok`` holds on every rank."""
    return reduce_max(dist, 0.0 if ok else 1.0) == 0.0


def measure_converter(sets: ConverterSets, steps: int, warmup: int, dev, dist=None, sampler=None) -> dict:
    """Time ``steps`` steps after ``warmup`` (CUDA events inside the replayed
    graphs, max over ranks, a barrier and a synchronize on both sides) and
    check every used buffer set against the oracle."""
    import contextlib

    import torch

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for i in range(max(3, sets.n_sets)):
            sets.launch(i)
    torch.cuda.synchronize(dev)
    warm_launches = warmup * sets.calls
    timed_launches = steps * sets.calls
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with sampler if sampler is not None else contextlib.nullcontext():
        seconds = _replay_seconds(sets.launch, warm_launches, timed_launches, stream, dev)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    per_step_s = reduce_max(dist, seconds) / steps
    used = {i % sets.n_sets for i in range(max(3, sets.n_sets) + warm_launches + timed_launches)}
    ok = _all_ranks(dist, sets.bit_exact(used))
    return {"per_step_s": per_step_s, "per_call_s": per_step_s / sets.calls, "bit_exact": ok}


# Calls per timing of isolated_us_per_call, whatever --steps is: the figure
# is the difference of two timings, which 20 calls leave noisy.
ISOLATED_CALLS = 200


def measure_isolated(sets: ConverterSets, steps: int, warmup: int, dev) -> float:
    """Seconds one converter call adds between a producer kernel that writes
    its tokens and a consumer kernel that reads its output, with no other
    converter call around it: [producer, converter, consumer] per step,
    minus [producer, consumer] per step, over rotating sets. Programmatic
    dependent launch cannot overlap the call with a previous converter call
    here, so this is the latency of one call in a pipeline."""
    import torch

    sources = [b["tokens"].clone() for b, _ in sets.sets]
    sinks = [torch.empty_like(b["out"]) for b, _ in sets.sets]

    def with_call(i: int) -> None:
        k = i % sets.n_sets
        bufs, call = sets.sets[k]
        bufs["tokens"].copy_(sources[k])  # producer: writes the converter's input
        call()
        sinks[k].copy_(bufs["out"])  # consumer: reads the converter's output

    def without_call(i: int) -> None:
        k = i % sets.n_sets
        bufs, _ = sets.sets[k]
        bufs["tokens"].copy_(sources[k])
        sinks[k].copy_(bufs["out"])

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    warm = max(3, warmup) * sets.calls
    timed = steps * sets.calls
    # Median of three alternating pairs.
    diffs = sorted(_replay_seconds(with_call, warm, timed, stream, dev) -
                   _replay_seconds(without_call, warm, timed, stream, dev) for _ in range(3))
    return diffs[1] / timed


# Launch shapes of the copy-floor sweep: (elements per thread, threads per
# CTA, most CTAs per SM with 0 for no limit).
COPY_FLOOR_SHAPES = tuple((run, threads, per_sm) for run, threads in
                          ((8, 128), (8, 256), (8, 512), (8, 1024), (16, 128), (16, 256), (16, 512))
                          for per_sm in (0, 1, 2, 4))


def measure_copy_floor(sets: ConverterSets, steps: int, warmup: int, dev, dist, per_call_s: float) -> dict:
    """The floor a converter call runs against: each call's tokens copied to
    its output buffer by silkern_copy_floor_v1 (the converter's loads,
    stores and launch mode, none of its work), over the same rotating sets,
    timed like the converter for every launch shape of COPY_FLOOR_SHAPES
    (max over ranks); the fastest shape is the floor. Overwrites the sets'
    outputs, so it runs after their check."""
    import torch

    from silkern_b200.kernels import copy_floor

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    shapes = {}
    for run, threads, per_sm in COPY_FLOOR_SHAPES:
        def launch(i: int, run=run, threads=threads, per_sm=per_sm) -> None:
            bufs, _ = sets.sets[i % sets.n_sets]
            copy_floor(bufs["tokens"], bufs["out"], run=run, threads=threads, ctas_per_sm=per_sm)

        seconds = _replay_seconds(launch, max(3, warmup) * sets.calls, steps * sets.calls, stream, dev)
        shapes[f"{run}x{threads}/{per_sm}"] = reduce_max(dist, seconds) / (steps * sets.calls) * 1e6
    best = min(shapes, key=shapes.get)
    floor_us = shapes[best]
    moved = 2 * 4 * sum(int(b["tokens"].numel()) for b, _ in sets.sets[:sets.calls]) / sets.calls
    return {
        "us_per_call": floor_us,
        "shape": best,
        "bytes_per_call": int(moved),
        "gbs": moved / floor_us / 1e3,
        "frac_of_peak": moved / floor_us / 1e3 / _peaks()["hbm_gbs"],
        "converter_frac_of_floor": floor_us / (per_call_s * 1e6),
        "us_per_call_by_shape": shapes,
        "what": "tokens copied to out (the converter's loads, stores and launch mode, none of its work), "
                "back to back over the same rotating sets; fastest of the launch shapes (elements per thread "
                "x threads per CTA / most CTAs per SM, 0 for no limit)",
    }


def run_ours(args, rank: int, world: int, local_rank: int, dist) -> dict | None:
    import torch

    from silkern_b200 import _native

    config = args.config
    impl = "atomic" if args.impl == "atomic" else "ours"
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    plan = shard_plan(rank, world, config)
    sets = ConverterSets(config, plan, dev, impl=impl, rows=args.rows)
    calls = sets.calls
    sampler = ClockSampler(local_rank)
    timing = measure_converter(sets, args.steps, args.warmup, dev, dist, sampler)
    per_step_s, per_call_s = timing["per_step_s"], timing["per_call_s"]
    bytes_per_call = sets.bytes_per_call
    indices_per_call = sets.indices_per_call
    n_sets = sets.n_sets
    headline_cases = sets.cases[:calls]

    floor = None
    if impl == "ours":
        floor = measure_copy_floor(sets, args.steps, args.warmup, dev, dist, per_call_s)
    isolated = None
    if impl == "ours" and world == 1 and args.rows == 0:
        isolated = measure_isolated(sets, ISOLATED_CALLS, args.warmup, dev)
    del sets
    torch.cuda.empty_cache()

    extra = {}
    if impl == "ours" and args.rows == 0 and not args.headline_only:
        # The other workloads, timed the same way on this GPU's DCP rank.
        others = {}
        for other in sorted(WORKLOADS):
            if other == config:
                continue
            other_plan = shard_plan(rank, world, other)
            other_sets = ConverterSets(other, other_plan, dev)
            t = measure_converter(other_sets, args.steps, args.warmup, dev, dist)
            others[str(other)] = {
                "workload": WORKLOADS[other]["desc"],
                "us_per_call": t["per_call_s"] * 1e6,
                "value": world * other_sets.calls * other_sets.indices_per_call / t["per_step_s"] / 1e9,
                "unit": UNIT,
                "bit_exact": t["bit_exact"],
                "dcp_rank": f"gpu_index % {WORKLOADS[other]['dcp_size']}",
                "frac": other_sets.bytes_per_call / t["per_call_s"] / 1e9 / _peaks()["hbm_gbs"],
            }
            del other_sets
            torch.cuda.empty_cache()
        extra["configs"] = others
        if world == 1:
            extra["triton_reference"] = _triton_sub(config, args, dev)
        extra["replay_gate"] = _replay_gate_sub(rank, world, dev, dist)

    e2e = run_e2e(args, headline_cases, dev, dist) if impl == "ours" else None

    peaks = _peaks()
    achieved = bytes_per_call / per_call_s / 1e9
    traffic = _traffic(config) if args.rows == 0 else {"bytes": None, "source": "captures are of the default rows"}
    workload = _workload_config(config, world, n_sets)
    if args.rows > 0:
        workload["rows_per_call"] = args.rows
        workload["workload"] += f"; {args.rows} rows per call, the config's rows repeated"
    frac = achieved / peaks["hbm_gbs"]
    result = {
        **({"impl": "atomic-baseline"} if impl == "atomic" else {}),
        "metric": METRIC if config == 3 else f"Gindices/s per B200, config {config}",
        "value": world * calls * indices_per_call / per_step_s / 1e9,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_step_s * 1e3,
        "us_per_call": per_call_s * 1e6,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int32",
        "data": f"synthetic (seeded; config {config} shapes)",
        "config": workload,
        "bit_exact": timing["bit_exact"],
        "hbm_gbs": achieved,
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": frac,
            "traffic": traffic["bytes"],
            "traffic_source": traffic["source"],
            "dram_gbs": None if traffic["bytes"] is None else traffic["bytes"] / per_call_s / 1e9,
            "algorithmic_bytes_per_call": bytes_per_call,
            "peak_source": peaks["source"],
            "regime": "bandwidth" if frac >= 0.6 else
                      "latency and issue: one call moves too few bytes to fill HBM, see us_per_call",
            "timing": "CUDA events recorded inside the replayed graphs around the timed calls, per call",
        },
        "isolated_us_per_call": None if isolated is None else isolated * 1e6,
        "copy_floor": floor,
        "gpu_launches": args.steps * calls,
        **extra,
        "e2e": e2e,
        "clocks": sampler.summary(),
        "library": _native.LIB_PATH,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = _cpu_baseline(config, _host_threads())
    return result if rank == 0 else None


def _replay_gate_sub(rank: int, world: int, dev, dist) -> dict:
    """Config 5's decode step on this GPU's DCP rank: 48 converter calls of
    128 x 2048 (dcp 8), each layer on its own seeded selection, captured once
    and replayed 10,000 times, every layer of every replay compared with the
    oracle on the device; pointers and the allocator checked at replay 0, 1,
    10, 100, 1000 and 10000. Every rank runs it; the line reports all ranks."""
    import oracle
    from silkern_b200.verify import GATE_REPLAYS, decode_step_gate

    plan = shard_plan(rank, world, 5)
    layers = [_case(5, seed=plan["base_seed"] + 7000 + layer, dcp_rank=plan["dcp_rank"])
              for layer in range(WORKLOADS[5]["calls"])]
    expected = [oracle.localize(c.req_ids, c.block_table, c.tokens, threads=4, **c.geometry()) for c in layers]
    gate = decode_step_gate(layers, expected=expected, replays=GATE_REPLAYS)
    return {
        "workload": WORKLOADS[5]["desc"],
        "layers": len(layers),
        "replays": _min_over_ranks(dist, gate.replays),
        "mismatches": int(reduce_max(dist, max(gate.mismatches, 0) if gate.error is None else 1 << 30)),
        "checkpoints": sorted(gate.checkpoints),
        "ok": _all_ranks(dist, gate.ok),
        "converter_step_us": reduce_max(dist, gate.step_us or 0.0),
        "dcp_rank": "gpu_index % 8",
        "error": gate.error,
    }


def _triton_sub(config: int, args, dev) -> dict:
    """The reference's own Triton launcher on the same workload, same
    rotation and timing, in this process (a comparison beside the headline)."""
    import torch

    ref_silkern = _reference_package()
    if ref_silkern is None:
        return {"unavailable": "reference package not present in baseline/_ref"}
    try:
        sets = ConverterSets(config, shard_plan(0, 1, config), dev, impl="triton", ref_silkern=ref_silkern)
        t = measure_converter(sets, args.steps, args.warmup, dev)
        isolated = measure_isolated(sets, ISOLATED_CALLS, args.warmup, dev)
    except Exception as exc:  # the comparison arm must not take the headline down
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
    finally:
        torch.cuda.empty_cache()
    return {
        "us_per_call": t["per_call_s"] * 1e6,
        "isolated_us_per_call": isolated * 1e6,
        "bit_exact": t["bit_exact"],
        "source": "reference silkern.localize_rowwise / localize_hierarchical (Triton) from baseline/_ref",
    }


def _stack_rows(case, rows: int):
    """`case` with `rows` selection rows: its own rows repeated in order (the
    requests and the block table unchanged)."""
    import dataclasses

    import numpy as np

    reps = -(-rows // case.batch)
    return dataclasses.replace(case, req_ids=np.ascontiguousarray(np.tile(case.req_ids, reps)[:rows]),
                               tokens=np.ascontiguousarray(np.tile(case.tokens, (reps, 1))[:rows]))


# End-to-end steps when --e2e-steps is not given, at least: the step is bound
# by the host link, and 20 steps over a few streams are mostly the pipeline's
# fill and drain (one box: 132.8 us per step over 20 steps on 4 streams, 59.3
# over 200).
E2E_MIN_STEPS = 200
# Pinned host bytes the end-to-end lanes may hold in all (each lane has its
# own inputs and outputs).
E2E_LANE_BYTES = 1 << 30


def run_e2e(args, cases, dev, dist) -> dict:
    """Same metric through the public API, host inputs in and results out every step."""
    import torch

    from silkern_b200.workspace import workspace_shapes

    steps = args.e2e_steps if args.e2e_steps > 0 else max(args.steps, E2E_MIN_STEPS)
    arm = WORKLOADS[args.config]["arm"]
    lanes = []
    h2d = d2h = 0
    # Every lane holds its own pinned and device copy of a step's buffers:
    # at most E2E_LANE_BYTES of them in all.
    lane_bytes = sum(4 * (c.req_ids.size + c.block_table.size + 2 * c.tokens.size + c.batch) for c in cases)
    n_lanes = max(1, min(args.e2e_lanes, E2E_LANE_BYTES // max(1, lane_bytes)))
    for lane_index in range(n_lanes):
        stream = torch.cuda.Stream(device=dev)
        jobs = []
        for case in cases:
            batch, width = case.tokens.shape
            n_req, n_table = case.req_ids.size, case.block_table.size
            n_in = n_req + n_table + case.tokens.size
            host_in = torch.empty(n_in, dtype=torch.int32).pin_memory()
            host_in[:n_req] = torch.as_tensor(case.req_ids)
            host_in[n_req:n_req + n_table] = torch.as_tensor(case.block_table.ravel())
            host_in[n_req + n_table:] = torch.as_tensor(case.tokens.ravel())
            # Inputs share one device buffer (one H2D copy); the two outputs must
            # not share storage, so they come back in two D2H copies.
            dev_in = torch.empty(n_in, dtype=torch.int32, device=dev)
            bufs = {
                "req": dev_in[:n_req],
                "table": dev_in[n_req:n_req + n_table].view(case.block_table.shape),
                "tokens": dev_in[n_req + n_table:].view(batch, width),
                "out": torch.empty((batch, width), dtype=torch.int32, device=dev),
                "counts": torch.empty(batch, dtype=torch.int32, device=dev),
            }
            if arm == "hierarchical_stable":
                # The hierarchical entry point wants every buffer in its own
                # storage: the inputs land in one staging buffer and are split
                # into their own tensors on the device.
                bufs["req"] = torch.empty(n_req, dtype=torch.int32, device=dev)
                bufs["table"] = torch.empty(case.block_table.shape, dtype=torch.int32, device=dev)
                bufs["tokens"] = torch.empty((batch, width), dtype=torch.int32, device=dev)
                bufs["staging"] = dev_in
                for name, shape in workspace_shapes(batch, width, tile_size=case.tile_size).items():
                    bufs[name] = torch.empty(shape, dtype=torch.int32, device=dev)
            host_out = torch.empty((batch, width), dtype=torch.int32).pin_memory()
            host_counts = torch.empty(batch, dtype=torch.int32).pin_memory()
            jobs.append((host_in, dev_in, bufs, host_out, host_counts,
                         _make_call(arm, bufs, case.geometry(), case.tile_size)))
            if lane_index == 0:
                h2d += 4 * n_in
                d2h += 4 * (batch * width + batch)
        lanes.append((stream, jobs))

    def step(i: int) -> None:
        stream, jobs = lanes[i % n_lanes]
        with torch.cuda.stream(stream):
            for host_in, dev_in, bufs, host_out, host_counts, call in jobs:
                dev_in.copy_(host_in, non_blocking=True)
                if "staging" in bufs:
                    n_req, n_table = bufs["req"].numel(), bufs["table"].numel()
                    bufs["req"].copy_(dev_in[:n_req])
                    bufs["table"].view(-1).copy_(dev_in[n_req:n_req + n_table])
                    bufs["tokens"].view(-1).copy_(dev_in[n_req + n_table:])
                call()
                host_out.copy_(bufs["out"], non_blocking=True)
                host_counts.copy_(bufs["counts"], non_blocking=True)

    for i in range(max(3, min(args.warmup, 8))):
        step(i)
    torch.cuda.synchronize(dev)

    def timed(run_step) -> float:
        """Seconds per step over `steps` steps, max over ranks."""
        if dist is not None:
            dist.barrier()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        current = torch.cuda.current_stream(dev)
        current.synchronize()
        start.record(current)
        for stream, _ in lanes:
            stream.wait_event(start)
        for i in range(steps):
            run_step(i)
        for stream, _ in lanes:
            current.wait_stream(stream)
        end.record(current)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        return reduce_max(dist, start.elapsed_time(end)) / 1e3 / steps

    # Eager: every step issued from Python (copies, launcher, copies).
    eager = timed(step)
    # Captured: one step per lane recorded once (H2D from the pinned inputs,
    # the public launcher, D2H of out and counts) and replayed, as a decode
    # step runs under CUDA graphs; the copies still move every step's bytes.
    graphs = []
    for lane_index, (stream, _) in enumerate(lanes):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step(lane_index)
        graphs.append(graph)
    torch.cuda.synchronize(dev)

    def replay(i: int) -> None:
        stream, _ = lanes[i % n_lanes]
        with torch.cuda.stream(stream):
            graphs[i % n_lanes].replay()

    captured = timed(replay)
    del graphs
    # The host link's ceiling: the same captured copies on the same lanes and
    # buffers, without the converter call.
    link_graphs = []
    for lane_index, (stream, jobs) in enumerate(lanes):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for host_in, dev_in, bufs, host_out, host_counts, _ in jobs:
                dev_in.copy_(host_in, non_blocking=True)
                host_out.copy_(bufs["out"], non_blocking=True)
                host_counts.copy_(bufs["counts"], non_blocking=True)
        link_graphs.append(graph)
    torch.cuda.synchronize(dev)

    def replay_link(i: int) -> None:
        stream, _ = lanes[i % n_lanes]
        with torch.cuda.stream(stream):
            link_graphs[i % n_lanes].replay()

    link = timed(replay_link)
    del link_graphs
    world = dist.get_world_size() if dist is not None else 1
    indices = len(cases) * cases[0].batch * cases[0].width
    return {
        "value": world * indices / captured / 1e9,
        "unit": UNIT,
        "h2d_bytes_per_step": h2d,
        "d2h_bytes_per_step": d2h,
        "steps": steps,
        "us_per_step": captured * 1e6,
        "path": "silkern_b200 public launchers with host copies in and out every step, captured per "
                f"stream (CUDA graph) and replayed on {n_lanes} alternating streams, pinned host buffers",
        "eager_us_per_step": eager * 1e6,
        "eager_value": world * indices / eager / 1e9,
        "link_us_per_step": link * 1e6,
        "link_gbs_per_gpu": (h2d + d2h) / link / 1e9,
    }


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=2000)
    parser.add_argument("--warmup", type=int, default=64)
    parser.add_argument("--impl", choices=["ours", "reference", "triton", "vllm", "fused", "atomic", "link"],
                        default="ours")
    parser.add_argument("--config", type=int, choices=sorted(WORKLOADS), default=3)
    parser.add_argument("--e2e-steps", type=int, default=0,
                        help=f"end-to-end steps (default: --steps, at least {E2E_MIN_STEPS})")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--batch", type=int, default=0, help="rows of the fused arm (default 256)")
    parser.add_argument("--rows", type=int, default=0,
                        help="rows per converter call: the workload's rows repeated (default: its own batch)")
    parser.add_argument("--e2e-lanes", type=int, default=8,
                        help="streams the end-to-end steps alternate over, each with its own buffers")
    parser.add_argument("--headline-only", action="store_true",
                        help="skip the other workloads, the Triton comparison and the replay gate")
    args = parser.parse_args(argv)
    if args.steps < 1 or args.warmup < 0:
        parser.error("--steps must be >= 1 and --warmup >= 0")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl in ("reference", "triton", "vllm", "fused", "link"):
        result = {"reference": run_reference, "triton": run_triton, "vllm": run_vllm,
                  "fused": run_fused, "link": run_link}[args.impl](args, rank, world)
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
        result = run_ours(args, rank, world, local_rank, dist)  # also --impl atomic
    finally:
        if dist is not None:
            dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
