"""Generate the golden fixtures from the reference implementation itself.

    python tests/golden/make_golden.py --reference <checkout of the reference> [--skip-config5]

Runs in a container that has the reference checkout (read-only is fine) and
triton; it is not needed on a GPU machine. For every case it records the
sha256 of the inputs and of the outputs of

* the reference's ``silkern.localize_reference`` (silkern/contract.py:67-158),
* the reference's Triton kernels run by the Triton CPU interpreter
  (``TRITON_INTERPRET=1``), launched with the launch parameters of
  silkern/kernels.py:411-434 (row-wise) and :560-633 (hierarchical, whose
  tile_counts/tile_offsets are recorded too),

where a digest is sha256 over the little-endian int32 bytes of ``out`` then
``counts`` (``silkern_b200.workloads.digest``). Inputs come from this
repository's generators (``silkern_b200.verify._random_case`` and
``silkern_b200.workloads.config_case``), so the tests can regenerate them and
check ``input_sha256`` first. Config 1 is also stored as full arrays in
``config1.npz``.

Outputs: tests/golden/golden.json and tests/golden/config1.npz.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _setup(reference: str):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.dont_write_bytecode = True
    # The reference package is named `silkern`, like this repository's alias
    # package: put the reference first so `import silkern` resolves to it.
    sys.path.insert(0, reference)
    sys.path.append(REPO)
    import silkern  # noqa: F401  (the reference)

    assert os.path.abspath(silkern.__file__).startswith(os.path.abspath(reference)), silkern.__file__


def _next_pow2(n: int) -> int:
    p = 1
    while p < n:
        p *= 2
    return p


def triton_rowwise(torch, req, table, tokens, *, block_size, dcp_size, dcp_rank, dcp_interleave,
                   compact):
    from silkern.kernels import _rowwise_kernel  # the reference's kernel

    batch, width = tokens.shape
    out = torch.empty_like(tokens)
    counts = torch.empty(batch, dtype=torch.int32)
    _rowwise_kernel[(batch,)](
        req, table, tokens, out, counts,
        table.stride(0), table.stride(1), tokens.stride(0), tokens.stride(1),
        out.stride(0), out.stride(1),
        WIDTH=width, PADDED_WIDTH=_next_pow2(width), BLOCK_TABLE_WIDTH=table.shape[1],
        BLOCK_SIZE=block_size, DCP_SIZE=dcp_size, DCP_RANK=dcp_rank,
        DCP_INTERLEAVE=dcp_interleave, COMPACT_TO_FRONT=compact and dcp_size > 1, num_warps=8,
    )
    return out, counts


def triton_hierarchical(torch, req, table, tokens, *, block_size, dcp_size, dcp_rank,
                        dcp_interleave, compact, tile_size):
    from silkern.kernels import (
        _fill_output_kernel,
        _map_tiles_kernel,
        _scatter_tiles_kernel,
        _tile_prefix_kernel,
    )

    batch, width = tokens.shape
    tiles = (width + tile_size - 1) // tile_size
    out = torch.empty_like(tokens)
    counts = torch.empty(batch, dtype=torch.int32)
    mapped = torch.empty_like(tokens)
    positions = torch.empty_like(tokens)
    tile_counts = torch.empty((batch, tiles), dtype=torch.int32)
    tile_offsets = torch.empty((batch, tiles), dtype=torch.int32)
    do_compact = compact and dcp_size > 1
    _map_tiles_kernel[(batch, tiles)](
        req, table, tokens, out, mapped, positions, tile_counts,
        table.stride(0), table.stride(1), tokens.stride(0), tokens.stride(1),
        out.stride(0), out.stride(1), mapped.stride(0), mapped.stride(1),
        positions.stride(0), positions.stride(1), tile_counts.stride(0), tile_counts.stride(1),
        WIDTH=width, BLOCK_TABLE_WIDTH=table.shape[1], BLOCK_SIZE=block_size,
        DCP_SIZE=dcp_size, DCP_RANK=dcp_rank, DCP_INTERLEAVE=dcp_interleave,
        TILE_SIZE=tile_size, DIRECT_OUTPUT=not do_compact, num_warps=4,
    )
    _tile_prefix_kernel[(batch,)](
        tile_counts, tile_offsets, counts,
        tile_counts.stride(0), tile_counts.stride(1), tile_offsets.stride(0),
        tile_offsets.stride(1), NUM_TILES=tiles, PADDED_TILES=_next_pow2(tiles), num_warps=1,
    )
    if do_compact:
        elements = batch * width
        _fill_output_kernel[((elements + 255) // 256,)](out, elements, BLOCK=256, num_warps=4)
        _scatter_tiles_kernel[(batch, tiles)](
            out, mapped, positions, tile_counts, tile_offsets,
            out.stride(0), out.stride(1), mapped.stride(0), mapped.stride(1),
            positions.stride(0), positions.stride(1), tile_counts.stride(0),
            tile_counts.stride(1), tile_offsets.stride(0), tile_offsets.stride(1),
            WIDTH=width, TILE_SIZE=tile_size, num_warps=4,
        )
    return out, counts, tile_counts, tile_offsets


def record(np, torch, entry, req_ids, block_table, rows, *, geometry, compact=True,
           run_rowwise=True, run_hierarchical=True, tile_size=128):
    from silkern import localize_reference  # the reference oracle

    from silkern_b200.workloads import digest

    req = np.asarray(req_ids, dtype=np.int32)
    table = np.asarray(block_table, dtype=np.int32)
    tokens = np.asarray(rows, dtype=np.int32)
    h = __import__("hashlib").sha256()
    for array in (req, table, tokens):
        h.update(np.ascontiguousarray(array, dtype="<i4").tobytes())
    entry["input_sha256"] = h.hexdigest()
    entry["compact_valid_to_front"] = compact
    expected_out, expected_counts = localize_reference(
        req.tolist(), table.tolist(), tokens.tolist(), compact_valid_to_front=compact, **geometry
    )
    entry["oracle_sha256"] = digest(np.asarray(expected_out, dtype=np.int32),
                                    np.asarray(expected_counts, dtype=np.int32))
    t_req, t_table, t_tokens = (torch.from_numpy(np.ascontiguousarray(a)) for a in (req, table, tokens))
    if run_rowwise:
        out, counts = triton_rowwise(torch, t_req, t_table, t_tokens, compact=compact, **geometry)
        entry["triton_rowwise_sha256"] = digest(out.numpy(), counts.numpy())
    if run_hierarchical:
        out, counts, tc, to = triton_hierarchical(torch, t_req, t_table, t_tokens, compact=compact,
                                                  tile_size=tile_size, **geometry)
        entry["tile_size"] = tile_size
        entry["triton_hierarchical_sha256"] = digest(out.numpy(), counts.numpy())
        entry["triton_tiles_sha256"] = digest(tc.numpy(), to.numpy())
    return expected_out, expected_counts


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", required=True,
                        help="path of a checkout of the reference repository (its silkern package)")
    parser.add_argument("--skip-config5", action="store_true")
    args = parser.parse_args(argv)
    _setup(args.reference)

    import numpy as np
    import torch

    from silkern_b200.verify import DEFAULT_MATRIX, _random_case
    from silkern_b200.workloads import config_case

    cases = []
    started = time.time()

    def adversarial(case_id, *, width, batch, block_size, gen_dcp, seed, geometries, compact=True,
                    tile_size=128):
        req_ids, block_table, rows = _random_case(width=width, batch=batch, block_size=block_size,
                                                  dcp_size=gen_dcp, seed=seed)
        for dcp_size, dcp_rank, interleave in geometries:
            geometry = {"block_size": block_size, "dcp_size": dcp_size, "dcp_rank": dcp_rank,
                        "dcp_interleave": interleave}
            entry = {"id": f"{case_id}/d{dcp_size}r{dcp_rank}i{interleave}", "kind": "random_case",
                     "width": width, "batch": batch, "gen_dcp_size": gen_dcp, "seed": seed,
                     **geometry}
            record(np, torch, entry, req_ids, block_table, rows, geometry=geometry,
                   compact=compact, tile_size=tile_size,
                   run_rowwise=width <= 4096, run_hierarchical=width <= 4096)
            cases.append(entry)

    # test_kernels_gpu.py:126-159 parametrization (seed 650000 + width*31 + dcp*7 + rank)
    for width in (1, 63, 128, 129, 513, 1024, 2048, 4096):
        for dcp_size, dcp_rank, interleave in ((1, 0, 1), (2, 1, 2), (4, 3, 4), (8, 7, 1)):
            adversarial(f"widths/w{width}", width=width, batch=3, block_size=64, gen_dcp=dcp_size,
                        seed=650000 + width * 31 + dcp_size * 7 + dcp_rank,
                        geometries=[(dcp_size, dcp_rank, interleave)])
    # test_kernels_gpu.py:162-188: every rank and grouped interleave at width 257
    for dcp_size in (1, 2, 4, 8):
        adversarial(f"ranks/d{dcp_size}", width=257, batch=4, block_size=64, gen_dcp=dcp_size,
                    seed=651000 + dcp_size,
                    geometries=[(dcp_size, r, il) for il in (1, 2, 4) for r in range(dcp_size)])
    # test_kernels_gpu.py:191-211: non-compacting column semantics
    adversarial("noncompact", width=513, batch=3, block_size=32, gen_dcp=4, seed=652001,
                geometries=[(1, 0, 4), (4, 2, 2)], compact=False)
    # test_kernels_gpu.py:232-240 (canaries) and :312-320 (graph replay)
    adversarial("canaries", width=513, batch=3, block_size=64, gen_dcp=4, seed=653001,
                geometries=[(4, 3, 4)])
    adversarial("replay", width=2048, batch=8, block_size=64, gen_dcp=4, seed=654001,
                geometries=[(4, 2, 2)])
    # hierarchical tile sizes the reference supports
    for tile in (64, 256):
        adversarial(f"tiles{tile}", width=1000, batch=3, block_size=64, gen_dcp=4, seed=655000 + tile,
                    geometries=[(4, 1, 1)], tile_size=tile)
    # the conformance matrix with its seeds (silkern/verify.py:389-447 derivation)
    for index, g in enumerate(DEFAULT_MATRIX):
        adversarial(f"matrix/{index}", width=g["width"], batch=5, block_size=g["block_size"],
                    gen_dcp=g["dcp_size"], seed=20260803 + index,
                    geometries=[(g["dcp_size"], g["dcp_rank"], g["dcp_interleave"])])
    print(f"adversarial cases done in {time.time() - started:.1f}s", file=sys.stderr)

    def config(config_id, *, seed, ranks, rowwise, hierarchical, batch=None, tile_size=None):
        for rank in ranks:
            case = config_case(config_id, seed=seed, dcp_rank=rank, batch=batch)
            entry = {"id": f"config{config_id}/s{seed}/r{rank}" + (f"/b{batch}" if batch else ""),
                     "kind": "config", "config": config_id, "seed": seed, "batch_limit": batch,
                     **case.geometry()}
            expected = record(np, torch, entry, case.req_ids, case.block_table, case.tokens,
                              geometry=case.geometry(), run_rowwise=rowwise,
                              run_hierarchical=hierarchical, tile_size=tile_size or case.tile_size)
            cases.append(entry)
            yield case, expected

    # Config 1: the CPU-runnable case, both ranks, full arrays kept.
    arrays = {}
    for case, (out, counts) in config(1, seed=0, ranks=(0, 1), rowwise=True, hierarchical=True):
        arrays["req_ids"] = case.req_ids
        arrays["block_table"] = case.block_table
        arrays["tokens"] = case.tokens
        arrays[f"out_rank{case.dcp_rank}"] = np.asarray(out, dtype=np.int32)
        arrays[f"counts_rank{case.dcp_rank}"] = np.asarray(counts, dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "config1.npz"), **arrays)
    for _ in config(2, seed=2, ranks=(0, 1), rowwise=True, hierarchical=False):
        pass
    for _ in config(3, seed=3, ranks=(0, 1, 2, 3), rowwise=False, hierarchical=False):
        pass
    for _ in config(3, seed=3, ranks=(0, 3), rowwise=True, hierarchical=True, batch=24):
        pass
    for _ in config(4, seed=4, ranks=tuple(range(8)), rowwise=False, hierarchical=False):
        pass
    for _ in config(4, seed=4, ranks=(0, 7), rowwise=False, hierarchical=True, batch=4):
        pass
    print(f"configs 1-4 done in {time.time() - started:.1f}s", file=sys.stderr)
    if not args.skip_config5:
        for layer in range(48):
            for _ in config(5, seed=5000 + layer, ranks=(0, 7), rowwise=False, hierarchical=False):
                pass
        for _ in config(5, seed=5000, ranks=(1, 2, 3, 4, 5, 6), rowwise=True, hierarchical=False,
                        batch=16):
            pass
    print(f"all cases done in {time.time() - started:.1f}s", file=sys.stderr)

    meta = {
        "reference": "StevenWang-CY/silkern",
        "generator": "tests/golden/make_golden.py",
        "digest": "sha256 over little-endian int32 bytes of out then counts "
                  "(tiles: tile_counts then tile_offsets)",
        "oracle": "silkern.localize_reference (silkern/contract.py:67-158)",
        "triton": "reference Triton kernels under TRITON_INTERPRET=1 with the launch parameters "
                  "of silkern/kernels.py:411-434 and :560-633",
    }
    with open(os.path.join(HERE, "golden.json"), "w") as fh:
        json.dump({"meta": meta, "cases": cases}, fh, indent=1)
    print(f"{len(cases)} cases written", file=sys.stderr)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
