"""The fused top-k + localization kernel against its CPU oracle, bit for bit.

The oracle (``oracle.topk``) selects by brute-force partition and localizes
with the converter's C oracle (silkern/contract.py:67-158). Cases cover row
lengths at every edge (0, 1, top_k, top_k + 1, the full width, out of range),
scores with heavy ties, all-equal rows, infinities, signed zeros and NaNs,
every launch geometry, unaligned and padded logits rows, bad request ids,
graph replay, and vLLM's own radix top-k where it is installed.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.topk import select_positions, topk_localize as oracle_topk  # noqa: E402
from silkern_b200 import LocalizationError, localize_rowwise, topk_localize  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA is required", allow_module_level=True)

DEV = torch.device("cuda", 0)


def _values(rng, kind, shape):
    if kind == "normal":
        return rng.standard_normal(shape).astype(np.float32)
    if kind == "ties":
        return rng.integers(-3, 4, size=shape).astype(np.float32)
    if kind == "equal":
        return np.full(shape, 0.25, dtype=np.float32)
    if kind == "special":
        pool = np.array([math.inf, -math.inf, 0.0, -0.0, 1.0, -1.0, np.nan, 1e-40, -1e-40, 3.0],
                        dtype=np.float32)
        return pool[rng.integers(0, len(pool), size=shape)]
    raise ValueError(kind)


def _lens(rng, batch, width, top_k):
    edges = [0, 1, top_k, top_k + 1, width, max(width - 1, 0)]
    lens = rng.integers(0, width + 1, size=batch)
    lens[: min(batch, len(edges))] = [min(e, width) for e in edges[:batch]]
    return lens.astype(np.int32)


def _table(rng, rows, width):
    return rng.integers(-2, 1 << 16, size=(rows, width)).astype(np.int32)


def _dev(a):
    return torch.as_tensor(np.ascontiguousarray(a)).to(DEV)


def _run(logits_t, lens, req, table, top_k, *, positions=True, status=None, **kw):
    batch = logits_t.shape[0]
    out = torch.full((batch, top_k), 0x5A5A5A5A, dtype=torch.int32, device=DEV)
    counts = torch.full((batch,), 0x5A5A5A5A, dtype=torch.int32, device=DEV)
    pos = torch.full((batch, top_k), 0x5A5A5A5A, dtype=torch.int32, device=DEV) if positions else None
    topk_localize(logits_t, _dev(lens), _dev(req), _dev(table), out, counts, positions=pos,
                  status=status, **kw)
    torch.cuda.synchronize()
    return (pos.cpu().numpy() if positions else None), out.cpu().numpy(), counts.cpu().numpy()


GEOMETRIES = [
    dict(block_size=64, dcp_size=1, dcp_rank=0),
    dict(block_size=64, dcp_size=2, dcp_rank=1),
    dict(block_size=64, dcp_size=4, dcp_rank=3, compact_valid_to_front=False),
    dict(block_size=32, dcp_size=8, dcp_rank=5),
    dict(block_size=6, dcp_size=3, dcp_rank=1, dcp_interleave=2),
]
SHAPES = [(1, 100, 64), (3, 2048, 2048), (4, 4097, 2048), (6, 8192, 1), (5, 10000, 7),
          (8, 65536, 2048), (2, 131072, 16384), (2, 262144, 2048)]


KINDS = ["normal", "ties", "equal", "special"]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_matches_oracle(shape, kind) -> None:
    batch, width, top_k = shape
    rng = np.random.default_rng(7200 + 10 * SHAPES.index(shape) + KINDS.index(kind))
    logits = _values(rng, kind, (batch, width))
    lens = _lens(rng, batch, width, top_k)
    table = _table(rng, 9, 1 + width // 64)
    req = rng.integers(0, 9, size=batch).astype(np.int32)
    geometry = GEOMETRIES[(SHAPES.index(shape) + len(kind)) % len(GEOMETRIES)]
    pos, out, counts = _run(_dev(logits), lens, req, table, top_k, **geometry)
    want_pos, want_out, want_counts = oracle_topk(logits, lens, req, table, top_k=top_k, threads=8,
                                                  **geometry)
    assert np.array_equal(pos, want_pos)
    assert np.array_equal(out, want_out)
    assert np.array_equal(counts, want_counts)


@pytest.mark.parametrize("threads", [512, 1024])
@pytest.mark.parametrize("kind", ["normal", "ties"])
@pytest.mark.parametrize(("capacity", "stage"), [(0, 0), (0, 1), (1000, -1), (1500, 1), (20000, 0)])
def test_internal_paths(capacity, stage, kind, threads) -> None:
    """Both selection paths (a capacity of top_k forces the whole-row path),
    both table sources and both CTA shapes."""
    width, top_k, batch = 20000, 1000, 5
    rng = np.random.default_rng(7300 + capacity + stage + len(kind))
    logits = _values(rng, kind, (batch, width))
    lens = _lens(rng, batch, width, top_k)
    table = _table(rng, 5, 200)
    req = np.arange(batch, dtype=np.int32)
    kw = dict(block_size=64, dcp_size=2, dcp_rank=0)
    pos, out, counts = _run(_dev(logits), lens, req, table, top_k, candidate_capacity=capacity,
                            stage_table=stage, cta_threads=threads, **kw)
    want = oracle_topk(logits, lens, req, table, top_k=top_k, **kw)
    assert np.array_equal(pos, want[0]) and np.array_equal(out, want[1]) and np.array_equal(counts, want[2])


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("shape", SHAPES[1:6], ids=lambda s: "x".join(map(str, s)))
def test_small_cta_shape_matches_oracle(shape, kind) -> None:
    """Batches this small launch 1024-thread CTAs; the 512-thread shape of
    larger batches, pinned, gives the same rows."""
    batch, width, top_k = shape
    rng = np.random.default_rng(7400 + 10 * SHAPES.index(shape) + KINDS.index(kind))
    logits = _values(rng, kind, (batch, width))
    lens = _lens(rng, batch, width, top_k)
    table = _table(rng, 9, 1 + width // 64)
    req = rng.integers(0, 9, size=batch).astype(np.int32)
    geometry = GEOMETRIES[(SHAPES.index(shape) + len(kind) + 1) % len(GEOMETRIES)]
    pos, out, counts = _run(_dev(logits), lens, req, table, top_k, cta_threads=512, **geometry)
    want = oracle_topk(logits, lens, req, table, top_k=top_k, threads=8, **geometry)
    assert np.array_equal(pos, want[0]) and np.array_equal(out, want[1]) and np.array_equal(counts, want[2])


def _bin_taken_whole_rows(rng, last_pass, batch, width, top_k):
    """Rows whose radix select ends at `last_pass` because the threshold bin
    there holds exactly the keys still needed. Order keys split 11/11/10 bits:
    an 11-bit bin spans [1024, 1280) at exponent 10, a 22-bit bin 0.125 there.
    """
    logits = rng.standard_normal((batch, width)).astype(np.float32)  # all below 10
    for r in range(batch):
        cols = rng.permutation(width)
        if last_pass == 0:
            # top_k distinct scores alone in [1024, 1280)
            logits[r, cols[:top_k]] = rng.uniform(1024.0, 1279.0, size=top_k)
        elif last_pass == 1:
            # top_k - 10 high scores; the threshold's 11-bit bin holds 30, of
            # which 10 share the top 22-bit bin [1100, 1100.125)
            logits[r, cols[:top_k - 10]] = rng.uniform(2048.0, 2559.0, size=top_k - 10)
            logits[r, cols[top_k - 10:top_k]] = 1100.0 + 0.01 * np.arange(10)
            logits[r, cols[top_k:top_k + 20]] = rng.uniform(1030.0, 1090.0, size=20)
        else:
            # the 22-bit bin [1100, 1100.125) holds 12 with 8 needed: 3 above
            # the threshold and exactly 5 equal to it, taken with no tie cut
            logits[r, cols[:top_k - 8]] = rng.uniform(2048.0, 2559.0, size=top_k - 8)
            logits[r, cols[top_k - 8:top_k - 5]] = 1100.0625
            logits[r, cols[top_k - 5:top_k]] = 1100.03
            logits[r, cols[top_k:top_k + 4]] = 1100.0
    return logits


@pytest.mark.parametrize("capacity", [0, 1000], ids=["list", "whole_row"])
@pytest.mark.parametrize("last_pass", [0, 1, 2])
def test_threshold_bin_taken_whole(last_pass, capacity) -> None:
    """The select ends early when a pass's threshold bin is taken whole."""
    width, top_k, batch = 20000, 1000, 3
    rng = np.random.default_rng(7330 + last_pass)
    logits = _bin_taken_whole_rows(rng, last_pass, batch, width, top_k)
    lens = np.full(batch, width, dtype=np.int32)
    table = _table(rng, batch, 400)
    req = np.arange(batch, dtype=np.int32)
    kw = dict(block_size=64, dcp_size=2, dcp_rank=1)
    pos, out, counts = _run(_dev(logits), lens, req, table, top_k, candidate_capacity=capacity,
                            cta_threads=512 if last_pass == 1 else 0, **kw)
    want = oracle_topk(logits, lens, req, table, top_k=top_k, **kw)
    assert np.array_equal(pos, want[0]) and np.array_equal(out, want[1]) and np.array_equal(counts, want[2])


@pytest.mark.parametrize("stage", [0, 1])
def test_physical_slots_wrap_like_int32_lanes(stage) -> None:
    """Table entries over the whole int32 range: the slot arithmetic overflows
    and wraps mod 2**32, as in the converter and the reference's int32 lanes."""
    batch, width, top_k = 4, 30000, 2048
    rng = np.random.default_rng(7340 + stage)
    logits = rng.standard_normal((batch, width)).astype(np.float32)
    lens = np.array([width, 20000, 2048, 2500], dtype=np.int32)
    table = rng.integers(-(2**31), 2**31, size=(batch, 200), dtype=np.int64).astype(np.int32)
    req = np.array([3, 1, 0, 2], dtype=np.int32)
    kw = dict(block_size=48, dcp_size=3, dcp_rank=2, dcp_interleave=3)
    assert (table.astype(np.int64) * 48 > 2**31 - 1).any()  # the case overflows
    pos, out, counts = _run(_dev(logits), lens, req, table, top_k, stage_table=stage, **kw)
    want = oracle_topk(logits, lens, req, table, top_k=top_k, **kw)
    assert np.array_equal(pos, want[0]) and np.array_equal(out, want[1]) and np.array_equal(counts, want[2])


def test_estimate_misses_fall_back_exactly() -> None:
    """Rows whose sampled columns are unrepresentative: 1000 of the sampled
    float4 groups' columns score high, so the floor lands above all but those
    1000 and fewer than top_k scores clear it."""
    batch, width, top_k = 4, 32768, 2048
    rng = np.random.default_rng(7350)
    logits = rng.standard_normal((batch, width)).astype(np.float32)
    cols = np.arange(width)
    sampled = cols[(cols // 4) % 8 == 0]
    logits[:, sampled[:1000]] += 10.0
    lens = np.array([width, width - 3, 5000, 2049], dtype=np.int32)
    table = _table(rng, 4, 600)
    req = np.arange(batch, dtype=np.int32)
    kw = dict(block_size=16, dcp_size=4, dcp_rank=1)
    pos, out, counts = _run(_dev(logits), lens, req, table, top_k, **kw)
    want = oracle_topk(logits, lens, req, table, top_k=top_k, **kw)
    assert np.array_equal(pos, want[0]) and np.array_equal(out, want[1]) and np.array_equal(counts, want[2])


@pytest.mark.parametrize("layout", ["offset1", "stride_odd", "stride_padded"])
def test_unaligned_and_padded_rows(layout) -> None:
    batch, width, top_k = 4, 9000, 512
    rng = np.random.default_rng(7400)
    logits = _values(rng, "normal", (batch, width))
    if layout == "offset1":  # rows start 4 bytes past a 16-byte boundary: plain loads
        base = torch.empty(batch * width + 1, dtype=torch.float32, device=DEV)
        view = base[1:].view(batch, width)
    else:
        stride = width + (3 if layout == "stride_odd" else 8)
        base = torch.full((batch, stride), float("nan"), dtype=torch.float32, device=DEV)
        view = base[:, :width]
    view.copy_(torch.as_tensor(logits))
    lens = _lens(rng, batch, width, top_k)
    table = _table(rng, 4, 64)
    req = np.arange(batch, dtype=np.int32)
    kw = dict(block_size=64, dcp_size=2, dcp_rank=1)
    pos, out, counts = _run(view, lens, req, table, top_k, **kw)
    want = oracle_topk(logits, lens, req, table, top_k=top_k, **kw)
    assert np.array_equal(pos, want[0]) and np.array_equal(out, want[1]) and np.array_equal(counts, want[2])


def test_without_positions_output() -> None:
    batch, width, top_k = 3, 5000, 700
    rng = np.random.default_rng(7500)
    logits = _values(rng, "normal", (batch, width))
    lens = np.array([5000, 300, 4000], dtype=np.int32)
    table = _table(rng, 3, 100)
    req = np.arange(batch, dtype=np.int32)
    kw = dict(block_size=64, dcp_size=4, dcp_rank=2)
    _, out, counts = _run(_dev(logits), lens, req, table, top_k, positions=False, **kw)
    want = oracle_topk(logits, lens, req, table, top_k=top_k, **kw)
    assert np.array_equal(out, want[1]) and np.array_equal(counts, want[2])


def test_status_flags_bad_lengths_and_requests() -> None:
    batch, width, top_k = 4, 3000, 100
    rng = np.random.default_rng(7600)
    logits = _values(rng, "normal", (batch, width))
    lens = np.array([-5, 3000, 7000, 50], dtype=np.int32)
    table = _table(rng, 3, 50)
    req = np.array([0, 1, 2, 0], dtype=np.int32)
    kw = dict(block_size=64, dcp_size=2, dcp_rank=0)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    pos, out, counts = _run(_dev(logits), lens, req, table, top_k, status=status, **kw)
    assert int(status.item()) == 2  # lengths clamped and flagged; requests fine
    want = oracle_topk(logits, lens, req, table, top_k=top_k, **kw)
    assert np.array_equal(pos, want[0]) and np.array_equal(out, want[1]) and np.array_equal(counts, want[2])

    bad_req = np.array([0, 7, -1, 0], dtype=np.int32)
    status.zero_()
    pos, out, counts = _run(_dev(logits), np.clip(lens, 0, width), bad_req, table, top_k, status=status, **kw)
    assert int(status.item()) == 1
    assert (out[1] == -1).all() and (out[2] == -1).all() and counts[1] == 0 and counts[2] == 0
    rows = select_positions(logits, np.clip(lens, 0, width), top_k)
    assert np.array_equal(pos, rows)  # selection does not depend on the request


def test_graph_replay_is_bitwise_stable() -> None:
    batch, width, top_k = 16, 65536, 2048
    rng = np.random.default_rng(7700)
    logits_t = _dev(_values(rng, "normal", (batch, width)))
    lens_t = _dev(_lens(rng, batch, width, top_k))
    table_t = _dev(_table(rng, batch, 256))
    req_t = _dev(np.arange(batch, dtype=np.int32))
    out = torch.empty((batch, top_k), dtype=torch.int32, device=DEV)
    counts = torch.empty(batch, dtype=torch.int32, device=DEV)
    kw = dict(block_size=64, dcp_size=4, dcp_rank=1)

    def op():
        topk_localize(logits_t, lens_t, req_t, table_t, out, counts, **kw)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        op()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    first = (out.clone(), counts.clone())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(4):
            op()
    allocated = torch.cuda.memory_allocated()
    for _ in range(25):
        out.fill_(-7)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, first[0]) and torch.equal(counts, first[1])
    assert torch.cuda.memory_allocated() == allocated


@pytest.mark.parametrize("kind", ["normal", "ties"])
@pytest.mark.parametrize("above_sm_count", [False, True])
def test_batches_from_half_the_sms_match_oracle(kind, above_sm_count) -> None:
    """From half a row per SM each CTA starts its row streaming into L2 before
    it waits on the previous grid (1024-thread CTAs up to the SM count,
    512-thread ones above it); those batches match the oracle too."""
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    batch = sms + 12 if above_sm_count else sms // 2 + 3
    width, top_k = 4096, 256
    rng = np.random.default_rng(9100 + 2 * KINDS.index(kind) + int(above_sm_count))
    logits = _values(rng, kind, (batch, width))
    lens = _lens(rng, batch, width, top_k)
    table = _table(rng, 11, 1 + width // 64)
    req = rng.integers(0, 11, size=batch).astype(np.int32)
    geometry = dict(block_size=64, dcp_size=4, dcp_rank=1)
    pos, out, counts = _run(_dev(logits), lens, req, table, top_k, **geometry)
    want = oracle_topk(logits, lens, req, table, top_k=top_k, threads=8, **geometry)
    assert np.array_equal(pos, want[0]) and np.array_equal(out, want[1]) and np.array_equal(counts, want[2])


def test_row_lengths_written_by_the_previous_grid() -> None:
    """The length the kernel reads before waiting on the previous grid is only
    a prefetch hint: here the previous grid (a converter call, which lets its
    dependents start at once) is still writing the lengths. Its counts are the
    top-k's row lengths, back to back in one stream, after each round resets
    them to a value past the row; every round matches the oracle on the final
    lengths."""
    import oracle

    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    batch, conv_width, top_k = sms + 12, 2048, 128
    rng = np.random.default_rng(9200)
    conv_geometry = dict(block_size=64, dcp_size=2, dcp_rank=0)
    conv_req = np.arange(batch, dtype=np.int32)
    conv_table = rng.integers(0, 1 << 16, size=(batch, 64)).astype(np.int32)
    tokens = rng.integers(-1, 8192, size=(batch, conv_width)).astype(np.int32)
    _, lens = oracle.localize(conv_req, conv_table, tokens, **conv_geometry)
    assert lens.min() > top_k and lens.max() <= conv_width  # rows past top_k: the sampled path

    logits = rng.standard_normal((batch, conv_width)).astype(np.float32)
    table = _table(rng, 7, 1 + conv_width // 64)
    req = rng.integers(0, 7, size=batch).astype(np.int32)
    geometry = dict(block_size=64, dcp_size=4, dcp_rank=2)
    want = oracle_topk(logits, lens, req, table, top_k=top_k, threads=8, **geometry)

    conv_in = [_dev(a) for a in (conv_req, conv_table, tokens)]
    conv_out = torch.empty((batch, conv_width), dtype=torch.int32, device=DEV)
    seq_lens = torch.empty(batch, dtype=torch.int32, device=DEV)
    logits_t, req_t, table_t = _dev(logits), _dev(req), _dev(table)
    for _ in range(4):
        out = torch.full((batch, top_k), 0x5A5A5A5A, dtype=torch.int32, device=DEV)
        counts = torch.full((batch,), 0x5A5A5A5A, dtype=torch.int32, device=DEV)
        pos = torch.full((batch, top_k), 0x5A5A5A5A, dtype=torch.int32, device=DEV)
        seq_lens.fill_(5 * conv_width)  # past the row until the converter writes it
        localize_rowwise(*conv_in, conv_out, seq_lens, **conv_geometry)
        topk_localize(logits_t, seq_lens, req_t, table_t, out, counts, positions=pos, **geometry)
        torch.cuda.synchronize()
        assert np.array_equal(seq_lens.cpu().numpy(), lens)
        assert np.array_equal(pos.cpu().numpy(), want[0])
        assert np.array_equal(out.cpu().numpy(), want[1]) and np.array_equal(counts.cpu().numpy(), want[2])


def test_matches_vllm_radix_topk_then_converter() -> None:
    """vLLM's decode top-k (``torch.ops._C.persistent_topk``) selects the same sets.

    Scores are distinct (a permutation), so the top-k set is unique; vLLM's
    output order is its own, so rows are compared sorted, and our converter
    on vLLM's sorted selection must reproduce the fused output.
    """
    pytest.importorskip("vllm._custom_ops")
    batch, width, top_k = 32, 65536, 2048
    rng = np.random.default_rng(7800)
    logits = np.stack([rng.permutation(width) for _ in range(batch)]).astype(np.float32)
    lens = rng.integers(1024, width + 1, size=batch).astype(np.int32)
    lens[:3] = [top_k, top_k - 5, width]
    table = _table(rng, batch, 256)
    req = np.arange(batch, dtype=np.int32)
    kw = dict(block_size=64, dcp_size=4, dcp_rank=2)
    logits_t, lens_t = _dev(logits), _dev(lens)
    pos, out, counts = _run(logits_t, lens, req, table, top_k, **kw)

    vllm_rows = torch.empty((batch, top_k), dtype=torch.int32, device=DEV)
    workspace = torch.zeros(1024 * 1024, dtype=torch.uint8, device=DEV)
    torch.ops._C.persistent_topk(logits_t, lens_t, vllm_rows, workspace, top_k, int(lens.max()))
    torch.cuda.synchronize()
    got = vllm_rows.cpu().numpy()
    sorted_rows = np.full_like(got, -1)
    for b in range(batch):
        n = min(int(lens[b]), top_k)
        sorted_rows[b, :n] = np.sort(got[b, :n])
    assert np.array_equal(sorted_rows, pos)
    conv_out = torch.empty_like(vllm_rows)
    conv_counts = torch.empty(batch, dtype=torch.int32, device=DEV)
    localize_rowwise(_dev(req), _dev(table), _dev(sorted_rows), conv_out, conv_counts, **kw)
    torch.cuda.synchronize()
    assert np.array_equal(conv_out.cpu().numpy(), out)
    assert np.array_equal(conv_counts.cpu().numpy(), counts)


def test_launcher_rejections() -> None:
    logits = torch.zeros((2, 100), dtype=torch.float32, device=DEV)
    lens = torch.full((2,), 100, dtype=torch.int32, device=DEV)
    req = torch.zeros(2, dtype=torch.int32, device=DEV)
    table = torch.zeros((1, 4), dtype=torch.int32, device=DEV)
    out = torch.empty((2, 16), dtype=torch.int32, device=DEV)
    counts = torch.empty(2, dtype=torch.int32, device=DEV)
    kw = dict(block_size=64, dcp_size=2, dcp_rank=0)
    with pytest.raises(LocalizationError, match="float32"):
        topk_localize(logits.double(), lens, req, table, out, counts, **kw)
    with pytest.raises(LocalizationError, match="one element per row"):
        topk_localize(logits, lens[:1], req, table, out, counts, **kw)
    with pytest.raises(LocalizationError, match="must not share storage"):
        topk_localize(logits, lens, req, table, out, out.view(-1)[:2], **kw)
    with pytest.raises(LocalizationError, match="unit column stride"):
        topk_localize(logits.t(), lens, req, table, out, counts, **kw)
    with pytest.raises(LocalizationError, match="top_k exceeds"):
        topk_localize(logits, lens, req, table, torch.empty((2, 16385), dtype=torch.int32, device=DEV),
                      counts, **kw)
    with pytest.raises(LocalizationError, match="invalid dcp configuration"):
        topk_localize(logits, lens, req, table, out, counts, block_size=64, dcp_size=2, dcp_rank=2)
