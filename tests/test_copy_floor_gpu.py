"""The copy-floor reference kernel: an exact copy at every size, offset and CTA shape."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from silkern_b200.kernels import copy_floor  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA is required", allow_module_level=True)


@pytest.mark.parametrize("ctas_per_sm", [0, 1, 4])
@pytest.mark.parametrize("run", [8, 16])
@pytest.mark.parametrize("threads", [32, 256, 1024])
@pytest.mark.parametrize("n", [1, 7, 8, 255, 4096, 524288 + 13])
@pytest.mark.parametrize("offset", [0, 1, 4])
def test_copy_floor_copies_exactly(ctas_per_sm, run, threads, n, offset) -> None:
    gen = torch.Generator().manual_seed(n * 31 + offset)
    base_src = torch.randint(-(2**31), 2**31 - 1, (n + 8,), generator=gen, dtype=torch.int32).cuda()
    base_dst = torch.full((n + 8,), 7, dtype=torch.int32, device="cuda")
    src = base_src[offset:offset + n]
    dst = base_dst[offset:offset + n]
    copy_floor(src, dst, run=run, threads=threads, ctas_per_sm=ctas_per_sm)
    torch.cuda.synchronize()
    assert torch.equal(dst, src)
    # Nothing outside the destination view is written.
    assert torch.all(base_dst[:offset] == 7) and torch.all(base_dst[offset + n:] == 7)
