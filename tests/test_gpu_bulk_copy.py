"""The TMA bulk-copy diagnostic kernel (global -> this CTA's shared memory -> global) against
torch's copy: byte-exact over sizes that end mid-stage and mid-chunk, guard bytes
untouched, misaligned requests refused.  It also times the copy against the load/store copy
core on one buffer larger than L2.

Marked gpu_extended (run with `pytest -m gpu_extended` on a B200 box) until it has run there.
"""
from __future__ import annotations

import pytest

from conftest import gpu_count

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu_extended


@pytest.fixture(scope="module")
def dev():
    if gpu_count() < 1:
        pytest.skip("no GPU")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


@pytest.mark.parametrize("n", [16, 4096, 32768, 32768 + 16, 5 * 32768 + 48, (64 << 20) + 4096])
def test_bulk_copy_is_byte_exact(dev, n):
    from ugdr_b200 import ops

    g = torch.Generator(device=dev).manual_seed(n)
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g)
    dst = torch.zeros(n + 64, dtype=torch.uint8, device=dev)
    ops.bulk_copy_ms(dst[:n], src, iters=1)
    torch.cuda.synchronize()
    assert torch.equal(dst[:n], src)
    assert int(dst[n:].sum()) == 0


def test_bulk_copy_refuses_misaligned(dev):
    from ugdr_b200 import ops

    src = torch.zeros(4096, dtype=torch.uint8, device=dev)
    dst = torch.zeros(4096, dtype=torch.uint8, device=dev)
    with pytest.raises(RuntimeError):
        ops.bulk_copy_ms(dst[8:], src[:1000], iters=1)


def test_bulk_copy_rate_against_the_copy_core(dev):
    from ugdr_b200 import ops

    n = 1 << 30
    src = torch.ones(n, dtype=torch.uint8, device=dev)
    dst = torch.empty(n, dtype=torch.uint8, device=dev)
    t_bulk = ops.bulk_copy_ms(dst, src, iters=10)
    t_core = ops.grid_copy_ms(dst, src, iters=10)
    gbs = lambda t: 2 * n / (t * 1e-3) / 1e9  # noqa: E731  read + write bytes
    print(f"bulk copy {gbs(t_bulk):.0f} GB/s, copy core {gbs(t_core):.0f} GB/s (1 GiB, read + write)")
    assert torch.equal(dst[:4096], src[:4096])
    assert t_bulk > 0 and t_core > 0
