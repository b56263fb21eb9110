"""ugdr_x_moe_route_noalloc, the MoE routing entry point for callers that may not allocate
device memory (its scratch lives in a fixed array inside libugdr), called through its exported C
symbol and checked against ugdr_x_moe_route, whose scratch the caller allocates.

Collected last on purpose: a run that stops at the first failure has run everything else."""
from __future__ import annotations

import ctypes as C

import pytest

from conftest import gpu_count

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _lib():
    from ugdr_b200 import _native as N

    L = N.lib()
    f = L.ugdr_x_moe_route_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_uint64, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    g = L.ugdr_x_moe_route
    g.restype = C.c_int
    g.argtypes = [C.c_void_p, C.c_uint64, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]
    L.ugdr_x_moe_route_scratch_bytes.restype = C.c_size_t
    L.ugdr_x_moe_route_scratch_bytes.argtypes = [C.c_uint64, C.c_int]
    return L


def _run(L, fn, ids, nexp, scratch=None):
    rows = ids.numel()
    counts = torch.full((nexp,), -7, dtype=torch.int32, device="cuda")
    pos = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if scratch is None:
        rc = fn(C.c_void_p(ids.data_ptr()), rows, nexp, C.c_void_p(counts.data_ptr()), C.c_void_p(pos.data_ptr()), s)
    else:
        rc = fn(C.c_void_p(ids.data_ptr()), rows, nexp, C.c_void_p(counts.data_ptr()), C.c_void_p(pos.data_ptr()),
                C.c_void_p(scratch.data_ptr()), scratch.numel(), s)
    torch.cuda.synchronize()
    return rc, counts, pos


def test_noalloc_route_matches_allocating_route_twice():
    if gpu_count() < 1:
        pytest.skip("no GPU")
    torch.cuda.set_device(0)
    L = _lib()
    gen = torch.Generator(device="cuda").manual_seed(11)
    # Two calls in a row with different shapes: the second must not see the first's leftovers.
    for tokens, nexp, topk in ((16384, 256, 8), (3000, 64, 4)):
        ids = torch.randint(0, nexp, (tokens * topk,), dtype=torch.int32, device="cuda", generator=gen)
        scratch = torch.empty(L.ugdr_x_moe_route_scratch_bytes(ids.numel(), nexp), dtype=torch.uint8, device="cuda")
        rc_ref, c_ref, p_ref = _run(L, L.ugdr_x_moe_route, ids, nexp, scratch)
        rc, c, p = _run(L, L.ugdr_x_moe_route_noalloc, ids, nexp)
        assert rc_ref == 0 and rc == 0
        assert torch.equal(c, c_ref)  # integer outputs: exact match
        assert torch.equal(p, p_ref)


def test_noalloc_route_rejects_oversized_calls():
    if gpu_count() < 1:
        pytest.skip("no GPU")
    torch.cuda.set_device(0)
    L = _lib()
    rows = 4096 * 300  # 300 blocks x 256 experts > 65536 entries
    ids = torch.zeros(rows, dtype=torch.int32, device="cuda")
    rc, c, _ = _run(L, L.ugdr_x_moe_route_noalloc, ids, 256)
    assert rc != 0
    assert int((c == -7).sum()) == 256  # nothing was launched
