"""Collective kernels against plain torch fp32 references: MoE routing (1 GPU), allreduce and
the MoE all-to-all on 1 rank and on 2 ranks (one process per GPU, gloo for the handle exchange)."""
from __future__ import annotations

import os

import pytest

from conftest import gpu_count

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def one_gpu():
    if gpu_count() < 1:
        pytest.skip("no GPU")
    torch.cuda.set_device(0)


@pytest.mark.parametrize("tokens,experts,topk", [(1, 8, 2), (1000, 256, 8), (16384, 256, 8), (5000, 64, 3)])
def test_moe_route_matches_reference(one_gpu, tokens, experts, topk):
    from ugdr_b200.models.moe import reference_positions, route
    from ugdr_b200.parallel.collectives import moe_route

    ids, _ = route(tokens, experts, topk, seed=tokens)
    counts, pos = moe_route(ids, experts)
    rc, rp = reference_positions(ids, experts)
    assert torch.equal(counts, rc)
    assert torch.equal(pos, rp)


def test_moe_route_rejects_out_of_range_ids(one_gpu):
    from ugdr_b200.parallel.collectives import moe_route

    ids = torch.tensor([[0, 5], [9, 1], [-1, 0]], dtype=torch.int32, device="cuda")
    counts, pos = moe_route(ids, 8)
    assert counts.tolist() == [2, 1, 0, 0, 0, 1, 0, 0]
    assert pos.tolist() == [[0, 0], [-1, 0], [-1, 1]]


@pytest.mark.parametrize("tokens,hidden,experts,topk", [(1, 8, 4, 1), (777, 1024, 64, 8), (300, 7168, 256, 3)])
def test_pack_grouped_and_grouped_weighted_sum(one_gpu, tokens, hidden, experts, topk):
    """ugdr_x_moe_pack_grouped places row (t, k) at start[e] + pos exactly (a permutation, bit for
    bit), and ugdr_x_moe_weighted_sum_grouped on that layout matches an fp32 torch weighted sum."""
    from ugdr_b200.models.moe import route
    from ugdr_b200.parallel.collectives import moe_route
    from ugdr_b200.parallel.verbs_collectives import _moe_lib

    L = _moe_lib()
    ids, w = route(tokens, experts, topk, seed=tokens + hidden)
    counts, pos = moe_route(ids, experts)
    x = torch.randn(tokens, hidden, device="cuda").to(torch.bfloat16)
    ids_d = ids.reshape(-1).to(torch.int32).contiguous()
    pos_d = pos.reshape(-1).to(torch.int32).contiguous()
    c64 = counts.to(torch.int64)
    start = torch.cumsum(c64, 0) - c64
    rows = torch.full((tokens * topk, hidden), float("nan"), device="cuda", dtype=torch.bfloat16)
    s = torch.cuda.current_stream().cuda_stream
    assert L.ugdr_x_moe_pack_grouped(rows.data_ptr(), x.data_ptr(), ids_d.data_ptr(), pos_d.data_ptr(),
                                     start.data_ptr(), tokens, topk, hidden * 2, 0, s) == 0
    torch.cuda.synchronize()
    idx = start[ids_d.long()] + pos_d.long()
    assert torch.equal(torch.sort(idx).values, torch.arange(tokens * topk, device="cuda"))
    assert torch.equal(rows[idx], x.repeat_interleave(topk, dim=0))
    wf = w.reshape(-1).to(device="cuda", dtype=torch.float32).contiguous()
    out = torch.empty(tokens, hidden, device="cuda", dtype=torch.bfloat16)
    assert L.ugdr_x_moe_weighted_sum_grouped(out.data_ptr(), rows.data_ptr(), ids_d.data_ptr(), pos_d.data_ptr(),
                                             start.data_ptr(), wf.data_ptr(), tokens, topk, hidden * 2, 0, s) == 0
    torch.cuda.synchronize()
    ref = (x.float().unsqueeze(1) * wf.view(tokens, topk, 1)).sum(1)
    assert torch.allclose(out.float(), ref, atol=1e-2, rtol=1e-2)


def _single_rank_group(nbytes):
    from ugdr_b200.parallel.peers import PeerGroup

    return PeerGroup(nbytes, 0, 1, lambda x: [x])


def test_allreduce_single_rank_is_identity(one_gpu):
    from ugdr_b200.parallel.collectives import allreduce_bf16

    g = _single_rank_group(1 << 20)
    x = g.view(torch.bfloat16, 1 << 19)
    x.copy_(torch.randn(1 << 19, device="cuda").to(torch.bfloat16))
    ref = x.clone()
    allreduce_bf16(g, 1 << 19)
    torch.cuda.synchronize()
    g.check_status()
    assert torch.equal(x, ref)


def test_missing_peer_times_out_with_status(one_gpu):
    """A bounded cross-GPU wait that runs out: a 2-rank peer set in one process whose "peer"
    buffers are local allocations that nothing signals.  The allreduce's waits give up after the
    configured bound, the kernel reports status 1 and returns, and the GPU stays usable."""
    import ctypes as C
    import time

    from ugdr_b200.parallel.collectives import allreduce_bf16
    from ugdr_b200.parallel.peers import MAX_RANKS, SLOTS, lib

    L = lib()
    L.ugdr_x_set_collective_wait_ns.restype = C.c_uint64
    L.ugdr_x_set_collective_wait_ns.argtypes = [C.c_uint64]
    g = _single_rank_group(1 << 20)
    fake_buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    fake_sig = torch.zeros(SLOTS * MAX_RANKS, dtype=torch.int64, device="cuda")
    g.ps.n = 2
    g.ps.buf[1] = fake_buf.data_ptr()
    g.ps.signal[1] = fake_sig.data_ptr()
    old = L.ugdr_x_set_collective_wait_ns(2_000_000)  # 2 ms
    try:
        torch.cuda.synchronize()
        t0 = time.monotonic()
        allreduce_bf16(g, 1 << 19)
        torch.cuda.synchronize()
        elapsed = time.monotonic() - t0
    finally:
        L.ugdr_x_set_collective_wait_ns(old)
    assert int(g.status.item()) == 1
    assert elapsed < 2.0
    # The context is intact: an ordinary single-rank call still works.
    g.status.zero_()
    g.ps.n = 1
    x = g.view(torch.bfloat16, 1024)
    x.fill_(1.5)
    allreduce_bf16(g, 1024)
    torch.cuda.synchronize()
    g.check_status()
    assert torch.all(x == 1.5)


def test_moe_all_to_all_single_rank(one_gpu):
    from ugdr_b200.models.moe import route
    from ugdr_b200.parallel.collectives import MoEAllToAll

    tokens, hidden, topk, experts = 512, 1024, 4, 16
    recv = tokens * topk
    g = _single_rank_group(MoEAllToAll.required_bytes(1, experts, hidden, recv))
    a2a = MoEAllToAll(g, tokens, hidden, topk, experts, recv)
    x = torch.randn(tokens, hidden, device="cuda").to(torch.bfloat16)
    ids, w = route(tokens, experts, topk, seed=1)
    a2a.dispatch(x, ids)
    out = a2a.combine(w)
    torch.cuda.synchronize()
    g.check_status()
    # Rows landed grouped by expert, in token order inside each group.
    rv = a2a.recv_view()
    flat = ids.reshape(-1).long()
    order = torch.sort(flat, stable=True).indices
    assert torch.equal(rv[:recv], x[order // topk])
    ref = (x.float() * w.sum(-1, keepdim=True)).to(torch.bfloat16)
    assert torch.allclose(out.float(), ref.float(), atol=2e-2, rtol=1e-2)


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world)

        def exchange(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        from ugdr_b200.models.moe import route
        from ugdr_b200.parallel.collectives import MoEAllToAll, allreduce_bf16
        from ugdr_b200.parallel.peers import PeerGroup

        # allreduce: bf16 inputs, fp32 reference, several calls in a row
        n = (3 << 20) + 8
        g = PeerGroup(n * 2, rank, world, exchange)
        for it in range(3):
            xs = [torch.randn(n, generator=torch.Generator().manual_seed(100 * it + r)).to(torch.bfloat16)
                  for r in range(world)]
            v = g.view(torch.bfloat16, n)
            v.copy_(xs[rank].cuda())
            torch.cuda.synchronize()
            dist.barrier()
            allreduce_bf16(g, n)
            torch.cuda.synchronize()
            g.check_status()
            ref = sum(x.float() for x in xs)
            # One rounding of an fp32 sum: within half a bf16 ulp (2^-8 relative), plus fp32
            # summation-order noise near zero.
            bad = (v.float().cpu() - ref).abs() > ref.abs() * 2.0 ** -8 + 1e-4
            assert not bool(bad.any()), f"allreduce: {int(bad.sum())} elements beyond half a bf16 ulp"
        # The same through NVLS multicast memory (reduction inside the NVSwitch), when available.
        from ugdr_b200.parallel import nvls

        if nvls.supported():
            sig = PeerGroup(4096, rank, world, exchange)
            buf = nvls.NvlsBuffer(n * 2, rank, world, exchange)
            errs = []
            try:
                for it in range(3):
                    xs = [torch.randn(n, generator=torch.Generator().manual_seed(500 + 100 * it + r)).to(
                        torch.bfloat16) for r in range(world)]
                    v = buf.view(torch.bfloat16, n)
                    v.copy_(xs[rank].cuda())
                    torch.cuda.synchronize()
                    dist.barrier()
                    nvls.allreduce_bf16_nvls(sig, buf, n)
                    torch.cuda.synchronize()
                    sig.check_status()
                    ref = sum(x.float() for x in xs)
                    errs.append((v.float().cpu() - ref).abs().max().item() / (1 + ref.abs().max().item()))
                    del v
            finally:
                buf.close()  # collective, before any rank can leave with memory bound
            sig.close()
            assert max(errs) <= 0.05 / 8, f"NVLS allreduce errors {errs}"
        # MoE all-to-all
        tokens, hidden, topk, experts = 1024, 2048, 8, 32
        recv = tokens * topk * world
        mg = PeerGroup(MoEAllToAll.required_bytes(world, experts, hidden, recv), rank, world, exchange)
        a2a = MoEAllToAll(mg, tokens, hidden, topk, experts, recv)
        x = torch.randn(tokens, hidden, generator=torch.Generator().manual_seed(rank)).to(torch.bfloat16).cuda()
        ids, w = route(tokens, experts, topk, seed=7 + rank)
        for _ in range(2):
            a2a.dispatch(x, ids)
            out = a2a.combine(w)
        torch.cuda.synchronize()
        mg.check_status()
        ref = (x.float() * w.sum(-1, keepdim=True)).to(torch.bfloat16)
        assert torch.allclose(out.float(), ref.float(), atol=3e-2, rtol=2e-2)
        # Receive side, row for row: this rank's experts in order, inside each the source ranks in
        # order, inside each source its rows of that expert in (token, k) order.
        from ugdr_b200.models.moe import reference_positions

        used = int(a2a.recv_used.item())
        epr = experts // world
        parts = []
        srcs = []
        for s_ in range(world):
            xs_ = torch.randn(tokens, hidden, generator=torch.Generator().manual_seed(s_)).to(torch.bfloat16).cuda()
            ids_s, _ = route(tokens, experts, topk, seed=7 + s_)
            srcs.append((xs_, ids_s))
        for e in range(rank * epr, (rank + 1) * epr):
            for xs_, ids_s in srcs:
                _, pos_s = reference_positions(ids_s, experts)
                flat = ids_s.reshape(-1)
                sel = (flat == e).nonzero().reshape(-1)
                order = sel[torch.argsort(pos_s.reshape(-1)[sel])]
                parts.append(xs_[order // topk])
        want = torch.cat(parts)
        assert used == want.shape[0], (used, want.shape)
        assert torch.equal(a2a.recv_view()[:used], want), "receive area differs from the expected permutation"
        dist.barrier()
        q.put((rank, "ok"))
    except BaseException as e:  # report to the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_rank_allreduce_and_moe(world):
    """Allreduce (fused kernel and NVLS) against an fp32 sum, and the MoE receive areas row for row
    against the expected permutation, on 2, 4 and 8 GPUs (skipped when the box has fewer)."""
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + world + os.getpid() % 200
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    results = {}
    try:
        for _ in ps:
            r, msg = q.get(timeout=300)
            results[r] = msg
    finally:
        for p in ps:
            p.join(60)
            if p.is_alive():
                p.kill()
    assert results == {r: "ok" for r in range(world)}, results
