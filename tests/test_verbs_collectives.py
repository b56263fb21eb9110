"""Allreduce on the verbs (ugdr_x_verbs_allreduce_bf16) as separate processes over gloo.

CPU: 2 and 3 ranks on the host engine (host memory), uneven sizes, several calls in a row; the
result must equal, bit for bit, the fp32 sum x_0 + ... + x_{n-1} of every rank's seeded input
rounded once to bf16.  GPU (marked gpu): the same on the executors, one GPU per rank, when the
box has that many GPUs.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import gpu_count


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(rank: int, count: int, call: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(1000 * call + rank)
    return torch.randn(count, generator=g).to(torch.bfloat16)


def _expected(world: int, count: int, call: int) -> torch.Tensor:
    acc = torch.zeros(count, dtype=torch.float32)
    for q in range(world):
        acc += _inputs(q, count, call).float()
    return acc.to(torch.bfloat16)


def _worker(rank: int, world: int, port: int, gpu: bool, counts: list, pieces: int, errq) -> None:
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    daemon = None
    try:
        from ugdr_b200.parallel.verbs_collectives import VerbsGroup, shared_daemon

        def bcast(obj):
            lst = [obj]
            dist.broadcast_object_list(lst, src=0)
            return lst[0]

        def exchange(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        if gpu:
            torch.cuda.set_device(rank)
        daemon = shared_daemon(rank, world, bcast, gpus=world if gpu else 0)
        g = VerbsGroup(rank, world, rank if gpu else 0, max(counts), exchange, pieces=pieces,
                       device_kind=1 if gpu else 0)
        try:
            for call, count in enumerate(counts):
                g.buf[:count].copy_(_inputs(rank, count, call).to(g.buf.device))
                if gpu:
                    torch.cuda.synchronize()
                dist.barrier()
                g.allreduce(count)
                got = g.buf[:count].cpu()
                want = _expected(world, count, call)
                bad = (got.view(torch.int16) != want.view(torch.int16)).nonzero()
                if bad.numel():
                    i = int(bad[0])
                    raise AssertionError(f"rank {rank} call {call}: {bad.numel()} elements differ, first {i}: "
                                         f"{got[i].item()} != {want[i].item()}")
            dist.barrier()
        finally:
            g.close()
        dist.barrier()
    except BaseException as e:  # report to the parent, which asserts
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        if daemon is not None:
            daemon.stop()
        dist.destroy_process_group()


def _run(world: int, gpu: bool, counts: list, pieces: int) -> None:
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, gpu, counts, pieces, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


@pytest.mark.parametrize("world,counts,pieces", [(2, [4096, 1000, 8], 3), (3, [3 * 8 * 50 + 5, 77], 2)])
def test_verbs_allreduce_on_the_host_engine(world, counts, pieces):
    _run(world, False, counts, pieces)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_verbs_allreduce_on_the_executors(world):
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run(world, True, [(1 << 24) + 40, 3 * 8 * 1000 + 3], 4)


# ---- MoE all-to-all on the verbs ------------------------------------------------------------------


def _moe_inputs(rank: int, T: int, H: int, K: int, E: int, call: int, dev):
    from ugdr_b200.models.moe import route

    g = torch.Generator().manual_seed(10_000 * call + 10 + rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids, w = route(T, E, K, seed=10_000 * call + 20 + rank, device="cpu")
    if call >= 2:  # skewed: every token picks among K experts only, so most expert groups are empty
        allowed = torch.tensor([e * E // K for e in range(K - 1)] + [E - 1], dtype=torch.int32)
        ids = allowed[torch.argsort(torch.rand(T, K, generator=g), dim=1)]
    return x.to(dev), ids.to(dev), w.to(dev)


def _moe_expected_recv(q: int, world: int, T: int, H: int, K: int, E: int, call: int) -> torch.Tensor:
    """Owner q's receive area: its experts in order, inside each the source ranks in order, inside
    each source its rows of that expert in (token, k) order."""
    from ugdr_b200.models.moe import reference_positions

    epr = E // world
    parts = []
    srcs = [_moe_inputs(s, T, H, K, E, call, "cpu") for s in range(world)]
    for e in range(q * epr, (q + 1) * epr):
        for s in range(world):
            x, ids, _ = srcs[s]
            counts, pos = reference_positions(ids, E)
            flat = ids.reshape(-1)
            sel = (flat == e).nonzero().reshape(-1)
            order = sel[torch.argsort(pos.reshape(-1)[sel])]
            parts.append(x[order // K])
    return torch.cat(parts) if parts else torch.empty(0, H, dtype=torch.bfloat16)


def _moe_worker(rank: int, world: int, port: int, gpu: bool, shape: tuple, calls: int, errq) -> None:
    import torch.distributed as dist

    T, H, K, E = shape
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    daemon = None
    try:
        from ugdr_b200.parallel.verbs_collectives import VerbsMoE, moe_group, shared_daemon

        def bcast(obj):
            lst = [obj]
            dist.broadcast_object_list(lst, src=0)
            return lst[0]

        def exchange(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        dev = f"cuda:{rank}" if gpu else "cpu"
        if gpu:
            torch.cuda.set_device(rank)
        daemon = shared_daemon(rank, world, bcast, gpus=world if gpu else 0)
        g = moe_group(rank, world, rank if gpu else 0, T, K, E, exchange, device_kind=1 if gpu else 0)
        moe = VerbsMoE(g, T, H, K, E, recv_rows=T * K * world)
        try:
            for call in range(calls):
                x, ids, w = _moe_inputs(rank, T, H, K, E, call, dev)
                # The calls alternate the packed dispatch (one WRITE per expert group) and the
                # 32-SGE gathers, on the host engine and on the executors.
                moe.dispatch(x, ids, packed=call % 2 == 0)
                got = moe.recv_view().cpu()
                want = _moe_expected_recv(rank, world, T, H, K, E, call)
                assert got.shape == want.shape, (got.shape, want.shape)
                assert torch.equal(got, want), f"rank {rank} call {call}: receive area differs"
                out = moe.combine(w)
                if gpu:
                    torch.cuda.synchronize()
                # Rows read back, grouped by expert in position order: row (t, k) at start[e] + pos.
                idx = (moe.start_d[moe.ids_d.long()] + moe.pos_d.long()).cpu()
                back = moe.back.cpu()[idx]
                assert torch.equal(back, x.cpu().repeat_interleave(K, dim=0)), f"rank {rank}: rows read back differ"
                ref = x.cpu().float() * w.cpu().sum(-1, keepdim=True)
                assert torch.allclose(out.cpu().float(), ref, atol=2e-2, rtol=1e-2), f"rank {rank}: combine"
                dist.barrier()
        finally:
            moe.close()
            g.close()
        dist.barrier()
    except BaseException as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        if daemon is not None:
            daemon.stop()
        dist.destroy_process_group()


def _run_moe(world: int, gpu: bool, shape: tuple, calls: int) -> None:
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_moe_worker, args=(r, world, port, gpu, shape, calls, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


@pytest.mark.parametrize("world,shape", [(2, (64, 64, 4, 8)), (3, (50, 32, 2, 6))])
def test_verbs_moe_exact_permutation_on_the_host_engine(world, shape):
    """Every owner's receive area equals, row for row, the expected expert-grouped permutation of
    every rank's tokens; combine reads every row back to its (token, k) slot and weights it.
    Calls 2 and 3 route to a few experts only (most groups empty), packed and gathered."""
    _run_moe(world, False, shape, calls=4)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_verbs_moe_exact_permutation_on_the_executors(world):
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run_moe(world, True, (512, 1024, 8, 32), calls=2)


# ---- allreduce through NVLink SHARP on the verbs (multicast MR) -----------------------------------


def _nvls_worker(rank: int, world: int, port: int, count: int, errq) -> None:
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    daemon = None
    try:
        from ugdr_b200.parallel import nvls
        from ugdr_b200.parallel.verbs_collectives import VerbsGroup, shared_daemon

        def bcast(obj):
            lst = [obj]
            dist.broadcast_object_list(lst, src=0)
            return lst[0]

        def exchange(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        torch.cuda.set_device(rank)
        daemon = shared_daemon(rank, world, bcast)
        g = VerbsGroup(rank, world, rank, 8, exchange, pieces=1)
        buf = nvls.NvlsBuffer(count * 2, rank, world, exchange)
        try:
            for call in range(2):
                v = buf.view(torch.bfloat16, count)
                v.copy_(_inputs(rank, count, call).cuda())
                torch.cuda.synchronize()
                g.allreduce_nvls(buf, count)
                got = v.cpu()
                want = _expected(world, count, call).float()
                # The switch accumulates in fp32 in its own order and rounds once.
                bad = (got.float() - want).abs() > want.abs() * 2.0 ** -7 + 1e-3
                assert not bool(bad.any()), f"rank {rank} call {call}: {int(bad.sum())} elements off"
                del v
                dist.barrier()
        finally:
            g.release_multicast()  # the daemon's mapping goes before any rank unbinds
            dist.barrier()
            buf.close()
            g.close()
        dist.barrier()
    except BaseException as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        if daemon is not None:
            daemon.stop()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_verbs_nvls_allreduce_on_the_executors(world):
    """One WRITE_SUM_BF16 per rank from and to its shard of a multicast MR: the executor's
    multimem loads have the NVSwitch sum, its multimem stores broadcast."""
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from ugdr_b200.parallel import nvls

    if not nvls.supported(0):
        pytest.skip("no NVLS multicast on this box")
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nvls_worker, args=(r, world, port, (1 << 22) + 64, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_multicast_mr_needs_a_gpu_context(cpu_daemon):
    """The host engine cannot reach NVLink multicast memory: registration is refused."""
    from ugdr_b200 import verbs as V

    ctx = V.Context(V.find_device(kind=0))
    pd = ctx.alloc_pd()
    r, w = os.pipe()
    try:
        with pytest.raises(V.UgdrError):
            pd.reg_mr_multicast(1 << 21, 1 << 21, 1, r)
        with pytest.raises(V.UgdrError):
            pd.reg_mr_multicast(1 << 21, 1 << 21, 1, -1)
    finally:
        os.close(r)
        os.close(w)
        pd.dealloc()
        ctx.close()


def test_verbs_collectives_example_on_host_memory():
    """examples/verbs_collectives.py runs end to end on the host-memory device (2 ranks, torchrun)."""
    import subprocess
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
                        os.path.join(repo, "examples", "verbs_collectives.py"), "--cpu"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "verbs collectives ok on 2 ranks (host memory)" in r.stdout


def test_packed_dispatch_and_pack_reject_missing_arguments():
    """The packed dispatch refuses a missing group, descriptor or count table (EINVAL) and the
    pack refuses missing pointers (cudaErrorInvalidValue) before touching any device."""
    import errno

    from ugdr_b200.parallel.verbs_collectives import _moe_lib

    L = _moe_lib()
    assert L.ugdr_x_verbs_moe_dispatch_packed(None, None, None, 0) == errno.EINVAL
    assert L.ugdr_x_moe_pack_grouped(None, None, None, None, None, 16, 2, 32, 0, None) == 1
