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
