"""Collectives on the verbs API from PyTorch: a bf16 allreduce and an MoE dispatch + combine whose
every byte moves as RDMA work requests that the daemon runs, each checked against plain torch.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/verbs_collectives.py          # GPUs
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/verbs_collectives.py --cpu    # host memory

One process per rank; torch.distributed (gloo) only starts the shared daemon, exchanges the QP
numbers and rkeys, and gathers the reference inputs for the checks.  With --cpu the same
schedules run on the daemon's host-memory device, so the example needs no GPU.
"""
from __future__ import annotations

import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from ugdr_b200.models.moe import reference_positions  # noqa: E402
from ugdr_b200.parallel.verbs_collectives import VerbsGroup, VerbsMoE, moe_group, shared_daemon  # noqa: E402


def main() -> None:
    cpu = "--cpu" in sys.argv
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = "cpu" if cpu else f"cuda:{local}"
    if not cpu:
        torch.cuda.set_device(local)

    def bcast(obj):
        lst = [obj]
        dist.broadcast_object_list(lst, src=0)
        return lst[0]

    def exchange(obj):
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    # One daemon for every rank.  The MoE part runs kernels of its own between work requests, so
    # the executors leave the GPU after 50 us without work instead of holding its time slice.
    daemon = shared_daemon(rank, world, bcast, gpus=0 if cpu else world, idle_exit_us=50)
    kind = 0 if cpu else 1
    try:
        # --- allreduce: WRITE_WITH_IMM reduce-scatter, WRITE_SUM_BF16, WRITE_WITH_IMM all-gather -----
        count = 1 << 20
        g = VerbsGroup(rank, world, 0 if cpu else local, count, exchange, pieces=4, device_kind=kind)
        gen = torch.Generator().manual_seed(rank)
        x = torch.randn(count, generator=gen).to(torch.bfloat16)
        g.buf[:count].copy_(x.to(g.buf.device))
        every = [None] * world
        dist.all_gather_object(every, x)
        expect = torch.stack([t.float() for t in every]).sum(0).to(torch.bfloat16)
        if not cpu:
            torch.cuda.synchronize()
        dist.barrier()
        g.allreduce(count)
        assert torch.equal(g.buf[:count].cpu(), expect), "allreduce differs from the fp32 sum rounded once"
        g.close()

        # --- MoE: route, send every (token, k) row to its expert's owner, read back and combine ------
        tokens, hidden, topk, nexp = 1024, 512, 4, 8 * world
        mg = moe_group(rank, world, 0 if cpu else local, tokens, topk, nexp, exchange, device_kind=kind)
        moe = VerbsMoE(mg, tokens, hidden, topk, nexp, recv_rows=tokens * topk * world)
        h = torch.randn(tokens, hidden, generator=gen).to(torch.bfloat16).to(dev)
        ids = torch.stack([torch.randperm(nexp, generator=gen)[:topk] for _ in range(tokens)]).to(torch.int32).to(dev)
        w = torch.softmax(torch.randn(tokens, topk, generator=gen), dim=-1).to(dev)
        moe.dispatch(h, ids)
        # The owner's receive area holds its experts' rows, grouped by expert then source rank: an
        # expert layer would run on moe.recv_view() here (identity in this example).
        got_rows = int(moe.recv_view().shape[0])
        counts, _ = reference_positions(ids.cpu(), nexp)
        mine = [None] * world
        dist.all_gather_object(mine, counts)
        epr = nexp // world
        want_rows = int(sum(int(c[rank * epr:(rank + 1) * epr].sum()) for c in mine))
        assert got_rows == want_rows, (got_rows, want_rows)
        out = moe.combine(w)
        if not cpu:
            torch.cuda.synchronize()
        ref = h.float() * w.sum(-1, keepdim=True)
        assert torch.allclose(out.float(), ref, atol=2e-2, rtol=1e-2), "combine differs from sum_k w * row"
        moe.close()
        mg.close()
        dist.barrier()
        if rank == 0:
            print(f"verbs collectives ok on {world} ranks ({'host memory' if cpu else 'GPUs'})")
    finally:
        dist.barrier()
        if daemon is not None:
            daemon.stop()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
