"""Collectives on ugdr-b200 from PyTorch: a fused bf16 allreduce and an MoE dispatch + combine over
NVLink peer memory, each checked against a plain torch fp32 computation.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/collectives.py

One process per GPU; torch.distributed (NCCL) only exchanges the IPC handles that build the peer
group and gathers the reference inputs for the checks.
"""
from __future__ import annotations

import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from ugdr_b200.parallel.collectives import MoEAllToAll, allreduce_bf16  # noqa: E402
from ugdr_b200.parallel.peers import PeerGroup  # noqa: E402


def main() -> None:
    dist.init_process_group("nccl")
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))

    def exchange(obj):
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    # --- allreduce: 4 Mi bf16 elements in the symmetric buffer, summed in place -----------------
    count = 4 << 20
    tokens, hidden, topk, nexp = 2048, 1024, 4, 8 * world
    recv_rows = tokens * topk * world  # enough for any routing
    nbytes = max(count * 2, MoEAllToAll.required_bytes(world, nexp, hidden, recv_rows))
    group = PeerGroup(nbytes, rank, world, exchange)
    x = group.view(torch.bfloat16, count)
    g = torch.Generator(device="cuda").manual_seed(rank)
    x.copy_(torch.randn(count, device="cuda", generator=g).to(torch.bfloat16))
    every = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(every, x)
    expect = torch.stack([t.float() for t in every]).sum(0)
    torch.cuda.synchronize()
    allreduce_bf16(group, count)
    torch.cuda.synchronize()
    group.check_status()
    err = (x.float() - expect).abs().max().item()
    tol = 2 ** -7 * expect.abs().max().item() + 1e-2  # one bf16 rounding of the fp32 sum
    assert err <= tol, f"allreduce error {err} above {tol}"

    # --- MoE: route every token to topk experts, send the rows to their owners, combine ---------
    moe = MoEAllToAll(group, tokens, hidden, topk, nexp, recv_rows)
    h = torch.randn(tokens, hidden, device="cuda", generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(nexp, device="cuda", generator=g)[:topk] for _ in range(tokens)]).to(torch.int32)
    w = torch.softmax(torch.randn(tokens, topk, device="cuda", generator=g), dim=-1)
    moe.dispatch(h, ids)
    out = moe.combine(w)
    torch.cuda.synchronize()
    group.check_status()
    # Every expert here is the identity, so combine must return sum_k w[t, k] * h[t].
    ref = (w.sum(-1, keepdim=True) * h.float()).to(torch.bfloat16)
    merr = (out.float() - ref.float()).abs().max().item()
    assert merr <= 2 ** -6 * ref.float().abs().max().item() + 1e-2, f"MoE error {merr}"

    group.close()
    if rank == 0:
        print(f"ok: allreduce of {count} bf16 on {world} GPUs (max err {err:.3g}); "
              f"MoE {tokens} tokens x top-{topk} of {nexp} experts (max err {merr:.3g})")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
