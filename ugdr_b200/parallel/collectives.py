"""Collectives on symmetric peer buffers: fused-sum bf16 allreduce and the MoE all-to-all whose
dispatch / combine permutes are the NVLink transfers themselves."""
from __future__ import annotations

import ctypes as C

import torch

from .peers import PeerGroup, check, lib, stream_ptr


def allreduce_bf16(group: PeerGroup, count: int, offset: int = 0, ctas: int = 0,
                   stream: torch.cuda.Stream | None = None) -> None:
    """Sum `count` bf16 elements at byte `offset` of every rank's buffer, in place (fp32
    accumulation).  Enqueued on `stream`; every rank must make the same call."""
    rc = lib().ugdr_x_allreduce_bf16(C.byref(group.ps), offset, count, group.next_epoch(), ctas,
                                     stream_ptr(stream))
    check(rc, "ugdr_x_allreduce_bf16")


def moe_route(expert_ids: torch.Tensor, nexp: int, scratch: torch.Tensor | None = None,
              stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-expert row counts and each row's position within its expert group (row order)."""
    ids = expert_ids.reshape(-1).to(torch.int32).contiguous()
    rows = ids.numel()
    L = lib()
    need = L.ugdr_x_moe_route_scratch_bytes(rows, nexp)
    if scratch is None or scratch.numel() < need:
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=ids.device)
    counts = torch.empty(nexp, dtype=torch.int32, device=ids.device)
    pos = torch.empty(rows, dtype=torch.int32, device=ids.device)
    check(L.ugdr_x_moe_route(C.c_void_p(ids.data_ptr()), rows, nexp, C.c_void_p(counts.data_ptr()),
                             C.c_void_p(pos.data_ptr()), C.c_void_p(scratch.data_ptr()), scratch.numel(),
                             stream_ptr(stream)), "ugdr_x_moe_route")
    return counts, pos.view(expert_ids.shape)


class MoEAllToAll:
    """Expert-parallel token exchange.  Layout of each rank's symmetric buffer:
    [count table: world * nexp int32 | receive area: recv_rows rows of `hidden` bf16].

    dispatch(x, ids) sends every (token, k) row to the owner of expert ids[t, k], stored grouped
    by expert; combine(w) pulls them back and returns sum_k w[t, k] * row(t, k)."""

    def __init__(self, group: PeerGroup, tokens: int, hidden: int, topk: int, nexp: int,
                 recv_rows: int):
        if nexp % group.world:
            raise ValueError("experts must split evenly over ranks")
        self.g, self.tokens, self.hidden, self.topk, self.nexp = group, tokens, hidden, topk, nexp
        self.exp_per_rank = nexp // group.world
        self.row_bytes = hidden * 2
        self.table_off = 0
        table = group.world * nexp * 4
        self.recv_off = (table + 255) // 256 * 256
        self.recv_rows = recv_rows
        if self.recv_off + recv_rows * self.row_bytes > group.nbytes:
            raise ValueError("symmetric buffer too small for the receive area")
        dev = group.buf.device
        self.gbase = torch.zeros(nexp, dtype=torch.int64, device=dev)
        self.recv_used = torch.zeros(1, dtype=torch.int64, device=dev)
        self.scratch = torch.empty(max(1, lib().ugdr_x_moe_route_scratch_bytes(tokens * topk, nexp)),
                                   dtype=torch.uint8, device=dev)
        self.ids = None
        self.pos = None

    @staticmethod
    def required_bytes(world: int, nexp: int, hidden: int, recv_rows: int) -> int:
        return (world * nexp * 4 + 255) // 256 * 256 + recv_rows * hidden * 2

    def recv_view(self) -> torch.Tensor:
        return self.g.view(torch.bfloat16, self.recv_rows * self.hidden, self.recv_off).view(self.recv_rows,
                                                                                             self.hidden)

    def dispatch(self, x: torch.Tensor, expert_ids: torch.Tensor, ctas: int = 0,
                 stream: torch.cuda.Stream | None = None) -> None:
        assert x.dtype == torch.bfloat16 and x.is_contiguous() and x.shape == (self.tokens, self.hidden)
        L = lib()
        s = stream_ptr(stream)
        counts, pos = moe_route(expert_ids, self.nexp, self.scratch, stream)
        self.ids = expert_ids.reshape(-1).to(torch.int32).contiguous()
        self.pos = pos.reshape(-1)
        ep = self.g.next_epoch()
        check(L.ugdr_x_moe_layout(C.byref(self.g.ps), C.c_void_p(counts.data_ptr()), self.nexp,
                                  self.exp_per_rank, self.table_off, C.c_void_p(self.gbase.data_ptr()),
                                  C.c_void_p(self.recv_used.data_ptr()), ep, s), "ugdr_x_moe_layout")
        check(L.ugdr_x_moe_dispatch(C.byref(self.g.ps), C.c_void_p(x.data_ptr()), self.row_bytes,
                                    C.c_void_p(self.ids.data_ptr()), C.c_void_p(self.pos.data_ptr()),
                                    C.c_void_p(self.gbase.data_ptr()), self.tokens, self.topk, self.exp_per_rank,
                                    self.recv_off, self.recv_rows, ep, ctas, s), "ugdr_x_moe_dispatch")

    def combine(self, weights: torch.Tensor, out: torch.Tensor | None = None, ctas: int = 0,
                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        w = weights.reshape(-1).to(torch.float32).contiguous()
        if out is None:
            out = torch.empty(self.tokens, self.hidden, dtype=torch.bfloat16, device=w.device)
        check(lib().ugdr_x_moe_combine(C.byref(self.g.ps), C.c_void_p(out.data_ptr()), self.row_bytes,
                                       C.c_void_p(self.ids.data_ptr()), C.c_void_p(self.pos.data_ptr()),
                                       C.c_void_p(self.gbase.data_ptr()), C.c_void_p(w.data_ptr()), self.tokens,
                                       self.topk, self.exp_per_rank, self.recv_off, self.recv_rows,
                                       self.g.next_epoch(), ctas, stream_ptr(stream)), "ugdr_x_moe_combine")
        self._w = w
        return out
