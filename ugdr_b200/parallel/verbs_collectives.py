"""Collectives on the ugdr verbs (include/ugdr/verbs_collective.h), wired over torch.distributed.

    g = VerbsGroup(rank, world, local_gpu, count, exchange)   # one daemon serves every rank
    g.buf.copy_(x); g.allreduce(); x = g.buf

Every byte moves as a verbs work request run by the daemon's persistent executor on the rank's
GPU: WRITE_WITH_IMM into the owner's staging, one UGDR_X_WR_RDMA_WRITE_SUM_BF16 per piece (the
executor sums while it writes), WRITE_WITH_IMM back to every rank.  The schedule itself is the
native `ugdr_x_verbs_allreduce_bf16` (client-side C++ over the public verbs calls).

`exchange(obj)` must return the list of every rank's `obj` (an all_gather_object over a CPU
group).  The daemon is found through UGDR_DAEMON_SOCKET (see `shared_daemon`).
"""
from __future__ import annotations

import ctypes as C
import os

import torch

from .. import _native as N
from .. import verbs as V

MAX_RANKS = 8
MAX_PIECES = 64


class _Peer(C.Structure):
    _fields_ = [("to", C.c_void_p), ("frm", C.c_void_p), ("buf_addr", C.c_uint64), ("buf_rkey", C.c_uint32),
                ("stage_rkey", C.c_uint32), ("stage_addr", C.c_uint64)]


class _Group(C.Structure):
    _fields_ = [("rank", C.c_int), ("n", C.c_int), ("cq", C.c_void_p), ("self_to", C.c_void_p),
                ("buf_addr", C.c_uint64), ("buf_lkey", C.c_uint32), ("buf_rkey", C.c_uint32),
                ("stage_addr", C.c_uint64), ("stage_lkey", C.c_uint32), ("pad", C.c_uint32),
                ("stage_bytes", C.c_uint64), ("epoch", C.c_uint32), ("pad2", C.c_uint32),
                ("peer", _Peer * MAX_RANKS)]


def _lib():
    L = N.lib()
    if not getattr(L, "_vcoll_sigs", False):
        L.ugdr_x_verbs_allreduce_stage_bytes.restype = C.c_uint64
        L.ugdr_x_verbs_allreduce_stage_bytes.argtypes = [C.c_uint64, C.c_int]
        L.ugdr_x_verbs_allreduce_bf16.restype = C.c_int
        L.ugdr_x_verbs_allreduce_bf16.argtypes = [C.POINTER(_Group), C.c_uint64, C.c_int, C.c_uint64]
        L._vcoll_sigs = True
    return L


def shared_daemon(rank: int, world: int, bcast, gpus: int | None = None):
    """Rank 0 starts one daemon owning `gpus` (default: world) GPUs, or only the host-memory
    device when gpus == 0; every rank points UGDR_DAEMON_SOCKET at it.  Returns rank 0's Daemon
    (None elsewhere); stop it after every rank closed its group."""
    gpus = world if gpus is None else gpus
    d = V.Daemon(gpus=gpus, cpu_device=gpus == 0) if rank == 0 else None
    path = bcast(d.socket_path if d else None)
    os.environ["UGDR_DAEMON_SOCKET"] = path
    return d


class VerbsGroup:
    """A rank's QPs, CQ and registered buffers for the verbs collectives (one GPU per rank)."""

    def __init__(self, rank: int, world: int, gpu: int, count: int, exchange, pieces: int = 8,
                 device_kind: int = 1):
        if not 1 <= world <= MAX_RANKS or not 1 <= pieces <= MAX_PIECES:
            raise ValueError("world must be 1..8 and pieces 1..64")
        self.rank, self.world, self.count, self.pieces = rank, world, count, pieces
        L = _lib()
        dev = V.find_device(gpu=gpu) if device_kind == 1 else V.find_device(kind=0)
        self.ctx = V.Context(dev)
        self.pd = self.ctx.alloc_pd()
        depth = 2 * pieces + 4
        self.cq = self.ctx.create_cq(2 * pieces * world + pieces + world + 64)
        stage_bytes = max(int(L.ugdr_x_verbs_allreduce_stage_bytes(count, world)), 16)
        self._host = []
        if device_kind == 1:
            self.buf = torch.empty(count, dtype=torch.bfloat16, device=f"cuda:{gpu}")
            self.stage = torch.empty(stage_bytes, dtype=torch.uint8, device=f"cuda:{gpu}")
            torch.cuda.synchronize(gpu)
        else:  # host engine: daemon-shareable host memory
            hb, hs = V.HostBuffer(max(2 * count, 16)), V.HostBuffer(stage_bytes)
            self._host = [hb, hs]
            self.buf = torch.from_numpy(hb.view()).view(torch.bfloat16)[:count]
            self.stage = torch.from_numpy(hs.view())
        acc = N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE
        self.buf_mr = self.pd.reg_mr(self.buf.data_ptr(), max(2 * count, 2), acc)
        self.stage_mr = self.pd.reg_mr(self.stage.data_ptr(), self.stage.numel(), acc)
        self.to = {q: self.pd.create_qp(self.cq, max_send_wr=depth, max_recv_wr=4) for q in range(world) if q != rank}
        self.frm = {q: self.pd.create_qp(self.cq, max_send_wr=4, max_recv_wr=depth) for q in range(world) if q != rank}
        self.self_to = self.pd.create_qp(self.cq, max_send_wr=depth, max_recv_wr=4, max_send_sge=MAX_RANKS)
        self.self_peer = self.pd.create_qp(self.cq, max_send_wr=4, max_recv_wr=4)
        V.connect_pair(self.self_to, self.self_peer, access=N.ACCESS_REMOTE_WRITE)
        for q in list(self.to.values()) + list(self.frm.values()):
            q.to_init(N.ACCESS_REMOTE_WRITE)
        info = exchange({"to": {q: qp.qpn for q, qp in self.to.items()},
                         "from": {q: qp.qpn for q, qp in self.frm.items()},
                         "buf": (self.buf.data_ptr(), self.buf_mr.rkey),
                         "stage": (self.stage.data_ptr(), self.stage_mr.rkey)})
        g = _Group()
        g.rank, g.n = rank, world
        g.cq, g.self_to = self.cq.h, self.self_to.h
        g.buf_addr, g.buf_lkey, g.buf_rkey = self.buf.data_ptr(), self.buf_mr.lkey, self.buf_mr.rkey
        g.stage_addr, g.stage_lkey, g.stage_bytes = self.stage.data_ptr(), self.stage_mr.lkey, self.stage.numel()
        for q in range(world):
            if q == rank:
                continue
            # rnr_retry 7: a peer that runs ahead waits for this rank's next receives.
            self.to[q].connect(info[q]["from"][rank], rnr_retry=7)
            self.frm[q].connect(info[q]["to"][rank], rnr_retry=7)
            p = g.peer[q]
            p.to, p.frm = self.to[q].h, self.frm[q].h
            p.buf_addr, p.buf_rkey = info[q]["buf"]
            p.stage_addr, p.stage_rkey = info[q]["stage"]
        self._g = g
        exchange(None)  # every rank connected before anyone posts

    def allreduce(self, count: int | None = None, pieces: int | None = None, timeout_s: float = 60.0) -> None:
        """In-place bf16 sum of the first `count` elements of `buf` over the group."""
        count = self.count if count is None else count
        if count > self.count:
            raise ValueError("count larger than the group's buffer")
        rc = _lib().ugdr_x_verbs_allreduce_bf16(C.byref(self._g), count, pieces or self.pieces, int(timeout_s * 1e9))
        if rc != 0:
            raise V.UgdrError(rc, f"ugdr_x_verbs_allreduce_bf16: {N.errname(rc)}")

    def close(self) -> None:
        for q in list(self.to.values()) + list(self.frm.values()) + [self.self_to, self.self_peer]:
            q.destroy()
        self.buf_mr.dereg()
        self.stage_mr.dereg()
        self.cq.destroy()
        self.pd.dealloc()
        self.ctx.close()
        for h in self._host:
            h.free()
