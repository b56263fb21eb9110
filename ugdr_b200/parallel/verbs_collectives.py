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


def shared_daemon(rank: int, world: int, bcast, gpus: int | None = None, idle_exit_us: int | None = None):
    """Rank 0 starts one daemon owning `gpus` (default: world) GPUs, or only the host-memory
    device when gpus == 0; every rank points UGDR_DAEMON_SOCKET at it.  Returns rank 0's Daemon
    (None elsewhere); stop it after every rank closed its group.

    idle_exit_us: how long each GPU's executor stays resident without work.  The executor is a
    kernel of the daemon's CUDA context, and kernels of different contexts share a GPU by time
    slices, so while it is resident every kernel of the ranks (routing, the MoE pack and weighted
    sum) first waits for a context switch.  Workloads that alternate their own kernels with
    collectives run faster with a short idle exit (the executor relaunches on the next WR):
    measured on one B200, an MoE step of 16,384 tokens took 7.8 ms with the daemon's 200 ms
    default and 3.2 ms with 50 us.  Back-to-back collectives with no kernels between them (the
    allreduce) are better served by the default (None), which saves the relaunches."""
    gpus = world if gpus is None else gpus
    d = V.Daemon(gpus=gpus, cpu_device=gpus == 0, idle_exit_us=idle_exit_us) if rank == 0 else None
    path = bcast(d.socket_path if d else None)
    os.environ["UGDR_DAEMON_SOCKET"] = path
    return d


class VerbsGroup:
    """A rank's QPs, CQ and registered buffers for the verbs collectives (one GPU per rank)."""

    def __init__(self, rank: int, world: int, gpu: int, count: int, exchange, pieces: int = 8,
                 device_kind: int = 1, send_depth: int = 0, max_sge: int = 1):
        if not 1 <= world <= MAX_RANKS or not 1 <= pieces <= MAX_PIECES:
            raise ValueError("world must be 1..8 and pieces 1..64")
        self.rank, self.world, self.count, self.pieces = rank, world, count, pieces
        self.device_kind = device_kind
        self._mc = {}
        L = _lib()
        dev = V.find_device(gpu=gpu) if device_kind == 1 else V.find_device(kind=0)
        self.ctx = V.Context(dev)
        self.pd = self.ctx.alloc_pd()
        depth = max(2 * pieces + 4, send_depth)
        self.exchange = exchange
        self.cq = self.ctx.create_cq(2 * pieces * world + pieces + 4 * world + 64)
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
        self.to = {q: self.pd.create_qp(self.cq, max_send_wr=depth, max_recv_wr=4, max_send_sge=max_sge)
                   for q in range(world) if q != rank}
        self.frm = {q: self.pd.create_qp(self.cq, max_send_wr=4, max_recv_wr=2 * pieces + 4)
                    for q in range(world) if q != rank}
        self.self_to = self.pd.create_qp(self.cq, max_send_wr=depth, max_recv_wr=4,
                                         max_send_sge=max(MAX_RANKS, max_sge))
        self.self_peer = self.pd.create_qp(self.cq, max_send_wr=4, max_recv_wr=4)
        remote = N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ
        V.connect_pair(self.self_to, self.self_peer, access=remote)
        for q in list(self.to.values()) + list(self.frm.values()):
            q.to_init(remote)
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

    def allreduce_nvls(self, nvbuf, count: int, timeout_s: float = 60.0) -> None:
        """In-place bf16 sum of the first `count` elements of an NVLS buffer (parallel.nvls.NvlsBuffer,
        each rank's data in its unicast view) through NVLink SHARP, on the verbs: the buffer is
        registered once as a multicast MR and every rank posts one WRITE_SUM_BF16 of its shard
        (ugdr_x_verbs_allreduce_bf16_mc)."""
        L = _lib()
        if not getattr(L, "_vcoll_mc_sig", False):
            L.ugdr_x_verbs_allreduce_bf16_mc.restype = C.c_int
            L.ugdr_x_verbs_allreduce_bf16_mc.argtypes = [C.POINTER(_Group), C.c_uint64, C.c_uint32, C.c_uint32,
                                                         C.c_uint64, C.c_uint64]
            L._vcoll_mc_sig = True
        mr = self._mc.get(id(nvbuf))
        if mr is None:
            acc = N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE
            mr = self.pd.reg_mr_multicast(int(nvbuf.h.mc), nvbuf.nbytes, acc, nvbuf.fd)
            self._mc[id(nvbuf)] = mr
        torch.cuda.synchronize()
        rc = L.ugdr_x_verbs_allreduce_bf16_mc(C.byref(self._g), int(nvbuf.h.mc), mr.lkey, mr.rkey, count,
                                              int(timeout_s * 1e9))
        if rc != 0:
            raise V.UgdrError(rc, f"ugdr_x_verbs_allreduce_bf16_mc: {N.errname(rc)}")

    def release_multicast(self) -> None:
        """Deregister the multicast MRs; every rank does this before its NVLS buffers close."""
        for mr in self._mc.values():
            mr.dereg()
        self._mc.clear()

    def close(self) -> None:
        self.release_multicast()
        for q in list(self.to.values()) + list(self.frm.values()) + [self.self_to, self.self_peer]:
            q.destroy()
        self.buf_mr.dereg()
        self.stage_mr.dereg()
        self.cq.destroy()
        self.pd.dealloc()
        self.ctx.close()
        for h in self._host:
            h.free()


class _Moe(C.Structure):
    _fields_ = [("tokens", C.c_int), ("topk", C.c_int), ("nexp", C.c_int), ("row_bytes", C.c_uint32),
                ("x_addr", C.c_uint64), ("x_lkey", C.c_uint32), ("recv_lkey", C.c_uint32),
                ("recv_addr", C.c_uint64), ("recv_rkey", C.c_uint32), ("back_lkey", C.c_uint32),
                ("recv_rows", C.c_uint64), ("back_addr", C.c_uint64), ("table", C.c_void_p),
                ("table_lkey", C.c_uint32), ("table_rkey", C.c_uint32),
                ("peer_recv_addr", C.c_uint64 * MAX_RANKS), ("peer_recv_rkey", C.c_uint32 * MAX_RANKS),
                ("peer_table_addr", C.c_uint64 * MAX_RANKS), ("peer_table_rkey", C.c_uint32 * MAX_RANKS),
                ("base", C.c_void_p), ("received", C.c_uint64)]


def _moe_lib():
    L = _lib()
    if not getattr(L, "_vmoe_sigs", False):
        L.ugdr_x_verbs_moe_wrs.restype = C.c_uint32
        L.ugdr_x_verbs_moe_wrs.argtypes = [C.c_uint64, C.c_int, C.c_int]
        L.ugdr_x_verbs_moe_dispatch.restype = C.c_int
        L.ugdr_x_verbs_moe_dispatch.argtypes = [C.POINTER(_Group), C.POINTER(_Moe), C.c_void_p, C.c_void_p,
                                                C.c_void_p, C.c_uint64]
        L.ugdr_x_verbs_moe_dispatch_packed.restype = C.c_int
        L.ugdr_x_verbs_moe_dispatch_packed.argtypes = [C.POINTER(_Group), C.POINTER(_Moe), C.c_void_p, C.c_uint64]
        L.ugdr_x_moe_pack_grouped.restype = C.c_int
        L.ugdr_x_moe_pack_grouped.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                              C.c_uint64, C.c_int, C.c_uint64, C.c_int, C.c_void_p]
        L.ugdr_x_verbs_moe_combine.restype = C.c_int
        L.ugdr_x_verbs_moe_combine.argtypes = [C.POINTER(_Group), C.POINTER(_Moe), C.c_uint64]
        L.ugdr_x_moe_weighted_sum_grouped.restype = C.c_int
        L.ugdr_x_moe_weighted_sum_grouped.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                      C.c_void_p, C.c_uint64, C.c_int, C.c_uint64, C.c_int,
                                                      C.c_void_p]
        L.ugdr_x_moe_weighted_sum.restype = C.c_int
        L.ugdr_x_moe_weighted_sum.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64, C.c_int, C.c_uint64,
                                              C.c_int, C.c_void_p]
        L._vmoe_sigs = True
    return L


def moe_group(rank: int, world: int, gpu: int, tokens: int, topk: int, nexp: int, exchange,
              device_kind: int = 1) -> VerbsGroup:
    """A VerbsGroup sized for VerbsMoE: 32-SGE send queues deep enough for one call's WRs."""
    depth = int(_moe_lib().ugdr_x_verbs_moe_wrs(tokens * topk, nexp, world)) + 8
    return VerbsGroup(rank, world, gpu, 8, exchange, pieces=1, send_depth=depth, max_sge=32,
                      device_kind=device_kind)


def _host_tensor(nbytes: int, dtype, shape, keep: list):
    hb = V.HostBuffer(max(nbytes, 16))
    keep.append(hb)
    return torch.from_numpy(hb.view()[:nbytes]).view(dtype).view(*shape)


class VerbsMoE:
    """MoE all-to-all on the verbs (ugdr_x_verbs_moe_dispatch / _combine).

    dispatch(x, ids) routes on the GPU (ugdr_x_moe_route), groups the rows by expert into `back`
    (ugdr_x_moe_pack_grouped) and sends each (owner, expert) group with one WRITE (on the host
    engine, or with packed=False, WRITEs whose 32-SGE lists gather the rows are the permute);
    `recv_view()[:received]` then holds this rank's experts' rows, grouped by expert and source
    rank.  combine(w) READs every (owner, expert) group back in one piece into `back` (grouped by
    expert) and returns sum_k w[t, k] * row(t, k), the unpermute being the gather of the
    weighted sum (ugdr_x_moe_weighted_sum_grouped).  Start the daemon with a short executor idle
    exit (shared_daemon(..., idle_exit_us=50)): the routing, pack and weighted-sum kernels are this
    process's, and they would otherwise wait for the resident executor's time slice."""

    def __init__(self, group: VerbsGroup, tokens: int, hidden: int, topk: int, nexp: int, recv_rows: int):
        if nexp % group.world:
            raise ValueError("experts must split evenly over ranks")
        self.g, self.tokens, self.hidden, self.topk, self.nexp = group, tokens, hidden, topk, nexp
        L = _moe_lib()
        self.row_bytes = hidden * 2
        self.gpu = group.device_kind == 1
        self._host = []
        if self.gpu:
            dev = torch.device("cuda", torch.cuda.current_device())
            self.x = torch.empty(tokens, hidden, dtype=torch.bfloat16, device=dev)
            self.recv = torch.empty(recv_rows, hidden, dtype=torch.bfloat16, device=dev)
            self.back = torch.empty(tokens * topk, hidden, dtype=torch.bfloat16, device=dev)
            torch.cuda.synchronize()
        else:  # host engine: daemon-shareable host memory, torch on the CPU
            rb = self.row_bytes
            self.x = _host_tensor(tokens * rb, torch.bfloat16, (tokens, hidden), self._host)
            self.recv = _host_tensor(recv_rows * rb, torch.bfloat16, (recv_rows, hidden), self._host)
            self.back = _host_tensor(tokens * topk * rb, torch.bfloat16, (tokens * topk, hidden), self._host)
        self.table = V.HostBuffer(group.world * nexp * 4)
        self.table.view()[:] = 0
        pd = group.pd
        lw, rw, rr = N.ACCESS_LOCAL_WRITE, N.ACCESS_REMOTE_WRITE, N.ACCESS_REMOTE_READ
        self.x_mr = pd.reg_mr(self.x.data_ptr(), self.x.numel() * 2, lw)
        self.recv_mr = pd.reg_mr(self.recv.data_ptr(), self.recv.numel() * 2, lw | rw | rr)
        self.back_mr = pd.reg_mr(self.back.data_ptr(), self.back.numel() * 2, lw)
        self.table_mr = pd.reg_mr(self.table.addr, self.table.length, lw | rw)
        import numpy as np

        self.base = np.zeros(nexp * group.world, dtype=np.uint64)
        info = group.exchange({"recv": (self.recv.data_ptr(), self.recv_mr.rkey),
                               "table": (self.table.addr, self.table_mr.rkey)})
        m = _Moe()
        m.tokens, m.topk, m.nexp, m.row_bytes = tokens, topk, nexp, self.row_bytes
        m.x_addr, m.x_lkey = self.x.data_ptr(), self.x_mr.lkey
        m.recv_addr, m.recv_lkey, m.recv_rkey, m.recv_rows = (self.recv.data_ptr(), self.recv_mr.lkey,
                                                              self.recv_mr.rkey, recv_rows)
        m.back_addr, m.back_lkey = self.back.data_ptr(), self.back_mr.lkey
        m.table, m.table_lkey, m.table_rkey = self.table.addr, self.table_mr.lkey, self.table_mr.rkey
        for q in range(group.world):
            m.peer_recv_addr[q], m.peer_recv_rkey[q] = info[q]["recv"]
            m.peer_table_addr[q], m.peer_table_rkey[q] = info[q]["table"]
        m.base = self.base.ctypes.data
        self._m = m
        self.scratch = None

    def recv_view(self) -> torch.Tensor:
        return self.recv[: int(self._m.received)]

    def dispatch(self, x: torch.Tensor | None, expert_ids: torch.Tensor, timeout_s: float = 60.0,
                 packed: bool | None = None) -> None:
        """Send every (token, k) row of x to its expert's owner.  On the GPU the default is the
        packed form: ugdr_x_moe_pack_grouped groups the rows by expert into `back` (each x row
        read once, straight from the caller's tensor) and every (owner, expert) group leaves as
        one contiguous WRITE.  packed=False gathers the rows with 32-SGE WRITEs from the
        registered x instead (the default on the host engine, where packed=True groups the rows
        with torch)."""
        packed = self.gpu if packed is None else packed
        src = self.x
        if x is not None:
            if packed and x.is_contiguous() and x.dtype == torch.bfloat16 and x.shape == self.x.shape \
                    and x.device == self.x.device:
                src = x
            else:
                self.x.copy_(x)
        if self.gpu:
            from .collectives import moe_route

            counts, pos = moe_route(expert_ids, self.nexp)
        else:
            from ..models.moe import reference_positions

            counts, pos = reference_positions(expert_ids, self.nexp)
        dev = self.x.device
        # The routing on the rows' device and each expert's first row in the expert-grouped area
        # (`back`): the pack, and the combine's grouped weighted sum, gather through them.
        self.ids_d = expert_ids.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
        self.pos_d = pos.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
        c64 = counts.to(device=dev, dtype=torch.int64)
        self.start_d = torch.cumsum(c64, 0) - c64
        L = _moe_lib()
        if packed and not self.gpu:  # host engine: the same grouping with torch
            self.back[self.start_d[self.ids_d.long()] + self.pos_d.long()] = src.repeat_interleave(self.topk, 0)
        elif packed:
            rc = L.ugdr_x_moe_pack_grouped(self.back.data_ptr(), src.data_ptr(), self.ids_d.data_ptr(),
                                           self.pos_d.data_ptr(), self.start_d.data_ptr(), self.tokens, self.topk,
                                           self.row_bytes, 0, torch.cuda.current_stream().cuda_stream)
            if rc != 0:
                raise RuntimeError(f"ugdr_x_moe_pack_grouped: cudaError {rc}")
        counts_h = counts.to(torch.int32).cpu().contiguous()  # synchronises: the rows and the routing are ready
        if packed:
            rc = L.ugdr_x_verbs_moe_dispatch_packed(C.byref(self.g._g), C.byref(self._m), counts_h.data_ptr(),
                                                    int(timeout_s * 1e9))
            name = "ugdr_x_verbs_moe_dispatch_packed"
        else:
            ids_h = expert_ids.reshape(-1).to(torch.int32).cpu().contiguous()
            pos_h = pos.reshape(-1).to(torch.int32).cpu().contiguous()
            rc = L.ugdr_x_verbs_moe_dispatch(C.byref(self.g._g), C.byref(self._m), ids_h.data_ptr(),
                                             pos_h.data_ptr(), counts_h.data_ptr(), int(timeout_s * 1e9))
            name = "ugdr_x_verbs_moe_dispatch"
        if rc != 0:
            raise V.UgdrError(rc, f"{name}: {N.errname(rc)}")

    def combine(self, weights: torch.Tensor, out: torch.Tensor | None = None, timeout_s: float = 60.0) -> torch.Tensor:
        L = _moe_lib()
        rc = L.ugdr_x_verbs_moe_combine(C.byref(self.g._g), C.byref(self._m), int(timeout_s * 1e9))
        if rc != 0:
            raise V.UgdrError(rc, f"ugdr_x_verbs_moe_combine: {N.errname(rc)}")
        w = weights.reshape(-1).to(device=self.x.device, dtype=torch.float32).contiguous()
        if not self.gpu:
            idx = (self.start_d[self.ids_d.long()] + self.pos_d.long())
            rows = self.back[idx].float().view(self.tokens, self.topk, self.hidden)
            res = (rows * w.view(self.tokens, self.topk, 1)).sum(1).to(torch.bfloat16)
            if out is not None:
                out.copy_(res)
                return out
            return res
        if out is None:
            out = torch.empty(self.tokens, self.hidden, dtype=torch.bfloat16, device=self.x.device)
        rc = L.ugdr_x_moe_weighted_sum_grouped(out.data_ptr(), self.back.data_ptr(), self.ids_d.data_ptr(),
                                               self.pos_d.data_ptr(), self.start_d.data_ptr(), w.data_ptr(),
                                               self.tokens, self.topk, self.row_bytes, 0,
                                               torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise RuntimeError(f"ugdr_x_moe_weighted_sum_grouped: cudaError {rc}")
        return out

    def close(self) -> None:
        for mr in (self.x_mr, self.recv_mr, self.back_mr, self.table_mr):
            mr.dereg()
        self.table.free()
        for h in self._host:
            h.free()
