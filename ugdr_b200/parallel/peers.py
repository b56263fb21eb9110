"""Symmetric peer buffers: every rank allocates the same-size buffer, exports it with CUDA IPC
(ugdr_x_ipc_export), and maps every other rank's buffer into its own context
(ugdr_x_ipc_open), giving the collective kernels direct NVLink load / store access.

Host-side coordination (handle exchange, barriers) uses torch.distributed with any backend that
carries Python objects (gloo here); the data path never touches the host.
"""
from __future__ import annotations

import ctypes as C

import torch

from .. import _native as N

MAX_RANKS = 8
SLOTS = 8  # signal slots: 0 allreduce end, 2 dispatch, 3 combine, 4 counts, 5 allreduce entry


class PeerSet(C.Structure):
    _fields_ = [
        ("buf", C.c_void_p * MAX_RANKS),
        ("signal", C.c_void_p * MAX_RANKS),
        ("arrive", C.c_void_p),
        ("status", C.c_void_p),
        ("n", C.c_int),
        ("rank", C.c_int),
    ]


_SIGS = {
    "ugdr_x_ipc_export": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint64)]),
    "ugdr_x_ipc_open": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "ugdr_x_ipc_close": (C.c_int, [C.c_void_p]),
    "ugdr_x_allreduce_bf16": (C.c_int, [C.POINTER(PeerSet), C.c_uint64, C.c_uint64, C.c_uint64, C.c_int,
                                        C.c_void_p]),
    "ugdr_x_moe_route_scratch_bytes": (C.c_size_t, [C.c_uint64, C.c_int]),
    "ugdr_x_moe_route": (C.c_int, [C.c_void_p, C.c_uint64, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_size_t, C.c_void_p]),
    "ugdr_x_moe_layout": (C.c_int, [C.POINTER(PeerSet), C.c_void_p, C.c_int, C.c_int, C.c_uint64, C.c_void_p,
                                    C.c_void_p, C.c_uint64, C.c_void_p]),
    "ugdr_x_moe_dispatch": (C.c_int, [C.POINTER(PeerSet), C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_uint64, C.c_int, C.c_int, C.c_uint64, C.c_uint64,
                                      C.c_uint64, C.c_int, C.c_void_p]),
    "ugdr_x_moe_combine": (C.c_int, [C.POINTER(PeerSet), C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_uint64, C.c_int, C.c_int, C.c_uint64,
                                     C.c_uint64, C.c_uint64, C.c_int, C.c_void_p]),
}


def lib() -> C.CDLL:
    L = N.lib()
    if not getattr(L, "_coll_sigs", False):
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        L._coll_sigs = True
    return L


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: cudaError {rc}")


def stream_ptr(stream: torch.cuda.Stream | None = None) -> C.c_void_p:
    s = stream or torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


class PeerGroup:
    """One rank's view of `nbytes` of symmetric device memory across `world` ranks.

    `exchange(obj)` must return the list of every rank's `obj` (e.g. dist.all_gather_object).
    """

    def __init__(self, nbytes: int, rank: int, world: int, exchange, device: int | None = None):
        if not 1 <= world <= MAX_RANKS:
            raise ValueError(f"1..{MAX_RANKS} ranks supported, got {world}")
        self.rank, self.world, self.nbytes = rank, world, nbytes
        self.device = torch.cuda.current_device() if device is None else device
        L = lib()
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self.signal = torch.zeros(SLOTS * MAX_RANKS, dtype=torch.int64, device=self.device)
        self.arrive = torch.zeros(SLOTS, dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        mine = []
        for t in (self.buf, self.signal):
            h = C.create_string_buffer(64)
            off = C.c_uint64()
            check(L.ugdr_x_ipc_export(C.c_void_p(t.data_ptr()), h, C.byref(off)), "ugdr_x_ipc_export")
            mine.append((h.raw, off.value))
        everyone = exchange(mine)
        self._opened: list[int] = []
        ps = PeerSet()
        for q in range(world):
            if q == rank:
                ps.buf[q] = self.buf.data_ptr()
                ps.signal[q] = self.signal.data_ptr()
                continue
            ptrs = []
            for raw, off in everyone[q]:
                base = C.c_void_p()
                check(L.ugdr_x_ipc_open(raw, C.byref(base)), "ugdr_x_ipc_open")
                self._opened.append(base.value)
                ptrs.append(base.value + off)
            ps.buf[q], ps.signal[q] = ptrs
        ps.arrive = self.arrive.data_ptr()
        ps.status = self.status.data_ptr()
        ps.n, ps.rank = world, rank
        self.ps = ps
        self.epoch = 0

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def view(self, dtype: torch.dtype, numel: int, offset: int = 0) -> torch.Tensor:
        """A tensor over this rank's symmetric buffer."""
        esz = torch.empty((), dtype=dtype).element_size()
        if offset % esz or offset + numel * esz > self.nbytes:
            raise ValueError("view outside the symmetric buffer")
        return self.buf[offset:offset + numel * esz].view(dtype)

    def check_status(self) -> None:
        st = int(self.status.item())
        if st:
            raise RuntimeError({1: "a peer did not arrive within the bounded wait",
                                2: "MoE receive area too small"}.get(st, f"status {st}"))

    def close(self) -> None:
        L = lib()
        for b in self._opened:
            L.ugdr_x_ipc_close(C.c_void_p(b))
        self._opened = []
