"""NVLink SHARP (NVLS) multicast buffers for the collectives.

Every rank binds `nbytes` of its own GPU memory to one multicast object (ugdr_x_nvls_*): the
unicast view is an ordinary tensor on this GPU, and the multicast view lets the allreduce kernel
reduce inside the NVSwitch (multimem.ld_reduce) and broadcast the result (multimem.st).

Rank 0 creates the object and passes its POSIX file descriptor to the other ranks over an
abstract Unix socket (SCM_RIGHTS); `exchange(obj)` (e.g. dist.all_gather_object) carries the
socket name and doubles as the barrier between the set-up phases.
"""
from __future__ import annotations

import ctypes as C
import os
import socket
import threading
import time

import torch

from .peers import PeerGroup, PeerSet, check, lib, stream_ptr


class Nvls(C.Structure):
    _fields_ = [
        ("mc_handle", C.c_uint64),
        ("mem_handle", C.c_uint64),
        ("uc", C.c_void_p),
        ("mc", C.c_void_p),
        ("bytes", C.c_uint64),
        ("device", C.c_int),
    ]


_SIGS = {
    "ugdr_x_nvls_supported": (C.c_int, [C.c_int]),
    "ugdr_x_nvls_create": (C.c_int, [C.c_int, C.c_uint64, C.POINTER(Nvls), C.POINTER(C.c_int)]),
    "ugdr_x_nvls_import": (C.c_int, [C.c_int, C.c_int, C.c_uint64, C.POINTER(Nvls)]),
    "ugdr_x_nvls_add_device": (C.c_int, [C.POINTER(Nvls)]),
    "ugdr_x_nvls_bind": (C.c_int, [C.POINTER(Nvls)]),
    "ugdr_x_nvls_release": (C.c_int, [C.POINTER(Nvls)]),
    "ugdr_x_allreduce_bf16_nvls": (C.c_int, [C.POINTER(PeerSet), C.POINTER(Nvls), C.c_uint64, C.c_uint64, C.c_uint64,
                                             C.c_int, C.c_void_p]),
}


def _lib() -> C.CDLL:
    L = lib()
    if not getattr(L, "_nvls_sigs", False):
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        L._nvls_sigs = True
    return L


def supported(device: int | None = None) -> bool:
    dev = torch.cuda.current_device() if device is None else device
    return bool(_lib().ugdr_x_nvls_supported(dev))


def _serve_fd(name: str, fd: int, clients: int, timeout: float, ready: threading.Event, errors: list) -> None:
    try:
        with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as srv:
            srv.bind("\0" + name)
            srv.listen(clients)
            srv.settimeout(timeout)
            ready.set()
            for _ in range(clients):
                conn, _ = srv.accept()
                with conn:
                    socket.send_fds(conn, [b"F"], [fd])
    except Exception as e:  # reported by the caller after join()
        ready.set()
        errors.append(e)


def _fetch_fd(name: str, timeout: float) -> int:
    deadline = time.monotonic() + timeout
    while True:
        try:
            with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as s:
                s.settimeout(timeout)
                s.connect("\0" + name)
                _, fds, _, _ = socket.recv_fds(s, 1, 1)
                return fds[0]
        except (ConnectionRefusedError, FileNotFoundError):
            if time.monotonic() > deadline:
                raise
            time.sleep(0.01)


class NvlsBuffer:
    """`nbytes` (rounded up to the multicast granularity) of NVLS memory on every rank."""

    def __init__(self, nbytes: int, rank: int, world: int, exchange, timeout: float = 60.0):
        L = _lib()
        self.rank, self.world = rank, world
        self._exchange = exchange
        self.h = Nvls()
        fd = C.c_int(-1)
        name = None
        server = None
        errors: list = []
        if rank == 0:
            check(L.ugdr_x_nvls_create(world, nbytes, C.byref(self.h), C.byref(fd)), "ugdr_x_nvls_create")
            name = f"ugdr-nvls-{os.getpid()}-{os.urandom(6).hex()}"
            ready = threading.Event()
            server = threading.Thread(target=_serve_fd, args=(name, fd.value, world - 1, timeout, ready, errors),
                                      daemon=True)
            server.start()
            ready.wait(timeout)
        name = exchange(name)[0]
        # The object's descriptor stays open: registering the buffer with the verbs daemon
        # (ugdr_x_reg_mr_multicast) hands the daemon a duplicate of it.
        self.fd = -1
        if rank != 0:
            got = _fetch_fd(name, timeout)
            try:
                check(L.ugdr_x_nvls_import(got, world, nbytes, C.byref(self.h)), "ugdr_x_nvls_import")
            except BaseException:
                os.close(got)
                raise
            self.fd = got
        if server is not None:
            server.join(timeout)
            self.fd = fd.value
            if errors:
                raise RuntimeError(f"passing the NVLS descriptor failed: {errors[0]}")
        check(L.ugdr_x_nvls_add_device(C.byref(self.h)), "ugdr_x_nvls_add_device")
        exchange(None)  # every GPU added before any memory is bound
        check(L.ugdr_x_nvls_bind(C.byref(self.h)), "ugdr_x_nvls_bind")
        exchange(None)  # every GPU bound before the multicast view is used
        self.nbytes = int(self.h.bytes)
        self.tensor = _wrap(self.h.uc, self.nbytes, int(self.h.device), self)

    def view(self, dtype: torch.dtype, numel: int, offset: int = 0) -> torch.Tensor:
        esz = torch.empty((), dtype=dtype).element_size()
        if offset % esz or offset + numel * esz > self.nbytes:
            raise ValueError("view outside the NVLS buffer")
        return self.tensor[offset:offset + numel * esz].view(dtype)

    def close(self) -> None:
        """Collective: every rank's work on the buffer is finished before any rank unbinds."""
        if self.h.mc_handle:
            torch.cuda.synchronize()
            self._exchange(None)
            _lib().ugdr_x_nvls_release(C.byref(self.h))
        if self.fd >= 0:
            os.close(self.fd)
            self.fd = -1


class _Raw:
    """__cuda_array_interface__ over raw device memory, keeping its owner alive."""

    def __init__(self, ptr: int, nbytes: int, owner):
        self.owner = owner
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def _wrap(ptr: int, nbytes: int, device: int, owner) -> torch.Tensor:
    with torch.cuda.device(device):
        return torch.as_tensor(_Raw(ptr, nbytes, owner), device=f"cuda:{device}")


def allreduce_bf16_nvls(group: PeerGroup, buf: NvlsBuffer, count: int, offset: int = 0, ctas: int = 0,
                        stream: torch.cuda.Stream | None = None) -> None:
    """In-place sum of `count` bf16 elements at byte `offset` of every rank's NVLS buffer (the
    reduction runs in the NVSwitch, fp32 accumulation).  `group` provides the signal words."""
    rc = _lib().ugdr_x_allreduce_bf16_nvls(C.byref(group.ps), C.byref(buf.h), offset, count, group.next_epoch(),
                                          ctas, stream_ptr(stream))
    check(rc, "ugdr_x_allreduce_bf16_nvls")
