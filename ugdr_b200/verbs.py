"""Pythonic wrappers over the ugdr verbs C ABI (libugdr.so via ctypes).

Every call goes through the native library: the wrappers only build the C records, check
return codes and raise `UgdrError` with the errno the library reported.  Object lifetimes
follow the verbs rules the daemon enforces (children before parents; EBUSY otherwise).
"""
from __future__ import annotations

import contextlib
import ctypes as C
import os
import signal
import subprocess
import tempfile
import time
from dataclasses import dataclass
from pathlib import Path

from . import _native as N


class UgdrError(OSError):
    pass


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise UgdrError(rc, f"{what}: {N.errname(rc)}")


def _check_ptr(p, what: str):
    if not p:
        e = N.errno()
        raise UgdrError(e, f"{what}: {N.errname(e)}")
    return p


# ---- daemon process ---------------------------------------------------------------------------


class Daemon:
    """Run `ugdr_daemon` as a child process on a private socket.

    `gpus`: how many GPUs it owns (None = all visible, 0 = host engine only).  With `export`
    (the default) the socket path is set as UGDR_DAEMON_SOCKET so this process's verbs calls reach
    it, and `stop()` puts the variable back as it was, so a nested daemon (one a benchmark helper
    starts and stops) leaves the outer daemon's clients pointing at the outer socket.  Helpers
    that only hand the socket to child processes pass `export=False`.
    """

    def __init__(self, gpus: int | None = None, socket_path: str | None = None,
                 ctas: int | None = None, idle_exit_us: int | None = None,
                 cpu_device: bool = True, env: dict | None = None, log_path: str | None = None,
                 export: bool = True):
        self._dir = None
        self._exported = False
        self._prev_socket = None
        if socket_path is None:
            self._dir = tempfile.mkdtemp(prefix="ugdr-")
            socket_path = os.path.join(self._dir, "ugdr.sock")
        self.socket_path = socket_path
        args = [str(N.DAEMON_PATH), "--socket", socket_path]
        if gpus is not None:
            args += ["--gpus", str(gpus)]
        ctas = ctas if ctas is not None else os.environ.get("UGDR_EXECUTOR_CTAS")
        if ctas is not None:
            args += ["--ctas", str(ctas)]
        if idle_exit_us is not None:
            args += ["--idle-exit-us", str(idle_exit_us)]
        if not cpu_device:
            args += ["--no-cpu-device"]
        if not N.DAEMON_PATH.exists():
            raise RuntimeError(f"{N.DAEMON_PATH} missing: build the native tree first")
        # The daemon's stderr goes to a file (a pipe nobody drains could block its threads).
        log_dir = os.environ.get("UGDR_DAEMON_LOG_DIR") or self._dir or tempfile.gettempdir()
        self.log_path = log_path or tempfile.mkstemp(prefix=f"ugdr-daemon-{os.getpid()}-", suffix=".log",
                                                     dir=log_dir)[1]
        self._log = open(self.log_path, "w")
        self.proc = subprocess.Popen(args, env=env, stderr=self._log, stdout=self._log)
        deadline = time.time() + 120
        while not os.path.exists(socket_path):
            if self.proc.poll() is not None:
                raise RuntimeError(f"ugdr_daemon exited ({self.proc.returncode}): {self.log_text()}")
            if time.time() > deadline:
                self.stop()
                raise RuntimeError("ugdr_daemon did not create its socket")
            time.sleep(0.01)
        if export:
            self._prev_socket = os.environ.get("UGDR_DAEMON_SOCKET")
            os.environ["UGDR_DAEMON_SOCKET"] = socket_path
            self._exported = True

    def stop(self, timeout: float = 30.0) -> int:
        if self.proc.poll() is None:
            self.proc.send_signal(signal.SIGTERM)
            try:
                self.proc.wait(timeout)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
        self._log.close()
        if self._exported and os.environ.get("UGDR_DAEMON_SOCKET") == self.socket_path:
            if self._prev_socket is None:
                os.environ.pop("UGDR_DAEMON_SOCKET", None)
            else:
                os.environ["UGDR_DAEMON_SOCKET"] = self._prev_socket
        self._exported = False
        if self._dir:
            with contextlib.suppress(OSError):
                os.unlink(self.socket_path)
            with contextlib.suppress(OSError):
                os.rmdir(self._dir)
        return self.proc.returncode

    def log_text(self) -> str:
        try:
            with open(self.log_path) as f:
                return f.read()
        except OSError:
            return ""

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.stop()


# ---- objects ----------------------------------------------------------------------------------


@dataclass
class Device:
    name: str
    kind: int  # 0 cpu, 1 gpu
    gpu: int
    handle: int


def get_devices() -> list[Device]:
    L = N.lib()
    n = C.c_int(0)
    lst = _check_ptr(L.ugdr_get_device_list(C.byref(n)), "ugdr_get_device_list")
    out = []
    for i in range(n.value):
        info = N.DeviceInfo()
        _check(L.ugdr_x_query_device(lst[i], C.byref(info)), "ugdr_x_query_device")
        out.append(Device(info.name.decode(), info.kind, info.gpu_ordinal, lst[i]))
    # The list's proxies stay valid until freed; keep the list alive for the process.
    _device_lists.append(lst)
    return out


_device_lists: list = []


def find_device(name: str | None = None, gpu: int | None = None, kind: int | None = None) -> Device:
    for d in get_devices():
        if name is not None and d.name == name:
            return d
        if gpu is not None and d.kind == 1 and d.gpu == gpu:
            return d
        if kind is not None and name is None and gpu is None and d.kind == kind:
            return d
    raise UgdrError(19, f"no ugdr device matching name={name} gpu={gpu} kind={kind}")


class Context:
    def __init__(self, device: Device):
        self.device = device
        self.h = _check_ptr(N.lib().ugdr_open_device(device.handle), "ugdr_open_device")

    def __enter__(self) -> "Context":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def close(self) -> None:
        if N.lib().ugdr_close_device(self.h) != 0:
            e = N.errno()
            raise UgdrError(e, f"ugdr_close_device: {N.errname(e)}")

    def alloc_pd(self) -> "Pd":
        return Pd(self)

    def create_cq(self, cqe: int) -> "CompletionQueue":
        return CompletionQueue(self, cqe)

    def stats(self, reset: bool = False) -> N.EngineStats:
        st = N.EngineStats()
        _check(N.lib().ugdr_x_query_engine_stats(self.h, C.byref(st), int(reset)), "engine stats")
        return st

    def trace(self, records_per_cta: int) -> None:
        """Keep up to `records_per_cta` executor events per CTA from the next launch on (0: off)."""
        _check(N.lib().ugdr_x_engine_trace(self.h, records_per_cta), "ugdr_x_engine_trace")

    def trace_dump(self, path: str) -> tuple[int, int]:
        """Write the kept events (Chrome trace JSON) to `path`; returns (kept, dropped)."""
        k, d = C.c_uint64(), C.c_uint64()
        _check(N.lib().ugdr_x_engine_trace_dump(self.h, path.encode(), C.byref(k), C.byref(d)),
               "ugdr_x_engine_trace_dump")
        return k.value, d.value

    def hold(self, on: bool) -> None:
        _check(N.lib().ugdr_x_engine_hold(self.h, int(on)), "engine hold")


def daemon_stats() -> dict:
    """Live objects in the daemon over all sessions, and its device count."""
    st = N.DaemonStats()
    _check(N.lib().ugdr_x_query_daemon_stats(C.byref(st)), "ugdr_x_query_daemon_stats")
    return {f: int(getattr(st, f)) for f, _ in st._fields_}


def timed_drain(contexts: list[Context], expected: list[int], timeout_ms: int = 60000) -> list[float]:
    n = len(contexts)
    arr = (C.c_void_p * n)(*[c.h for c in contexts])
    exp = (C.c_uint64 * n)(*expected)
    out = (C.c_float * n)()
    _check(N.lib().ugdr_x_timed_drain(arr, n, exp, timeout_ms, out), "timed drain")
    return [out[i] for i in range(n)]


class Pd:
    def __init__(self, ctx: Context):
        self.ctx = ctx
        self.h = _check_ptr(N.lib().ugdr_alloc_pd(ctx.h), "ugdr_alloc_pd")

    def __enter__(self) -> "Pd":
        return self

    def __exit__(self, *exc) -> None:
        self.dealloc()

    def dealloc(self) -> None:
        _check(N.lib().ugdr_dealloc_pd(self.h), "ugdr_dealloc_pd")

    def reg_mr(self, addr: int, length: int, access: int) -> "MemoryRegion":
        return MemoryRegion(self, addr, length, access)

    def reg_mr_multicast(self, mc_addr: int, length: int, access: int, mc_fd: int) -> "MemoryRegion":
        """An NVLS multicast object as an MR (see ugdr_x_reg_mr_multicast)."""
        return MemoryRegion(self, mc_addr, length, access, mc_fd=mc_fd)

    def create_qp(self, send_cq: "CompletionQueue", recv_cq: "CompletionQueue | None" = None,
                  max_send_wr: int = 128, max_recv_wr: int = 128, max_send_sge: int = 1,
                  max_recv_sge: int = 1, sq_sig_all: bool = False) -> "QueuePair":
        return QueuePair(self, send_cq, recv_cq or send_cq, max_send_wr, max_recv_wr,
                         max_send_sge, max_recv_sge, sq_sig_all)


class MemoryRegion:
    def __init__(self, pd: Pd, addr: int, length: int, access: int, mc_fd: int = -1):
        self.pd = pd
        if mc_fd >= 0:  # an NVLink multicast object (ugdr_x_reg_mr_multicast); addr: its multicast view
            self.p = _check_ptr(N.lib().ugdr_x_reg_mr_multicast(pd.h, C.c_void_p(addr), length, access, mc_fd),
                                "ugdr_x_reg_mr_multicast")
        else:
            self.p = _check_ptr(N.lib().ugdr_reg_mr(pd.h, C.c_void_p(addr), length, access), "ugdr_reg_mr")
        self.addr = addr
        self.length = length
        self.lkey = self.p.contents.lkey
        self.rkey = self.p.contents.rkey

    def __enter__(self) -> "MemoryRegion":
        return self

    def __exit__(self, *exc) -> None:
        self.dereg()

    def dereg(self) -> None:
        _check(N.lib().ugdr_dereg_mr(self.p), "ugdr_dereg_mr")


@dataclass
class Completion:
    wr_id: int
    status: int
    opcode: int
    byte_len: int
    imm_data: int
    qp_num: int
    wc_flags: int


class CompletionQueue:
    def __init__(self, ctx: Context, cqe: int):
        self.ctx = ctx
        self.h = _check_ptr(N.lib().ugdr_create_cq(ctx.h, cqe, None, None, 0), "ugdr_create_cq")
        self._buf = (N.Wc * 256)()

    def __enter__(self) -> "CompletionQueue":
        return self

    def __exit__(self, *exc) -> None:
        self.destroy()

    def destroy(self) -> None:
        _check(N.lib().ugdr_destroy_cq(self.h), "ugdr_destroy_cq")

    def poll(self, n: int = 256) -> list[Completion]:
        n = min(n, 256)
        got = N.lib().ugdr_poll_cq(self.h, n, self._buf)
        if got < 0:
            raise UgdrError(-got, f"ugdr_poll_cq: {N.errname(-got)}")
        return [Completion(w.wr_id, w.status, w.opcode, w.byte_len, w.imm_data, w.qp_num, w.wc_flags)
                for w in self._buf[:got]]

    def wait(self, count: int, timeout: float = 30.0) -> list[Completion]:
        """At least `count` completions (the C library busy-polls; no Python loop per poll)."""
        out: list[Completion] = []
        deadline = time.time() + timeout
        while len(out) < count:
            want = min(count - len(out), 256)
            left_ns = max(0, int((deadline - time.time()) * 1e9))
            got = N.lib().ugdr_x_poll_cq_wait(self.h, want, want, self._buf, left_ns)
            if got < 0:
                raise UgdrError(-got, f"ugdr_x_poll_cq_wait: {N.errname(-got)}")
            out += [Completion(w.wr_id, w.status, w.opcode, w.byte_len, w.imm_data, w.qp_num, w.wc_flags)
                    for w in self._buf[:got]]
            if len(out) < count and time.time() > deadline:
                raise TimeoutError(f"got {len(out)} of {count} completions")
        return out


class QueuePair:
    def __init__(self, pd: Pd, send_cq: CompletionQueue, recv_cq: CompletionQueue, max_send_wr: int,
                 max_recv_wr: int, max_send_sge: int, max_recv_sge: int, sq_sig_all: bool):
        self.pd = pd
        a = N.QpInitAttr(send_cq.h, recv_cq.h, max_send_wr, max_recv_wr, max_send_sge, max_recv_sge,
                         N.QPT_RC, int(sq_sig_all))
        self.h = _check_ptr(N.lib().ugdr_create_qp(pd.h, C.byref(a)), "ugdr_create_qp")
        info = N.QpConnInfo()
        _check(N.lib().ugdr_query_qp_conn_info(self.h, C.byref(info)), "conn info")
        self.qpn = info.qp_num

    def __enter__(self) -> "QueuePair":
        return self

    def __exit__(self, *exc) -> None:
        self.destroy()

    def destroy(self) -> None:
        _check(N.lib().ugdr_destroy_qp(self.h), "ugdr_destroy_qp")

    def modify(self, attr: N.QpAttr, mask: int) -> int:
        return N.lib().ugdr_modify_qp(self.h, C.byref(attr), mask)

    def to_init(self, access: int = N.ACCESS_REMOTE_WRITE) -> None:
        a = N.QpAttr(qp_state=N.QPS_INIT, qp_access_flags=access)
        _check(self.modify(a, N.QP_STATE | N.QP_ACCESS_FLAGS), "modify INIT")

    def to_error(self) -> None:
        _check(self.modify(N.QpAttr(qp_state=N.QPS_ERR), N.QP_STATE), "modify ERR")

    def connect(self, remote_qpn: int, timeout: int = 14, retry_cnt: int = 7, rnr_retry: int = 7,
                min_rnr_timer: int = 12) -> None:
        info = N.QpConnInfo(remote_qpn)
        a = N.QpAttr(timeout=timeout, retry_cnt=retry_cnt, rnr_retry=rnr_retry,
                     min_rnr_timer=min_rnr_timer)
        _check(N.lib().ugdr_connect_qp(self.h, C.byref(info), C.byref(a), N.CONNECT_MASK), "connect")

    def query(self) -> tuple[N.QpAttr, N.QpInitAttr]:
        a, ia = N.QpAttr(), N.QpInitAttr()
        mask = (N.QP_STATE | N.QP_CUR_STATE | N.QP_ACCESS_FLAGS | N.QP_TIMEOUT | N.QP_RETRY_CNT
                | N.QP_RNR_RETRY | N.QP_MIN_RNR_TIMER)
        _check(N.lib().ugdr_query_qp(self.h, C.byref(a), mask, C.byref(ia)), "ugdr_query_qp")
        return a, ia

    def stats(self) -> N.QpStats:
        """Per-QP counters: ring cursors (posted / retired / consumed) and the engine's byte,
        error and RNR counts."""
        st = N.QpStats()
        _check(N.lib().ugdr_x_query_qp_stats(self.h, C.byref(st)), "ugdr_x_query_qp_stats")
        return st

    # -- posting --
    def post_send_raw(self, wrs: list[N.SendWr]) -> tuple[int, int]:
        """Post a chain; returns (rc, index of bad_wr or -1)."""
        for i in range(len(wrs) - 1):
            wrs[i].next = C.pointer(wrs[i + 1])
        if wrs:
            wrs[-1].next = None
        bad = C.POINTER(N.SendWr)()
        rc = N.lib().ugdr_post_send(self.h, C.byref(wrs[0]), C.byref(bad))
        idx = -1
        if rc != 0 and bad:
            addr = C.addressof(bad.contents)
            idx = next((i for i, w in enumerate(wrs) if C.addressof(w) == addr), -1)
        return rc, idx

    @staticmethod
    def make_send_wr(opcode: int, sges: list[tuple[int, int, int]], remote_addr: int = 0, rkey: int = 0,
                     wr_id: int = 0, signaled: bool = True, imm: int = 0, compare_add: int = 0,
                     swap: int = 0) -> N.SendWr:
        sg = (N.Sge * max(1, len(sges)))(*[N.Sge(a, l, k) for a, l, k in sges])
        w = N.SendWr()
        w.wr_id = wr_id
        w.sg_list = C.cast(sg, C.POINTER(N.Sge)) if sges else None
        w.num_sge = len(sges)
        w.opcode = opcode
        w.send_flags = N.SEND_SIGNALED if signaled else 0
        w.imm_data = imm
        if opcode in (N.WR_ATOMIC_CMP_AND_SWP, N.WR_ATOMIC_FETCH_AND_ADD):
            w.wr.atomic.remote_addr = remote_addr
            w.wr.atomic.rkey = rkey
            w.wr.atomic.compare_add = compare_add
            w.wr.atomic.swap = swap
        else:
            w.wr.rdma.remote_addr = remote_addr
            w.wr.rdma.rkey = rkey
        w._keep = sg  # keep the SGE array alive with the WR
        return w

    def post_send(self, opcode: int, sges: list[tuple[int, int, int]], **kw) -> None:
        rc, _ = self.post_send_raw([self.make_send_wr(opcode, sges, **kw)])
        _check(rc, "ugdr_post_send")

    def post_write(self, local: tuple[int, int, int], remote_addr: int, rkey: int, **kw) -> None:
        self.post_send(N.WR_RDMA_WRITE, [local], remote_addr=remote_addr, rkey=rkey, **kw)

    def post_read(self, local: tuple[int, int, int], remote_addr: int, rkey: int, **kw) -> None:
        self.post_send(N.WR_RDMA_READ, [local], remote_addr=remote_addr, rkey=rkey, **kw)

    def post_recv(self, wr_id: int, sges: list[tuple[int, int, int]] = ()) -> None:
        rc, _ = self.post_recv_raw([self.make_recv_wr(wr_id, list(sges))])
        _check(rc, "ugdr_post_recv")

    @staticmethod
    def make_recv_wr(wr_id: int, sges: list[tuple[int, int, int]]) -> N.RecvWr:
        sg = (N.Sge * max(1, len(sges)))(*[N.Sge(a, l, k) for a, l, k in sges])
        w = N.RecvWr()
        w.wr_id = wr_id
        w.sg_list = C.cast(sg, C.POINTER(N.Sge)) if sges else None
        w.num_sge = len(sges)
        w._keep = sg
        return w

    def post_recv_raw(self, wrs: list[N.RecvWr]) -> tuple[int, int]:
        for i in range(len(wrs) - 1):
            wrs[i].next = C.pointer(wrs[i + 1])
        wrs[-1].next = None
        bad = C.POINTER(N.RecvWr)()
        rc = N.lib().ugdr_post_recv(self.h, C.byref(wrs[0]), C.byref(bad))
        idx = -1
        if rc != 0 and bad:
            addr = C.addressof(bad.contents)
            idx = next((i for i, w in enumerate(wrs) if C.addressof(w) == addr), -1)
        return rc, idx


def connect_pair(a: QueuePair, b: QueuePair, access: int = N.ACCESS_REMOTE_WRITE, **kw) -> None:
    """Bring two QPs to RTS bound to each other."""
    a.to_init(access)
    b.to_init(access)
    a.connect(b.qpn, **kw)
    b.connect(a.qpn, **kw)


class HostBuffer:
    """Host memory the daemon can reach (memfd-backed, from ugdr_x_alloc_host)."""

    def __init__(self, length: int):
        self.length = length
        self.addr = _check_ptr(N.lib().ugdr_x_alloc_host(length), "ugdr_x_alloc_host")

    def view(self):
        import numpy as np

        return np.ctypeslib.as_array((C.c_uint8 * self.length).from_address(self.addr))

    def __enter__(self) -> "HostBuffer":
        return self

    def __exit__(self, *exc) -> None:
        self.free()

    def free(self) -> None:
        _check(N.lib().ugdr_x_free_host(C.c_void_p(self.addr)), "ugdr_x_free_host")
