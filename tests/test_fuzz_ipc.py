"""Robustness of the daemon's control socket against malformed clients (reference suite semantics:
tests/unit/ipc_protocol_test.cpp - truncation, bad magic - extended to random input).

Hypothesis sends random datagrams over raw SOCK_SEQPACKET connections:
- pure noise;
- envelopes with a valid magic and random method, flags, lengths and fd counts;
- well-formed envelopes whose RPC payloads are random bytes.

The daemon may answer with an error or drop the session, but it must stay up and keep serving a
well-behaved client.
"""
from __future__ import annotations

import os
import socket
import struct
import subprocess

import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

from ugdr_b200 import _native as N  # noqa: E402
from ugdr_b200 import verbs as V  # noqa: E402

MAGIC = 0x49504331


def envelope(method: int, flags: int, req: int, status: int, plen: int, nfd: int) -> bytes:
    return struct.pack(">IHHIIQiII", MAGIC, 1, 0, method, flags, req, status, plen, nfd)


@st.composite
def datagrams(draw):
    kind = draw(st.sampled_from(["noise", "envelope", "rpc"]))
    if kind == "noise":
        return draw(st.binary(min_size=0, max_size=256))
    method = draw(st.sampled_from(list(range(0, 17)) + [32, 33, 34, 35, 0xFFFFFFFF]))
    payload = draw(st.binary(min_size=0, max_size=200))
    if kind == "envelope":
        plen = draw(st.sampled_from([len(payload), len(payload) + 1, 0, 1 << 20, (1 << 32) - 1]))
        nfd = draw(st.sampled_from([0, 1, 16, 17, 1 << 31]))
        return envelope(method, draw(st.integers(0, 3)), draw(st.integers(0, 1 << 63)), 0, plen, nfd) + payload
    # rpc: a consistent envelope around a random (possibly prefix-valid) request body
    body = struct.pack(">HHQQII", 1, 0, draw(st.integers(0, 1 << 63)), draw(st.integers(0, 1 << 63)),
                       draw(st.integers(0, 0xFFFFFFFF)), draw(st.integers(0, 300))) + payload
    return envelope(method, 0, draw(st.integers(0, 1 << 63)), 0, len(body), 0) + body


@pytest.fixture(scope="module")
def daemon(tmp_path_factory):
    sock = str(tmp_path_factory.mktemp("fuzz") / "ugdr.sock")
    d = V.Daemon(gpus=0, socket_path=sock)
    yield d
    d.stop()


def _healthy(d) -> bool:
    env = dict(os.environ, UGDR_DAEMON_SOCKET=d.socket_path)
    r = subprocess.run([str(N.LIB_DIR / "ugdr_client")], env=env, capture_output=True, text=True, timeout=30)
    return r.returncode == 0 and "kind=cpu" in r.stdout


@settings(max_examples=300, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(msgs=st.lists(datagrams(), min_size=1, max_size=4))
def test_daemon_survives_malformed_clients(daemon, msgs):
    s = socket.socket(socket.AF_UNIX, socket.SOCK_SEQPACKET)
    s.settimeout(2.0)
    try:
        s.connect(daemon.socket_path)
        for m in msgs:
            try:
                s.send(m)
                s.recv(1 << 16)  # an error reply, or nothing if the daemon dropped the session
            except (socket.timeout, ConnectionError, OSError):
                break
    finally:
        s.close()
    assert daemon.proc.poll() is None, daemon.log_text()[-2000:]


def test_daemon_still_serves_after_fuzzing(daemon):
    assert daemon.proc.poll() is None
    assert _healthy(daemon)


def _fd_count(pid: int) -> int:
    return len(os.listdir(f"/proc/{pid}/fd"))


def test_fds_sent_with_bad_requests_are_not_leaked(daemon):
    """Descriptors attached (SCM_RIGHTS) to malformed or refused requests are closed by the daemon:
    its descriptor count returns to where it was after many such requests."""
    import array

    assert _healthy(daemon)
    before = _fd_count(daemon.proc.pid)
    for i in range(200):
        s = socket.socket(socket.AF_UNIX, socket.SOCK_SEQPACKET)
        s.settimeout(2.0)
        fds = [os.memfd_create(f"leak{i}_{k}") for k in range(3)]
        try:
            s.connect(daemon.socket_path)
            kind = i % 4
            if kind == 0:  # garbage bytes with descriptors
                msg = os.urandom(40)
            elif kind == 1:  # valid envelope, unknown method, descriptor count matching
                msg = envelope(999, 0, i, 0, 0, 3)
            elif kind == 2:  # register-MR method with a truncated body
                msg = envelope(6, 0, i, 0, 8, 3) + b"\0" * 8
            else:  # well-formed register-MR request for a PD that does not exist
                opaque = struct.pack(">B3xQQQ", 1, 0x10000, 4096, 0)
                body = struct.pack(">HHQQII", 1, 0, 0x0300000100000001, 4096, 1, len(opaque)) + opaque
                msg = envelope(6, 0, i, 0, len(body), 3) + body
            s.sendmsg([msg], [(socket.SOL_SOCKET, socket.SCM_RIGHTS, array.array("i", fds))])
            try:
                s.recv(1 << 16)
            except (socket.timeout, OSError):
                pass
        except (ConnectionError, OSError):
            pass
        finally:
            s.close()
            for fd in fds:
                os.close(fd)
    assert daemon.proc.poll() is None
    assert _healthy(daemon)
    import time

    deadline = time.time() + 5
    while _fd_count(daemon.proc.pid) > before + 2 and time.time() < deadline:
        time.sleep(0.05)
    assert _fd_count(daemon.proc.pid) <= before + 2, (before, _fd_count(daemon.proc.pid))


def test_objects_of_a_vanished_client_release_their_descriptors(daemon):
    """A client that registers host MRs and creates CQs and QPs (each backed by a memfd the daemon
    holds) and then exits without destroying anything: session reclaim closes every descriptor."""
    import sys
    import time

    assert _healthy(daemon)
    before = _fd_count(daemon.proc.pid)
    code = (
        "import os\n"
        "from ugdr_b200 import verbs as V, _native as N\n"
        "ctx = V.Context(V.find_device(kind=0))\n"
        "pd = ctx.alloc_pd()\n"
        "cqs = [ctx.create_cq(64) for _ in range(4)]\n"
        "qps = [pd.create_qp(cqs[i % 4], max_send_wr=16, max_recv_wr=16) for i in range(8)]\n"
        "bufs = [V.HostBuffer(1 << 16) for _ in range(4)]\n"
        "mrs = [pd.reg_mr(b.addr, 1 << 16, N.ACCESS_LOCAL_WRITE) for b in bufs]\n"
        "print('held', flush=True)\n"
        "input()\n"
        "os._exit(0)\n")
    env = dict(os.environ, UGDR_DAEMON_SOCKET=daemon.socket_path,
               PYTHONPATH=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    p = subprocess.Popen([sys.executable, "-c", code], env=env, stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                         stderr=subprocess.PIPE, text=True)
    try:
        assert p.stdout.readline().strip() == "held", p.stderr.read()
        # The daemon now holds the rings and MR regions (4 CQs + 8 x 2 QP rings + 4 MRs).
        assert _fd_count(daemon.proc.pid) >= before + 20, (before, _fd_count(daemon.proc.pid))
        p.stdin.write("\n")
        p.stdin.flush()
        assert p.wait(timeout=60) == 0
    finally:
        if p.poll() is None:
            p.kill()
            p.wait()
    deadline = time.time() + 10
    while _fd_count(daemon.proc.pid) > before + 2 and time.time() < deadline:
        time.sleep(0.05)
    assert _fd_count(daemon.proc.pid) <= before + 2, (before, _fd_count(daemon.proc.pid))
    assert _healthy(daemon)


def test_descriptor_exhaustion_refuses_the_request_and_keeps_the_session(tmp_path):
    """At its descriptor limit the daemon answers EMFILE to a registration whose region
    descriptor it could not receive; the client's session survives, and once MRs are freed
    registration works again."""
    import errno
    import resource

    d = V.Daemon(gpus=0, socket_path=str(tmp_path / "d.sock"))
    try:
        env_sock = os.environ.get("UGDR_DAEMON_SOCKET")
        os.environ["UGDR_DAEMON_SOCKET"] = d.socket_path
        ctx = V.Context(V.find_device(kind=0))
        pd = ctx.alloc_pd()
        buf = V.HostBuffer(1 << 16)
        have = _fd_count(d.proc.pid)
        resource.prlimit(d.proc.pid, resource.RLIMIT_NOFILE, (have + 40, have + 40))
        mrs, err = [], None
        for _ in range(200):
            try:
                mrs.append(pd.reg_mr(buf.addr, 4096, N.ACCESS_LOCAL_WRITE))
            except V.UgdrError as e:
                err = e
                break
        assert err is not None and err.errno == errno.EMFILE, err
        assert 20 <= len(mrs) <= 40
        # A new connection at the limit is accepted on a reserved descriptor and closed at once.
        s = socket.socket(socket.AF_UNIX, socket.SOCK_SEQPACKET)
        s.settimeout(5.0)
        s.connect(d.socket_path)
        assert s.recv(64) == b""
        s.close()
        for m in mrs[:8]:
            m.dereg()
        again = pd.reg_mr(buf.addr, 4096, N.ACCESS_LOCAL_WRITE)  # same session, still connected
        again.dereg()
        for m in mrs[8:]:
            m.dereg()
        pd.dealloc()
        ctx.close()
        buf.free()
        assert d.proc.poll() is None
    finally:
        if env_sock is None:
            os.environ.pop("UGDR_DAEMON_SOCKET", None)
        else:
            os.environ["UGDR_DAEMON_SOCKET"] = env_sock
        d.stop()


def test_client_at_its_descriptor_limit_gets_emfile_and_leaves_no_orphan(daemon):
    """A client at its own descriptor limit cannot receive a new CQ's ring: ugdr_create_cq fails
    with EMFILE, the library destroys the CQ the daemon made for it, and the connection stays
    usable."""
    import sys
    import time

    code = (
        "import os, resource\n"
        "from ugdr_b200 import verbs as V\n"
        "ctx = V.Context(V.find_device(kind=0))\n"
        "n = len(os.listdir('/proc/self/fd'))\n"
        "resource.setrlimit(resource.RLIMIT_NOFILE, (n + 6, resource.getrlimit(resource.RLIMIT_NOFILE)[1]))\n"
        "cqs, err = [], None\n"
        "while err is None and len(cqs) < 50:\n"
        "    try:\n"
        "        cqs.append(ctx.create_cq(16))\n"
        "    except V.UgdrError as e:\n"
        "        err = e.errno\n"
        "print(len(cqs), err, flush=True)\n"
        "input()\n"
        "cqs[0].destroy()\n"
        "print('ok', ctx.create_cq(16) is not None, flush=True)\n"
        "os._exit(0)\n")
    env = dict(os.environ, UGDR_DAEMON_SOCKET=daemon.socket_path,
               PYTHONPATH=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    before = _fd_count(daemon.proc.pid)
    p = subprocess.Popen([sys.executable, "-c", code], env=env, stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                         stderr=subprocess.PIPE, text=True)
    try:
        made, err = p.stdout.readline().split()
        assert err == str(__import__("errno").EMFILE) and 1 <= int(made) < 50
        time.sleep(0.1)
        # The daemon holds the client's session socket and one ring descriptor per CQ the client
        # kept, none for the refused one.
        assert _fd_count(daemon.proc.pid) == before + 1 + int(made), (before, made, _fd_count(daemon.proc.pid))
        p.stdin.write("\n")
        p.stdin.flush()
        assert p.stdout.readline().strip() == "ok True"
        assert p.wait(timeout=60) == 0
    finally:
        if p.poll() is None:
            p.kill()
            p.wait()


def test_a_client_that_never_reads_replies_cannot_stall_the_daemon(tmp_path):
    """A client that floods requests and never reads the replies fills its socket's buffer; the
    daemon drops that session instead of blocking on it, and keeps serving everyone else."""
    import threading

    d = V.Daemon(gpus=0, socket_path=str(tmp_path / "d.sock"))
    try:
        flood = socket.socket(socket.AF_UNIX, socket.SOCK_SEQPACKET)
        flood.connect(d.socket_path)
        flood.settimeout(0.5)
        body = struct.pack(">HHQQII", 1, 0, 0, 0, 0, 0)
        sent = 0
        try:
            for i in range(200000):  # list-devices requests; their replies pile up unread
                flood.send(envelope(1, 0, i, 0, len(body), 0) + body)
                sent += 1
        except (socket.timeout, BlockingIOError, ConnectionError, OSError):
            pass
        assert sent > 100
        ok = threading.Event()

        def probe():
            ok.set() if _healthy(d) else None

        t = threading.Thread(target=probe)
        t.start()
        t.join(timeout=20)
        assert ok.is_set(), "daemon stopped serving other clients"
        flood.close()
        assert d.proc.poll() is None
    finally:
        d.stop()


def test_a_daemon_that_never_answers_times_out_the_call(tmp_path):
    """A listener that accepts and never replies: with UGDR_RPC_TIMEOUT_MS set, the client's first
    call (ugdr_client lists the devices) fails quickly instead of hanging."""
    import sys
    import time

    path = str(tmp_path / "mute.sock")
    srv = socket.socket(socket.AF_UNIX, socket.SOCK_SEQPACKET)
    srv.bind(path)
    srv.listen(4)
    try:
        env = {k: v for k, v in os.environ.items() if not k.startswith("UGDR_")}
        env.update(UGDR_DAEMON_SOCKET=path, UGDR_RPC_TIMEOUT_MS="300")
        t0 = time.time()
        r = subprocess.run([str(N.LIB_DIR / "ugdr_client")], env=env, capture_output=True, text=True, timeout=30)
        assert r.returncode != 0 and time.time() - t0 < 10, (r.stdout, r.stderr)
    finally:
        srv.close()
