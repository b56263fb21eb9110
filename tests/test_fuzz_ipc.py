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
