"""Property test of the host-memory engine against a pure-Python model of the verbs semantics.

The host engine is the byte-exact oracle the GPU executor is tested against, so its semantics
are pinned here independently.  Hypothesis draws random WR streams:
- RDMA WRITE, WRITE_WITH_IMM and READ with 1-4 SGEs of random lengths and offsets (unaligned);
- FETCH_ADD and CMP_AND_SWP on 8-byte aligned counters;
- signaled and unsignaled WRs;
- now and then a fault: a bad lkey, a remote range past the MR end, or a misaligned atomic.

The model predicts:
- every byte of both buffers;
- the send completions (wr_id, status, opcode, byte_len) in order, with unsignaled successes
  silent;
- the error that moves the QP to ERR, and the FLUSH_ERR of every WR after it;
- the receive completions of the immediates.
"""
from __future__ import annotations

import struct

import numpy as np
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

from ugdr_b200 import _native as N  # noqa: E402
from ugdr_b200 import verbs as V  # noqa: E402

LEN = 1 << 14  # bytes per buffer
ACC = N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ | N.ACCESS_REMOTE_ATOMIC
REMOTE = N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ | N.ACCESS_REMOTE_ATOMIC
CTR = LEN - 256  # counters live in the last 256 bytes of the remote buffer (32 of them)
WC_OP = {N.WR_RDMA_WRITE: N.WC_RDMA_WRITE, N.WR_RDMA_WRITE_WITH_IMM: N.WC_RDMA_WRITE,
         N.WR_RDMA_READ: N.WC_RDMA_READ, N.WR_ATOMIC_FETCH_AND_ADD: N.WC_FETCH_ADD,
         N.WR_ATOMIC_CMP_AND_SWP: N.WC_COMP_SWAP}


@st.composite
def wr_stream(draw):
    n = draw(st.integers(1, 24))
    wrs = []
    for i in range(n):
        kind = draw(st.sampled_from(["write", "imm", "read", "faa", "cas"]))
        signaled = draw(st.booleans())
        fault = draw(st.sampled_from([None] * 12 + ["lkey", "range", "align"]))
        if kind in ("faa", "cas"):
            ctr = draw(st.integers(0, 31))
            if fault == "align":
                ctr = min(ctr, 30)  # the misaligned 8 bytes stay inside the MR (else: access error first)
            wrs.append(dict(kind=kind, signaled=signaled, fault=fault if fault != "range" else None,
                            ctr=ctr, local=draw(st.integers(0, 255)) * 8,
                            operand=draw(st.integers(0, 5)), swap=draw(st.integers(0, 1 << 40))))
            continue
        nsge = draw(st.integers(1, 4))
        sges = []
        for _ in range(nsge):
            ln = draw(st.integers(0, 700))
            off = draw(st.integers(0, CTR - 1 - ln))
            sges.append((off, ln))
        total = sum(ln for _, ln in sges)
        roff = draw(st.integers(0, CTR - 1 - total))
        wrs.append(dict(kind=kind, signaled=signaled, fault=fault if fault != "align" else None, sges=sges,
                        roff=roff, imm=draw(st.integers(0, (1 << 32) - 1))))
    return wrs


def model(wrs, loc0: np.ndarray, rem0: np.ndarray):
    """Expected (local bytes, remote bytes, send CQEs, recv CQEs) after the stream."""
    loc, rem = loc0.copy(), rem0.copy()
    send, recv = [], []
    err = False
    for i, w in enumerate(wrs):
        op = {"write": N.WR_RDMA_WRITE, "imm": N.WR_RDMA_WRITE_WITH_IMM, "read": N.WR_RDMA_READ,
              "faa": N.WR_ATOMIC_FETCH_AND_ADD, "cas": N.WR_ATOMIC_CMP_AND_SWP}[w["kind"]]
        if err:
            send.append((i, N.WC_WR_FLUSH_ERR, WC_OP[op], 0))
            continue
        status = N.WC_SUCCESS
        # Zero-length SGEs touch no memory, so their lkey is not checked (as on an HCA).
        if w["fault"] == "lkey" and (w["kind"] in ("faa", "cas") or any(ln for _, ln in w["sges"])):
            status = N.WC_LOC_PROT_ERR
        elif w["fault"] == "range":
            status = N.WC_REM_ACCESS_ERR
        elif w["fault"] == "align":
            status = N.WC_REM_INV_REQ_ERR
        if status != N.WC_SUCCESS:
            send.append((i, status, WC_OP[op], 0))
            err = True
            continue
        if w["kind"] in ("faa", "cas"):
            a = CTR + 8 * w["ctr"]
            old = int(rem[a:a + 8].view(np.uint64)[0])
            if w["kind"] == "faa":
                new = (old + w["operand"]) & ((1 << 64) - 1)
            else:
                new = w["swap"] if old == w["operand"] else old
            rem[a:a + 8] = np.frombuffer(struct.pack("<Q", new), dtype=np.uint8)
            loc[w["local"]:w["local"] + 8] = np.frombuffer(struct.pack("<Q", old), dtype=np.uint8)
            total = 8
        else:
            total = sum(ln for _, ln in w["sges"])
            pos = w["roff"]
            for off, ln in w["sges"]:
                if w["kind"] == "read":
                    loc[off:off + ln] = rem[pos:pos + ln]
                else:
                    rem[pos:pos + ln] = loc[off:off + ln]
                pos += ln
            if w["kind"] == "imm":
                recv.append((1000 + i, total, w["imm"]))
        if w["signaled"]:
            send.append((i, N.WC_SUCCESS, WC_OP[op], total))
    return loc, rem, send, recv, err


@pytest.fixture(scope="module")
def daemon():
    d = V.Daemon(gpus=0)
    yield d
    d.stop()


@settings(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(wrs=wr_stream(), seed=st.integers(0, 1 << 30))
def test_host_engine_matches_the_model(daemon, wrs, seed):
    ctx = V.Context(V.find_device(kind=0))
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(256)
    a = pd.create_qp(cq, max_send_wr=64, max_recv_wr=64, max_send_sge=4, max_recv_sge=1)
    b = pd.create_qp(cq, max_send_wr=64, max_recv_wr=64, max_send_sge=4, max_recv_sge=1)
    V.connect_pair(a, b, access=REMOTE)
    lb, rb = V.HostBuffer(LEN), V.HostBuffer(LEN)
    lv, rv = lb.view(), rb.view()
    rng = np.random.default_rng(seed)
    lv[:] = rng.integers(0, 256, LEN, dtype=np.uint8)
    rv[:] = rng.integers(0, 256, LEN, dtype=np.uint8)
    rv[CTR:] = 0
    loc0, rem0 = lv.copy(), rv.copy()
    lm, rm = pd.reg_mr(lb.addr, LEN, ACC), pd.reg_mr(rb.addr, LEN, ACC)
    try:
        for i, w in enumerate(wrs):
            if w["kind"] == "imm":
                b.post_recv(1000 + i)
        raw = []
        for i, w in enumerate(wrs):
            lkey = lm.lkey ^ 0x2 if w["fault"] == "lkey" else lm.lkey
            if w["kind"] in ("faa", "cas"):
                op = N.WR_ATOMIC_FETCH_AND_ADD if w["kind"] == "faa" else N.WR_ATOMIC_CMP_AND_SWP
                raddr = rb.addr + CTR + 8 * w["ctr"] + (4 if w["fault"] == "align" else 0)
                raw.append(V.QueuePair.make_send_wr(op, [(lb.addr + w["local"], 8, lkey)], remote_addr=raddr,
                                                    rkey=rm.rkey, wr_id=i, signaled=w["signaled"],
                                                    compare_add=w["operand"], swap=w["swap"]))
            else:
                op = {"write": N.WR_RDMA_WRITE, "imm": N.WR_RDMA_WRITE_WITH_IMM, "read": N.WR_RDMA_READ}[w["kind"]]
                sges = [(lb.addr + off, ln, lkey) for off, ln in w["sges"]]
                roff = LEN - 8 if w["fault"] == "range" else w["roff"]
                total = sum(ln for _, ln in w["sges"])
                if w["fault"] == "range" and total <= 8:
                    sges[0] = (sges[0][0], 64, lkey)  # make the range really overrun the MR
                    w["sges"][0] = (w["sges"][0][0], 64)
                raw.append(V.QueuePair.make_send_wr(op, sges, remote_addr=rb.addr + roff, rkey=rm.rkey, wr_id=i,
                                                    signaled=w["signaled"], imm=w["imm"]))
        # A signaled zero-length WRITE closes the stream, so there is always a completion that
        # comes after every WR above has run (or been flushed).
        raw.append(V.QueuePair.make_send_wr(N.WR_RDMA_WRITE, [], remote_addr=rb.addr, rkey=rm.rkey,
                                            wr_id=len(wrs), signaled=True))
        rc, bad = a.post_send_raw(raw)
        assert rc == 0 and bad == -1
        loc, rem, send, recv, err = model(wrs, loc0, rem0)
        send.append((len(wrs), N.WC_WR_FLUSH_ERR if err else N.WC_SUCCESS, N.WC_RDMA_WRITE, 0))
        got = cq.wait(len(send) + len(recv), timeout=30)
        got_send = [(w.wr_id, w.status, w.opcode, w.byte_len) for w in got if w.opcode != N.WC_RECV_RDMA_WITH_IMM]
        got_recv = [(w.wr_id, w.byte_len, w.imm_data) for w in got
                    if w.opcode == N.WC_RECV_RDMA_WITH_IMM and w.status == N.WC_SUCCESS]
        assert got_send == send
        assert got_recv == recv
        assert np.array_equal(lv, loc)
        assert np.array_equal(rv, rem)
        assert cq.poll() == [] or err  # nothing extra (flushes of the responder RQ come only after ERR)
    finally:
        for q in (a, b):
            q.destroy()
        lm.dereg()
        rm.dereg()
        cq.destroy()
        pd.dealloc()
        ctx.close()
        lb.free()
        rb.free()
