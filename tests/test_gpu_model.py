"""The sm_100a executor against the same Python model of the verbs semantics as the host engine
(tests/test_cpu_model.py): random multi-SGE WRITE / WRITE_WITH_IMM / READ and atomic streams
with faults, on GPU memory, with every byte and completion compared.

Marked gpu_extended: run with `pytest -m gpu_extended` on a B200 box.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import gpu_count

hypothesis = pytest.importorskip("hypothesis")
torch = pytest.importorskip("torch")
from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

from test_cpu_model import ACC, CTR, LEN, REMOTE, model, wr_stream  # noqa: E402
from ugdr_b200 import _native as N  # noqa: E402
from ugdr_b200 import verbs as V  # noqa: E402

pytestmark = pytest.mark.gpu_extended


@pytest.fixture(scope="module")
def gpu_daemon():
    if gpu_count() < 1:
        pytest.skip("no GPU")
    torch.cuda.set_device(0)
    d = V.Daemon(gpus=1)
    yield d
    d.stop()


@settings(max_examples=80, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(wrs=wr_stream(), seed=st.integers(0, 1 << 30))
def test_executor_matches_the_model(gpu_daemon, wrs, seed):
    ctx = V.Context(V.find_device(gpu=0))
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(256)
    a = pd.create_qp(cq, max_send_wr=64, max_recv_wr=64, max_send_sge=4, max_recv_sge=1)
    b = pd.create_qp(cq, max_send_wr=64, max_recv_wr=64, max_send_sge=4, max_recv_sge=1)
    V.connect_pair(a, b, access=REMOTE)
    rng = np.random.default_rng(seed)
    loc0 = rng.integers(0, 256, LEN, dtype=np.uint8)
    rem0 = rng.integers(0, 256, LEN, dtype=np.uint8)
    rem0[CTR:] = 0
    lt = torch.from_numpy(loc0.copy()).cuda()
    rt = torch.from_numpy(rem0.copy()).cuda()
    torch.cuda.synchronize()
    la, ra = lt.data_ptr(), rt.data_ptr()
    lm, rm = pd.reg_mr(la, LEN, ACC), pd.reg_mr(ra, LEN, ACC)
    try:
        for i, w in enumerate(wrs):
            if w["kind"] == "imm":
                b.post_recv(1000 + i)
        raw = []
        for i, w in enumerate(wrs):
            lkey = lm.lkey ^ 0x2 if w["fault"] == "lkey" else lm.lkey
            if w["kind"] in ("faa", "cas"):
                op = N.WR_ATOMIC_FETCH_AND_ADD if w["kind"] == "faa" else N.WR_ATOMIC_CMP_AND_SWP
                raddr = ra + CTR + 8 * w["ctr"] + (4 if w["fault"] == "align" else 0)
                raw.append(V.QueuePair.make_send_wr(op, [(la + w["local"], 8, lkey)], remote_addr=raddr, rkey=rm.rkey,
                                                    wr_id=i, signaled=w["signaled"], compare_add=w["operand"],
                                                    swap=w["swap"]))
            else:
                op = {"write": N.WR_RDMA_WRITE, "imm": N.WR_RDMA_WRITE_WITH_IMM, "read": N.WR_RDMA_READ}[w["kind"]]
                if w["fault"] == "range" and sum(ln for _, ln in w["sges"]) <= 8:
                    w["sges"][0] = (w["sges"][0][0], 64)
                sges = [(la + off, ln, lkey) for off, ln in w["sges"]]
                roff = LEN - 8 if w["fault"] == "range" else w["roff"]
                raw.append(V.QueuePair.make_send_wr(op, sges, remote_addr=ra + roff, rkey=rm.rkey, wr_id=i,
                                                    signaled=w["signaled"], imm=w["imm"]))
        raw.append(V.QueuePair.make_send_wr(N.WR_RDMA_WRITE, [], remote_addr=ra, rkey=rm.rkey, wr_id=len(wrs),
                                            signaled=True))
        rc, bad = a.post_send_raw(raw)
        assert rc == 0 and bad == -1
        loc, rem, send, recv, err = model(wrs, loc0, rem0)
        send.append((len(wrs), N.WC_WR_FLUSH_ERR if err else N.WC_SUCCESS, N.WC_RDMA_WRITE, 0))
        got = cq.wait(len(send) + len(recv), timeout=60)
        got_send = [(w.wr_id, w.status, w.opcode, w.byte_len) for w in got if w.opcode != N.WC_RECV_RDMA_WITH_IMM]
        got_recv = [(w.wr_id, w.byte_len, w.imm_data) for w in got
                    if w.opcode == N.WC_RECV_RDMA_WITH_IMM and w.status == N.WC_SUCCESS]
        torch.cuda.synchronize()
        assert got_send == send
        assert got_recv == recv
        assert np.array_equal(lt.cpu().numpy(), loc)
        assert np.array_equal(rt.cpu().numpy(), rem)
    finally:
        for q in (a, b):
            q.destroy()
        lm.dereg()
        rm.dereg()
        cq.destroy()
        pd.dealloc()
        ctx.close()
