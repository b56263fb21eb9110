"""UGDR_X_WR_RDMA_WRITE_SUM_BF16: an RDMA WRITE of the elementwise bf16 sum of the WR's SGEs.

The same checks run on the host engine (CPU, host memory) and on the sm_100a executor (GPU
memory, marked gpu): results against an fp32 torch sum rounded to bf16, in place and out of
place, inline (<= 4 KiB) and chunked sizes, 16-byte aligned and 2-byte aligned addresses, and
the error completions of malformed WRs.  Guard bytes around every destination stay untouched.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import gpu_count
from ugdr_b200 import _native as N
from ugdr_b200 import verbs as V

ACC = N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ
SUM = N.WR_X_RDMA_WRITE_SUM_BF16
GUARD = 64


def _expected(srcs: list[np.ndarray]) -> np.ndarray:
    """bf16 of the fp32 sum in SGE order (numpy bf16 words in, words out)."""
    acc = torch.zeros(srcs[0].size, dtype=torch.float32)
    for s in srcs:
        acc += torch.from_numpy(s.astype(np.int16)).view(torch.bfloat16).float()
    return acc.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)


class Mem:
    """One registered byte region, in host memory (host engine) or on a GPU (executor)."""

    def __init__(self, pd, nbytes: int, gpu: bool):
        self.gpu = gpu
        if gpu:
            self.t = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
            torch.cuda.synchronize()
            self.addr = self.t.data_ptr()
            self.hb = None
        else:
            self.hb = V.HostBuffer(nbytes)
            self.addr = self.hb.addr
            self.hb.view()[:] = 0
        self.mr = pd.reg_mr(self.addr, nbytes, ACC)

    def write(self, off: int, data: np.ndarray) -> None:
        b = data.view(np.uint8)
        if self.gpu:
            self.t[off:off + b.size].copy_(torch.from_numpy(b.copy()))
            torch.cuda.synchronize()
        else:
            self.hb.view()[off:off + b.size] = b

    def read(self, off: int, n: int) -> np.ndarray:
        if self.gpu:
            torch.cuda.synchronize()
            return self.t[off:off + n].cpu().numpy().copy()
        return self.hb.view()[off:off + n].copy()

    def close(self) -> None:
        self.mr.dereg()
        if self.hb is not None:
            self.hb.free()


def _run(ctx, gpu: bool) -> None:
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(256)
    a = pd.create_qp(cq, max_send_wr=64, max_recv_wr=16, max_send_sge=8)
    b = pd.create_qp(cq, max_send_wr=64, max_recv_wr=16, max_send_sge=8)
    V.connect_pair(a, b, access=N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ)
    rng = np.random.default_rng(7)
    big = 3 << 20
    src = Mem(pd, 8 * big + 4096, gpu)
    dst = Mem(pd, big + 2 * GUARD + 4096, gpu)
    try:
        cases = [  # (elements, number of SGEs, source misalignment in bytes, destination misalignment)
            (8, 1, 0, 0), (1000, 3, 0, 0), (2048, 8, 0, 0),  # inline
            (big // 2, 4, 0, 0), (big // 2, 7, 0, 0),  # chunked
            (40000, 2, 2, 6), (3, 5, 2, 0),  # 2-byte aligned only
        ]
        for i, (ne, k, smis, dmis) in enumerate(cases):
            nb = 2 * ne
            words = [rng.normal(size=ne).astype(np.float32) for _ in range(k)]
            srcs = [torch.from_numpy(w).to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16) for w in words]
            offs = [j * (nb + 4096) // 4096 * 4096 + smis for j in range(k)]
            for o, s in zip(offs, srcs):
                src.write(o, s)
            guard = rng.integers(0, 256, nb + 2 * GUARD, dtype=np.uint8)
            dst.write(dmis, guard)
            sges = [(src.addr + o, nb, src.mr.lkey) for o in offs]
            a.post_send(SUM, sges, remote_addr=dst.addr + dmis + GUARD, rkey=dst.mr.rkey, wr_id=i)
            wc = cq.wait(1, timeout=60)[0]
            assert (wc.wr_id, wc.status, wc.opcode, wc.byte_len) == (i, N.WC_SUCCESS, N.WC_RDMA_WRITE, nb), (i, wc)
            got = dst.read(dmis, nb + 2 * GUARD)
            assert np.array_equal(got[:GUARD], guard[:GUARD]) and np.array_equal(got[GUARD + nb:], guard[GUARD + nb:])
            assert np.array_equal(got[GUARD:GUARD + nb].view(np.uint16), _expected(srcs)), f"case {i}"

        # In place: the destination is the first SGE.
        ne = 300000
        srcs = [torch.randn(ne).to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16) for _ in range(3)]
        offs = [0, 1 << 20, 2 << 20]
        for o, s in zip(offs, srcs):
            src.write(o, s)
        a.post_send(SUM, [(src.addr + o, 2 * ne, src.mr.lkey) for o in offs], remote_addr=src.addr, rkey=src.mr.rkey,
                    wr_id=50)
        assert cq.wait(1, timeout=60)[0].status == N.WC_SUCCESS
        assert np.array_equal(src.read(0, 2 * ne).view(np.uint16), _expected(srcs))

        # Malformed WRs: each completes in error and moves the QP to ERR, so use fresh pairs.
        bad = [
            ([(src.addr, 64, src.mr.lkey), (src.addr + 4096, 66, src.mr.lkey)], dst.addr, N.WC_LOC_LEN_ERR),
            ([(src.addr, 63, src.mr.lkey), (src.addr + 4096, 63, src.mr.lkey)], dst.addr, N.WC_LOC_LEN_ERR),
            ([(src.addr + 1, 64, src.mr.lkey)], dst.addr, N.WC_LOC_PROT_ERR),
            ([(src.addr, 64, src.mr.lkey)], dst.addr + 1, N.WC_REM_INV_REQ_ERR),
        ]
        for j, (sges, raddr, want) in enumerate(bad):
            c = pd.create_qp(cq, max_send_wr=8, max_recv_wr=8, max_send_sge=8)
            d = pd.create_qp(cq, max_send_wr=8, max_recv_wr=8, max_send_sge=8)
            V.connect_pair(c, d, access=N.ACCESS_REMOTE_WRITE)
            c.post_send(SUM, sges, remote_addr=raddr, rkey=dst.mr.rkey, wr_id=100 + j)
            wc = cq.wait(1, timeout=60)[0]
            assert (wc.wr_id, wc.status) == (100 + j, want), wc
            c.destroy()
            d.destroy()
    finally:
        for q in (a, b):
            q.destroy()
        src.close()
        dst.close()
        cq.destroy()
        pd.dealloc()


def test_write_sum_on_the_host_engine(cpu_daemon):
    ctx = V.Context(V.find_device(kind=0))
    try:
        _run(ctx, gpu=False)
    finally:
        ctx.close()


@pytest.mark.gpu
def test_write_sum_on_the_executor():
    if gpu_count() < 1:
        pytest.skip("no GPU")
    torch.cuda.set_device(0)
    with V.Daemon(gpus=1):
        ctx = V.Context(V.find_device(gpu=0))
        try:
            _run(ctx, gpu=True)
        finally:
            ctx.close()
