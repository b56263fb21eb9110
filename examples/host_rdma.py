"""A ugdr client in Python over the daemon's host-memory engine (no GPU needed): WRITE with three
SGEs gathered into one remote range, WRITE_WITH_IMM consuming a posted receive, and FETCH_ADD.

    python examples/host_rdma.py

The same calls work on GPU memory: register torch CUDA tensors (tensor.data_ptr()) on a context
of a GPU device (V.find_device(gpu=0)), and start the daemon with gpus=N.
"""
from __future__ import annotations

import os
import struct
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from ugdr_b200 import _native as N  # noqa: E402
from ugdr_b200 import verbs as V  # noqa: E402


def main() -> int:
    with V.Daemon(gpus=0):
        ctx = V.Context(V.find_device(kind=0))
        pd = ctx.alloc_pd()
        cq = ctx.create_cq(64)
        a = pd.create_qp(cq, max_send_sge=4)
        b = pd.create_qp(cq, max_recv_wr=16)
        V.connect_pair(a, b, access=N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_ATOMIC)
        buf = V.HostBuffer(1 << 16)
        mem = buf.view()  # numpy uint8 view of the buffer

        def put(off: int, data: bytes) -> None:
            mem[off:off + len(data)] = np.frombuffer(data, dtype=np.uint8)

        mr = pd.reg_mr(buf.addr, buf.length, N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_ATOMIC)

        # Gather three pieces into [8192, 8192 + 9).
        put(0, b"abc")
        put(100, b"def")
        put(200, b"ghi")
        pieces = [(buf.addr, 3, mr.lkey), (buf.addr + 100, 3, mr.lkey), (buf.addr + 200, 3, mr.lkey)]
        a.post_send(N.WR_RDMA_WRITE, pieces, remote_addr=buf.addr + 8192, rkey=mr.rkey, wr_id=1)
        assert cq.wait(1)[0].status == N.WC_SUCCESS
        assert bytes(mem[8192:8201]) == b"abcdefghi"

        # WRITE_WITH_IMM: the responder's receive completes with the immediate.
        b.post_recv(wr_id=77)
        a.post_send(N.WR_RDMA_WRITE_WITH_IMM, [(buf.addr, 3, mr.lkey)], remote_addr=buf.addr + 9000,
                    rkey=mr.rkey, wr_id=2, imm=0xC0FFEE)
        wcs = {w.wr_id: w for w in cq.wait(2)}
        assert wcs[77].opcode == N.WC_RECV_RDMA_WITH_IMM and wcs[77].imm_data == 0xC0FFEE

        # FETCH_ADD on an 8-byte counter; the old value lands in the local SGE.
        put(12288, struct.pack("<Q", 40))
        a.post_send(N.WR_ATOMIC_FETCH_AND_ADD, [(buf.addr + 12296, 8, mr.lkey)], remote_addr=buf.addr + 12288,
                    rkey=mr.rkey, wr_id=3, compare_add=2)
        assert cq.wait(1)[0].status == N.WC_SUCCESS
        assert struct.unpack("<QQ", bytes(mem[12288:12304])) == (42, 40)

        for q in (a, b):
            q.destroy()
        mr.dereg()
        cq.destroy()
        pd.dealloc()
        ctx.close()
        buf.free()
    print("gather WRITE, WRITE_WITH_IMM and FETCH_ADD ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
