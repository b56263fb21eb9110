"""Device trace of the executor (ugdr_x_engine_trace / _dump): events recorded in the kernel with
%globaltimer stamps, written by the daemon as Chrome trace-event JSON.

Marked gpu_extended (run with `pytest -m gpu_extended` on a B200 box) until it has run there.
"""
from __future__ import annotations

import json

import pytest

from conftest import gpu_count

torch = pytest.importorskip("torch")

from ugdr_b200 import _native as N  # noqa: E402
from ugdr_b200 import verbs as V  # noqa: E402

pytestmark = pytest.mark.gpu_extended

ACC = N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ


def test_trace_records_batches_and_chunks(tmp_path):
    if gpu_count() < 1:
        pytest.skip("no GPU")
    torch.cuda.set_device(0)
    with V.Daemon(gpus=1):
        ctx = V.Context(V.find_device(gpu=0))
        pd = ctx.alloc_pd()
        cq = ctx.create_cq(512)
        a = pd.create_qp(cq, max_send_wr=256, max_recv_wr=16)
        b = pd.create_qp(cq, max_send_wr=256, max_recv_wr=16)
        V.connect_pair(a, b, access=N.ACCESS_REMOTE_WRITE)
        n = 8 << 20
        src = torch.ones(n, dtype=torch.uint8, device="cuda")
        dst = torch.zeros(n, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        ms, md = pd.reg_mr(src.data_ptr(), n, ACC), pd.reg_mr(dst.data_ptr(), n, ACC)
        ctx.trace(4096)
        for i in range(64):
            a.post_write((src.data_ptr(), 256, ms.lkey), dst.data_ptr() + 256 * i, md.rkey, wr_id=i)
        a.post_write((src.data_ptr(), n, ms.lkey), dst.data_ptr(), md.rkey, wr_id=99)
        assert all(w.status == N.WC_SUCCESS for w in cq.wait(65, 60))
        path = tmp_path / "trace.json"
        kept, dropped = ctx.trace_dump(str(path))
        ctx.trace(0)
        doc = json.loads(path.read_text())
        ev = doc["traceEvents"]
        assert kept == len(ev) and kept > 0 and dropped == 0
        names = {e["name"] for e in ev}
        assert "chunk" in names and ({"fast_batch", "retire"} & names)
        assert all(e["dur"] >= 0 and e["ts"] >= 0 for e in ev)
        # Every WR above 64 B is copied in chunks: the 64 small ones and the large one.
        assert sum(e["args"]["value"] for e in ev if e["name"] == "chunk") == n + 64 * 256
        with pytest.raises(V.UgdrError):  # off again: nothing to dump
            ctx.trace_dump(str(path))
