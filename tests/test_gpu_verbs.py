"""GPU data path through the public verbs API: the sm_100a executor against byte-exact
expectations (the same checks the CPU engine passes in test_cpu_engine.py)."""
from __future__ import annotations

import pytest

from conftest import gpu_count

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def gpu_env():
    if gpu_count() < 1:
        pytest.skip("no GPU")
    from ugdr_b200 import verbs as V

    torch.cuda.set_device(0)
    d = V.Daemon(gpus=1)
    yield V
    d.stop()


def _setup(V, N, depth=256, max_sge=1, access=None):
    access = access or (N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ | N.ACCESS_REMOTE_ATOMIC)
    ctx = V.Context(V.find_device(gpu=0))
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(depth * 2)
    a = pd.create_qp(cq, max_send_wr=depth, max_send_sge=max_sge, max_recv_wr=depth)
    b = pd.create_qp(cq, max_send_wr=depth, max_send_sge=max_sge, max_recv_wr=depth)
    V.connect_pair(a, b, access=access)
    return ctx, pd, cq, a, b


ACC_ALL = None


def _acc(N):
    return N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ | N.ACCESS_REMOTE_ATOMIC


@pytest.mark.parametrize("size,soff,doff", [(8, 0, 0), (1, 3, 5), (4096, 0, 0), (4097, 1, 1),
                                            (65536, 16, 32), (1 << 20, 7, 3), ((32 << 20) + 5, 0, 16),
                                            ((1 << 20) + 3, 32, 0), (100003, 5, 37)])
def test_write_read_sizes(gpu_env, size, soff, doff):
    V = gpu_env
    from ugdr_b200 import _native as N

    ctx, pd, cq, a, b = _setup(V, N)
    n = size + 64
    g = torch.Generator(device="cuda").manual_seed(size)
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda", generator=g)
    dst = torch.zeros(n, dtype=torch.uint8, device="cuda")
    back = torch.zeros(n, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ms, md, mb = (pd.reg_mr(t.data_ptr(), n, _acc(N)) for t in (src, dst, back))
    a.post_write((src.data_ptr() + soff, size, ms.lkey), dst.data_ptr() + doff, md.rkey, wr_id=7)
    wc = cq.wait(1, 60)[0]
    assert (wc.status, wc.wr_id, wc.opcode, wc.byte_len) == (N.WC_SUCCESS, 7, N.WC_RDMA_WRITE, size)
    a.post_read((back.data_ptr() + soff, size, mb.lkey), dst.data_ptr() + doff, md.rkey, wr_id=8)
    wc = cq.wait(1, 60)[0]
    assert (wc.status, wc.opcode) == (N.WC_SUCCESS, N.WC_RDMA_READ)
    torch.cuda.synchronize()
    exp = torch.zeros_like(dst)
    exp[doff:doff + size] = src[soff:soff + size]
    assert torch.equal(dst, exp), "WRITE payload or guard bytes wrong"
    exp2 = torch.zeros_like(back)
    exp2[soff:soff + size] = src[soff:soff + size]
    assert torch.equal(back, exp2), "READ payload or guard bytes wrong"


def test_multi_sge_gather_and_imm(gpu_env):
    V = gpu_env
    from ugdr_b200 import _native as N

    ctx, pd, cq, a, b = _setup(V, N, max_sge=16)
    import random

    rng = random.Random(3)
    sizes = [int(2 ** rng.uniform(6, 16)) for _ in range(16)]
    total = sum(sizes)
    src = torch.randint(0, 256, (total + 4096 * 16,), dtype=torch.uint8, device="cuda")
    dst = torch.zeros(total + 256, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ms, md = pd.reg_mr(src.data_ptr(), src.numel(), _acc(N)), pd.reg_mr(dst.data_ptr(), dst.numel(), _acc(N))
    sges, off, pieces = [], 0, []
    for i, s in enumerate(sizes):
        sges.append((src.data_ptr() + off, s, ms.lkey))
        pieces.append(src[off:off + s])
        off += s + 4096
    b.post_recv(wr_id=555)
    a.post_send(N.WR_RDMA_WRITE_WITH_IMM, sges, remote_addr=dst.data_ptr() + 128, rkey=md.rkey,
                wr_id=9, imm=0xABCD1234)
    wcs = cq.wait(2, 60)
    by_op = {w.opcode: w for w in wcs}
    send, recv = by_op[N.WC_RDMA_WRITE], by_op[N.WC_RECV_RDMA_WITH_IMM]
    assert send.status == N.WC_SUCCESS and send.wr_id == 9
    assert recv.status == N.WC_SUCCESS and recv.wr_id == 555 and recv.byte_len == total
    assert recv.imm_data == 0xABCD1234 and recv.wc_flags & N.WC_WITH_IMM and recv.qp_num == b.qpn
    torch.cuda.synchronize()
    assert torch.equal(dst[128:128 + total], torch.cat(pieces))
    assert int(dst[:128].sum()) == 0 and int(dst[128 + total:].sum()) == 0


def test_atomics(gpu_env):
    V = gpu_env
    from ugdr_b200 import _native as N

    ctx, pd, cq, a, b = _setup(V, N)
    ctr = torch.zeros(4096, dtype=torch.int64, device="cuda")
    ctr[5] = 100
    old = torch.zeros(64, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    mc, mo = pd.reg_mr(ctr.data_ptr(), ctr.numel() * 8, _acc(N)), pd.reg_mr(old.data_ptr(), 512, _acc(N))
    for i in range(10):
        a.post_send(N.WR_ATOMIC_FETCH_AND_ADD, [(old.data_ptr() + 8 * i, 8, mo.lkey)],
                    remote_addr=ctr.data_ptr() + 40, rkey=mc.rkey, compare_add=3, wr_id=i)
    wcs = cq.wait(10, 60)
    assert all(w.status == N.WC_SUCCESS and w.opcode == N.WC_FETCH_ADD for w in wcs)
    torch.cuda.synchronize()
    assert int(ctr[5]) == 130
    assert old[:10].tolist() == [100 + 3 * i for i in range(10)]
    # compare-and-swap: succeeds once, then fails (value already swapped)
    for i, cmp in enumerate((130, 130)):
        a.post_send(N.WR_ATOMIC_CMP_AND_SWP, [(old.data_ptr() + 8 * (20 + i), 8, mo.lkey)],
                    remote_addr=ctr.data_ptr() + 40, rkey=mc.rkey, compare_add=cmp, swap=7, wr_id=50 + i)
    wcs = cq.wait(2, 60)
    assert all(w.status == N.WC_SUCCESS and w.opcode == N.WC_COMP_SWAP for w in wcs)
    torch.cuda.synchronize()
    assert int(ctr[5]) == 7 and old[20:22].tolist() == [130, 7]


def test_remote_access_error_and_flush(gpu_env):
    V = gpu_env
    from ugdr_b200 import _native as N

    ctx, pd, cq, a, b = _setup(V, N)
    src = torch.ones(4096, dtype=torch.uint8, device="cuda")
    dst = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ms = pd.reg_mr(src.data_ptr(), 4096, _acc(N))
    md = pd.reg_mr(dst.data_ptr(), 4096, N.ACCESS_LOCAL_WRITE)  # no remote write
    b.post_recv(wr_id=77)
    raw = [V.QueuePair.make_send_wr(N.WR_RDMA_WRITE, [(src.data_ptr(), 64, ms.lkey)], remote_addr=dst.data_ptr(),
                                    rkey=md.rkey, wr_id=1 + i, signaled=i == 0) for i in range(2)]
    assert a.post_send_raw(raw) == (0, -1)  # one chain: posting on a QP already in ERR is refused
    wcs = cq.wait(2, 60)
    assert wcs[0].wr_id == 1 and wcs[0].status == N.WC_REM_ACCESS_ERR
    assert wcs[1].wr_id == 2 and wcs[1].status == N.WC_WR_FLUSH_ERR
    attr, _ = a.query()
    assert attr.qp_state == N.QPS_ERR
    b.to_error()
    w = cq.wait(1, 60)[0]
    assert w.wr_id == 77 and w.status == N.WC_WR_FLUSH_ERR
    torch.cuda.synchronize()
    assert int(dst.sum()) == 0


def test_many_qps_queue_depth(gpu_env):
    V = gpu_env
    from ugdr_b200 import _native as N

    ctx = V.Context(V.find_device(gpu=0))
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(4096)
    qps = [pd.create_qp(cq, max_send_wr=64) for _ in range(32)]
    for i in range(0, 32, 2):
        V.connect_pair(qps[i], qps[i + 1])
    n = 1 << 16
    src = torch.randint(0, 256, (n * 16,), dtype=torch.uint8, device="cuda")
    dst = torch.zeros(n * 16 * 64, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ms, md = pd.reg_mr(src.data_ptr(), src.numel(), _acc(N)), pd.reg_mr(dst.data_ptr(), dst.numel(), _acc(N))
    k = 0
    for d in range(64):
        for q in range(0, 32, 2):
            qps[q].post_write((src.data_ptr() + (q // 2) * n, n, ms.lkey),
                              dst.data_ptr() + k * n, md.rkey, wr_id=k)
            k += 1
    wcs = cq.wait(k, 120)
    assert sorted(w.wr_id for w in wcs) == list(range(k))
    assert all(w.status == N.WC_SUCCESS for w in wcs)
    torch.cuda.synchronize()
    view = dst.view(k, n)
    for i in (0, 1, 17, k - 1):
        q = (i % 16)
        assert torch.equal(view[i], src[q * n:(q + 1) * n])


@pytest.fixture(scope="module")
def gpu2_env():
    if gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    from ugdr_b200 import verbs as V

    d = V.Daemon(gpus=2)
    yield V
    d.stop()


def test_cross_gpu_write_read_imm_atomics(gpu2_env):
    """Requester on GPU 0, responder memory / QP / CQ on GPU 1: the GPU 0 executor stores over
    NVLink into GPU 1 memory, consumes GPU 1's RQ and fills GPU 1's receive CQ."""
    V = gpu2_env
    from ugdr_b200 import _native as N

    acc = _acc(N)
    c0, c1 = V.Context(V.find_device(gpu=0)), V.Context(V.find_device(gpu=1))
    p0, p1 = c0.alloc_pd(), c1.alloc_pd()
    q0c, q1c = c0.create_cq(256), c1.create_cq(256)
    a = p0.create_qp(q0c, max_send_wr=64)
    b = p1.create_qp(q1c, max_send_wr=64)
    V.connect_pair(a, b, access=N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ | N.ACCESS_REMOTE_ATOMIC)
    n = (8 << 20) + 3
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda:0")
    back = torch.zeros(n, dtype=torch.uint8, device="cuda:0")
    dst = torch.zeros(n + 64, dtype=torch.uint8, device="cuda:1")
    ctr = torch.zeros(16, dtype=torch.int64, device="cuda:1")
    old = torch.zeros(16, dtype=torch.int64, device="cuda:0")
    torch.cuda.synchronize(0)
    torch.cuda.synchronize(1)
    ms, mb, mo = (p0.reg_mr(t.data_ptr(), t.numel() * t.element_size(), acc) for t in (src, back, old))
    md, mc = (p1.reg_mr(t.data_ptr(), t.numel() * t.element_size(), acc) for t in (dst, ctr))
    b.post_recv(wr_id=42)
    a.post_send(N.WR_RDMA_WRITE_WITH_IMM, [(src.data_ptr(), n, ms.lkey)], remote_addr=dst.data_ptr() + 32,
                rkey=md.rkey, wr_id=1, imm=7)
    w = q0c.wait(1, 60)[0]
    assert (w.status, w.wr_id, w.byte_len) == (N.WC_SUCCESS, 1, n)
    r = q1c.wait(1, 60)[0]
    assert (r.status, r.wr_id, r.opcode, r.imm_data, r.byte_len) == (N.WC_SUCCESS, 42, N.WC_RECV_RDMA_WITH_IMM, 7, n)
    a.post_read((back.data_ptr(), n, mb.lkey), dst.data_ptr() + 32, md.rkey, wr_id=2)
    assert q0c.wait(1, 60)[0].status == N.WC_SUCCESS
    for i in range(8):
        a.post_send(N.WR_ATOMIC_FETCH_AND_ADD, [(old.data_ptr() + 8 * i, 8, mo.lkey)],
                    remote_addr=ctr.data_ptr(), rkey=mc.rkey, compare_add=1 << i, wr_id=10 + i)
    assert all(x.status == N.WC_SUCCESS for x in q0c.wait(8, 60))
    torch.cuda.synchronize(0)
    torch.cuda.synchronize(1)
    assert torch.equal(dst[32:32 + n].cpu(), src.cpu()) and int(dst[:32].sum()) == 0
    assert int(dst[32 + n:].sum()) == 0
    assert torch.equal(back, src)
    assert int(ctr[0]) == 255 and sorted(old[:8].tolist()) == sorted([sum(1 << j for j in range(i)) for i in range(8)])


@pytest.mark.parametrize("dst_gpu", [0, 1])
def test_verbs_stress_16sge_imm_atomics(dst_gpu):
    """The verbs-feature stress workload at reduced size: per QP an interleave of 16-SGE WRITE / WRITE_WITH_IMM
    (SGE sizes log-uniform 64 B..64 KiB, random offsets) and fetch-add / compare-swap on a
    4096-entry counter array; ugdr_perf checks every gathered byte, immediate, CAS result and
    final counter value."""
    if gpu_count() < dst_gpu + 1:
        pytest.skip(f"needs {dst_gpu + 1} GPU(s)")
    from ugdr_b200.utils.perf import run

    out = run(["stress", "--src-gpu", "0", "--dst-gpu", str(dst_gpu), "--qps", "16", "--depth", "64",
               "--sges", "16", "--rounds", "2"], timeout=600)
    assert out and out[-1]["correct"], out


def test_copy_core_alignment_matrix():
    """The executor's warp copy core (reference parity: the copy-core alignment matrix of
    tests/integration/persistent_copy_test.cpp): every (source offset, destination offset, size)
    copies exactly its bytes - guard bytes on both sides of the destination stay untouched - for
    the byte, 4-byte, 16-byte and 32-byte bodies."""
    if gpu_count() < 1:
        pytest.skip("no GPU")
    import ctypes as C

    from ugdr_b200 import _native as N

    L = N.lib()
    L.ugdr_x_copy_core_test.restype = C.c_int
    L.ugdr_x_copy_core_test.argtypes = [C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p]
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(5)
    src = torch.randint(0, 256, (1 << 20,), dtype=torch.uint8, device="cuda", generator=g)
    dst = torch.empty((1 << 20) + 256, dtype=torch.uint8, device="cuda")
    sizes = [0, 1, 3, 15, 16, 17, 31, 32, 33, 63, 64, 65, 255, 4095, 4096, 4097, 4127, 65536 + 7, 300001]
    offs = [0, 1, 4, 15, 16, 17, 31, 32, 33]
    for n in sizes:
        for so in offs:
            for do in offs:
                dst.fill_(0xD3)
                base = 64 + do
                rc = L.ugdr_x_copy_core_test(C.c_void_p(dst.data_ptr() + base), C.c_void_p(src.data_ptr() + so), n,
                                             None)
                assert rc == 0
                torch.cuda.synchronize()
                assert torch.equal(dst[base:base + n], src[so:so + n]), (n, so, do)
                assert bool((dst[:base] == 0xD3).all()) and bool((dst[base + n:] == 0xD3).all()), (n, so, do)


def test_qp_stats_on_the_executor(gpu_env):
    """Per-QP counters kept by the executor: bytes of retired successful WRs (inline, lane-parallel
    and chunked sizes) and the error plus flush completions of a QP that went to ERR."""
    V = gpu_env
    from ugdr_b200 import _native as N

    ctx, pd, cq, a, b = _setup(V, N)
    n = 2 << 20
    src = torch.ones(n, dtype=torch.uint8, device="cuda")
    dst = torch.zeros(n, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ms, md = pd.reg_mr(src.data_ptr(), n, _acc(N)), pd.reg_mr(dst.data_ptr(), n, _acc(N))
    sizes = [8, 100, 4097, 65536, 1 << 20]
    for i, sz in enumerate(sizes):
        a.post_write((src.data_ptr(), sz, ms.lkey), dst.data_ptr(), md.rkey, wr_id=i)
    assert all(w.status == N.WC_SUCCESS for w in cq.wait(len(sizes), 60))
    st = a.stats()
    assert (st.send_posted, st.send_retired, st.bytes, st.error_completions) == (5, 5, sum(sizes), 0)
    raw = [V.QueuePair.make_send_wr(N.WR_RDMA_WRITE, [(src.data_ptr(), 64, ms.lkey)], remote_addr=dst.data_ptr(),
                                    rkey=md.rkey ^ (2 if i == 0 else 0), wr_id=10 + i) for i in range(2)]
    assert a.post_send_raw(raw) == (0, -1)  # one chain: posting on a QP already in ERR is refused
    wcs = cq.wait(2, 60)
    assert [w.status for w in wcs] == [N.WC_REM_ACCESS_ERR, N.WC_WR_FLUSH_ERR]
    st = a.stats()
    assert (st.send_retired, st.bytes, st.error_completions, st.state) == (7, sum(sizes), 2, N.QPS_ERR)


def test_mr_deregistration_keeps_the_executor_running(gpu_env):
    """Deregistering an MR that no in-flight WR uses finishes by a grace period while another QP
    keeps streaming: the executor is not stopped (no extra launch), the stream's bytes are right,
    and the engine counts the deregistrations as live ones."""
    V = gpu_env
    import gc

    from ugdr_b200 import _native as N

    # Objects of earlier tests on this daemon are released now, not mid-test: destroying a QP or
    # a CQ still stops the executor, which would show up as a relaunch below.
    gc.collect()
    ctx, pd, cq, a, b = _setup(V, N, depth=512)
    n = 64 << 20
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    dst = torch.zeros(n, dtype=torch.uint8, device="cuda")
    spare = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ms, md = pd.reg_mr(src.data_ptr(), n, _acc(N)), pd.reg_mr(dst.data_ptr(), n, _acc(N))
    a.post_write((src.data_ptr(), 4096, ms.lkey), dst.data_ptr(), md.rkey, wr_id=0)
    assert cq.wait(1, 60)[0].status == N.WC_SUCCESS  # the executor is up
    st0 = ctx.stats()
    chunk = 1 << 20
    posted = 0
    done = 0
    deregs = 0
    while done < 256:
        while posted < 256 and posted - done < 64:
            off = (posted % 64) * chunk
            a.post_write((src.data_ptr() + off, chunk, ms.lkey), dst.data_ptr() + off, md.rkey, wr_id=posted)
            posted += 1
        if deregs < 8:  # an unrelated MR comes and goes under the stream
            pd.reg_mr(spare.data_ptr(), spare.numel(), _acc(N)).dereg()
            deregs += 1
        wcs = cq.wait(1, 60)
        assert all(w.status == N.WC_SUCCESS for w in wcs)
        done += len(wcs)
    st1 = ctx.stats()
    torch.cuda.synchronize()
    assert torch.equal(dst, src)
    assert st1.mr_detach_live - st0.mr_detach_live == deregs, (st0.mr_detach_live, st1.mr_detach_live)
    assert st1.mr_detach_quiesced == st0.mr_detach_quiesced
    assert st1.launches == st0.launches  # never stopped and relaunched
    for q in (a, b):
        q.destroy()
    ms.dereg()
    md.dereg()
    cq.destroy()
    pd.dealloc()
    ctx.close()


def test_qp_and_cq_destruction_keeps_the_executor_running(gpu_env):
    """QPs and CQs created, used and destroyed while another QP streams: the executor is never
    stopped (no relaunch), every short-lived pair's WRs complete correctly, and the stream's bytes
    are right.  The destroyed objects' rings and slots are released once the executor is idle."""
    V = gpu_env
    import gc

    from ugdr_b200 import _native as N

    gc.collect()
    ctx, pd, cq, a, b = _setup(V, N, depth=512)
    n = 64 << 20
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    dst = torch.zeros(n, dtype=torch.uint8, device="cuda")
    small = torch.randint(0, 256, (1 << 16,), dtype=torch.uint8, device="cuda")
    small_dst = torch.zeros_like(small)
    torch.cuda.synchronize()
    ms, md = pd.reg_mr(src.data_ptr(), n, _acc(N)), pd.reg_mr(dst.data_ptr(), n, _acc(N))
    ss, sd = pd.reg_mr(small.data_ptr(), small.numel(), _acc(N)), pd.reg_mr(small_dst.data_ptr(), small.numel(), _acc(N))
    a.post_write((src.data_ptr(), 4096, ms.lkey), dst.data_ptr(), md.rkey, wr_id=0)
    assert cq.wait(1, 60)[0].status == N.WC_SUCCESS  # the executor is up
    st0 = ctx.stats()
    chunk = 1 << 20
    posted = done = cycles = 0
    while done < 256:
        while posted < 256 and posted - done < 64:
            off = (posted % 64) * chunk
            a.post_write((src.data_ptr() + off, chunk, ms.lkey), dst.data_ptr() + off, md.rkey, wr_id=posted)
            posted += 1
        if cycles < 6:  # a short-lived pair with its own CQ comes and goes under the stream
            cq2 = ctx.create_cq(64)
            c = pd.create_qp(cq2, max_send_wr=16, max_recv_wr=16)
            d = pd.create_qp(cq2, max_send_wr=16, max_recv_wr=16)
            V.connect_pair(c, d, access=N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ)
            k = 4096 * (cycles + 1)
            c.post_write((small.data_ptr(), k, ss.lkey), small_dst.data_ptr(), sd.rkey, wr_id=1000 + cycles)
            wc = cq2.wait(1, 60)[0]
            assert (wc.wr_id, wc.status) == (1000 + cycles, N.WC_SUCCESS), wc
            torch.cuda.synchronize()
            assert torch.equal(small_dst[:k], small[:k])
            c.destroy()
            d.destroy()
            cq2.destroy()
            cycles += 1
        wcs = cq.wait(1, 60)
        assert all(w.status == N.WC_SUCCESS for w in wcs)
        done += len(wcs)
    st1 = ctx.stats()
    torch.cuda.synchronize()
    assert cycles == 6
    assert torch.equal(dst, src)
    assert st1.launches == st0.launches, (st0.launches, st1.launches)  # never stopped and relaunched
    for q in (a, b):
        q.destroy()
    for m in (ms, md, ss, sd):
        m.dereg()
    cq.destroy()
    pd.dealloc()
    ctx.close()


def test_cross_gpu_qp_destruction_keeps_both_executors_running(gpu2_env):
    """A cross-GPU pair (requester on GPU 0, responder on GPU 1, WRITE_WITH_IMM into GPU 1's RQ and
    receive CQ) is created, used and destroyed six times while a GPU 0 loopback stream runs.  The
    responder's destruction unbinds the GPU 0 requester while GPU 0's executor runs and waits for
    its grace period: neither executor is stopped, and every byte and completion is right."""
    V = gpu2_env
    import gc

    from ugdr_b200 import _native as N

    gc.collect()
    acc = _acc(N)
    c0, c1 = V.Context(V.find_device(gpu=0)), V.Context(V.find_device(gpu=1))
    p0, p1 = c0.alloc_pd(), c1.alloc_pd()
    cq0 = c0.create_cq(1024)
    a = p0.create_qp(cq0, max_send_wr=512)
    b = p0.create_qp(cq0, max_send_wr=512)
    V.connect_pair(a, b, access=N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ)
    n = 64 << 20
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda:0")
    dst = torch.zeros(n, dtype=torch.uint8, device="cuda:0")
    small = torch.randint(0, 256, (1 << 16,), dtype=torch.uint8, device="cuda:0")
    far = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda:1")
    torch.cuda.synchronize(0)
    torch.cuda.synchronize(1)
    ms, md, ss = (p0.reg_mr(t.data_ptr(), t.numel(), acc) for t in (src, dst, small))
    mf = p1.reg_mr(far.data_ptr(), far.numel(), acc)
    a.post_write((src.data_ptr(), 4096, ms.lkey), dst.data_ptr(), md.rkey, wr_id=0)
    assert cq0.wait(1, 60)[0].status == N.WC_SUCCESS  # GPU 0's executor is up
    cqx, cqy = c0.create_cq(64), c1.create_cq(64)
    x0 = p0.create_qp(cqx, max_send_wr=16)
    y0 = p1.create_qp(cqy, max_send_wr=16)
    V.connect_pair(x0, y0, access=N.ACCESS_REMOTE_WRITE)
    y0.post_recv(wr_id=7)
    x0.post_send(N.WR_RDMA_WRITE_WITH_IMM, [(small.data_ptr(), 4096, ss.lkey)], remote_addr=far.data_ptr(),
                 rkey=mf.rkey, wr_id=7, imm=7)
    assert cqx.wait(1, 60)[0].status == N.WC_SUCCESS and cqy.wait(1, 60)[0].status == N.WC_SUCCESS  # GPU 1's too
    s0, s1 = c0.stats(), c1.stats()
    chunk = 1 << 20
    posted = done = cycles = 0
    while done < 256:
        while posted < 256 and posted - done < 64:
            off = (posted % 64) * chunk
            a.post_write((src.data_ptr() + off, chunk, ms.lkey), dst.data_ptr() + off, md.rkey, wr_id=posted)
            posted += 1
        if cycles < 6:
            x = p0.create_qp(cqx, max_send_wr=16)
            y = p1.create_qp(cqy, max_send_wr=16)
            V.connect_pair(x, y, access=N.ACCESS_REMOTE_WRITE)
            k = 4096 * (cycles + 1)
            y.post_recv(wr_id=100 + cycles)
            x.post_send(N.WR_RDMA_WRITE_WITH_IMM, [(small.data_ptr(), k, ss.lkey)], remote_addr=far.data_ptr(),
                        rkey=mf.rkey, wr_id=100 + cycles, imm=cycles)
            w = cqx.wait(1, 60)[0]
            r = cqy.wait(1, 60)[0]
            assert (w.wr_id, w.status) == (100 + cycles, N.WC_SUCCESS), w
            assert (r.wr_id, r.status, r.imm_data, r.byte_len) == (100 + cycles, N.WC_SUCCESS, cycles, k), r
            torch.cuda.synchronize(1)
            assert torch.equal(far[:k].cpu(), small[:k].cpu())
            y.destroy()  # the responder first: its GPU 0 requester is unbound live
            x.destroy()
            cycles += 1
        wcs = cq0.wait(1, 60)
        assert all(wc.status == N.WC_SUCCESS for wc in wcs)
        done += len(wcs)
    t0, t1 = c0.stats(), c1.stats()
    torch.cuda.synchronize(0)
    assert cycles == 6
    assert torch.equal(dst, src)
    assert (t0.launches, t1.launches) == (s0.launches, s1.launches), (s0.launches, t0.launches, s1.launches, t1.launches)
    for q in (a, b, x0, y0):
        q.destroy()
    for m in (ms, md, ss, mf):
        m.dereg()
    for c in (cq0, cqx, cqy):
        c.destroy()
    p0.dealloc()
    p1.dealloc()
    c0.close()
    c1.close()


def test_kernel_attributes_report_every_kernel():
    """cudaFuncGetAttributes + occupancy for every kernel of the library: each fits its launch
    block size; the persistent executor keeps one 256-thread CTA (8 warps) per SM, whose register
    budget (up to 255 per thread) holds its state without spilling."""
    if gpu_count() < 1:
        pytest.skip("no GPU")
    from ugdr_b200 import ops

    torch.cuda.set_device(0)
    attrs = {a["name"]: a for a in ops.kernel_attributes()}
    assert {"executor_kernel", "allreduce_nvls_kernel<4>", "dispatch_kernel", "combine_kernel<8>"} <= set(attrs)
    for a in attrs.values():
        assert a["blocks_per_sm"] >= 1 and a["threads_per_block"] <= a["max_threads_per_block"], a
    ex = attrs["executor_kernel"]
    assert ex["threads_per_block"] == 256 and ex["registers_per_thread"] <= 255 and ex["blocks_per_sm"] == 1, ex
