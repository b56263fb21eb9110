"""Public verbs API end to end against a real ugdr_daemon process, host-memory engine only (no
GPU).  Mirrors the reference's integration suite (tests/integration/*_client_server_test.cpp,
control_plane_acceptance_test.cpp) and adds the data path the reference only runs on a GPU."""
from __future__ import annotations

import ctypes as C
import errno
import multiprocessing as mp
import os
import random
import time

import numpy as np
import pytest

from ugdr_b200 import _native as N
from ugdr_b200 import verbs as V

ACC = N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ | N.ACCESS_REMOTE_ATOMIC
REMOTE = N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ | N.ACCESS_REMOTE_ATOMIC


def _pair(depth=128, max_sge=4, rnr_retry=7, min_rnr_timer=1, cq_depth=512):
    ctx = V.Context(V.find_device(kind=0))
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(cq_depth)
    a = pd.create_qp(cq, max_send_wr=depth, max_recv_wr=depth, max_send_sge=max_sge, max_recv_sge=max_sge)
    b = pd.create_qp(cq, max_send_wr=depth, max_recv_wr=depth, max_send_sge=max_sge, max_recv_sge=max_sge)
    V.connect_pair(a, b, access=REMOTE, rnr_retry=rnr_retry, min_rnr_timer=min_rnr_timer)
    return ctx, pd, cq, a, b


def test_config0_cpu_plumbing_10k_writes(cpu_daemon):
    """CPU-only plumbing workload: 1 PD, 2 host MRs of 1 MiB, 1 QP of depth 128, 10,000 RDMA_WRITEs of
    4 KiB at seeded random 4 KiB-aligned offsets, payload uniform uint8 from seed 0."""
    ctx, pd, cq, a, b = _pair(depth=128, cq_depth=256)
    n = 1 << 20
    src, dst = V.HostBuffer(n), V.HostBuffer(n)
    sv, dv = src.view(), dst.view()
    sv[:] = np.random.default_rng(0).integers(0, 256, n, dtype=np.uint8)
    ms, md = pd.reg_mr(src.addr, n, ACC), pd.reg_mr(dst.addr, n, ACC)
    rng = random.Random(0)
    expect = np.zeros(n, dtype=np.uint8)
    done, posted, total = 0, 0, 10_000
    t0 = time.perf_counter()
    while done < total:
        while posted < total and posted - done < 128:
            so, do = rng.randrange(256) * 4096, rng.randrange(256) * 4096
            a.post_write((src.addr + so, 4096, ms.lkey), dst.addr + do, md.rkey, wr_id=posted)
            expect[do:do + 4096] = sv[so:so + 4096]
            posted += 1
        for w in cq.poll():
            assert w.status == N.WC_SUCCESS and w.wr_id == done
            done += 1
    dt = time.perf_counter() - t0
    assert np.array_equal(dv, expect)
    print(f"config0: {total} x 4 KiB WRITEs in {dt * 1e3:.1f} ms ({total / dt / 1e6:.3f} MWR/s)")


def test_a_polled_completion_frees_its_send_slot(cpu_daemon):
    """A full SQ: once a completion has been polled, the next post must find its slot free at once
    (the engine returns the SQ slot before it publishes the CQE, as an HCA retires a WQE first)."""
    ctx, pd, cq, a, b = _pair(depth=4, cq_depth=64)
    buf = V.HostBuffer(1 << 16)
    mr = pd.reg_mr(buf.addr, 1 << 16, ACC)
    try:
        posted = done = 0
        while posted < 4:  # fill the SQ
            a.post_write((buf.addr, 8, mr.lkey), buf.addr + 4096, mr.rkey, wr_id=posted)
            posted += 1
        while done < 2000:
            got = cq.wait(1, timeout=10)
            assert got and all(w.status == N.WC_SUCCESS for w in got)
            done += len(got)
            for _ in got:  # every polled completion is a slot that must take a new WR at once
                a.post_write((buf.addr, 8, mr.lkey), buf.addr + 4096, mr.rkey, wr_id=posted)
                posted += 1
        assert len(cq.wait(posted - done, timeout=10)) == posted - done
    finally:
        a.destroy()
        b.destroy()
        mr.dereg()
        cq.destroy()
        pd.dealloc()
        ctx.close()
        buf.free()


def test_qp_stats_count_wrs_bytes_rnr_and_errors(cpu_daemon):
    """ugdr_x_query_qp_stats: ring cursors, payload bytes, one RNR wait episode, and the error plus
    flush completions of a QP that went to ERR."""
    ctx, pd, cq, a, b = _pair(depth=32, cq_depth=128)  # rnr_retry 7: wait for a receive forever
    buf = V.HostBuffer(1 << 16)
    mr = pd.reg_mr(buf.addr, 1 << 16, ACC)
    try:
        for i in range(10):
            a.post_write((buf.addr, 100, mr.lkey), buf.addr + 4096, mr.rkey, wr_id=i)
        assert len(cq.wait(10, timeout=10)) == 10
        st = a.stats()
        assert (st.send_posted, st.send_retired, st.bytes, st.error_completions) == (10, 10, 1000, 0)
        assert st.state == N.QPS_RTS
        a.post_send(N.WR_RDMA_WRITE_WITH_IMM, [(buf.addr, 64, mr.lkey)], remote_addr=buf.addr + 8192, rkey=mr.rkey,
                    wr_id=50, imm=7)
        deadline = time.time() + 10
        while a.stats().rnr_waits == 0 and time.time() < deadline:
            time.sleep(0.001)
        assert a.stats().rnr_waits == 1 and a.stats().send_retired == 10
        b.post_recv(900)
        got = cq.wait(2, timeout=10)
        assert sorted(w.wr_id for w in got) == [50, 900]
        sa, sb = a.stats(), b.stats()
        assert (sa.send_retired, sa.bytes, sa.rnr_waits) == (11, 1064, 1)
        assert (sb.recv_posted, sb.recv_consumed, sb.send_posted) == (1, 1, 0)
        # A bad lkey moves the QP to ERR; the two WRs behind it (same chain: posting on an ERR QP
        # is refused) are flushed.
        raw = [V.QueuePair.make_send_wr(N.WR_RDMA_WRITE, [(buf.addr, 8, mr.lkey ^ (2 if i == 0 else 0))],
                                        remote_addr=buf.addr, rkey=mr.rkey, wr_id=60 + i) for i in range(3)]
        assert a.post_send_raw(raw) == (0, -1)
        got = cq.wait(3, timeout=10)
        assert [w.status for w in got] == [N.WC_LOC_PROT_ERR, N.WC_WR_FLUSH_ERR, N.WC_WR_FLUSH_ERR]
        sa = a.stats()
        assert (sa.send_posted, sa.send_retired, sa.error_completions, sa.bytes) == (14, 14, 3, 1064)
        assert sa.state == N.QPS_ERR
    finally:
        a.destroy()
        b.destroy()
        mr.dereg()
        cq.destroy()
        pd.dealloc()
        ctx.close()
        buf.free()


def test_engine_trace_is_a_gpu_feature(cpu_daemon):
    """The device trace exists on GPU contexts only: the host-memory device answers EOPNOTSUPP."""
    import errno

    ctx = V.Context(V.find_device(kind=0))
    try:
        for call in (lambda: ctx.trace(16), lambda: ctx.trace_dump("/nonexistent/trace.json")):
            with pytest.raises(V.UgdrError) as e:
                call()
            assert e.value.errno == errno.EOPNOTSUPP
    finally:
        ctx.close()


def test_poll_cq_wait_returns_on_count_or_timeout(cpu_daemon):
    """ugdr_x_poll_cq_wait: returns as soon as the minimum is there, or with what it has once the
    timeout passes; CompletionQueue.wait raises TimeoutError past its own deadline."""
    ctx, pd, cq, a, b = _pair(depth=16, cq_depth=64)
    buf = V.HostBuffer(8192)
    mr = pd.reg_mr(buf.addr, 8192, ACC)
    try:
        wc = (N.Wc * 8)()
        t0 = time.perf_counter()
        assert N.lib().ugdr_x_poll_cq_wait(cq.h, 1, 8, wc, 5_000_000) == 0
        assert time.perf_counter() - t0 >= 0.004
        assert N.lib().ugdr_x_poll_cq_wait(cq.h, 2, 1, wc, 0) == -errno.EINVAL
        for i in range(3):
            a.post_write((buf.addr, 8, mr.lkey), buf.addr + 4096, mr.rkey, wr_id=i)
        got = N.lib().ugdr_x_poll_cq_wait(cq.h, 3, 8, wc, 10_000_000_000)
        assert got == 3 and [wc[i].wr_id for i in range(3)] == [0, 1, 2]
        with pytest.raises(TimeoutError):
            cq.wait(1, timeout=0.05)
    finally:
        a.destroy()
        b.destroy()
        mr.dereg()
        cq.destroy()
        pd.dealloc()
        ctx.close()
        buf.free()


def test_write_with_imm_consumes_rq_in_order(cpu_daemon):
    ctx, pd, cq, a, b = _pair()
    buf = V.HostBuffer(1 << 16)
    m = pd.reg_mr(buf.addr, 1 << 16, ACC)
    for i in range(3):
        b.post_recv(wr_id=100 + i)
    for i in range(3):
        a.post_send(N.WR_RDMA_WRITE_WITH_IMM, [(buf.addr, 64 * (i + 1), m.lkey)], remote_addr=buf.addr + 4096,
                    rkey=m.rkey, wr_id=i, imm=0x10 + i, signaled=(i != 1))
    wcs = cq.wait(5, 10)
    recv = [w for w in wcs if w.opcode == N.WC_RECV_RDMA_WITH_IMM]
    send = [w for w in wcs if w.opcode == N.WC_RDMA_WRITE]
    assert [w.wr_id for w in recv] == [100, 101, 102]
    assert [w.imm_data for w in recv] == [0x10, 0x11, 0x12]
    assert [w.byte_len for w in recv] == [64, 128, 192]
    assert all(w.wc_flags & N.WC_WITH_IMM and w.qp_num == b.qpn for w in recv)
    assert [w.wr_id for w in send] == [0, 2]  # the unsignaled WR produces no send completion


def test_rnr_retry_exhausted(cpu_daemon):
    ctx, pd, cq, a, b = _pair(rnr_retry=2, min_rnr_timer=1)  # 10 us timer, 2 retries
    buf = V.HostBuffer(8192)
    m = pd.reg_mr(buf.addr, 8192, ACC)
    a.post_send(N.WR_RDMA_WRITE_WITH_IMM, [(buf.addr, 8, m.lkey)], remote_addr=buf.addr + 64, rkey=m.rkey,
                wr_id=5, imm=1, signaled=False)
    a.post_write((buf.addr, 8, m.lkey), buf.addr + 128, m.rkey, wr_id=6)
    wcs = cq.wait(2, 10)
    assert (wcs[0].wr_id, wcs[0].status) == (5, N.WC_RNR_RETRY_EXC_ERR)  # error WCs ignore signaling
    assert (wcs[1].wr_id, wcs[1].status) == (6, N.WC_WR_FLUSH_ERR)
    assert a.query()[0].qp_state == N.QPS_ERR
    # ERR refuses new sends.
    rc, bad = a.post_send_raw([a.make_send_wr(N.WR_RDMA_WRITE, [(buf.addr, 8, m.lkey)], buf.addr, m.rkey)])
    assert rc == 22 and bad == 0


def test_infinite_rnr_waits_for_receive(cpu_daemon):
    ctx, pd, cq, a, b = _pair(rnr_retry=7)
    buf = V.HostBuffer(8192)
    m = pd.reg_mr(buf.addr, 8192, ACC)
    a.post_send(N.WR_RDMA_WRITE_WITH_IMM, [(buf.addr, 16, m.lkey)], remote_addr=buf.addr + 64, rkey=m.rkey,
                wr_id=1, imm=9)
    time.sleep(0.05)
    assert cq.poll() == []  # stalled, not failed
    b.post_recv(wr_id=2)
    wcs = cq.wait(2, 10)
    assert sorted((w.wr_id, w.status) for w in wcs) == [(1, 0), (2, 0)]


def test_modify_to_err_flushes_sq_and_rq(cpu_daemon):
    ctx, pd, cq, a, b = _pair()
    for i in range(4):
        b.post_recv(wr_id=i)
    b.to_error()
    wcs = cq.wait(4, 10)
    assert [w.wr_id for w in wcs] == [0, 1, 2, 3]
    assert all(w.status == N.WC_WR_FLUSH_ERR for w in wcs)
    rc, _ = b.post_recv_raw([b.make_recv_wr(9, [])])
    assert rc == 22


def test_access_and_protection_errors(cpu_daemon):
    ctx, pd, cq, a, b = _pair()
    buf = V.HostBuffer(8192)
    ro = pd.reg_mr(buf.addr, 4096, N.ACCESS_LOCAL_WRITE)  # no remote access
    rw = pd.reg_mr(buf.addr + 4096, 4096, ACC)
    a.post_write((buf.addr + 4096, 8, rw.lkey), buf.addr, ro.rkey, wr_id=1)
    assert cq.wait(1, 10)[0].status == N.WC_REM_ACCESS_ERR
    ctx2, pd2, cq2, c, d = _pair()
    c.post_write((buf.addr + 4096, 8, rw.lkey), buf.addr + 4096, rw.rkey, wr_id=2)  # lkey of another PD
    assert cq2.wait(1, 10)[0].status == N.WC_LOC_PROT_ERR
    ctx3, pd3, cq3, e, f = _pair()
    m3 = pd3.reg_mr(buf.addr + 4096, 4096, ACC)
    e.post_write((buf.addr + 4096, 8, m3.lkey), buf.addr + 4096 + 4090, m3.rkey, wr_id=3)  # runs past the MR
    assert cq3.wait(1, 10)[0].status == N.WC_REM_ACCESS_ERR


def test_api_error_domains(cpu_daemon):
    L = N.lib()
    ctx = V.Context(V.find_device(kind=0))
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(8)
    assert L.ugdr_close_device(ctx.h) == -1 and N.errno() == 16  # EBUSY with live children
    assert L.ugdr_poll_cq(None, 1, None) == -22
    assert L.ugdr_create_cq(ctx.h, 0, None, None, 0) is None and N.errno() == 22
    assert not L.ugdr_reg_mr(pd.h, C.c_void_p(12345), 8, 1)  # malloc-style host memory
    assert N.errno() == 95
    cq.destroy()
    assert L.ugdr_destroy_cq(cq.h) == 22  # repeated destroy
    pd.dealloc()
    ctx.close()
    assert L.ugdr_close_device(ctx.h) == -1 and N.errno() == 22


def _client_b(path, q):
    os.environ["UGDR_DAEMON_SOCKET"] = path
    ctx = V.Context(V.find_device(kind=0))
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(8)
    qp = pd.create_qp(cq)
    qp.to_init(N.ACCESS_REMOTE_WRITE)
    q.put(qp.qpn)
    q.get()  # wait for the peer to connect, then exit without cleanup (session reclaim)


def test_two_clients_connect_and_disconnect_reclaim(cpu_daemon):
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    p = mpc.Process(target=_client_b, args=(cpu_daemon.socket_path, q))
    p.start()
    remote_qpn = q.get(timeout=60)
    ctx = V.Context(V.find_device(kind=0))
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(8)
    a = pd.create_qp(cq)
    a.to_init(N.ACCESS_REMOTE_WRITE)
    a.connect(remote_qpn)  # cross-session, same daemon
    assert a.query()[0].qp_state == N.QPS_RTS
    q.put("done")
    p.join(30)
    assert p.exitcode == 0
    # The other client's QP was reclaimed with its session: a new connect cannot find it.
    b = pd.create_qp(cq)
    b.to_init(N.ACCESS_REMOTE_WRITE)
    deadline = time.time() + 5
    while True:
        rc = N.lib().ugdr_connect_qp(b.h, C.byref(N.QpConnInfo(remote_qpn)),
                                     C.byref(N.QpAttr(timeout=14, retry_cnt=7, rnr_retry=7, min_rnr_timer=1)),
                                     N.CONNECT_MASK)
        if rc == 2 or time.time() > deadline:
            break
        time.sleep(0.05)
    assert rc == 2  # ENOENT


def test_killed_client_does_not_take_the_daemon_down(cpu_daemon):
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    p = mpc.Process(target=_client_b, args=(cpu_daemon.socket_path, q))
    p.start()
    q.get(timeout=60)
    p.kill()
    p.join(30)
    assert cpu_daemon.proc.poll() is None
    assert V.find_device(kind=0).name == "ugdr_cpu0"


def test_engine_stats_count_work(cpu_daemon):
    ctx, pd, cq, a, b = _pair()
    buf = V.HostBuffer(1 << 16)
    m = pd.reg_mr(buf.addr, 1 << 16, ACC)
    ctx.stats(reset=True)
    for i in range(10):
        a.post_write((buf.addr, 1000, m.lkey), buf.addr + 8192, m.rkey, wr_id=i)
    cq.wait(10, 10)
    st = ctx.stats()
    assert st.wrs_completed >= 10 and st.bytes_moved >= 10_000


def test_cli_doctor_reports_the_build():
    from ugdr_b200.cli import doctor

    rep = doctor()
    assert rep["libugdr"] and rep["daemon"]
    assert "gpus" in rep or "torch_error" in rep


def test_config3_stress_on_the_host_engine():
    """Verbs-feature stress semantics on the host-memory engine: 16-SGE WRITE / WRITE_WITH_IMM with
    log-uniform SGE sizes, fetch-add and compare-swap on a 4096-entry counter array; every byte,
    immediate, CAS result and counter is checked by ugdr_perf."""
    from ugdr_b200.utils.perf import run

    out = run(["stress", "--src-gpu", "-1", "--dst-gpu", "-1", "--qps", "16", "--depth", "64", "--sges", "16",
               "--rounds", "2"], gpus=0, timeout=300)
    assert out and out[-1]["correct"] and out[-1]["wrs"] == 2048, out


def test_concurrent_stress_clients_meet_at_the_barriers():
    """Two stress clients against one daemon run their rounds between a shared start and finish
    barrier (the stress-all launcher's protocol) and both verify."""
    from ugdr_b200.utils.perf import stress_all

    res = stress_all(0, ["--qps", "8", "--depth", "32", "--sges", "16", "--rounds", "2"], timeout=300,
                     host_clients=2)
    agg = res["aggregate"]
    assert agg["correct"] and agg["clients"] == 2 and agg["wrs"] == 2 * 2 * 8 * 32, agg


def test_daemon_death_is_reported_and_a_restarted_daemon_serves_new_objects(tmp_path):
    """Failure detection on the host (reference: stale handles fail with EINVAL after a
    reconnect, src/api/api.cpp connection epoch).  A daemon killed with SIGKILL leaves the client
    with errors, not hangs: control calls on its objects fail promptly.  A new daemon on the same
    socket path serves new objects, and handles from the dead daemon stay invalid."""
    import signal

    sock = str(tmp_path / "ugdr.sock")
    d = V.Daemon(gpus=0, socket_path=sock)
    ctx, pd, cq, a, b = _pair(depth=16, cq_depth=64)
    buf = V.HostBuffer(1 << 16)
    mr = pd.reg_mr(buf.addr, 1 << 16, ACC)
    a.post_write((buf.addr, 8, mr.lkey), buf.addr + 4096, mr.rkey, wr_id=1)
    assert cq.wait(1, timeout=10)[0].status == N.WC_SUCCESS
    d.proc.send_signal(signal.SIGKILL)
    d.proc.wait(10)
    t0 = time.perf_counter()
    with pytest.raises(V.UgdrError):
        a.to_error()  # a control call on an object of the dead daemon
    with pytest.raises(V.UgdrError):
        ctx.alloc_pd()
    assert time.perf_counter() - t0 < 5.0
    # A restarted daemon on the same path: new objects work, old handles stay invalid.
    os.unlink(sock)
    d2 = V.Daemon(gpus=0, socket_path=sock)
    try:
        ctx2, pd2, cq2, a2, b2 = _pair(depth=16, cq_depth=64)
        buf2 = V.HostBuffer(1 << 16)
        mr2 = pd2.reg_mr(buf2.addr, 1 << 16, ACC)
        buf2.view()[:8] = np.arange(8, dtype=np.uint8)
        a2.post_write((buf2.addr, 8, mr2.lkey), buf2.addr + 4096, mr2.rkey, wr_id=7)
        wc = cq2.wait(1, timeout=10)[0]
        assert wc.status == N.WC_SUCCESS and wc.wr_id == 7
        assert np.array_equal(buf2.view()[4096:4104], np.arange(8, dtype=np.uint8))
        with pytest.raises(V.UgdrError):
            pd.reg_mr(buf.addr, 4096, ACC)  # a PD of the dead daemon
    finally:
        d2.stop()
        d.stop()  # reaps the killed process and closes its log


def test_nested_daemon_leaves_the_outer_socket_in_place():
    """A daemon started and stopped inside another's lifetime (as benchmark helpers do) puts
    UGDR_DAEMON_SOCKET back when it stops, so clients of the outer daemon keep working; a daemon
    started with export=False never touches the variable."""
    outer = V.Daemon(gpus=0)
    try:
        assert os.environ["UGDR_DAEMON_SOCKET"] == outer.socket_path
        assert any(d.kind == 0 for d in V.get_devices())
        with V.Daemon(gpus=0) as inner:
            assert os.environ["UGDR_DAEMON_SOCKET"] == inner.socket_path
        assert os.environ["UGDR_DAEMON_SOCKET"] == outer.socket_path
        with V.Daemon(gpus=0, export=False) as quiet:
            assert os.environ["UGDR_DAEMON_SOCKET"] == outer.socket_path != quiet.socket_path
        assert os.environ["UGDR_DAEMON_SOCKET"] == outer.socket_path
        devs = V.get_devices()  # reaches the outer daemon, whose socket still exists
        assert any(d.kind == 0 for d in devs)
        ctx, pd, cq, a, b = _pair(depth=16, cq_depth=64)
        buf = V.HostBuffer(1 << 16)
        mr = pd.reg_mr(buf.addr, 1 << 16, ACC)
        buf.view()[:8] = np.arange(8, dtype=np.uint8)
        a.post_write((buf.addr, 8, mr.lkey), buf.addr + 4096, mr.rkey, wr_id=3)
        assert cq.wait(1, timeout=10)[0].status == N.WC_SUCCESS
    finally:
        outer.stop()


def test_smoke_binaries(tmp_path):
    """Reference smoke checks (tests/smoke): the client without a daemon reports an errno and
    fails; the daemon prints its usage; with a daemon, the client lists its devices."""
    import subprocess

    env = dict(os.environ, UGDR_DAEMON_SOCKET=str(tmp_path / "none.sock"))
    r = subprocess.run([str(N.LIB_DIR / "ugdr_client")], env=env, capture_output=True, text=True, timeout=30)
    assert r.returncode != 0 and "no daemon" in r.stderr
    r = subprocess.run([str(N.DAEMON_PATH), "--help"], capture_output=True, text=True, timeout=30)
    assert r.returncode == 0 and "usage: ugdr_daemon" in r.stdout
    with V.Daemon(gpus=0, socket_path=str(tmp_path / "d.sock")):
        env = dict(os.environ, UGDR_DAEMON_SOCKET=str(tmp_path / "d.sock"))
        r = subprocess.run([str(N.LIB_DIR / "ugdr_client")], env=env, capture_output=True, text=True, timeout=30)
        assert r.returncode == 0 and "kind=cpu" in r.stdout, r.stdout + r.stderr


def test_c_example_client(tmp_path):
    """examples/write_read.c builds as C11 against the public header and runs WRITE, READ and
    FETCH_ADD through a daemon's host-memory engine."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = str(tmp_path / "write_read")
    subprocess.run([cc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", os.path.join(repo, "include"),
                    os.path.join(repo, "examples", "write_read.c"), "-L", str(N.LIB_DIR), "-lugdr",
                    f"-Wl,-rpath,{N.LIB_DIR}", "-o", exe], check=True, capture_output=True, text=True)
    with V.Daemon(gpus=0, socket_path=str(tmp_path / "d.sock")):
        env = dict(os.environ, UGDR_DAEMON_SOCKET=str(tmp_path / "d.sock"))
        r = subprocess.run([exe, "ugdr_cpu0"], env=env, capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


def test_ring_benchmark_moves_every_descriptor():
    """ugdr_perf ring: producer and consumer threads over one shared ring, batch 1 and 32; the
    consumer's checksum proves every descriptor arrived once and in order."""
    import json
    import subprocess

    for batch in (1, 32):
        r = subprocess.run([str(N.LIB_DIR / "ugdr_perf"), "ring", "--batch", str(batch), "--wrs", "200000"],
                           capture_output=True, text=True, timeout=120)
        out = [json.loads(line) for line in r.stdout.splitlines() if line.startswith("{")]
        assert r.returncode == 0 and out and out[-1]["correct"], r.stdout + r.stderr


def test_python_example_runs():
    """examples/host_rdma.py runs end to end (gather WRITE, WRITE_WITH_IMM, FETCH_ADD)."""
    import subprocess
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = {k: v for k, v in os.environ.items() if k != "UGDR_DAEMON_SOCKET"}
    r = subprocess.run([sys.executable, os.path.join(repo, "examples", "host_rdma.py")], capture_output=True,
                       text=True, timeout=120, env=env)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


def test_engine_bench_runs_every_case():
    """ugdr_engine_bench (in-process host engine): the eight metadata cases and the four payload
    cases run to completion, move the payload (the binary byte-checks it) and report rates."""
    import subprocess

    exe = str(N.LIB_DIR / "ugdr_engine_bench")
    r = subprocess.run([exe, "metadata", "--wr-bytes", "64"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("benchmark=engine_metadata")]
    assert len(lines) == 8
    for ln in lines:
        f = dict(kv.split("=", 1) for kv in ln.split())
        assert f["completed_wr"] == "262144" and float(f["MWR_per_s"]) > 0
        assert int(f["wc"]) == (262144 if f["signaling"] == "every_wr" else 262144 // 32)
    r = subprocess.run([exe, "payload", "--iters", "2000"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("benchmark=engine_payload")]
    assert len(lines) == 4 and all("parent_MWR_per_s=" in ln for ln in lines)


def test_make_install_layout_and_pkg_config(tmp_path):
    """`make install PREFIX=...` gives headers, libugdr.so, ugdr.pc and the binaries; the C example
    builds from pkg-config flags alone and runs against the installed daemon."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None or shutil.which("make") is None or shutil.which("pkg-config") is None:
        pytest.skip("needs cc, make and pkg-config")
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    prefix = tmp_path / "usr"
    r = subprocess.run(["make", "install", f"PREFIX={prefix}"], cwd=repo, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    for rel in ("include/ugdr/api.hpp", "include/ugdr/collective.h", "lib/libugdr.so", "lib/pkgconfig/ugdr.pc",
                "bin/ugdr_daemon", "bin/ugdr_client"):
        assert (prefix / rel).exists(), rel
    env = dict(os.environ, PKG_CONFIG_PATH=str(prefix / "lib" / "pkgconfig"))
    flags = subprocess.run(["pkg-config", "--cflags", "--libs", "ugdr"], env=env, capture_output=True, text=True,
                           check=True).stdout.split()
    exe = str(tmp_path / "write_read")
    subprocess.run([cc, "-std=c11", os.path.join(repo, "examples", "write_read.c"), "-o", exe, *flags], check=True,
                   capture_output=True, text=True)
    sock = str(tmp_path / "d.sock")
    d = subprocess.Popen([str(prefix / "bin" / "ugdr_daemon"), "--socket", sock, "--gpus", "0"],
                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    try:
        deadline = time.time() + 20
        while not os.path.exists(sock) and time.time() < deadline:
            time.sleep(0.02)
        r = subprocess.run([exe, "ugdr_cpu0"], env=dict(os.environ, UGDR_DAEMON_SOCKET=sock), capture_output=True,
                           text=True, timeout=60)
        assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
    finally:
        d.terminate()
        d.wait(timeout=30)


def test_pip_install_ships_the_native_build(tmp_path):
    """`pip install .` (offline, no build isolation) runs make and ships libugdr.so and the daemon
    as package data: the installed package starts its own daemon and lists the host device from
    a directory outside the source tree."""
    import subprocess
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    site = tmp_path / "site"
    r = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
                        "--target", str(site), repo], capture_output=True, text=True, timeout=900)
    if r.returncode != 0 and "No module named pip" in r.stderr:
        pytest.skip("pip not available")
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    code = ("from ugdr_b200 import verbs as V, _native as N\n"
            "assert str(N.LIB_DIR).startswith(%r), N.LIB_DIR\n"
            "with V.Daemon(gpus=0):\n"
            "    print(sorted(d.name for d in V.get_devices()))\n") % str(site)
    env = {k: v for k, v in os.environ.items() if not k.startswith("UGDR_")}
    env["PYTHONPATH"] = str(site)
    r = subprocess.run([sys.executable, "-c", code], cwd=str(tmp_path), env=env, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0 and "ugdr_cpu0" in r.stdout, r.stdout + r.stderr


def test_object_churn_holds_memory_and_descriptors_flat(cpu_daemon):
    """Thousands of create / connect / post / destroy cycles (CQ, two QPs, an MR): the daemon's
    resident memory and descriptor count and this client's resident memory stay flat once warm
    (destroyed proxies sit in a bounded quarantine; the daemon frees every object)."""
    def rss_kb(pid: int) -> int:
        with open(f"/proc/{pid}/status") as f:
            return next(int(ln.split()[1]) for ln in f if ln.startswith("VmRSS"))

    ctx = V.Context(V.find_device(kind=0))
    pd = ctx.alloc_pd()
    buf = V.HostBuffer(1 << 16)
    dpid = cpu_daemon.proc.pid
    try:
        marks = {}
        for it in range(3000):
            cq = ctx.create_cq(64)
            a = pd.create_qp(cq, max_send_wr=16, max_recv_wr=16)
            b = pd.create_qp(cq, max_send_wr=16, max_recv_wr=16)
            V.connect_pair(a, b, access=N.ACCESS_REMOTE_WRITE)
            mr = pd.reg_mr(buf.addr, 4096, N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE)
            a.post_write((buf.addr, 8, mr.lkey), buf.addr + 64, mr.rkey, wr_id=it)
            assert cq.wait(1, 10)[0].status == N.WC_SUCCESS
            a.destroy()
            b.destroy()
            mr.dereg()
            cq.destroy()
            if it in (1000, 2999):
                marks[it] = (rss_kb(dpid), len(os.listdir(f"/proc/{dpid}/fd")), rss_kb(os.getpid()))
        (d0, f0, c0), (d1, f1, c1) = marks[1000], marks[2999]
        assert f1 <= f0 and c1 - c0 < 4096, marks
        # An instrumented daemon (the sanitizer suite sets UGDR_DAEMON_BIN) keeps freed blocks in
        # its allocator's quarantine, so its resident size grows by design; LeakSanitizer checks
        # that daemon instead.
        if not os.environ.get("UGDR_DAEMON_BIN"):
            assert d1 - d0 < 2048, marks
    finally:
        pd.dealloc()
        ctx.close()
        buf.free()


def test_examples_byte_compile():
    """Every Python example at least compiles (the GPU ones run on a B200 box)."""
    import py_compile

    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "examples")
    for name in sorted(os.listdir(root)):
        if name.endswith(".py"):
            py_compile.compile(os.path.join(root, name), doraise=True)


def test_control_plane_latency_benchmark():
    """ugdr_perf control on the host device: every life-cycle operation is timed and reported."""
    from ugdr_b200.utils import perf

    rows = [r for r in perf.run(["control", "--src-gpu", "-1", "--iters", "50"], gpus=0)
            if r.get("benchmark") == "ugdr_control"]
    assert len(rows) == 1
    for op in ("cq_create", "cq_destroy", "qp_create", "qp_destroy", "qp_connect_pair", "mr_register",
               "mr_deregister", "query_qp"):
        assert 0 < rows[0][f"{op}_p50_us"] <= rows[0][f"{op}_p99_us"], op


def test_forked_child_gets_its_own_session(cpu_daemon):
    """After fork the child does not talk over its parent's session: its first control call opens
    a new connection, the parent's objects are stale there (EINVAL), and the parent keeps working."""
    import errno

    ctx = V.Context(V.find_device(kind=0))
    pd = ctx.alloc_pd()
    r, w = os.pipe()
    pid = os.fork()
    if pid == 0:  # child
        code = 1
        try:
            os.close(r)
            try:
                ctx.alloc_pd()
                code = 2  # the parent's context must be stale in the child
            except V.UgdrError as e:
                if e.errno == errno.EINVAL:
                    names = [d.name for d in V.get_devices()]  # a fresh session works
                    code = 0 if "ugdr_cpu0" in names else 3
        finally:
            os.write(w, bytes([code]))
            os._exit(0)
    os.close(w)
    code = os.read(r, 1)
    os.close(r)
    os.waitpid(pid, 0)
    assert code == b"\x00", code
    pd2 = ctx.alloc_pd()  # the parent's session is intact
    pd2.dealloc()
    pd.dealloc()
    ctx.close()


def test_wr_length_limit_is_four_gib_minus_one(cpu_daemon):
    """A WR may gather up to 4 GiB - 1 bytes (byte_len is 32 bits; the reference's limit): 2.25 GiB
    passes the length check (and then fails on the small remote MR), 4.25 GiB is LOC_LEN_ERR.
    The SGEs repeat one untouched 300 MiB region, so nothing is copied."""
    ctx = V.Context(V.find_device(kind=0))
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(64)
    mk = lambda: pd.create_qp(cq, max_send_wr=8, max_recv_wr=8, max_send_sge=32, max_recv_sge=1)  # noqa: E731
    big, small = V.HostBuffer(300 << 20), V.HostBuffer(4096)
    lm = pd.reg_mr(big.addr, 300 << 20, ACC)
    rm = pd.reg_mr(small.addr, 4096, ACC)
    try:
        for nsge, want in ((9, N.WC_REM_ACCESS_ERR), (17, N.WC_LOC_LEN_ERR)):
            a, b = mk(), mk()
            V.connect_pair(a, b, access=REMOTE)
            sges = [(big.addr, 256 << 20, lm.lkey)] * nsge
            wr = V.QueuePair.make_send_wr(N.WR_RDMA_WRITE, sges, remote_addr=small.addr, rkey=rm.rkey, wr_id=nsge)
            assert a.post_send_raw([wr]) == (0, -1)
            w = cq.wait(1, 30)[0]
            assert (w.wr_id, w.status) == (nsge, want)
            a.destroy()
            b.destroy()
    finally:
        lm.dereg()
        rm.dereg()
        cq.destroy()
        pd.dealloc()
        ctx.close()
        big.free()
        small.free()


def test_latency_and_bandwidth_sweeps_run_on_the_host_device():
    """ugdr_perf latency / bw with --src-gpu -1 --dst-gpu -1 use the host-memory device and host
    buffers end to end (byte-checked by the binary)."""
    from ugdr_b200.utils import perf

    lat = [r for r in perf.run(["latency", "--src-gpu", "-1", "--dst-gpu", "-1", "--bytes", "4096", "--iters", "500"],
                               gpus=0) if r.get("benchmark") == "ugdr_latency"]
    assert len(lat) == 1 and lat[0]["correct"] and lat[0]["p50_us"] > 0
    bw = [r for r in perf.run(["bw", "--src-gpu", "-1", "--dst-gpu", "-1", "--min", "8", "--max", "64K", "--qd", "16",
                               "--bytes-per-size", "4M"], gpus=0) if r.get("benchmark") == "ugdr_bw"]
    assert len(bw) >= 2 and all(r["correct"] for r in bw)


def test_python_objects_are_context_managers(cpu_daemon):
    """Each verbs object releases itself at the end of a `with` block, innermost first."""
    with V.Context(V.find_device(kind=0)) as ctx, ctx.alloc_pd() as pd, ctx.create_cq(64) as cq, \
            V.HostBuffer(8192) as buf, pd.reg_mr(buf.addr, 8192, ACC) as mr, \
            pd.create_qp(cq, max_send_wr=8, max_recv_wr=8) as a, pd.create_qp(cq, max_send_wr=8, max_recv_wr=8) as b:
        V.connect_pair(a, b, access=REMOTE)
        buf.view()[:8] = 7
        a.post_write((buf.addr, 8, mr.lkey), buf.addr + 4096, mr.rkey, wr_id=1)
        assert cq.wait(1, 10)[0].status == N.WC_SUCCESS
        assert bytes(buf.view()[4096:4104]) == b"\x07" * 8
    with pytest.raises(V.UgdrError):  # everything above is gone
        pd.dealloc()


def test_daemon_stats_count_live_objects(tmp_path):
    """ugdr_x_query_daemon_stats counts every session's live objects and follows creation,
    destruction and the reclaim of a vanished client."""
    import subprocess
    import sys

    with V.Daemon(gpus=0, socket_path=str(tmp_path / "d.sock")) as d:
        old = os.environ.get("UGDR_DAEMON_SOCKET")
        os.environ["UGDR_DAEMON_SOCKET"] = d.socket_path
        try:
            base = V.daemon_stats()
            assert base["devices"] == 1 and base["qps"] == 0
            with V.Context(V.find_device(kind=0)) as ctx, ctx.alloc_pd() as pd, ctx.create_cq(16) as cq:
                with pd.create_qp(cq, max_send_wr=4, max_recv_wr=4):
                    st = V.daemon_stats()
                    assert (st["contexts"], st["pds"], st["cqs"], st["qps"]) == (1, 1, 1, 1)
            code = ("from ugdr_b200 import verbs as V\n"
                    "ctx = V.Context(V.find_device(kind=0)); pd = ctx.alloc_pd(); cq = ctx.create_cq(8)\n"
                    "print(V.daemon_stats()['cqs'])\n")
            env = dict(os.environ, PYTHONPATH=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
            r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=60)
            assert r.stdout.strip() == "1", r.stderr
            import time

            deadline = time.time() + 10
            while V.daemon_stats()["cqs"] != 0 and time.time() < deadline:
                time.sleep(0.02)
            assert V.daemon_stats() == base  # the vanished client's objects were reclaimed
        finally:
            if old is None:
                os.environ.pop("UGDR_DAEMON_SOCKET", None)
            else:
                os.environ["UGDR_DAEMON_SOCKET"] = old
