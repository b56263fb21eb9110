#!/usr/bin/env python
"""Headline benchmark: all-pairs RDMA WRITE bandwidth through the ugdr verbs API.

Workload (the all-pairs configuration, weak-scaled): every GPU holds one 256 MiB bf16 MR (N(0,1),
seeded by rank) of eight 32 MiB slices, plus a 512 MiB receive MR (two sets of eight slots, used by
alternate steps).  One step = every GPU RDMA_WRITEs 7 distinct slices over 7 QPs: WR k of rank r
sends slice k to peer (r + 1 + k mod (N - 1)) % N, into that GPU's receive slot (dst + 1 + k) % 8
of the step's set, so every inbound WR of a step lands in its own slot.  With N = 8 this is exactly "a 32 MiB slice to each of its 7
peers"; with fewer GPUs the same 7 x 32 MiB per GPU cycle over the N - 1 peers, so all traffic
crosses NVLink.  N = 1 has no peer: the WRs are loopback copies inside the GPU, and each WR of
the run gets its own source slice and destination slot so that no step is served from L2.
Per-GPU work is fixed, so scaling is weak; each step reads 224 MiB and writes 224 MiB per GPU,
more than the 126 MB L2.

`value` is device-timed: the daemon launches every GPU's executor together for the K timed steps
(all WRs of the K steps are queued first), brackets each launch with CUDA events on its
launching stream, and the step time is the max over GPUs.  `e2e` runs the same steps through the
public API with the persistent executors: per step each rank posts 7 WRs (the WQEs travel
host->device from the pinned shared ring) and polls 7 CQEs (device->host).

`--impl reference` runs the reference's own client->daemon benchmark binary, built unmodified
from the reference sources into baseline/_ref (configure-time flags only), one process per GPU.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

SLOT_MIB = 32
SLOTS = 8
PEERS = 7
BASELINE_GBPS = None  # no published number exists for this configuration
_DAEMON = None  # rank 0's daemon, kept for its log when a run fails


def peer_of(rank: int, k: int, world: int) -> int:
    """Destination of WR k: the peers in turn (never the sender itself unless it is alone)."""
    if world == 1:
        return rank
    return (rank + 1 + k % (world - 1)) % world


def sender_of(rank: int, k: int, world: int) -> int:
    """The rank whose WR k lands on `rank` (inverse of peer_of for a fixed k)."""
    if world == 1:
        return rank
    return (rank - 1 - k % (world - 1)) % world


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return world, rank, local


class Comm:
    """Host-side coordination between ranks (gloo): barriers, object exchange, max-reduce."""

    def __init__(self, world: int, rank: int):
        self.world, self.rank = world, rank
        self.dist = None
        if world > 1:
            import torch.distributed as dist

            dist.init_process_group("gloo")
            self.dist = dist

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def bcast(self, obj):
        if not self.dist:
            return obj
        lst = [obj]
        self.dist.broadcast_object_list(lst, src=0)
        return lst[0]

    def gather(self, obj):
        if not self.dist:
            return [obj]
        out = [None] * self.world
        self.dist.all_gather_object(out, obj)
        return out

    def max(self, x: float) -> float:
        return max(self.gather(x))

    def close(self):
        if self.dist:
            self.dist.destroy_process_group()


def run_ugdr(args, comm: Comm, world: int, rank: int, local: int) -> dict | None:
    import torch

    from ugdr_b200 import _native as N
    from ugdr_b200 import verbs as V
    from ugdr_b200.utils.clocks import ClockSampler

    global _DAEMON
    torch.cuda.set_device(local)
    daemon = None
    if rank == 0:
        daemon = _DAEMON = V.Daemon(gpus=world, cpu_device=False)
        path = daemon.socket_path
    else:
        path = None
    path = comm.bcast(path)
    os.environ["UGDR_DAEMON_SOCKET"] = path

    slot = SLOT_MIB << 20
    K, W = args.steps, args.warmup
    depth = K + W + 4
    # N = 1 has no peer: every WR is a loopback copy inside the GPU.  The executor runs many
    # queued steps at once, so with the 8-slice MR consecutive steps would re-read and re-write
    # the same slices while they sit in L2; instead every WR of the run gets its own source slice
    # and destination slot (capped at 448 slices, 14 GiB per MR), so each one moves HBM bytes.
    loop = world == 1
    nslices = min(PEERS * (K + W), 448) if loop else SLOTS
    total = nslices * slot
    # Receive MR: with peers, two sets of 8 slots used by alternate steps.  A QP's WRs take effect
    # in posting order, so a WR into the slot the previous step's WR on that QP is still writing
    # would wait for it; alternating sets lets two steps per QP be in flight.
    rcv_total = total if loop else 2 * total

    ctx = V.Context(V.find_device(gpu=local))
    pd = ctx.alloc_pd()
    cq = ctx.create_cq(2 * PEERS * depth + 64)
    # Source MR: 256 MiB of N(0,1) bf16 seeded by rank; WR k reads its own slice k, so one step
    # reads 7 distinct 32 MiB slices (224 MiB, larger than L2).  Receive MR: where peers write.
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    src_buf = torch.randn(total // 2, dtype=torch.bfloat16, device="cuda", generator=gen)
    rcv_buf = torch.zeros(rcv_total // 2, dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    acc = N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE
    src_mr = pd.reg_mr(src_buf.data_ptr(), total, acc)
    rcv_mr = pd.reg_mr(rcv_buf.data_ptr(), rcv_total, acc)
    req = [pd.create_qp(cq, max_send_wr=depth) for _ in range(PEERS)]
    rsp = [pd.create_qp(cq, max_send_wr=4) for _ in range(PEERS)]
    for q in req + rsp:
        q.to_init(N.ACCESS_REMOTE_WRITE)
    info = comm.gather({"addr": rcv_buf.data_ptr(), "rkey": rcv_mr.rkey,
                        "rsp": [q.qpn for q in rsp], "req": [q.qpn for q in req]})
    for k in range(PEERS):
        req[k].connect(info[peer_of(rank, k, world)]["rsp"][k])
        rsp[k].connect(info[sender_of(rank, k, world)]["req"][k])
    comm.barrier()

    # Work requests are built once per distinct (step pattern, QP) and reused: a step's WRs differ
    # only in their slices, which repeat with period 2 (N > 1) or nslices / 7 (N = 1).
    period = nslices // PEERS if loop else 2
    wr_cache: dict[tuple[int, int], object] = {}

    def step_wr(step_id: int, k: int):
        key = (step_id % period, k)
        w = wr_cache.get(key)
        if w is None:
            dst = peer_of(rank, k, world)
            sidx = k
            dslot = (dst + 1 + k) % SLOTS + SLOTS * (step_id % 2)
            if loop:
                sidx = dslot = (step_id * PEERS + k) % nslices
            w = V.QueuePair.make_send_wr(N.WR_RDMA_WRITE, [(src_buf.data_ptr() + sidx * slot, slot, src_mr.lkey)],
                                         remote_addr=info[dst]["addr"] + dslot * slot, rkey=info[dst]["rkey"],
                                         wr_id=k)
            wr_cache[key] = w
        return w

    def post_step(step_id: int):
        for k in range(PEERS):
            rc, _ = req[k].post_send_raw([step_wr(step_id, k)])
            if rc != 0:
                raise RuntimeError(f"rank {rank}: ugdr_post_send failed ({rc})")

    all_ctx = None
    if rank == 0:
        all_ctx = [V.Context(V.find_device(gpu=g)) for g in range(world)]

    def drain(steps: int, base: int) -> float:
        ctx.hold(True)
        comm.barrier()
        for s in range(steps):
            post_step(base + s)
        comm.barrier()
        ms = None
        if rank == 0:
            ms = max(V.timed_drain(all_ctx, [PEERS * steps] * world, timeout_ms=300000))
        ms = comm.bcast(ms)
        wcs = cq.wait(PEERS * steps, timeout=120)
        bad = [w for w in wcs if w.status != N.WC_SUCCESS]
        if bad:
            raise RuntimeError(f"rank {rank}: {len(bad)} failed completions, first {bad[0]}")
        ctx.hold(False)
        return ms

    # Warm-up (untimed), then verify every inbound slot against the sender's source slice.
    drain(W, 0)
    comm.barrier()
    torch.cuda.synchronize()
    ok = True
    rcv_bytes = rcv_buf.view(torch.uint8)
    if loop:
        n = min(PEERS * W, nslices) * slot
        ok &= torch.equal(rcv_bytes[:n], src_buf.view(torch.uint8)[:n])
    for k in range(PEERS if not loop else 0):
        src = sender_of(rank, k, world)
        dslot = (rank + 1 + k) % SLOTS
        g = torch.Generator(device="cuda").manual_seed(1234 + src)
        ref = torch.randn(total // 2, dtype=torch.bfloat16, device="cuda", generator=g).view(torch.uint8)
        ok &= torch.equal(rcv_bytes[dslot * slot:(dslot + 1) * slot], ref[k * slot:(k + 1) * slot])
        del ref
    ok = all(comm.gather(bool(ok)))

    # Device-timed region.
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    if all_ctx:
        for c in all_ctx:
            c.stats(reset=True)
    if sampler:
        sampler.__enter__()
    t_ms = drain(K, W)
    if sampler:
        sampler.__exit__(None, None, None)
    clocks = sampler.summary() if sampler else None
    diag = None
    if all_ctx:
        diag = []
        for c in all_ctx:
            st = c.stats()
            diag.append({f: int(getattr(st, f)) for f, _ in st._fields_})

    # End-to-end through the public API (persistent executors).
    for s in range(W):
        post_step(s)
        cq.wait(PEERS, timeout=60)
    comm.barrier()
    # Up to four steps in flight: new steps are posted before older steps' completions are
    # polled, as a streaming client would; every step still posts its 7 WQEs and reads its 7 CQEs.
    inflight = 4
    e2e_bad = 0
    t0 = time.perf_counter()
    for s in range(min(inflight, K)):
        post_step(s)
    for s in range(K):
        wcs = cq.wait(PEERS, timeout=60)
        e2e_bad += sum(1 for w in wcs if w.status != N.WC_SUCCESS)
        if s + inflight < K:
            post_step(s + inflight)
    t_e2e = time.perf_counter() - t0
    t_e2e = comm.max(t_e2e)
    if e2e_bad:
        raise RuntimeError(f"rank {rank}: {e2e_bad} failed completions in the end-to-end loop")

    step_bytes = world * PEERS * slot
    value = step_bytes * K / (t_ms / 1e3) / 1e9
    e2e = step_bytes * K / t_e2e / 1e9
    stats = ctx.stats()
    comm.barrier()
    for q in req + rsp:
        q.destroy()
    src_mr.dereg()
    rcv_mr.dereg()
    cq.destroy()
    pd.dealloc()
    ctx.close()
    if all_ctx:
        for c in all_ctx:
            c.close()
    comm.barrier()
    daemon_log = ""
    if daemon:
        daemon.stop()
        daemon_log = daemon.log_text()
    if rank != 0:
        return None
    wqe_bytes = 64  # one 64-byte send slot per WR (40 B header + 1 SGE, rounded)
    cqe_bytes = 32
    return {
        "metric": "rdma_write_allpairs_aggregate_GBps",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(t_ms / K, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None if BASELINE_GBPS is None else round(value / BASELINE_GBPS, 3),
        "dtype": "bf16",
        "data": "synthetic: N(0,1) bf16 MR per GPU, seeded by rank; payload verified after warm-up",
        "config": {
            "model": "ugdr all-pairs RDMA_WRITE (BASELINE configs[2])",
            "global_batch": world * PEERS,
            "seq_len": slot,
            "parallelism": f"{world} GPU(s) x {PEERS} QPs, 32 MiB per WR",
            "mr_bytes_per_gpu": total,
            "rcv_mr_bytes_per_gpu": rcv_total,
            "l2": ("inputs larger than L2: every WR of the run has its own 32 MiB source slice and destination slot"
                   if loop else
                   "inputs larger than L2: 7 distinct 32 MiB source slices (224 MiB) read + 224 MiB written per GPU per step"),
            "timing": "CUDA events around each GPU's executor launch, max over GPUs",
            "correct": bool(ok),
        },
        "clocks": clocks,
        "e2e": {"value": round(e2e, 2), "unit": "GB/s",
                "h2d_bytes_per_step": world * PEERS * wqe_bytes,
                "d2h_bytes_per_step": world * PEERS * cqe_bytes,
                "path": "ugdr_post_send -> persistent executor -> ugdr_poll_cq, four steps in flight, wall clock, "
                        "max over ranks"},
        "gpu_launches": world,
        "executor_launches_rank0": int(stats.launches),
        "engine_stats_timed": diag,
        "daemon_log_tail": daemon_log[-2000:] if daemon_log else "",
    }


def run_reference(args, comm: Comm, world: int, rank: int, local: int) -> dict | None:
    exe = os.path.join(REPO, "baseline", "_ref", "build", "benchmarks", "ugdr_client_daemon_cuda_benchmark")
    if not os.path.exists(exe):
        out = {"impl": "reference", "unavailable": "reference benchmark binary not built in baseline/_ref"}
        return out if rank == 0 else None
    env = dict(os.environ)
    env["CUDA_VISIBLE_DEVICES"] = str(local)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    wr = SLOT_MIB << 20
    # The reference runs queue depth 64 per batch; size its batches to ~ the same bytes as ours.
    batches = max(1, (args.steps * PEERS * wr) // (64 * wr))
    cmd = [exe, "--wr-bytes", str(wr), "--warmup-batches", str(max(1, args.warmup // 4)),
           "--bandwidth-batches", str(batches), "--latency-warmup", "2", "--latency-iterations", "20"]
    comm.barrier()
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=1800)
    gbps = None
    for line in res.stdout.splitlines():
        m = re.search(r"phase=bandwidth.*logical_payload_GB_per_s=([0-9.]+)", line)
        if m:
            gbps = float(m.group(1))
    got = comm.gather(gbps)
    if rank != 0:
        return None
    if any(g is None for g in got):
        return {"impl": "reference", "unavailable": f"reference benchmark failed (rc={res.returncode}): "
                f"{(res.stderr or res.stdout)[-300:]!r}"}
    value = sum(got)
    return {
        "impl": "reference",
        "metric": "rdma_write_allpairs_aggregate_GBps",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (reference's own seeded payload)",
        "config": {"model": "reference client->daemon CUDA benchmark, 32 MiB WRs, QD 64, same-GPU target",
                   "per_gpu_GBps": got, "batches": batches,
                   "timing": "reference's own wall clock (steady_clock) per process, summed over GPUs"},
        # The reference's number is already end to end: its client posts WRs into the shared
        # ring through the public API and polls their CQEs; the daemon's host worker feeds the
        # copy kernel.  One WQE goes host->device and one CQE device->host per WR, as in ours.
        "e2e": {"value": round(value, 2), "unit": "GB/s",
                "h2d_bytes_per_step": world * PEERS * 64,
                "d2h_bytes_per_step": world * PEERS * 32,
                "path": "reference ugdr_post_send -> daemon worker -> persistent copy kernel -> ugdr_poll_cq, "
                        "QD 64, wall clock per process, summed over GPUs"},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ugdr", "reference"], default="ugdr")
    args = ap.parse_args()
    world, rank, local = dist_env()
    if world != args.gpus and not (world == 1 and args.gpus == 1):
        if world == 1:
            raise SystemExit("--gpus N > 1 must be launched with torchrun (one rank per GPU)")
    comm = Comm(world, rank)
    try:
        if args.impl == "reference":
            out = run_reference(args, comm, world, rank, local)
        else:
            out = run_ugdr(args, comm, world, rank, local)
    except BaseException:
        if _DAEMON is not None:
            _DAEMON.stop()
            print("---- ugdr_daemon log ----\n" + _DAEMON.log_text()[-4000:], file=sys.stderr)
        raise
    finally:
        comm.close()
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
