"""Collectives benchmark - launch one rank per GPU:

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m ugdr_b200.parallel.bench [--op allreduce|moe|p2p|all] [--api peer|verbs|both] [--iters K]

* allreduce: 1 GiB bf16 per rank, N(0,1) seeded by rank; ugdr's one-kernel fused-sum allreduce
  over peer memory and (N >= 2, when the GPUs support multicast) its NVLS allreduce that sums in
  the NVSwitch, vs NCCL all_reduce on the same tensor size.  Reports both, the faster as
  `ugdr_best_ms`, algbw (bytes / time) and busbw (x 2(N-1)/N).
* p2p: NCCL send / recv from rank 0 to rank 1 for 8 B .. 1 GiB (the baseline of the verbs
  WRITE / READ sweep, which ugdr_b200.utils.perf runs).
* moe: 16,384 tokens x 7,168 bf16 per rank, top-8 of 256 experts from uniform router logits;
  one step = dispatch + combine (experts are the identity).  ugdr fuses the permutes into the
  NVLink stores / loads; the NCCL baseline is all_to_all_single with the permutes as separate
  torch kernels and the split sizes exchanged first.
Times are CUDA-event durations of K back-to-back iterations on each rank, max over ranks.  The
first ugdr call is checked against a torch fp32 reference.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from ..models.moe import MoEConfig, route
from .collectives import MoEAllToAll, allreduce_bf16
from . import nvls
from .peers import PeerGroup


def _timed(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    t = torch.tensor([ms], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=_GLOO)
    return float(t.item())


_GLOO = None


def bench_allreduce(rank, world, iters, warmup, nbytes=1 << 30, impl="all", ctas=0) -> dict:
    count = nbytes // 2

    def exchange(obj):
        out = [None] * world
        dist.all_gather_object(out, obj, group=_GLOO)
        return out

    g = PeerGroup(nbytes, rank, world, exchange)
    x = g.view(torch.bfloat16, count)
    gen = torch.Generator(device="cuda").manual_seed(rank)
    x.copy_(torch.randn(count, generator=gen, device="cuda", dtype=torch.float32).to(torch.bfloat16))
    # Correctness on a 1 Mi-element window against an fp32 sum of every rank's seeded input.
    lo = (count // 3) // 8 * 8
    ref = torch.zeros(1 << 20, dtype=torch.float32, device="cuda")
    for r in range(world):
        gr = torch.Generator(device="cuda").manual_seed(r)
        ref += torch.randn(count, generator=gr, device="cuda", dtype=torch.float32).to(torch.bfloat16)[
            lo:lo + (1 << 20)].float()
    torch.cuda.synchronize()
    dist.barrier()
    allreduce_bf16(g, count)
    torch.cuda.synchronize()
    g.check_status()
    err = (x[lo:lo + (1 << 20)].float() - ref).abs().max().item()
    tol = 2 ** -7 * ref.abs().max().item() + 1e-2
    ok = err <= tol
    t_ugdr = _timed(lambda: allreduce_bf16(g, count, ctas=ctas), iters, warmup) if impl in ("all", "ring") else None
    g.check_status()
    g.close()
    del x
    # NVLS variant: the same data in multicast-bound memory, reduced inside the NVSwitch.
    nv = {}
    if impl in ("all", "nvls") and world >= 2 and nvls.supported():
        sig = PeerGroup(4096, rank, world, exchange)
        buf = nvls.NvlsBuffer(nbytes, rank, world, exchange)
        try:
            xn = buf.view(torch.bfloat16, count)
            xn.copy_(torch.randn(count, generator=torch.Generator(device="cuda").manual_seed(rank), device="cuda",
                                 dtype=torch.float32).to(torch.bfloat16))
            torch.cuda.synchronize()
            dist.barrier()
            nvls.allreduce_bf16_nvls(sig, buf, count)
            torch.cuda.synchronize()
            sig.check_status()
            err_n = (xn[lo:lo + (1 << 20)].float() - ref).abs().max().item()
            t_n = _timed(lambda: nvls.allreduce_bf16_nvls(sig, buf, count, ctas=ctas), iters, warmup)
            sig.check_status()
            del xn
        finally:
            buf.close()  # collective, before any rank can leave with memory bound
        sig.close()
        nv = {"ugdr_nvls_ms": round(t_n, 4), "ugdr_nvls_algbw_GBps": round(nbytes / t_n / 1e6, 1),
              "nvls_correct": bool(err_n <= tol), "nvls_max_err": err_n}
    y = torch.randn(count, device="cuda").to(torch.bfloat16)
    t_nccl = _timed(lambda: dist.all_reduce(y), iters, warmup) if impl == "all" else None
    bus = 2 * (world - 1) / world if world > 1 else 1.0
    out = {"op": "allreduce_bf16", "n_gpus": world, "bytes": nbytes, **nv, "correct": bool(ok), "max_err": err}
    if t_ugdr is not None:
        out.update({"ugdr_ring_ms": round(t_ugdr, 4), "ugdr_ring_algbw_GBps": round(nbytes / t_ugdr / 1e6, 1),
                    "ugdr_ring_busbw_GBps": round(bus * nbytes / t_ugdr / 1e6, 1)})
    best = min(t for t in (t_ugdr, nv.get("ugdr_nvls_ms")) if t is not None)
    out["ugdr_best_ms"] = round(best, 4)
    out["ugdr_best_path"] = "nvls" if nv and best == nv["ugdr_nvls_ms"] else "ring"
    if t_nccl is not None:
        out.update({"nccl_ms": round(t_nccl, 4), "nccl_algbw_GBps": round(nbytes / t_nccl / 1e6, 1),
                    "nccl_busbw_GBps": round(bus * nbytes / t_nccl / 1e6, 1),
                    "speedup_vs_nccl": round(t_nccl / best, 3)})
    return out


def bench_allreduce_verbs(rank, world, local, iters, warmup, nbytes=1 << 30, pieces=8) -> dict:
    """The allreduce on the verbs API (ugdr_x_verbs_allreduce_bf16): every byte is a WR that the
    daemon's executor on the rank's GPU runs, the sum is the executor's WRITE_SUM_BF16.  Checked
    bit for bit on a 1 Mi-element window against the fp32 sum of the seeded inputs rounded once.
    Timed two ways, max over ranks: the executor's own span on the GPU (from the last retire of
    the call before the timed ones to the last retire of the last one, %globaltimer, from the
    engine statistics) and the caller's wall clock per call."""
    import time

    from . import verbs_collectives as VC

    count = nbytes // 2

    def exchange(obj):
        out = [None] * world
        dist.all_gather_object(out, obj, group=_GLOO)
        return out

    def bcast(obj):
        lst = [obj]
        dist.broadcast_object_list(lst, src=0, group=_GLOO)
        return lst[0]

    daemon = VC.shared_daemon(rank, world, bcast)
    g = VC.VerbsGroup(rank, world, local, count, exchange, pieces=pieces)
    try:
        gen = torch.Generator(device="cuda").manual_seed(rank)
        g.buf.copy_(torch.randn(count, generator=gen, device="cuda", dtype=torch.float32).to(torch.bfloat16))
        lo = (count // 3) // 8 * 8
        ref = torch.zeros(1 << 20, dtype=torch.float32, device="cuda")
        for r in range(world):
            gr = torch.Generator(device="cuda").manual_seed(r)
            ref += torch.randn(count, generator=gr, device="cuda", dtype=torch.float32).to(torch.bfloat16)[
                lo:lo + (1 << 20)].float()
        torch.cuda.synchronize()
        dist.barrier(group=_GLOO)
        g.allreduce()
        exact = bool(torch.equal(g.buf[lo:lo + (1 << 20)], ref.to(torch.bfloat16)))
        for _ in range(warmup):
            g.allreduce()
        dist.barrier(group=_GLOO)
        g.allreduce()  # its last retire opens the timed span on the executor's clock
        st0 = g.ctx.stats()
        t0 = time.perf_counter()
        for _ in range(iters):
            g.allreduce()
        wall = (time.perf_counter() - t0) / iters * 1e3
        st = g.ctx.stats()
        dev = (int(st.last_end_ns) - int(st0.last_end_ns)) / 1e6 / iters
        t = torch.tensor([wall, dev], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=_GLOO)
        wall, dev = float(t[0]), float(t[1])
        dist.barrier(group=_GLOO)
        # The same sum through NVLink SHARP on the verbs: one WRITE_SUM_BF16 per rank over its shard
        # of a multicast MR (ugdr_x_verbs_allreduce_bf16_mc).
        mc = {}
        if world >= 2 and nvls.supported():
            nvbuf = nvls.NvlsBuffer(nbytes, rank, world, exchange)
            try:
                xv = nvbuf.view(torch.bfloat16, count)
                xv.copy_(torch.randn(count, generator=torch.Generator(device="cuda").manual_seed(rank),
                                     device="cuda", dtype=torch.float32).to(torch.bfloat16))
                torch.cuda.synchronize()
                dist.barrier(group=_GLOO)
                g.allreduce_nvls(nvbuf, count)
                torch.cuda.synchronize()
                err = (xv[lo:lo + (1 << 20)].float() - ref).abs()
                mc_ok = bool((err <= ref.abs() * 2.0 ** -7 + 1e-3).all())
                for _ in range(warmup):
                    g.allreduce_nvls(nvbuf, count)
                dist.barrier(group=_GLOO)
                g.allreduce_nvls(nvbuf, count)
                s0 = g.ctx.stats()
                t1 = time.perf_counter()
                for _ in range(iters):
                    g.allreduce_nvls(nvbuf, count)
                mwall = (time.perf_counter() - t1) / iters * 1e3
                s1 = g.ctx.stats()
                mdev = (int(s1.last_end_ns) - int(s0.last_end_ns)) / 1e6 / iters
                tt = torch.tensor([mwall, mdev], dtype=torch.float64)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX, group=_GLOO)
                mc = {"ugdr_verbs_nvls_ms": round(float(tt[1]), 4), "ugdr_verbs_nvls_wall_ms": round(float(tt[0]), 4),
                      "ugdr_verbs_nvls_algbw_GBps": round(nbytes / float(tt[1]) / 1e6, 1), "nvls_correct": mc_ok}
                del xv
            finally:
                g.release_multicast()
                dist.barrier(group=_GLOO)
                nvbuf.close()
    finally:
        g.close()
        dist.barrier(group=_GLOO)
        if daemon is not None:
            daemon.stop()
    bus = 2 * (world - 1) / world if world > 1 else 1.0
    return {"op": "allreduce_bf16_verbs", "n_gpus": world, "bytes": nbytes, "pieces": pieces, **mc,
            "ugdr_verbs_ms": round(dev, 4), "ugdr_verbs_wall_ms": round(wall, 4),
            "ugdr_verbs_algbw_GBps": round(nbytes / dev / 1e6, 1),
            "ugdr_verbs_busbw_GBps": round(bus * nbytes / dev / 1e6, 1),
            "correct_exact": exact,
            "timing": "executor span on the GPU (last retire of the previous call to last retire of the last "
                      "call) per call, and wall clock per call; max over ranks"}


def bench_p2p_nccl(rank, world, sizes, iters, warmup) -> list[dict]:
    """NCCL send/recv baseline for the point-to-point WRITE / READ sweep: rank 0 sends
    `size` bytes to rank 1, `iters` transfers back to back, device-timed, max over the pair."""
    out = []
    if world < 2:
        return out
    for size in sizes:
        buf = torch.empty(max(size, 1), dtype=torch.uint8, device="cuda")

        def step():
            if rank == 0:
                dist.send(buf, 1)
            elif rank == 1:
                dist.recv(buf, 0)

        n = max(4, min(2000, (8 << 30) // max(size, 1)))
        t = _timed(step, n, warmup)
        out.append({"op": "p2p_nccl", "bytes": size, "us_per_transfer": round(t * 1e3, 3),
                    "GBps": round(size / t / 1e6, 3)})
        del buf
    return out


def bench_moe(rank, world, iters, warmup, cfg: MoEConfig) -> dict:
    T, H, K, E = cfg.tokens, cfg.hidden, cfg.topk, cfg.experts

    def exchange(obj):
        out = [None] * world
        dist.all_gather_object(out, obj, group=_GLOO)
        return out

    recv = int(T * K * 1.25) + 4096
    g = PeerGroup(MoEAllToAll.required_bytes(world, E, H, recv), rank, world, exchange)
    a2a = MoEAllToAll(g, T, H, K, E, recv)
    gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
    x = torch.randn(T, H, generator=gen, device="cuda").to(torch.bfloat16)
    ids, w = route(T, E, K, seed=2000 + rank)

    def ugdr_step():
        a2a.dispatch(x, ids)
        return a2a.combine(w)

    out = ugdr_step()
    torch.cuda.synchronize()
    g.check_status()
    ref = (x.float() * w.sum(-1, keepdim=True))
    ok = torch.allclose(out.float(), ref, atol=3e-2, rtol=2e-2)
    t_ugdr = _timed(ugdr_step, iters, warmup)
    g.check_status()

    # NCCL baseline: permute by destination rank, exchange split sizes, all_to_all_single,
    # (identity experts), reverse all_to_all_single, weighted un-permute.
    epr = E // world
    flat = ids.reshape(-1).long()
    dst = flat // epr
    order = torch.argsort(dst, stable=True)
    send_counts = torch.bincount(dst, minlength=world)

    def nccl_step():
        send = x[order // K]  # permute kernel
        rc = torch.empty_like(send_counts)
        dist.all_to_all_single(rc, send_counts)
        in_splits = send_counts.tolist()
        out_splits = rc.tolist()
        recv_buf = torch.empty(sum(out_splits), H, dtype=x.dtype, device="cuda")
        dist.all_to_all_single(recv_buf, send, out_splits, in_splits)
        back = torch.empty_like(send)
        dist.all_to_all_single(back, recv_buf, in_splits, out_splits)
        o = torch.zeros(T, H, dtype=torch.float32, device="cuda")
        o.index_add_(0, order // K, back.float() * w.reshape(-1)[order, None])  # un-permute + weight
        return o.to(torch.bfloat16)

    t_nccl = _timed(nccl_step, iters, warmup)
    g.close()
    row_bytes = H * 2
    moved = 2 * T * K * row_bytes  # dispatch + combine rows per rank
    return {"op": "moe_dispatch_combine", "n_gpus": world, "tokens": T, "hidden": H, "topk": K, "experts": E,
            "ugdr_ms": round(t_ugdr, 4), "nccl_ms": round(t_nccl, 4),
            "ugdr_GBps_per_rank": round(moved / t_ugdr / 1e6, 1), "nccl_GBps_per_rank": round(moved / t_nccl / 1e6, 1),
            "speedup_vs_nccl": round(t_nccl / t_ugdr, 3), "correct": bool(ok)}


def bench_moe_verbs(rank, world, local, iters, warmup, cfg: MoEConfig) -> dict:
    """MoE dispatch + combine on the verbs (VerbsMoE): the permutes are the SGE lists of WRITEs
    and READs that the daemon's executors run; experts are the identity.  Checked against the
    fp32 reference of the same workload; timed by wall clock per step (routing, the host copy of
    the routing, both transfers and the weighted sum), max over ranks."""
    import time

    from . import verbs_collectives as VC

    T, H, K, E = cfg.tokens, cfg.hidden, cfg.topk, cfg.experts

    def exchange(obj):
        out = [None] * world
        dist.all_gather_object(out, obj, group=_GLOO)
        return out

    def bcast(obj):
        lst = [obj]
        dist.broadcast_object_list(lst, src=0, group=_GLOO)
        return lst[0]

    daemon = VC.shared_daemon(rank, world, bcast, idle_exit_us=50)  # see VerbsMoE
    g = VC.moe_group(rank, world, local, T, K, E, exchange)
    moe = VC.VerbsMoE(g, T, H, K, E, recv_rows=int(T * K * 1.25) + 4096)
    try:
        gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
        x = torch.randn(T, H, generator=gen, device="cuda").to(torch.bfloat16)
        ids, w = route(T, E, K, seed=2000 + rank)

        def step():
            moe.dispatch(x, ids)
            return moe.combine(w)

        out = step()
        torch.cuda.synchronize()
        ok = torch.allclose(out.float(), x.float() * w.sum(-1, keepdim=True), atol=3e-2, rtol=2e-2)
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        dist.barrier(group=_GLOO)
        t0 = time.perf_counter()
        td = tc = 0.0
        st0 = g.ctx.stats()
        for _ in range(iters):
            a = time.perf_counter()
            moe.dispatch(x, ids)
            b = time.perf_counter()
            moe.combine(w)
            torch.cuda.synchronize()
            td += b - a
            tc += time.perf_counter() - b
        ms = (time.perf_counter() - t0) / iters * 1e3
        st1 = g.ctx.stats()
        split = {"dispatch_ms": round(td / iters * 1e3, 3), "combine_ms": round(tc / iters * 1e3, 3),
                 "slow_wrs_per_step": (int(st1.slow_wrs) - int(st0.slow_wrs)) // iters,
                 "jobs_per_step": (int(st1.jobs_published) - int(st0.jobs_published)) // iters,
                 "order_waits_per_step": (int(st1.order_waits) - int(st0.order_waits)) // iters}
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=_GLOO)
        ms = float(t.item())
        dist.barrier(group=_GLOO)
    finally:
        moe.close()
        g.close()
        dist.barrier(group=_GLOO)
        if daemon is not None:
            daemon.stop()
    moved = 2 * T * K * H * 2
    return {"op": "moe_dispatch_combine_verbs", "n_gpus": world, "tokens": T, "hidden": H, "topk": K, "experts": E,
            "ugdr_verbs_ms": round(ms, 4), "ugdr_verbs_GBps_per_rank": round(moved / ms / 1e6, 1), **split,
            "correct": bool(ok), "timing": "wall clock per step (route + host copy of the routing + dispatch WRs + "
                                           "combine WRs + weighted sum), max over ranks"}


def main():
    global _GLOO
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="all", choices=["all", "allreduce", "moe", "p2p"])
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--ar-mib", type=int, default=1024, help="allreduce bytes per rank, MiB")
    ap.add_argument("--tokens", type=int, default=MoEConfig().tokens, help="MoE tokens per rank")
    ap.add_argument("--ar-impl", default="all", choices=["all", "ring", "nvls"],
                    help="allreduce paths to time (all: ring, NVLS when available, and NCCL)")
    ap.add_argument("--ctas", type=int, default=0, help="allreduce grid size (0: one CTA per SM)")
    ap.add_argument("--api", default="peer", choices=["peer", "verbs", "both"],
                    help="allreduce over peer-mapped buffers (one kernel), over the verbs (WRs run by the "
                         "daemon's executors), or both")
    ap.add_argument("--pieces", type=int, default=8, help="verbs allreduce: pipeline pieces per shard")
    args = ap.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    _GLOO = dist.new_group(backend="gloo")
    results = []
    if args.op in ("all", "allreduce"):
        if args.api in ("peer", "both"):
            results.append(bench_allreduce(rank, world, args.iters, args.warmup, args.ar_mib << 20, args.ar_impl,
                                           args.ctas))
        if args.api in ("verbs", "both"):
            results.append(bench_allreduce_verbs(rank, world, local, args.iters, args.warmup, args.ar_mib << 20,
                                                 args.pieces))
            if args.api == "verbs":  # the NCCL figure beside it
                y = torch.randn((args.ar_mib << 20) // 2, device="cuda").to(torch.bfloat16)
                t_nccl = _timed(lambda: dist.all_reduce(y), args.iters, args.warmup)
                r = results[-1]
                r["nccl_ms"] = round(t_nccl, 4)
                best = min(v for v in (r["ugdr_verbs_ms"], r.get("ugdr_verbs_nvls_ms")) if v is not None)
                r["ugdr_verbs_best_ms"] = best
                r["speedup_vs_nccl"] = round(t_nccl / best, 3)
                del y
    if args.op == "p2p":
        sizes = [1 << k for k in range(3, 31, 2)]
        results.extend(bench_p2p_nccl(rank, world, sizes, max(args.iters, 20), args.warmup))
    if args.op in ("all", "moe"):
        if args.api in ("peer", "both"):
            results.append(bench_moe(rank, world, args.iters, args.warmup, MoEConfig(tokens=args.tokens)))
        if args.api in ("verbs", "both"):
            results.append(bench_moe_verbs(rank, world, local, args.iters, args.warmup, MoEConfig(tokens=args.tokens)))
    if rank == 0:
        for r in results:
            print(json.dumps(r), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
