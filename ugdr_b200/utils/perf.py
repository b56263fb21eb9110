"""Run the native verbs benchmarks (ugdr_perf) against a private daemon.

    python -m ugdr_b200.utils.perf latency --src-gpu 0 --dst-gpu 1 --bytes 8
    python -m ugdr_b200.utils.perf bw --src-gpu 0 --dst-gpu 1 --op read --min 8 --max 1G
    python -m ugdr_b200.utils.perf posting --batch 32
    python -m ugdr_b200.utils.perf stress-all --gpus 8 --qps 64 --depth 128 --rounds 2

Prints the binary's key=value and JSON lines.  `--gpus N` sets how many GPUs the daemon owns
(default: every GPU named by --src-gpu / --dst-gpu; 0 for `posting`).
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

from .. import _native as N
from .. import verbs as V


def run(args: list[str], gpus: int | None = None, timeout: float = 1800) -> list[dict]:
    if gpus is None:
        ids = [int(args[i + 1]) for i, a in enumerate(args[:-1]) if a in ("--src-gpu", "--dst-gpu")]
        gpus = 0 if args and args[0] == "posting" else (max(ids) + 1 if ids else 1)
    exe = N.LIB_DIR / "ugdr_perf"
    lines: list[str] = []
    with V.Daemon(gpus=gpus, export=False) as d:
        env = dict(os.environ, UGDR_DAEMON_SOCKET=d.socket_path)
        proc = subprocess.Popen([str(exe), *args], env=env, stdout=subprocess.PIPE, text=True)
        for line in proc.stdout:  # stream: a run cut short still leaves its finished points
            sys.stdout.write(line)
            sys.stdout.flush()
            lines.append(line)
        rc = proc.wait(timeout)
        if rc != 0:
            sys.stderr.write(d.log_text())
            raise RuntimeError(f"ugdr_perf exited {rc}")
    return [json.loads(line) for line in lines if line.startswith("{")]


def stress_all(gpus: int, extra: list[str], timeout: float = 1800, host_clients: int = 2) -> dict:
    """The verbs-feature stress workload on every ordered GPU pair at once: one daemon owning `gpus` GPUs and
    one ugdr_perf stress client per (src, dst) pair, all running concurrently.  The clients meet
    at a start barrier after their set-up and at a finish barrier before their tear-down, so the
    timed rounds overlap and no client's tear-down (which quiesces executors) lands inside
    another's rounds.  With gpus == 0 the `host_clients` clients use the host-memory engine.
    Returns the per-pair JSON results and aggregates: WRs and bytes over the slowest client's
    time, and the summed posting rate."""
    import tempfile

    exe = N.LIB_DIR / "ugdr_perf"
    if gpus > 0:
        pairs = [(a, b) for a in range(gpus) for b in range(gpus) if a != b] or [(0, 0)]
    else:
        pairs = [(-1, -1)] * host_clients
    results = []
    with tempfile.TemporaryDirectory(prefix="ugdr-stress-") as sync, V.Daemon(gpus=gpus, export=False) as d:
        env = dict(os.environ, UGDR_DAEMON_SOCKET=d.socket_path)
        procs = [subprocess.Popen([str(exe), "stress", "--src-gpu", str(a), "--dst-gpu", str(b), *extra,
                                   "--seed", str(1 + i), "--sync-dir", sync, "--sync-n", str(len(pairs))],
                                  env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
                 for i, (a, b) in enumerate(pairs)]
        failed = []
        for (a, b), p in zip(pairs, procs):
            out, err = p.communicate(timeout=timeout)
            js = [json.loads(line) for line in out.splitlines() if line.startswith("{")]
            if p.returncode != 0 or not js:
                failed.append((a, b, p.returncode, err[-300:]))
            results.extend(js)
        if failed:
            sys.stderr.write(d.log_text())
    secs = [r["wrs"] / (r["complete_MWRps"] * 1e6) for r in results if r["complete_MWRps"] > 0]
    slowest = max(secs) if secs else float("nan")
    agg = {"benchmark": "ugdr_stress_all", "gpus": gpus, "clients": len(pairs),
           "wrs": sum(r["wrs"] for r in results),
           "complete_MWRps": round(sum(r["wrs"] for r in results) / slowest / 1e6, 3) if secs else None,
           "GBps": round(sum(r["GBps"] * t for r, t in zip(results, secs)) / slowest, 3) if secs else None,
           "post_MWRps_sum": round(sum(r["post_MWRps"] for r in results), 3),
           "slowest_client_s": round(slowest, 4) if secs else None,
           "correct": bool(results) and not failed and all(r["correct"] for r in results),
           "failed": failed}
    return {"pairs": results, "aggregate": agg}


if __name__ == "__main__":
    argv = sys.argv[1:]
    g = None
    if "--gpus" in argv:
        i = argv.index("--gpus")
        g = int(argv[i + 1])
        del argv[i:i + 2]
    if argv and argv[0] == "stress-all":
        res = stress_all(2 if g is None else g, argv[1:])
        for r in res["pairs"]:
            print(json.dumps(r))
        print(json.dumps(res["aggregate"]))
        sys.exit(0 if res["aggregate"]["correct"] else 2)
    run(argv, gpus=g)
