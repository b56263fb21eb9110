"""Run the reference's own client->daemon CUDA benchmark (built unmodified into baseline/_ref) over
a list of WR sizes on one GPU, for side-by-side tables with `ugdr_b200.utils.perf`.

    python -m ugdr_b200.utils.refbench --gpu 0 --sizes 8K,64K,1M,16M,64M
    python -m ugdr_b200.utils.refbench --gpu 0 --persistent-copy

Prints one JSON line per size: the reference's QD-64 post_send->poll_cq bandwidth and its QD-1
latency percentiles, parsed from its key=value output (benchmarks/client_daemon_cuda_benchmark.cpp
in the reference).  The reference copies inside one GPU only (it has no peer path).

`--persistent-copy` runs the reference's kernel-model matrix instead
(benchmarks/persistent_copy_benchmark.cpp `matrix`: direct_atomic, dynamic_sharded_spsc,
static_partition_spsc, warp_specialized and the selected warp_specialized_pipeline, same task
stream) and prints one JSON line per model: copy GB/s, MTask/s, task latency percentiles,
registers, occupancy and the benchmark's own correctness flag.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
EXE = os.path.join(REPO, "baseline", "_ref", "build", "benchmarks", "ugdr_client_daemon_cuda_benchmark")


def _size(s: str) -> int:
    m = re.fullmatch(r"(\d+)([KMG]?)", s.strip().upper())
    if not m:
        raise ValueError(s)
    return int(m.group(1)) << {"": 0, "K": 10, "M": 20, "G": 30}[m.group(2)]


def run(gpu: int, wr_bytes: int, timeout: float = 600) -> dict:
    if not os.path.exists(EXE):
        return {"impl": "reference", "wr_bytes": wr_bytes, "unavailable": "reference benchmark not built"}
    # ~256 MiB per bandwidth phase (queue depth 64 per batch), at least 4 batches.
    batches = max(4, (256 << 20) // (64 * wr_bytes))
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(gpu))
    cmd = [EXE, "--wr-bytes", str(wr_bytes), "--warmup-batches", "2", "--bandwidth-batches", str(batches),
           "--latency-warmup", "20", "--latency-iterations", "200"]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout)
    out = {"impl": "reference", "gpu": gpu, "wr_bytes": wr_bytes, "rc": res.returncode}
    for line in res.stdout.splitlines():
        kv = dict(re.findall(r"(\w+)=(\"[^\"]*\"|\S+)", line))
        if kv.get("phase") == "bandwidth":
            out["GBps"] = float(kv.get("logical_payload_GB_per_s", "nan"))
            out["MWRps"] = float(kv.get("parent_MWR_per_s", "nan"))
        elif kv.get("phase") == "latency":
            out["p50_us"] = float(kv["latency_p50_us"])
            out["p99_us"] = float(kv["latency_p99_us"])
    if res.returncode != 0:
        out["stderr"] = res.stderr[-300:]
    return out


PC_EXE = os.path.join(REPO, "baseline", "_ref", "build", "benchmarks", "ugdr_persistent_copy_benchmark")


def run_persistent_copy(gpu: int, timeout: float = 900) -> list[dict]:
    if not os.path.exists(PC_EXE):
        return [{"impl": "reference", "benchmark": "persistent_copy", "unavailable": "reference benchmark not built"}]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(gpu))
    res = subprocess.run([PC_EXE, "matrix"], env=env, capture_output=True, text=True, timeout=timeout)
    rows = []
    for line in res.stdout.splitlines():
        kv = dict(re.findall(r"(\w+)=(\S+)", line))
        if kv.get("benchmark") != "persistent_copy":
            continue
        rows.append({"impl": "reference", "benchmark": "persistent_copy", "gpu": gpu, "model": kv.get("model"),
                     "payload_bytes": int(kv.get("payload_bytes", 0)), "copy_warps": int(kv.get("copy_warps", 0)),
                     "GBps": float(kv.get("copy_GB_per_s", "nan")), "MTaskps": float(kv.get("task_MTask_per_s", "nan")),
                     "p50_us": float(kv.get("task_p50_us", "nan")), "p99_us": float(kv.get("task_p99_us", "nan")),
                     "registers": int(kv.get("registers_per_thread", 0)), "occupancy": float(kv.get("occupancy", 0)),
                     "correct": kv.get("correctness_passed") == "1", "valid": kv.get("measurement_valid") == "1"})
    if res.returncode != 0 or not rows:
        rows.append({"impl": "reference", "benchmark": "persistent_copy", "rc": res.returncode,
                     "stderr": res.stderr[-300:]})
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpu", type=int, default=0)
    ap.add_argument("--sizes", default="8K,64K,1M,16M,64M")
    ap.add_argument("--persistent-copy", action="store_true", help="the reference's kernel-model matrix")
    args = ap.parse_args()
    if args.persistent_copy:
        for row in run_persistent_copy(args.gpu):
            print(json.dumps(row), flush=True)
        return
    for s in args.sizes.split(","):
        print(json.dumps(run(args.gpu, _size(s))), flush=True)


if __name__ == "__main__":
    main()
