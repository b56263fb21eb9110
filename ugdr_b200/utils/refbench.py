"""Run the reference's own client->daemon CUDA benchmark (built unmodified into baseline/_ref) over
a list of WR sizes on one GPU, for side-by-side tables with `ugdr_b200.utils.perf`.

    python -m ugdr_b200.utils.refbench --gpu 0 --sizes 8K,64K,1M,16M,64M

Prints one JSON line per size: the reference's QD-64 post_send->poll_cq bandwidth and its QD-1
latency percentiles, parsed from its key=value output (benchmarks/client_daemon_cuda_benchmark.cpp
in the reference).  The reference copies inside one GPU only (it has no peer path).
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpu", type=int, default=0)
    ap.add_argument("--sizes", default="8K,64K,1M,16M,64M")
    args = ap.parse_args()
    for s in args.sizes.split(","):
        print(json.dumps(run(args.gpu, _size(s))), flush=True)


if __name__ == "__main__":
    main()
