"""Run the native verbs benchmarks (ugdr_perf) against a private daemon.

    python -m ugdr_b200.utils.perf latency --src-gpu 0 --dst-gpu 1 --bytes 8
    python -m ugdr_b200.utils.perf bw --src-gpu 0 --dst-gpu 1 --op read --min 8 --max 1G
    python -m ugdr_b200.utils.perf posting --batch 32

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
    with V.Daemon(gpus=gpus) as d:
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


if __name__ == "__main__":
    argv = sys.argv[1:]
    g = None
    if "--gpus" in argv:
        i = argv.index("--gpus")
        g = int(argv[i + 1])
        del argv[i:i + 2]
    run(argv, gpus=g)
