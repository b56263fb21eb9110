"""Build the native tree (libugdr.so, ugdr_daemon, test and benchmark binaries) in place."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]


def build(jobs: int | None = None, quiet: bool = True) -> None:
    """Run `make` at the repo root (sm_100a; nvcc cross-compiles without a GPU)."""
    jobs = jobs or max(1, min(16, os.cpu_count() or 1))
    cmd = ["make", "-C", str(REPO), f"-j{jobs}"]
    res = subprocess.run(cmd, capture_output=quiet, text=True)
    if res.returncode != 0:
        out = (res.stdout or "") + (res.stderr or "")
        raise RuntimeError(f"native build failed:\n{out[-6000:]}")
