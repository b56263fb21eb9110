"""Run every case of the native C++ test binary (rings, IPC envelope, RPC codec, handle
registry, WR posting, control plane, CPU engine) as its own pytest case.  No GPU needed."""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

BIN = Path(__file__).resolve().parents[1] / "ugdr_b200" / "_lib" / "ugdr_native_tests"


def _cases() -> list[str]:
    if not BIN.exists():
        from ugdr_b200.utils.build import build

        build()
    out = subprocess.run([str(BIN), "--list"], capture_output=True, text=True, check=True)
    return [c for c in out.stdout.split() if c]


@pytest.mark.parametrize("case", _cases())
def test_native(case):
    res = subprocess.run([str(BIN), case], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
