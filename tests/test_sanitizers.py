"""The native suite under AddressSanitizer + UndefinedBehaviorSanitizer and under ThreadSanitizer
(host code instrumented; CUDA objects unmodified).  This replaces compute-sanitizer for the host
paths: rings, IPC, control plane, CPU engine, visibility gate."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("kind", ["asan", "tsan"])
def test_native_suite_under_sanitizer(kind):
    if not os.path.exists("/usr/bin/g++") or shutil.which("make") is None:
        pytest.skip("system g++ with sanitizer runtimes not available")
    b = subprocess.run(["make", "-j16", kind], cwd=REPO, capture_output=True, text=True, timeout=900)
    assert b.returncode == 0, b.stdout[-2000:] + b.stderr[-2000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0", TSAN_OPTIONS="halt_on_error=1")
    r = subprocess.run([os.path.join(REPO, "build", "san", kind, "ugdr_native_tests")], cwd=REPO, env=env,
                       capture_output=True, text=True, timeout=900)
    report = r.stdout[-3000:] + r.stderr[-3000:]
    assert r.returncode == 0, report
    assert "Sanitizer" not in r.stderr, report
