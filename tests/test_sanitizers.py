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


@pytest.mark.parametrize("kind", ["asan", "tsan"])
def test_api_suites_against_a_sanitized_daemon(kind, tmp_path):
    """The public-API, model and fuzz suites against a daemon whose host code is instrumented:
    any sanitizer report in a daemon log (or a daemon that died of one) fails the test."""
    import sys

    if not os.path.exists("/usr/bin/g++") or shutil.which("make") is None:
        pytest.skip("system g++ with sanitizer runtimes not available")
    b = subprocess.run(["make", "-j16", kind], cwd=REPO, capture_output=True, text=True, timeout=900)
    assert b.returncode == 0, b.stdout[-2000:] + b.stderr[-2000:]
    logs = tmp_path / "logs"
    logs.mkdir()
    env = dict(os.environ, UGDR_DAEMON_BIN=os.path.join(REPO, "build", "san", kind, "ugdr_daemon"),
               UGDR_DAEMON_LOG_DIR=str(logs), ASAN_OPTIONS="detect_leaks=1:halt_on_error=1",
               TSAN_OPTIONS="halt_on_error=1")
    env.pop("UGDR_DAEMON_SOCKET", None)
    suites = [os.path.join(REPO, "tests", f) for f in ("test_cpu_api.py", "test_cpu_model.py", "test_fuzz_ipc.py")]
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", *suites], cwd=REPO,
                       env=env, capture_output=True, text=True, timeout=1800)
    reports = []
    for f in logs.iterdir():
        text = f.read_text(errors="replace")
        if "Sanitizer" in text or "runtime error" in text:
            reports.append(f"{f.name}: {text[-1500:]}")
    assert r.returncode == 0, r.stdout[-3000:] + "\n".join(reports)
    assert not reports, "\n".join(reports)
