"""Developer harness (parity: the reference's tools/ugdr CLI — doctor, build, test, smoke).

    python -m ugdr_b200.cli doctor      toolchain, GPUs, NVLink peer access, multicast support
    python -m ugdr_b200.cli build       make -j (libugdr.so, daemon, client, perf, native tests)
    python -m ugdr_b200.cli test [-m "not gpu"]   pytest over tests/
    python -m ugdr_b200.cli smoke       one WRITE + READ through a private daemon on cuda:0
    python -m ugdr_b200.cli lint        layering, public ABI/exports, client contracts, byte-compile
                                        (parity: the reference's tools/check_module_boundaries.py and
                                        tools/check_client_contracts.py)
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def doctor() -> dict:
    rep: dict = {"repo": REPO}
    for tool in ("nvcc", "g++", "make", "ncu"):
        rep[tool] = shutil.which(tool)
    try:
        out = subprocess.run(["nvcc", "--version"], capture_output=True, text=True).stdout
        rep["nvcc_version"] = out.strip().splitlines()[-1] if out else None
    except OSError:
        rep["nvcc_version"] = None
    from . import _native as N

    rep["libugdr"] = str(N.LIB_PATH) if N.LIB_PATH.exists() else None
    if os.environ.get("UGDR_DAEMON_SOCKET") and rep["libugdr"]:
        from . import verbs as V

        try:  # a running daemon: its devices and live objects
            rep["daemon_stats"] = V.daemon_stats()
            rep["daemon_devices"] = [d.name for d in V.get_devices()]
        except Exception as e:  # a report, not a failure
            rep["daemon_error"] = repr(e)
    rep["daemon"] = str(N.DAEMON_PATH) if N.DAEMON_PATH.exists() else None
    try:
        import torch

        rep["torch"] = torch.__version__
        n = torch.cuda.device_count() if torch.cuda.is_available() else 0
        rep["gpus"] = [torch.cuda.get_device_name(i) for i in range(n)]
        rep["capability"] = [".".join(map(str, torch.cuda.get_device_capability(i))) for i in range(n)]
        rep["peer_access"] = {f"{a}->{b}": torch.cuda.can_device_access_peer(a, b)
                              for a in range(n) for b in range(n) if a != b}
        if n and rep["libugdr"]:
            from .parallel import nvls

            rep["nvls_multicast"] = [nvls.supported(i) for i in range(n)]
            from . import ops

            rep["kernels"] = ops.kernel_attributes()
    except Exception as e:  # a report, not a failure
        rep["torch_error"] = repr(e)
    return rep


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="ugdr_b200.cli")
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("doctor")
    sub.add_parser("build")
    t = sub.add_parser("test")
    t.add_argument("-m", default="not gpu")
    sub.add_parser("smoke")
    sub.add_parser("lint")
    args = ap.parse_args(argv)
    if args.cmd == "doctor":
        print(json.dumps(doctor(), indent=1))
        return 0
    if args.cmd == "build":
        return subprocess.run(["make", "-j"], cwd=REPO).returncode
    if args.cmd == "test":
        return subprocess.run([sys.executable, "-m", "pytest", "tests", "-q", "-m", args.m], cwd=REPO).returncode
    if args.cmd == "smoke":
        sys.path.insert(0, REPO)
        import __graft_entry__

        __graft_entry__.smoke()
        print("smoke ok")
        return 0
    if args.cmd == "lint":
        import compileall

        ok = all(compileall.compile_dir(os.path.join(REPO, d), quiet=1) for d in ("ugdr_b200", "tests"))
        rc = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider",
                             "tests/test_module_boundaries.py", "tests/test_abi_contract.py",
                             "tests/test_contracts.py"], cwd=REPO).returncode
        return 0 if ok and rc == 0 else 1
    return 2


if __name__ == "__main__":
    sys.exit(main())
