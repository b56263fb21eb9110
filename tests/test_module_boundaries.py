"""Layering of the native sources (reference governance check: tools/check_module_boundaries.py).

Each csrc/<layer> may include only the layers listed here, so the client library never depends on
daemon internals and the wire-format layers stay free of CUDA and control logic.
"""
from __future__ import annotations

import os
import re

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

ALLOWED = {
    "common": {"common"},
    "queue": {"common", "queue"},
    "ipc": {"common", "ipc"},
    "control": {"common", "queue", "ipc", "control", "ugdr"},
    "api": {"common", "queue", "ipc", "control", "api", "ugdr"},
    "engine": {"common", "queue", "control", "engine", "ugdr"},
    "gpu": {"common", "queue", "control", "gpu", "ugdr"},
    "collective": {"collective", "ugdr"},
    "daemon": {"common", "queue", "ipc", "control", "engine", "gpu", "daemon", "ugdr"},
    "apps": {"ugdr"},
    "bench": {"ugdr", "queue", "common", "api", "control", "engine"},  # in-process benchmarks drive those layers
}
# Files of a layer that need no CUDA headers at all (wire formats and the control plane run in
# processes and tests without a GPU stack).
NO_CUDA = {"common", "queue", "ipc", "control"}

INCLUDE = re.compile(r'^\s*#\s*include\s+[<"]([^>"]+)[>"]', re.M)


def _sources(root: str = os.path.join(REPO, "csrc")):
    for layer in sorted(os.listdir(root)):
        d = os.path.join(root, layer)
        if not os.path.isdir(d):
            continue
        for name in sorted(os.listdir(d)):
            if name.endswith((".cpp", ".hpp", ".cu", ".h")):
                with open(os.path.join(d, name)) as f:
                    yield layer, name, INCLUDE.findall(f.read())


def test_every_layer_is_listed():
    layers = {layer for layer, _, _ in _sources()}
    assert layers <= set(ALLOWED), layers - set(ALLOWED)


def layering_violations(root: str = os.path.join(REPO, "csrc")) -> list[str]:
    bad = []
    for layer, name, incs in _sources(root):
        for inc in incs:
            if "/" not in inc:
                continue  # system and toolkit headers
            top = inc.split("/")[0]
            if top in ALLOWED and top not in ALLOWED[layer] or top == "ugdr" and "ugdr" not in ALLOWED[layer]:
                bad.append(f"csrc/{layer}/{name} includes {inc}")
    return bad


def test_includes_respect_the_layering():
    bad = layering_violations()
    assert not bad, "\n".join(bad)


def test_the_checker_rejects_a_forbidden_dependency(tmp_path):
    """The checker itself is exercised on a fixture tree: the wire-format layer including the
    control plane, and the client API including the GPU executor, must both be reported
    (reference: tests/integration/forbidden_dependency/ against check_module_boundaries.py)."""
    (tmp_path / "queue").mkdir()
    (tmp_path / "api").mkdir()
    (tmp_path / "queue" / "ring.cpp").write_text('#include "control/service.hpp"\n#include <vector>\n')
    (tmp_path / "api" / "runtime.cpp").write_text('#include "gpu/executor.hpp"\n#include "queue/ring.hpp"\n')
    bad = layering_violations(str(tmp_path))
    assert sorted(bad) == ["csrc/api/runtime.cpp includes gpu/executor.hpp",
                           "csrc/queue/ring.cpp includes control/service.hpp"]


def test_wire_and_control_layers_do_not_include_cuda():
    bad = []
    for layer, name, incs in _sources():
        if layer in NO_CUDA:
            bad += [f"csrc/{layer}/{name} includes {i}" for i in incs if i.startswith("cuda") or i == "cuda.h"]
    assert not bad, "\n".join(bad)
