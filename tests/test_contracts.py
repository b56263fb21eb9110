"""Client-contract governance (reference: tools/check_client_contracts.py and its manifest).

The tree passes its own manifest, and a copy of the tree with each kind of drift fails with the
matching message: an undeclared inventory entry, a new undocumented declaration, a dropped
compatible symbol, a header that `make install` does not ship, and a malformed manifest."""
from __future__ import annotations

import json
import shutil
from pathlib import Path

from ugdr_b200.utils import contracts as K

REPO = Path(__file__).resolve().parents[1]


def _manifest(root: Path) -> dict:
    return json.loads((root / "docs" / "contracts.json").read_text())


def _fixture(tmp_path: Path) -> Path:
    root = tmp_path / "tree"
    shutil.copytree(REPO / "include", root / "include")
    (root / "docs").mkdir(parents=True)
    shutil.copy(REPO / "docs" / "API.md", root / "docs" / "API.md")
    shutil.copy(REPO / "docs" / "contracts.json", root / "docs" / "contracts.json")
    shutil.copy(REPO / "Makefile", root / "Makefile")
    return root


def test_tree_satisfies_its_contract_manifest():
    errs = K.check(REPO, _manifest(REPO), check_exports=True)
    assert errs == [], errs


def test_fixture_copy_passes_then_each_drift_is_reported(tmp_path):
    root = _fixture(tmp_path)
    m = _manifest(root)
    assert K.check(root, m, check_exports=False) == []

    # A new declaration that is neither inventoried nor documented.
    h = root / "include" / "ugdr" / "collective.h"
    text = h.read_text()
    h.write_text(text.replace("#ifdef __cplusplus\n}", "int ugdr_x_new_thing(int a);\n#ifdef __cplusplus\n}", 1))
    errs = K.check(root, m, check_exports=False)
    assert any("declared but not in the inventory: ugdr_x_new_thing" in e for e in errs), errs
    assert any("not documented in docs/API.md: ugdr_x_new_thing" in e for e in errs), errs
    h.write_text(text)

    # An inventory entry the header does not declare.
    m2 = json.loads(json.dumps(m))
    m2["headers"]["include/ugdr/api.hpp"].append("ugdr_x_gone")
    assert any("listed but not declared: ugdr_x_gone" in e for e in K.check(root, m2, check_exports=False))

    # A reference-compatible function removed from the header.
    a = root / "include" / "ugdr" / "api.hpp"
    atext = a.read_text()
    a.write_text(atext.replace("ugdr_post_recv(", "ugdr_post_recv_renamed("))
    errs = K.check(root, m, check_exports=False)
    assert any("compatible symbol no longer declared: ugdr_post_recv" in e for e in errs), errs
    a.write_text(atext)

    # A public header that make install would not ship.
    mk = root / "Makefile"
    mtext = mk.read_text()
    mk.write_text(mtext.replace(" include/ugdr/route_noalloc.h", ""))
    errs = K.check(root, m, check_exports=False)
    assert any("does not ship public header: include/ugdr/route_noalloc.h" in e for e in errs), errs
    mk.write_text(mtext)

    # Malformed manifests.
    bad = dict(m)
    bad.pop("documentation")
    bad["extra"] = 1
    errs = K.check(root, bad, check_exports=False)
    assert "manifest missing field: documentation" in errs and "manifest has unknown field: extra" in errs
    esc = dict(m, documentation="../outside.md")
    assert any("leaves the repository" in e for e in K.check(root, esc, check_exports=False))


def test_cli_exit_codes(tmp_path, capsys):
    assert K.main(["--no-exports"]) == 0
    root = _fixture(tmp_path)
    (root / "docs" / "API.md").write_text("# empty\n")
    assert K.main(["--root", str(root), "--no-exports"]) == 1
    assert "not documented" in capsys.readouterr().out
