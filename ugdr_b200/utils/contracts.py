"""Client-contract checker: the public C surface, as reviewed, against the tree.

    python -m ugdr_b200.utils.contracts [--root DIR] [--no-exports]

The manifest (`docs/contracts.json`) is the reviewed inventory of the client contract:

  * `headers`: every public header and the exact set of `ugdr_*` functions it declares;
  * `compatible_symbols`: the reference's public functions, which must all stay declared (the
    verbs-shaped ABI is kept source compatible);
  * `documentation`: the API document in which every declared function must be named;
  * `library`: the built shared library, whose dynamic symbol table must export every declared
    function with C linkage (checked when the library exists, skipped otherwise).

The check also requires that `make install` ships every manifest header, so an installed
consumer gets every declaration the library exports.  It never changes the tree; it prints one
line per violation and exits 1 if there is any.

Parity: the reference's tools/check_client_contracts.py with tools/client-contracts.json (a
reviewed symbol inventory matched against its public header, plus required contract documents).
The checks here are written for this tree's layout: several headers, an installed-header list in
the Makefile, and the exported-symbol table of the built library.
"""
from __future__ import annotations

import argparse
import json
import re
import shutil
import subprocess
import sys
from pathlib import Path

FIELDS = {"schema_version", "library", "documentation", "compatible_symbols", "headers"}
_DECL = re.compile(r"\b(ugdr_[a-z0-9_]+)\s*\([^;{]*\)\s*(?:noexcept\s*)?(?:UGDR_[A-Z_]*NOEXCEPT\s*)?;")
_COMMENT = re.compile(r"/\*.*?\*/|//[^\n]*", re.S)


def declared(header_text: str) -> set[str]:
    """`ugdr_*` function declarations of a C header (comments stripped)."""
    return set(_DECL.findall(_COMMENT.sub("", header_text)))


def _rel(root: Path, value, field: str, errors: list[str]) -> Path | None:
    if not isinstance(value, str) or not value or Path(value).is_absolute():
        errors.append(f"{field} must be a repository-relative path")
        return None
    p = (root / value).resolve()
    try:
        p.relative_to(root.resolve())
    except ValueError:
        errors.append(f"{field} leaves the repository: {value}")
        return None
    return p


def exported_symbols(lib: Path) -> set[str] | None:
    nm = shutil.which("nm")
    if nm is None or not lib.exists():
        return None
    out = subprocess.run([nm, "-D", "--defined-only", str(lib)], capture_output=True, text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if ln.split()[-2:-1] == ["T"]}


def check(root: Path, manifest: dict, check_exports: bool = True) -> list[str]:
    errors: list[str] = []
    keys = set(manifest)
    errors += [f"manifest missing field: {k}" for k in sorted(FIELDS - keys)]
    errors += [f"manifest has unknown field: {k}" for k in sorted(keys - FIELDS)]
    if keys != FIELDS:
        return errors
    if manifest["schema_version"] != 1:
        errors.append("schema_version must be 1")

    headers = manifest["headers"]
    if not isinstance(headers, dict) or not headers:
        return errors + ["headers must be a non-empty object"]
    all_declared: set[str] = set()
    for rel, listed in headers.items():
        p = _rel(root, rel, f"headers[{rel!r}]", errors)
        if p is None:
            continue
        if not p.is_file():
            errors.append(f"public header is missing: {rel}")
            continue
        if not isinstance(listed, list) or not all(isinstance(s, str) for s in listed):
            errors.append(f"headers[{rel!r}] must be an array of names")
            continue
        if len(set(listed)) != len(listed):
            errors.append(f"headers[{rel!r}] lists a name twice")
        have = declared(p.read_text(encoding="utf-8"))
        errors += [f"{rel}: listed but not declared: {s}" for s in sorted(set(listed) - have)]
        errors += [f"{rel}: declared but not in the inventory: {s}" for s in sorted(have - set(listed))]
        dup = have & all_declared
        errors += [f"{rel}: declared in more than one public header: {s}" for s in sorted(dup)]
        all_declared |= have

    compat = manifest["compatible_symbols"]
    if not isinstance(compat, list) or not compat:
        errors.append("compatible_symbols must be a non-empty array")
    else:
        errors += [f"compatible symbol no longer declared: {s}" for s in compat if s not in all_declared]

    doc = _rel(root, manifest["documentation"], "documentation", errors)
    if doc is not None:
        if not doc.is_file():
            errors.append(f"documentation is missing: {manifest['documentation']}")
        else:
            text = doc.read_text(encoding="utf-8")
            errors += [f"not documented in {manifest['documentation']}: {s}" for s in sorted(all_declared)
                       if not re.search(r"\b" + re.escape(s) + r"\b", text)]

    makefile = root / "Makefile"
    if makefile.is_file():
        inst = [ln for ln in makefile.read_text(encoding="utf-8").splitlines() if "install -m 644" in ln]
        shipped = set(re.findall(r"(include/ugdr/[A-Za-z0-9_.]+)", " ".join(inst)))
        errors += [f"make install does not ship public header: {h}" for h in sorted(set(headers) - shipped)]
        errors += [f"make install ships a header outside the inventory: {h}" for h in sorted(shipped - set(headers))]
    else:
        errors.append("Makefile is missing")

    if check_exports:
        lib = _rel(root, manifest["library"], "library", errors)
        exp = exported_symbols(lib) if lib is not None else None
        if exp is not None:
            errors += [f"declared but not exported by {manifest['library']}: {s}" for s in sorted(all_declared - exp)]
    return errors


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--root", default=str(Path(__file__).resolve().parents[2]))
    ap.add_argument("--manifest", default="docs/contracts.json")
    ap.add_argument("--no-exports", action="store_true", help="skip the library's symbol table")
    args = ap.parse_args(argv)
    root = Path(args.root)
    try:
        manifest = json.loads((root / args.manifest).read_text(encoding="utf-8"))
    except (OSError, json.JSONDecodeError) as e:
        print(f"cannot read manifest: {e}")
        return 1
    errs = check(root, manifest, check_exports=not args.no_exports)
    for e in errs:
        print(e)
    if not errs:
        print("client contracts: ok")
    return 1 if errs else 0


if __name__ == "__main__":
    sys.exit(main())
