"""Build recipe for oracle/_ref: the reference's own `atlas` package in compiled form.

TEST INFRASTRUCTURE. Only tests/, __graft_entry__ (build, smoke) and bench.py's CPU baseline legs
use this module; the product path never does.

The reference (haelyons/proteus) is Python. The Python analogue of compiling a C reference from its
sources into a binary is byte-compiling its modules: `build()` compiles the hot-path modules of the
reference's `atlas/` package, where they lie in the reference checkout, into sourceless bytecode
files oracle/_ref/atlas/<module>.bytecode (the .pyc format under another suffix, since snapshots of
the repository leave .pyc files behind), which `load_reference_atlas` imports through a path finder
of its own. No source file is copied. oracle/_ref/ is git-ignored, so nothing of it
enters the history, but it is not excluded from the GPU-box snapshot, so the reference's own CPU
implementation can run there: as the timed reference arm of bench.py and as the second sink of the
dual-sink parity tests. The bytecode is tied to the interpreter version that built it (the GPU box
runs the same image); a mismatch makes `load_reference_atlas` raise ReferenceUnavailable.

  python -m oracle.build_ref [--ref <reference checkout>]

The reference checkout is found from --ref, the PROTEUS_REF environment variable, or the
`reference_path` recorded in BASELINE.json.
"""
from __future__ import annotations

import argparse
import importlib
import importlib.abc
import importlib.machinery
import importlib.util
import json
import os
import py_compile
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
OUT = Path(__file__).resolve().parent / "_ref"
# the reference modules on the hot path (atlas/__init__.py is empty); ruler / seqbaseline are out of scope
MODULES = ("__init__", "core", "reference", "data", "esm", "filter_triton", "stats_triton", "proftrace")


class ReferenceUnavailable(RuntimeError):
    pass


def reference_root(ref: str | os.PathLike | None = None) -> Path | None:
    """The reference checkout, or None when it is not on this machine."""
    cands = [ref, os.environ.get("PROTEUS_REF")]
    bj = ROOT / "BASELINE.json"
    if bj.exists():
        try:
            cands.append(json.loads(bj.read_text()).get("reference_path"))
        except (ValueError, OSError):
            pass
    for c in cands:
        if c and (Path(c) / "atlas" / "core.py").exists():
            return Path(c)
    return None


SUFFIX = ".bytecode"


def build(ref: str | os.PathLike | None = None, out: Path = OUT) -> Path | None:
    """Byte-compile the reference's hot-path modules into out/atlas/. Returns out, or None when the
    reference checkout is absent (then an earlier build, if any, is left as it is)."""
    root = reference_root(ref)
    if root is None:
        return None
    pkg = out / "atlas"
    pkg.mkdir(parents=True, exist_ok=True)
    for m in MODULES:
        src = root / "atlas" / f"{m}.py"
        if not src.exists():
            continue
        py_compile.compile(str(src), cfile=str(pkg / f"{m}{SUFFIX}"), dfile=f"atlas/{m}.py", doraise=True,
                           invalidation_mode=py_compile.PycInvalidationMode.UNCHECKED_HASH)
    (out / "BUILT_FROM").write_text(f"python {sys.version.split()[0]}\nmodules {' '.join(MODULES)}\n")
    return out


def available(out: Path = OUT) -> bool:
    return (out / "atlas" / f"core{SUFFIX}").exists()


class _CompiledReferenceFinder(importlib.abc.MetaPathFinder):
    """Finds `atlas` and `atlas.<module>` among the compiled files of oracle/_ref."""

    def __init__(self, out: Path):
        self.pkg = out / "atlas"

    def find_spec(self, fullname, path=None, target=None):
        if fullname != "atlas" and not fullname.startswith("atlas."):
            return None
        leaf = "__init__" if fullname == "atlas" else fullname.split(".", 1)[1]
        f = self.pkg / f"{leaf}{SUFFIX}"
        if "." in leaf or not f.exists():
            return None
        loader = importlib.machinery.SourcelessFileLoader(fullname, str(f))
        return importlib.util.spec_from_file_location(
            fullname, str(f), loader=loader, submodule_search_locations=[str(self.pkg)] if leaf == "__init__" else None)


_FINDER: _CompiledReferenceFinder | None = None


def load_reference_atlas(out: Path = OUT):
    """Import the compiled reference package and return its `atlas.core` module. Raises
    ReferenceUnavailable when oracle/_ref has not been built or was built by another interpreter."""
    global _FINDER
    if not available(out):
        raise ReferenceUnavailable("oracle/_ref has not been built (python -m oracle.build_ref, needs the reference)")
    mod = sys.modules.get("atlas.core")
    if mod is not None and str(getattr(mod, "__file__", "")).startswith(str(out)):
        return mod
    if "atlas" in sys.modules and not str(getattr(sys.modules["atlas"], "__file__", "")).startswith(str(out)):
        raise ReferenceUnavailable("another package named 'atlas' is already imported")
    if _FINDER is None:
        _FINDER = _CompiledReferenceFinder(out)
        sys.meta_path.insert(0, _FINDER)
    try:
        return importlib.import_module("atlas.core")
    except ImportError as e:  # bad magic number (other interpreter) and the like
        raise ReferenceUnavailable(f"compiled reference cannot be imported: {e}") from e


def load_reference_module(name: str, out: Path = OUT):
    """Another module of the compiled reference package (e.g. "reference", "data")."""
    load_reference_atlas(out)
    return importlib.import_module(f"atlas.{name}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None)
    a = ap.parse_args()
    out = build(a.ref)
    print(out if out else "reference checkout not found: nothing built")


if __name__ == "__main__":
    main()
