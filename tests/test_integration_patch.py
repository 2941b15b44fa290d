"""The reference-side patch of INTEGRATION.md routes the reference's own imports to this build.

The block between the `patch:begin` / `patch:end` markers of INTEGRATION.md is appended, in memory,
to the reference's atlas/core.py (the checkout is only read); the patched module must then export
this build's Atlas / AtlasConfig / BatchCtx, the reference's other modules (atlas.data imports
pack_tok from atlas.core) must still import, and PROTEUS_B200=0 must keep the reference's classes.
Runs on CPU; skipped where the reference checkout is absent.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

from oracle.build_ref import reference_root

ROOT = Path(__file__).resolve().parents[1]

_PROBE = r'''
import os, sys, types
ref, patch = sys.argv[1], sys.argv[2]
pkg = types.ModuleType("atlas")
pkg.__path__ = [os.path.join(ref, "atlas")]
sys.modules["atlas"] = pkg
path = os.path.join(ref, "atlas", "core.py")
src = open(path).read() + "\n" + patch + "\n"
mod = types.ModuleType("atlas.core")
mod.__package__ = "atlas"
mod.__file__ = path
sys.modules["atlas.core"] = mod
exec(compile(src, path, "exec"), mod.__dict__)
import atlas.data  # the reference's other modules import from the patched core
import proteus_b200.core as pc
print("B200" if (mod.Atlas is pc.Atlas and mod.AtlasConfig is pc.AtlasConfig and mod.BatchCtx is pc.BatchCtx)
      else "REFERENCE", mod.pack_tok is atlas.data.pack_tok)
'''


def _patch_text() -> str:
    text = (ROOT / "INTEGRATION.md").read_text()
    m = re.search(r"<!-- patch:begin -->\s*```python\n(.*?)```\s*<!-- patch:end -->", text, re.S)
    assert m, "INTEGRATION.md lost its patch markers"
    return m.group(1)


def _run(env_extra):
    ref = reference_root()
    if ref is None:
        pytest.skip("reference checkout not on this machine")
    env = dict(os.environ, PYTHONPATH=str(ROOT), **env_extra)
    r = subprocess.run([sys.executable, "-c", _PROBE, str(ref), _patch_text()], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    return r.stdout.split()


def test_patch_at_end_of_reference_core_routes_to_b200():
    assert _run({}) == ["B200", "True"]


def test_patch_can_be_switched_off():
    assert _run({"PROTEUS_B200": "0"}) == ["REFERENCE", "True"]
