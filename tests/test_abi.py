"""CPU checks of the C ABI boundary: the in-tree library loads and exports every symbol that
include/proteus_atlas.h declares, with the binding derived from the header (no compute calls)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

from proteus_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def test_header_declares_and_library_exports_every_symbol():
    lib = _lib.load()
    names = set(_lib.SIGNATURES)
    text = (ROOT / "include" / "proteus_atlas.h").read_text()
    declared = set(re.findall(r"\b(atlas_\w+)\s*\(", re.sub(r"/\*.*?\*/", " ", text, flags=re.S)))
    assert declared == names, declared ^ names
    for n in names:
        assert hasattr(lib, n), n
    assert lib.atlas_abi_version() >= 1


def test_argument_errors_are_reported_without_a_gpu():
    lib = _lib.load()
    # T < 0 is rejected on the host before any CUDA call
    rc = lib.atlas_filter_compact(None, 1, -1, 8, 8, None, None, None, None, None, None, None, 0, None)
    assert rc == 1
    assert b"bad shape" in lib.atlas_last_error()
    rc = lib.atlas_grouped_merge(None, None, None, 10, 300, None, None, None, None, None, 5, None, None, None)
    assert rc == 1 and b"K must be" in lib.atlas_last_error()


def test_dense_select_rejects_out_of_range_shapes_on_the_host():
    """atlas_dense_select checks its limits before any CUDA call: 1..8 bins, K and Kr up to 256, the
    staging bound 2K + 2*B*Kr <= 1024, at most 64 x 65535 valid rows (16-bit per-thread counts over
    at most 64 row ranges) and at most 65536 columns (256 strips of 256)."""
    lib = _lib.load()

    def call(T=1000, D=512, n_v=1000, B=5, K=100, Kr=32):
        args = [None, 1, T, D, D, 0, None, n_v, None, None, None, B, K, Kr, 1] + [None] * 6 + [0, 1] + \
               [None] * 5 + [0] + [None] * 5 + [0, None, 0, None, None, None]
        return lib.atlas_dense_select(*args)

    assert call(B=9) == 1 and b"B must be" in lib.atlas_last_error()
    assert call(K=300) == 1
    assert call(K=200, Kr=100) == 1 and b"staging area" in lib.atlas_last_error()
    assert call(T=64 * 65535 + 1, n_v=64 * 65535 + 1) == 1 and b"valid rows" in lib.atlas_last_error()
    assert call(D=65536 + 256) == 1 and b"D above" in lib.atlas_last_error()
    assert call(n_v=2000) == 1 and b"bad shape" in lib.atlas_last_error()  # more valid rows than rows


def test_workspace_size_queries():
    lib = _lib.load()
    assert lib.atlas_merge_ws_i32(4096, 100) >= 4 * 4096
    assert lib.atlas_merge_ws_bytes(1000) >= 20 * 1000
    # per-range partial counts (64 ranges x 18 counts x D), decisions, hard-column lists, keys in key order
    assert lib.atlas_dense_scratch_bytes(32768, 5120, 5, 1) >= 64 * 18 * 5120 * 4 + 32768 * 4
    assert lib.atlas_dense_scratch_bytes(65536, 5120, 5, 1) > lib.atlas_dense_scratch_bytes(32768, 5120, 5, 1)


def test_product_refuses_cpu_device():
    import pytest
    import torch

    from proteus_b200.core import Atlas, AtlasConfig
    from proteus_b200._lib import AtlasKernelError
    with pytest.raises(AtlasKernelError):
        Atlas(1, 8, torch.zeros(1, 2, 8, 5), AtlasConfig(), device="cpu")
