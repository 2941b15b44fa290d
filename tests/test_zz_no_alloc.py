"""The allocation-free grouped merge (atlas_grouped_merge_static) gives the same result as the
regular one (atlas_grouped_merge with a caller-provided workspace).

Some callers cannot allocate device memory — a host runtime that owns every device byte through its
own pool, or a call site that must not trigger cudaMalloc's implicit synchronisation — so the library
offers a merge whose workspace is a fixed array inside the library. This test calls it through the
C ABI, twice in a row on the same state (the second call runs on whatever the first left in the
shared array), and compares every output slot with the regular entry point's, exactly: merges of
integer keys have no tolerance. It sits in its own file, collected last, and works both alone in a
fresh process and after the rest of the suite.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
I64_MIN = torch.iinfo(torch.int64).min


def _state(G, K):
    return (torch.full((G, K), I64_MIN, dtype=torch.long, device=DEV),
            torch.full((G, K), -1, dtype=torch.long, device=DEV),
            torch.full((G, K), float("-inf"), device=DEV))


def _candidates(rng, G, n):
    g = torch.from_numpy(rng.integers(0, G, n).astype(np.int32)).to(DEV)
    sc = torch.from_numpy(rng.choice(2**50, n, replace=False).astype(np.int64) - 2**49).to(DEV)
    tok = torch.from_numpy(rng.integers(0, 2**32, n)).to(DEV)
    val = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(DEV)
    return g, sc, tok, val


@pytest.mark.parametrize("G,K,n", [(500, 100, 40000), (4096, 32, 100000), (37, 8, 300)])
def test_static_workspace_merge_equals_workspace_merge(G, K, n):
    from proteus_b200 import _lib
    from proteus_b200 import kernels as KN
    lib = _lib.load()
    rng = np.random.default_rng(G + K)
    ref = _state(G, K)
    got = _state(G, K)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # two calls in a row: the shared array keeps the first call's contents
        g, sc, tok, val = _candidates(rng, G, n)
        n_dev = torch.tensor([n], dtype=torch.int32, device=DEV)
        KN.grouped_merge_records(ref[0], ref[1], ref[2], K, g, sc, tok, val, n_dev, n)
        rc = lib.atlas_grouped_merge_static(got[0].data_ptr(), got[1].data_ptr(), got[2].data_ptr(), G, K,
                                            g.data_ptr(), sc.data_ptr(), tok.data_ptr(), val.data_ptr(),
                                            n_dev.data_ptr(), n, stream)
        assert rc == 0, lib.atlas_last_error()
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)


def test_static_workspace_rejects_oversized_requests():
    from proteus_b200 import _lib
    lib = _lib.load()
    rc = lib.atlas_grouped_merge_static(None, None, None, 1 << 20, 8, None, None, None, None, None, 10, None)
    assert rc == 1 and b"exceeds the static workspace limit" in lib.atlas_last_error()
    rc = lib.atlas_grouped_merge_static(None, None, None, 64, 8, None, None, None, None, None, 1 << 20, None)
    assert rc == 1 and b"exceeds the static workspace limit" in lib.atlas_last_error()
