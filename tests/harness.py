"""Shared test plumbing: drive an atlas over a stream, load golden fixtures, compare results with the
reference's tolerances (exact for ids, keys, counts and values; sums rtol=atol=1e-6 as in the
reference's tests/test_exactness.py:149-150; Gram by relative error)."""
from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
I64_MAX = np.iinfo(np.int64).max

EXACT = ["top_val", "top_tok", "res_tok", "res_key", "sub_bin", "enr", "ann_tot", "res_seed_limited", "res_seed_key"]
SCALARS = ["n_seen", "n_sub", "res_seeded_bins", "res_seed_limited_bins", "top_seed_short_groups"]


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz", allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def as_np(x):
    try:
        import torch
        if torch.is_tensor(x):
            if x.dtype == torch.bfloat16:
                x = x.float()
            return x.detach().cpu().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x)


def drive(atlas, stream, to_input=lambda h: h, make_ctx=None):
    """The reference's driver loop (tests/test_exactness.py:54-86) over a tests.streams.Stream."""
    for b in stream.batches:
        ctx = atlas.make_ctx(b.T, b.valid_rows, b.tok, b.ann) if make_ctx is None else make_ctx(atlas, b)
        Hb = [to_input(h) for h in b.H]
        atlas.begin_batch(ctx)
        for l, h in enumerate(Hb):
            atlas.observe(l, h)
        redo = atlas.end_batch()
        if redo:
            atlas.begin_batch(ctx, redo_layers=redo)
            for l, h in enumerate(Hb):
                atlas.observe(l, h)
            assert atlas.end_batch() == []


def compare(got: dict, want: dict, gram_tol=1e-5, sum_tol=1e-6, fields=None) -> list:
    """Differences between two result dicts as a list of strings (empty = equal)."""
    bad = []
    for k in EXACT:
        if k in want and (fields is None or k in fields):
            a, b = as_np(got[k]), np.asarray(want[k])
            if a.shape != b.shape or not np.array_equal(a, b):
                n = int((a != b).sum()) if a.shape == b.shape else -1
                bad.append(f"{k}: {n} entries differ")
    if "res_val" in want and (fields is None or "res_val" in fields):
        a, b = as_np(got["res_val"]), want["res_val"]
        if not np.array_equal(a, b, equal_nan=True):
            bad.append("res_val differs")
    for k in ("sub_sum", "sub_sq"):
        if k in want and (fields is None or k in fields):
            if not np.allclose(as_np(got[k]), want[k], rtol=sum_tol, atol=sum_tol):
                d = np.abs(as_np(got[k]) - want[k]).max()
                bad.append(f"{k}: max abs diff {d:.3g}")
    if "gram" in want and "gram" in got and (fields is None or "gram" in fields):
        a, b = as_np(got["gram"]).astype(np.float64), want["gram"].astype(np.float64)
        rel = float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-300))
        if not rel < gram_tol:
            bad.append(f"gram rel-max err {rel:.3g} >= {gram_tol}")
    for k in SCALARS:
        if k in want and k in got and (fields is None or k in fields):
            if int(got[k]) != int(want[k]):
                bad.append(f"{k}: {int(got[k])} != {int(want[k])}")
    return bad


def gram_frobenius_rel(got, want) -> float:
    a, b = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))
