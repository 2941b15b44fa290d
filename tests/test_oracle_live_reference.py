"""The oracle against the reference itself, live on the CPU. The reference's own Atlas
(atlas/core.py, byte-compiled into oracle/_ref; backend torch, stats v1, merge loop, device cpu)
and oracle/atlas_np.py are driven over the same randomised streams and must agree on every exact
field (ids, keys, values, bin masses, contingencies, counts) and on the moments within the
reference's 1e-6, for configurations the golden fixtures do not cover: overflowing layers (the
reference's dense redo), few bins, reservoir or subsample switched off, early-layer capacity,
values on a grid (ties broken by token id), seeded thresholds. Skipped where oracle/_ref has not
been built (it needs the reference checkout)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import atlas_np as O
from tests.harness import compare, drive
from tests.streams import make_stream, pilot_edges_np

CASES = {
    "overflow_3bins": dict(
        stream=dict(L=2, D=32, n_seq=140, seed=21), bins=(0.5, 0.9, 0.99), seeded=False,
        cfg=dict(K=5, Kr=3, cap_frac=0.002, rho_res=0.05, rho_sub=0.3, seed=4, enrich_levels=(1, 2))),
    "seeded_grid_ties": dict(
        stream=dict(L=2, D=24, n_seq=160, seed=22, grid=0.25, shuffle_order=True),
        bins=(0.5, 0.9, 0.99, 0.999, 0.9999), seeded=True,
        cfg=dict(K=12, Kr=6, rho_res=0.03, rho_sub=0.2, seed=9)),
    "no_reservoir": dict(
        stream=dict(L=2, D=32, n_seq=120, seed=23), bins=(0.5, 0.9, 0.99, 0.999), seeded=False,
        cfg=dict(K=7, Kr=4, reservoir=False, rho_sub=0.2, seed=1, enrich_levels=(2, 3))),
    "no_subsample_early_cap": dict(
        stream=dict(L=3, D=16, n_seq=150, seed=24), bins=(0.5, 0.9, 0.99, 0.999, 0.9999), seeded=True,
        cfg=dict(K=6, Kr=5, subsample=False, gram=False, cap_frac_early=0.001, early_layers=1, rho_res=0.05,
                 seed=2)),
}


def _reference():
    try:
        from oracle.build_ref import ReferenceUnavailable, load_reference_atlas
        return load_reference_atlas()
    except Exception as e:  # noqa: BLE001  (ReferenceUnavailable or an import failure)
        pytest.skip(f"the compiled reference is not available: {e}")


def _edges(st, probs):
    E = pilot_edges_np([np.concatenate([s[l] for s in st.seqs[:50]]) for l in range(st.L)])
    full = (0.5, 0.9, 0.99, 0.999, 0.9999)
    return np.ascontiguousarray(E[..., [full.index(p) for p in probs]])


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_live_reference(name):
    rc = _reference()
    case = CASES[name]
    st = make_stream(**case["stream"])
    E = _edges(st, case["bins"])
    kw = case["cfg"]
    n_annot = 7 if kw.get("subsample", True) else 0
    orc = O.AtlasOracle(st.L, st.D, E, O.OracleConfig(**kw), n_annot=n_annot)
    ref = rc.Atlas(st.L, st.D, torch.from_numpy(E), rc.AtlasConfig(backend="torch", stats_impl="v1",
                                                                  merge_impl="loop", **kw),
                   n_annot=n_annot, device="cpu")
    if case["seeded"]:
        Hp = [np.concatenate([s[l] for s in st.seqs[:60]]) for l in range(st.L)]
        n_total = int(sum(len(s[0]) for s in st.seqs))
        ts, rk = O.pilot_seeds(Hp, E, kw["K"], kw["Kr"], n_total)
        orc.seed(ts, rk)
        ref.seed(torch.from_numpy(np.asarray(ts)), torch.from_numpy(np.asarray(rk)))
    drive(orc, st)
    drive(ref, st, to_input=lambda h: torch.from_numpy(np.asarray(h, np.float32)),
          make_ctx=lambda a, b: a.make_ctx(b.T, torch.from_numpy(b.valid_rows), torch.from_numpy(b.tok),
                                           torch.from_numpy(b.ann) if b.ann is not None else None))
    want, got = orc.result(), ref.result()
    bad = compare(got, want, gram_tol=1e-5, sum_tol=1e-6)
    assert not bad, bad
    for k in ("dense_layer_batches", "redo_layers", "top_cand", "res_cand", "compacted"):
        assert int(got["stats"][k]) == int(want["stats"][k]), (k, got["stats"][k], want["stats"][k])
    if name == "overflow_3bins":
        assert int(want["stats"]["redo_layers"]) > 0  # the case exercises the dense redo
