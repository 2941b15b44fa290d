"""Bin counts other than five on the GPU. The dense kernels are compiled twice: exactly for the
reference's five edges, and once for any other count (1..8 bins, unused edges padded). Every other
GPU stream test uses five bins; here the CUDA Atlas runs three- and seven-bin streams, unseeded (the
first batch dense in every column) and seeded, with a cap that sends more layer-batches back to the
dense path, and must match the oracle on every exact field."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import atlas_np as O
from tests.harness import compare, drive
from tests.streams import make_stream
from tests.test_gpu_atlas import EXACT_FIELDS, run_cuda

pytestmark = pytest.mark.gpu

PROBS = {3: (0.5, 0.9, 0.99), 7: (0.3, 0.5, 0.7, 0.9, 0.99, 0.999, 0.9999)}


@pytest.mark.parametrize("bins,seeded", [(3, False), (7, True)])
def test_stream_with_other_bin_counts_matches_oracle(bins, seeded):
    st = make_stream(L=2, D=160, n_seq=70, seed=31 + bins, dtype="bf16", n_annot=5, bmin=6, bmax=18)
    E = O.pilot_edges([np.concatenate([s[l] for s in st.seqs[:25]]) for l in range(st.L)], probs=PROBS[bins])
    levels = (1, 2) if bins == 3 else (2, 4, 6)
    cfg = dict(K=6, Kr=3, rho_res=0.05, rho_sub=0.2, cap_frac=0.02, seed=5, enrich_levels=levels,
               stats_impl="v1", merge_impl="loop")
    seeds = None
    if seeded:
        Hp = [np.concatenate([s[l] for s in st.seqs[:25]]) for l in range(st.L)]
        seeds = O.pilot_seeds(Hp, E, cfg["K"], cfg["Kr"], int(sum(len(s[0]) for s in st.seqs)))
        seeds = (np.asarray(seeds[0]), np.asarray(seeds[1]))
    at = run_cuda(st, E, cfg, seeds, n_annot=5)
    got = at.result()
    oa = O.AtlasOracle(st.L, st.D, E, O.OracleConfig(**cfg), n_annot=5)
    if seeded:
        oa.seed(*seeds)
    drive(oa, st)
    want = oa.result()
    bad = compare(got, want, fields=EXACT_FIELDS)
    assert not bad, bad
    assert got["stats"]["dense_layer_batches"] == want["stats"]["dense_layer_batches"] >= 1
