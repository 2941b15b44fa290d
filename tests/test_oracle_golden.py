"""The CPU oracle (oracle/atlas_np.py) reproduces the reference implementation's own outputs
(tests/golden/*.npz, made by tests/golden/make_golden.py from the reference package)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import atlas_np as O
from tests.golden.make_golden import N_PILOT, STREAM_CASES, STREAM_CFG, STREAM_SHAPE
from tests.harness import compare, drive, golden
from tests.streams import make_stream, pilot_edges_np, stream_digest


def test_token_keys_golden():
    z = golden("keys")
    for seed in (0, 7, 0x1_0000_0005):
        assert np.array_equal(O.token_keys(z["tok"], seed), z[f"keys_seed{seed}"])


def test_top_key_golden():
    z = golden("keys")
    assert np.array_equal(O.top_key(z["s"], z["s_tok"]), z["top_key"])


def test_grouped_merge_golden():
    z = golden("grouped_merge")
    for case in range(3):
        G, K, rounds = (int(x) for x in z[f"c{case}_meta"])
        st = np.full((G, K), O.I64_MIN, np.int64)
        pt = np.full((G, K), -1, np.int64)
        pv = np.full((G, K), -np.inf, np.float32)
        for r in range(rounds):
            O.grouped_merge(st, [pt, pv], z[f"c{case}_r{r}_g"], z[f"c{case}_r{r}_s"],
                            [z[f"c{case}_r{r}_t"], z[f"c{case}_r{r}_v"]], K, pay_fill=[-1, -np.inf])
        assert np.array_equal(st, z[f"c{case}_state"])
        assert np.array_equal(pt, z[f"c{case}_tok"])
        assert np.array_equal(pv, z[f"c{case}_val"])


def test_stream_edges_match_reference_pilot():
    """pilot_edges_np (used to seed test streams) == the reference's pilot_edges."""
    st = make_stream(**STREAM_SHAPE)
    Hp = [np.concatenate([s[l] for s in st.seqs[:N_PILOT]]) for l in range(st.L)]
    assert np.array_equal(pilot_edges_np(Hp), golden("stream_bf16")["E"])


def _oracle_case(name):
    skw, ckw, seeded, _ = STREAM_CASES[name]
    z = golden(f"stream_{name}")
    st = make_stream(**STREAM_SHAPE, **skw)
    assert stream_digest(st) == str(z["digest"]), "stream rebuild differs from the fixture's"
    cfg = O.OracleConfig(**STREAM_CFG, **ckw)
    at = O.AtlasOracle(st.L, st.D, z["E"], cfg, n_annot=STREAM_SHAPE["n_annot"])
    if seeded:
        at.seed(z["top_seed"], z["res_seed_key"])
    drive(at, st)
    return at, at.result(), z


@pytest.mark.parametrize("name", list(STREAM_CASES))
def test_oracle_stream_matches_reference(name):
    at, got, z = _oracle_case(name)
    bad = compare(got, z)
    assert not bad, bad
    for k in ("batches", "dense_layer_batches", "redo_layers", "compacted", "elements", "top_cand", "res_cand"):
        assert got["stats"][k] == int(z["stat_" + k]), (k, got["stats"][k], int(z["stat_" + k]))


def test_oracle_offline_reference_matches():
    st = make_stream(**STREAM_SHAPE)
    z = golden("stream_bf16")
    Hall, toks, A = st.all_tokens()
    annf = np.zeros((toks.size, STREAM_SHAPE["n_annot"]), np.float32)
    r, c = np.nonzero(A >= 0)
    annf[r, A[r, c]] = 1
    ref = O.offline_reference(Hall, toks, z["E"], STREAM_CFG["K"], STREAM_CFG["Kr"], STREAM_CFG["rho_sub"],
                              STREAM_CFG["seed"], ann=annf)
    want = golden("offline")
    for k in ("top_val", "top_tok", "res_key", "res_tok", "sub_bin", "enr"):
        assert np.array_equal(ref[k], want[k]), k
    assert np.array_equal(ref["res_val"], want["res_val"], equal_nan=True)
    assert ref["n_sub"] == int(want["n_sub"])
    for k in ("sub_sum", "sub_sq", "gram"):
        assert np.allclose(ref[k], want[k], rtol=1e-9, atol=1e-9), k


def test_streamed_oracle_equals_offline_truth():
    """The reference's own exactness check (tests/test_exactness.py:106-152) on the oracle."""
    at, got, z = _oracle_case("bf16")
    want = golden("offline")
    assert np.array_equal(got["top_val"], want["top_val"])
    assert np.array_equal(got["top_tok"], want["top_tok"])
    rk = np.where(got["res_tok"] >= 0, got["res_key"], np.iinfo(np.int64).max)
    assert np.array_equal(rk, want["res_key"])
    assert np.array_equal(got["res_tok"], want["res_tok"])
    assert np.array_equal(got["sub_bin"].astype(np.float64), want["sub_bin"])
    assert np.array_equal(got["enr"].astype(np.float64), want["enr"])
    assert np.allclose(got["sub_sum"], want["sub_sum"], rtol=1e-6, atol=1e-6)
    rel = np.abs(got["gram"] - want["gram"]).max() / np.abs(want["gram"]).max()
    assert rel < 1e-5


def test_oracle_merge_from_matches_reference():
    z = golden("merge_from")
    from tests.streams import Stream
    st = make_stream(L=2, D=48, n_seq=400, seed=3, dtype="bf16", n_annot=5)
    assert stream_digest(st) == str(z["digest"])
    cfg = O.OracleConfig(K=8, Kr=4, rho_res=0.05, rho_sub=0.2, cap_frac=0.05, seed=11)
    shards = []
    for half in (0, 1):
        sub = Stream(st.L, st.D, st.dtype, st.lens, st.seqs, st.ann_full,
                     [b for i, b in enumerate(st.batches) if i % 2 == half], st.order)
        at = O.AtlasOracle(st.L, st.D, z["E"], cfg, n_annot=5)
        at.seed(z["top_seed"], z["res_seed_key"])
        drive(at, sub)
        for k in O.AtlasOracle._STATE + ["enr", "ann_tot"]:
            a = getattr(at, k)
            if k in ("sub_sum", "sub_sq"):  # fp32 batch sums in the reference: its sum tolerance
                assert np.allclose(a, z[f"s{half}_{k}"], rtol=1e-5, atol=1e-4), k
            else:
                assert np.array_equal(a, z[f"s{half}_{k}"], equal_nan=True), (half, k)
        shards.append(at)
    shards[0].merge_from(shards[1])
    got = shards[0].result()
    want = {k[2:]: v for k, v in z.items() if k.startswith("m_")}
    bad = compare(got, want)
    assert not bad, bad


def test_oracle_pilot_math_matches_reference():
    from tests.streams import pilot_inputs
    Hs, _ = pilot_inputs()
    z = golden("pilot")
    E = O.pilot_edges(Hs)
    assert np.array_equal(E, z["E"])
    ts, rk = O.pilot_seeds(Hs, E, 16, 8, n_total=10**6)
    assert np.array_equal(ts, z["top_seed_nogroups"]) and np.array_equal(rk, z["res_seed_key_nogroups"])
