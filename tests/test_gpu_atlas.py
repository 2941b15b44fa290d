"""Stream-level parity on the GPU: the CUDA Atlas over the reference-exactness streams must
reproduce the reference's own results (tests/golden/stream_*.npz) and the oracle, with the
top-K and reservoir contents bit-exact as token-id sets in key order,
counts and int8 contingencies bit-exact, moments within 1e-6 (relative to the column's L1 mass),
Gram within 1e-3 relative Frobenius error."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import atlas_np as O
from tests.golden.make_golden import STREAM_CASES, STREAM_CFG, STREAM_SHAPE
from tests.harness import as_np, compare, drive, golden, gram_frobenius_rel
from tests.streams import Stream, make_stream, stream_digest

pytestmark = pytest.mark.gpu
DEV = "cuda"
EXACT_FIELDS = ["top_val", "top_tok", "res_tok", "res_key", "res_val", "sub_bin", "enr", "ann_tot", "n_seen", "n_sub",
                "res_seed_limited", "res_seed_key", "res_seeded_bins", "res_seed_limited_bins", "top_seed_short_groups"]


def torch_dtype(name):
    return torch.bfloat16 if name == "bf16" else torch.float32


def run_cuda(stream: Stream, E, cfg_kw, seeds=None, n_annot=7, batches=None):
    from proteus_b200.core import Atlas, AtlasConfig
    cfg = AtlasConfig(**cfg_kw)
    at = Atlas(stream.L, stream.D, torch.from_numpy(E), cfg, n_annot=n_annot, device=DEV)
    if seeds is not None:
        at.seed(torch.from_numpy(seeds[0]), torch.from_numpy(seeds[1]))
    dt = torch_dtype(stream.dtype)
    st = stream if batches is None else Stream(stream.L, stream.D, stream.dtype, stream.lens, stream.seqs,
                                               stream.ann_full, batches, stream.order)
    drive(at, st, to_input=lambda h: torch.from_numpy(h).to(DEV).to(dt))
    at.check_errors()
    return at


def moments_ok(got, ref_sum, ref_sq, n_sub):
    """|sum - ref| <= 1e-6 * L1 mass of the column (bounded by sqrt(n * sum x^2))."""
    scale = np.sqrt(max(n_sub, 1) * np.asarray(ref_sq, np.float64)) + 1e-12
    ds = np.abs(as_np(got["sub_sum"]) - ref_sum)
    dq = np.abs(as_np(got["sub_sq"]) - ref_sq)
    return bool((ds <= 1e-6 * scale).all() and (dq <= 1e-6 * np.asarray(ref_sq) + 1e-12).all())


@pytest.mark.parametrize("name", list(STREAM_CASES))
def test_stream_matches_reference(name):
    skw, ckw, seeded, _ = STREAM_CASES[name]
    z = golden(f"stream_{name}")
    st = make_stream(**STREAM_SHAPE, **skw)
    assert stream_digest(st) == str(z["digest"])
    seeds = (z["top_seed"], z["res_seed_key"]) if seeded else None
    at = run_cuda(st, z["E"], dict(STREAM_CFG, **ckw), seeds, STREAM_SHAPE["n_annot"])
    got = at.result()
    bad = compare(got, z, fields=EXACT_FIELDS)
    assert not bad, bad
    # the Atlas.stats counters of the reference (core.py:198-199); top_cand / res_cand are left out:
    # in dense bursts the reference counts every element tied at the K-th value, this build the top-K
    for k in ("batches", "elements", "compacted", "redo_layers", "dense_layer_batches"):
        assert got["stats"][k] == int(z["stat_" + k]), (k, got["stats"][k], int(z["stat_" + k]))
    # moments and Gram against the oracle's fp64 sums / the reference's Gram
    oc = O.OracleConfig(**STREAM_CFG, **ckw)
    oa = O.AtlasOracle(st.L, st.D, z["E"], oc, n_annot=STREAM_SHAPE["n_annot"])
    if seeded:
        oa.seed(*seeds)
    drive(oa, st)
    assert moments_ok(got, oa.sub_sum, oa.sub_sq, oa.n_sub)
    assert gram_frobenius_rel(as_np(got["gram"]), z["gram"]) < 1e-3


def test_stream_vs_offline_truth():
    """The reference's exactness checks (tests/test_exactness.py:106-152) on the CUDA atlas."""
    z = golden("stream_bf16")
    st = make_stream(**STREAM_SHAPE)
    at = run_cuda(st, z["E"], STREAM_CFG, None, STREAM_SHAPE["n_annot"])
    got = at.result()
    want = golden("offline")
    assert np.array_equal(as_np(got["top_val"]), want["top_val"])
    assert np.array_equal(as_np(got["top_tok"]), want["top_tok"])
    rk = np.where(as_np(got["res_tok"]) >= 0, as_np(got["res_key"]), np.iinfo(np.int64).max)
    assert np.array_equal(rk, want["res_key"])
    assert np.array_equal(as_np(got["sub_bin"]).astype(np.float64), want["sub_bin"])
    assert np.array_equal(as_np(got["enr"]).astype(np.float64), want["enr"])
    assert moments_ok(got, want["sub_sum"], want["sub_sq"], int(want["n_sub"]))
    rel = np.abs(as_np(got["gram"]) - want["gram"]).max() / np.abs(want["gram"]).max()
    assert rel < 1e-5, rel


def test_checkpoint_roundtrip_and_resume():
    """state_dict -> load_state_dict mid-stream, then continue: identical to an uninterrupted run
    (the reference's resume contract, tests/test_resume_merge.py:104-132, without the subprocess)."""
    from proteus_b200.core import Atlas, AtlasConfig
    z = golden("stream_bf16_seeded")
    st = make_stream(**STREAM_SHAPE)
    seeds = (z["top_seed"], z["res_seed_key"])
    full = run_cuda(st, z["E"], STREAM_CFG, seeds)
    half = len(st.batches) // 2
    a = run_cuda(st, z["E"], STREAM_CFG, seeds, batches=st.batches[:half])
    sd = a.state_dict()
    assert all((not torch.is_tensor(v)) or v.device.type == "cpu" for v in sd.values())
    b = Atlas(st.L, st.D, torch.from_numpy(z["E"]), AtlasConfig(**STREAM_CFG), n_annot=7, device=DEV)
    b.load_state_dict(sd)
    drive(b, Stream(st.L, st.D, st.dtype, st.lens, st.seqs, st.ann_full, st.batches[half:], st.order),
          to_input=lambda h: torch.from_numpy(h).to(DEV).to(torch.bfloat16))
    ga, gb = full.result(), b.result()
    for k in ("top_val", "top_tok", "res_tok", "res_key", "sub_bin", "enr", "ann_tot"):
        assert torch.equal(ga[k], gb[k]), k
    assert torch.allclose(ga["res_val"], gb["res_val"], equal_nan=True, rtol=0, atol=0)
    assert ga["n_seen"] == gb["n_seen"]


def test_dense_path_wide_layer_matches_oracle():
    """The dense path over more columns than one resident wave of CTAs (D = 1280: each CTA takes
    several columns in turn). Unseeded, so the first batch is dense in every column; later batches
    filter, and the cap sends some layer-batches back to the dense path (4 dense, 3 filtered). Every
    exact field against the oracle on the same activations."""
    st = make_stream(L=1, D=1280, n_seq=90, seed=21, dtype="bf16", n_annot=5, bmin=6, bmax=20)
    E = O.pilot_edges([st.batches[0].H[0][st.batches[0].valid_rows]])
    cfg = dict(K=8, Kr=4, rho_res=0.05, rho_sub=0.2, cap_frac=0.05, seed=13, stats_impl="v1", merge_impl="loop")
    at = run_cuda(st, E, cfg, None, n_annot=5)
    got = at.result()
    oa = O.AtlasOracle(st.L, st.D, E, O.OracleConfig(**cfg), n_annot=5)
    drive(oa, st)
    want = oa.result()
    bad = compare(got, want, fields=EXACT_FIELDS)
    assert not bad, bad
    assert got["stats"]["dense_layer_batches"] == want["stats"]["dense_layer_batches"] >= 1


def test_merge_from_matches_reference():
    """Two CUDA shards over interleaved halves, seeded from the global stream, merged with the GPU
    merge_from == the reference's merged result (tests/test_resume_merge.py:47-98)."""
    z = golden("merge_from")
    st = make_stream(L=2, D=48, n_seq=400, seed=3, dtype="bf16", n_annot=5)
    assert stream_digest(st) == str(z["digest"])
    cfg = dict(K=8, Kr=4, rho_res=0.05, rho_sub=0.2, cap_frac=0.05, seed=11, stats_impl="v1", merge_impl="loop")
    seeds = (z["top_seed"], z["res_seed_key"])
    shards = [run_cuda(st, z["E"], cfg, seeds, n_annot=5, batches=[b for i, b in enumerate(st.batches) if i % 2 == h])
              for h in (0, 1)]
    for h, at in enumerate(shards):
        for k in ("top_k", "top_t", "res_s", "res_t", "sub_bin", "enr", "ann_tot"):
            assert np.array_equal(as_np(getattr(at, k)), z[f"s{h}_{k}"]), (h, k)
    shards[0].merge_from(shards[1])
    got = shards[0].result()
    want = {k[2:]: v for k, v in z.items() if k.startswith("m_")}
    bad = compare(got, want, fields=EXACT_FIELDS)
    assert not bad, bad


def test_kernel_api_dropins_run():
    """filter_candidates / sub_stats / gram_accumulate / grouped_merge keep the reference's call
    shapes and return types."""
    from proteus_b200 import kernels as KN
    H = torch.randn(100, 64, device=DEV).to(torch.bfloat16)
    rowmap = torch.arange(100, device=DEV)
    v, r, c, cnt = KN.filter_candidates(H, rowmap, torch.full((64,), 1.0, device=DEV),
                                        torch.full((64,), 1.0, device=DEV), 4096)
    assert v.dtype == torch.float32 and r.dtype == torch.int64 and c.dtype == torch.int64 and cnt.dim() == 0
    s, sq, cn, M = KN.sub_stats(H, torch.zeros(64, 5, device=DEV), torch.zeros(64, 5, device=DEV), (2, 3, 4))
    assert s.dtype == torch.float64 and cn.dtype == torch.int32 and M.shape == (2, 3, 64, 104)


def test_make_ctx_device_equals_host_make_ctx():
    """atlas_ctx_rows / atlas_ctx_annotations give every field of the host make_ctx (core.py:210-237):
    keys, row map, subsample and bulk rows in order, key order, transposed one-hots and their totals,
    on batches with padding rows, repeated and missing (-1) annotation ids, and an empty subsample."""
    from proteus_b200.core import Atlas, AtlasConfig
    rng = np.random.default_rng(5)
    at = Atlas(1, 64, torch.zeros(1, 2, 64, 5), AtlasConfig(K=8, Kr=4, rho_res=0.05, rho_sub=0.2, seed=9), n_annot=11,
               device=DEV)
    side = torch.cuda.Stream()
    for trial, (n_seq, lmax) in enumerate([(40, 300), (7, 1000), (1, 3), (300, 60)]):
        lens = rng.integers(1, lmax - 1, n_seq)
        T = n_seq * lmax + 17
        valid = np.concatenate([r * lmax + 1 + np.arange(n) for r, n in enumerate(lens)]).astype(np.int64)
        tok = np.concatenate([(1000 * trial + r) * 1024 + np.arange(n) for r, n in enumerate(lens)]).astype(np.int64)
        ann = rng.integers(-1, 11, (valid.size, 4)).astype(np.int64)
        ann[::5, 1] = ann[::5, 0]  # a class listed twice for one row
        h = at.make_ctx(T, torch.from_numpy(valid), torch.from_numpy(tok), torch.from_numpy(ann))
        d = at.make_ctx_device(T, torch.from_numpy(valid).pin_memory(), torch.from_numpy(tok).pin_memory(),
                               torch.from_numpy(ann).pin_memory(), stream=side)
        d.ready.synchronize()
        assert (d.n_v, d.n_s, d.n_r) == (h.n_v, h.n_s, h.n_r)
        for k in ("key", "rowmap32", "valid32", "sub_rows32", "res_rows32", "res_vidx32", "key_order32", "annT",
                  "ann_counts"):
            a, b = getattr(d, k), getattr(h, k)
            assert a.shape == b.shape and torch.equal(a.cpu(), b.cpu()), (trial, k)
        assert torch.equal(d.sub_idx.cpu(), h.sub_idx.cpu()) and torch.equal(d.res_in_sub.cpu(), h.res_in_sub.cpu())


def test_stream_with_device_make_ctx_matches_reference():
    """A golden stream with every context built by make_ctx_device on a side stream (as the prefetch
    thread of run_atlas does): the reference's result, bit for bit."""
    skw, ckw, seeded, _ = STREAM_CASES["bf16_seeded"]
    z = golden("stream_bf16_seeded")
    st = make_stream(**STREAM_SHAPE, **skw)
    from proteus_b200.core import Atlas, AtlasConfig
    at = Atlas(st.L, st.D, torch.from_numpy(z["E"]), AtlasConfig(**STREAM_CFG, **ckw),
               n_annot=STREAM_SHAPE["n_annot"], device=DEV)
    at.seed(torch.from_numpy(z["top_seed"]), torch.from_numpy(z["res_seed_key"]))
    side = torch.cuda.Stream()
    drive(at, st, to_input=lambda h: torch.from_numpy(h).to(DEV).to(torch.bfloat16),
          make_ctx=lambda a, b: a.make_ctx_device(b.T, torch.from_numpy(b.valid_rows), torch.from_numpy(b.tok),
                                                  torch.from_numpy(b.ann), stream=side))
    at.check_errors()
    bad = compare(at.result(), z, fields=EXACT_FIELDS)
    assert not bad, bad
