"""BASELINE config 0 (ESM-2 8M, 512 synthetic sequences, K=16, Kr=8, seeded from a 64-sequence
pilot, stats v1 + merge loop) — the exactness case, on the real ESM forward.

* CPU (set RUN_SLOW=1; ~10 min): the oracle over the CPU fp32 forward reproduces the reference's
  own result (tests/golden/c1_esm8m.npz, exact fields compared by sha256), and the oracle's pilot
  math reproduces the reference's edges and seeds on the real activations.
* GPU: the same forward on cuda:0, all 512 sequences, feeds the CUDA atlas, the oracle and the
  reference's own Atlas (compiled into oracle/_ref) from the same hook; every exact field must agree
  bit for bit, moments to 1e-6, Gram to 1e-3 Frobenius.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import atlas_np as O
from tests.c1 import C1, build_model, c1_batches, c1_sequences, forward_layers
from tests.golden.make_golden import C1_DIGEST_FIELDS, digest
from tests.harness import as_np, compare, golden, gram_frobenius_rel


def _pilot_edges_seeds(Hp, prot, n_total):
    """Edges and seeds: on the device pilot kernels for CUDA activations, the oracle's pilot math
    (pinned to the reference's) for CPU ones."""
    if Hp[0].is_cuda:
        from proteus_b200.pilot import pilot_edges, pilot_seeds
        E = torch.cat([pilot_edges([h]) for h in Hp])
        parts = [pilot_seeds([h], E[li:li + 1], C1["K"], C1["Kr"], n_total, groups=prot) for li, h in enumerate(Hp)]
        return E.cpu(), torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts])
    E = O.pilot_edges([h.numpy() for h in Hp])
    ts, rk = O.pilot_seeds([h.numpy() for h in Hp], E, C1["K"], C1["Kr"], n_total, groups=prot.numpy())
    return torch.from_numpy(E), torch.from_numpy(ts), torch.from_numpy(rk)


@pytest.mark.skipif(os.environ.get("RUN_SLOW") != "1", reason="~10 min on 8 cores; set RUN_SLOW=1")
def test_c1_oracle_matches_reference_on_cpu_forward():
    torch.set_num_threads(1)  # the fixture's forward ran single-threaded (bitwise-stable activations)
    z = golden("c1_esm8m")
    model = build_model()
    seqs = c1_sequences()
    Hp, prot = [[] for _ in range(C1["L"])], []
    for b in c1_batches(seqs, list(range(C1["n_pilot"]))):
        Hs = forward_layers(model, b)
        for l in range(C1["L"]):
            Hp[l].append(torch.from_numpy(Hs[l][b.valid_rows]))
        prot.append(torch.from_numpy(b.tok // 1024))
    Hp = [torch.cat(h) for h in Hp]
    E, ts, rk = _pilot_edges_seeds(Hp, torch.cat(prot), int(sum(len(s) for s in seqs)))
    assert np.array_equal(E.numpy(), z["E"]) and np.array_equal(ts.numpy(), z["top_seed"])
    cfg = O.OracleConfig(K=C1["K"], Kr=C1["Kr"], seed=0)
    at = O.AtlasOracle(C1["L"], C1["D"], E.numpy(), cfg, n_annot=C1["n_annot"])
    at.seed(ts.numpy(), rk.numpy())
    for b in c1_batches(seqs, list(range(len(seqs)))):
        Hs = forward_layers(model, b)
        ctx = at.make_ctx(b.T, b.valid_rows, b.tok, b.ann)
        at.begin_batch(ctx)
        for l in range(C1["L"]):
            at.observe(l, Hs[l])
        redo = at.end_batch()
        if redo:
            at.begin_batch(ctx, redo_layers=redo)
            for l in range(C1["L"]):
                at.observe(l, Hs[l])
            at.end_batch()
    got = at.result()
    for k in C1_DIGEST_FIELDS:
        assert digest(got[k]) == str(z["sha_" + k]), k
    assert got["n_seen"] == int(z["n_seen"]) and got["n_sub"] == int(z["n_sub"])
    assert np.allclose(got["sub_sum"], z["sub_sum"], rtol=1e-5, atol=1e-4)
    assert np.allclose(np.stack([np.diag(x) for x in got["gram"]]), z["gram_diag"], rtol=1e-5)


@pytest.mark.gpu
def test_c1_dual_sink_cuda_atlas_equals_oracle():
    """ESM-2 8M on cuda:0 (fp32), all 512 C1 sequences; pilot = the first 64 (also streamed), seeds
    for the whole stream (n_total over the 512). The same hook output feeds the CUDA atlas, the
    oracle and, where oracle/_ref holds the compiled reference, the reference's own
    Atlas(stats_impl="v1", merge_impl="loop", device="cuda")."""
    from proteus_b200.core import Atlas, AtlasConfig
    dev = "cuda:0"
    model = build_model(device=dev, dtype=torch.float32)
    seqs = c1_sequences()
    assert len(seqs) == C1["n_seq"] == 512
    Hp, prot = [[] for _ in range(C1["L"])], []
    for b in c1_batches(seqs, list(range(C1["n_pilot"]))):
        Hs = forward_layers(model, b, device=dev, keep_device=True)
        vr = torch.from_numpy(b.valid_rows).to(dev)
        for l in range(C1["L"]):
            Hp[l].append(Hs[l].index_select(0, vr))
        prot.append(torch.from_numpy(b.tok // 1024).to(dev))
    Hp = [torch.cat(h) for h in Hp]
    E, ts, rk = _pilot_edges_seeds(Hp, torch.cat(prot), int(sum(len(s) for s in seqs)))
    kw = dict(K=C1["K"], Kr=C1["Kr"], seed=0)
    cu = Atlas(C1["L"], C1["D"], E, AtlasConfig(stats_impl="v1", merge_impl="loop", **kw), n_annot=C1["n_annot"],
               device=dev)
    cu.seed(ts, rk)
    orc = O.AtlasOracle(C1["L"], C1["D"], E.numpy(), O.OracleConfig(**kw), n_annot=C1["n_annot"])
    orc.seed(ts.numpy(), rk.numpy())
    ref = None
    try:
        from oracle.build_ref import ReferenceUnavailable, load_reference_atlas
        rc = load_reference_atlas()
        ref = rc.Atlas(C1["L"], C1["D"], E, rc.AtlasConfig(backend="torch", stats_impl="v1", merge_impl="loop", **kw),
                       n_annot=C1["n_annot"], device=dev)
        ref.seed(ts, rk)
    except ReferenceUnavailable:
        pass
    n_batches = 0
    for b in c1_batches(seqs, list(range(len(seqs)))):
        n_batches += 1
        Hs = forward_layers(model, b, device=dev, keep_device=True)
        ctx_c = cu.make_ctx(b.T, b.valid_rows, b.tok, b.ann)
        ctx_o = orc.make_ctx(b.T, b.valid_rows, b.tok, b.ann)
        cu.begin_batch(ctx_c)
        orc.begin_batch(ctx_o)
        Hn = [h.float().cpu().numpy() for h in Hs]
        for l in range(C1["L"]):
            cu.observe(l, Hs[l])
            orc.observe(l, Hn[l])
        assert cu.end_batch() == []
        redo = orc.end_batch()
        if redo:
            orc.begin_batch(ctx_o, redo_layers=redo)
            for l in range(C1["L"]):
                orc.observe(l, Hn[l])
            orc.end_batch()
        if ref is not None:
            rctx = ref.make_ctx(b.T, torch.from_numpy(b.valid_rows), torch.from_numpy(b.tok), torch.from_numpy(b.ann))
            ref.begin_batch(rctx)
            for l in range(C1["L"]):
                ref.observe(l, Hs[l])
            rr = ref.end_batch()
            if rr:
                ref.begin_batch(rctx, redo_layers=rr)
                for l in rr:
                    ref.observe(l, Hs[l])
                ref.end_batch()
    cu.check_errors()
    got, want = cu.result(), orc.result()
    assert got["n_seen"] == sum(len(s) for s in seqs)
    fields = ["top_val", "top_tok", "res_tok", "res_key", "res_val", "sub_bin", "enr", "ann_tot", "n_seen", "n_sub",
              "res_seed_limited", "res_seeded_bins", "res_seed_limited_bins", "top_seed_short_groups"]
    bad = compare(got, want, fields=fields)
    assert not bad, bad
    scale = np.sqrt(max(want["n_sub"], 1) * want["sub_sq"]) + 1e-12
    assert (np.abs(as_np(got["sub_sum"]) - want["sub_sum"]) <= 1e-6 * scale).all()
    assert gram_frobenius_rel(as_np(got["gram"]), want["gram"]) < 1e-3
    if ref is not None:
        rres = ref.result()
        bad = compare(got, {k: as_np(v) if torch.is_tensor(v) else v for k, v in rres.items()}, fields=fields)
        assert not bad, ("vs the reference's own Atlas", bad)
        assert gram_frobenius_rel(as_np(got["gram"]), as_np(rres["gram"])) < 1e-3
    print(f"C1: {n_batches} batches, n_seen {got['n_seen']}, reference arm {'run' if ref is not None else 'absent'}")
