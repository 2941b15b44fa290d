"""Generate the golden fixtures that pin the oracle (and, through it, the CUDA product) to the
reference implementation itself.

Runs the reference's own `atlas` package (haelyons/proteus, imported read-only from --ref) on
seeded inputs and stores every result field in compressed .npz files next to this script:

  stream_<case>.npz   Atlas (stats v1, merge loop, backend torch, CPU) over tests/streams.py
                      streams: unseeded / seeded / tie-heavy shuffled / fp32 / too-tight seeds /
                      cap_frac_early — the matrix of the reference's tests/test_exactness.py:162-184
  offline.npz         reference.reference() ground truth for stream case "bf16"
  keys.npz            token_keys / top_key on edge values (core.py:46-71)
  grouped_merge.npz   grouped_merge on random states and candidates (core.py:75-104)
  merge_from.npz      two shard Atlases on interleaved halves + merged result (core.py:628-654)
  pilot.npz           pilot_edges / pilot_seeds with protein groups (reference.py:55-122)
  filter.npz          filter_candidates survivor sets + overflow count (filter_triton.py:65-86;
                      Triton interpreter on CPU)
  sub_stats.npz       sub_stats counts, sums, masks (stats_triton.py:77-117; interpreter)
  data_plan.npz       SwissProt batch plan, pilot plan, coverage and batch tensors on a dataset
                      with truncation, odd letters and deep annotation overlaps (atlas/data.py)
  c1_esm8m.npz        BASELINE config 0: ESM-2 8M random-init fp32 CPU forward feeding the
                      reference Atlas (stats v1, merge loop), pilot edges + seeds from 64 sequences

Usage (with a read-only checkout of the reference project; the path may also come from
the PROTEUS_REF environment variable):
  python tests/golden/make_golden.py --ref <path to the haelyons/proteus checkout> [--only c1]
"""
from __future__ import annotations

import argparse
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from tests.streams import make_stream, stream_digest  # noqa: E402

STREAM_CASES = {
    # name: (make_stream kwargs, cfg kwargs, seeded, seed_c)
    "bf16": (dict(dtype="bf16"), dict(), False, 4.0),
    "bf16_seeded": (dict(dtype="bf16"), dict(), True, 4.0),
    "bf16_grid_shuffled": (dict(dtype="bf16", grid=0.5, shuffle_order=True), dict(), False, 4.0),
    "bf16_grid_shuffled_seeded": (dict(dtype="bf16", grid=0.5, shuffle_order=True), dict(), True, 4.0),
    "fp32": (dict(dtype="fp32"), dict(), False, 4.0),
    "bf16_tight_seeds": (dict(dtype="bf16"), dict(), True, 0.25),
    "bf16_cap_early": (dict(dtype="bf16"), dict(cap_frac_early=0.5), False, 4.0),
}
STREAM_SHAPE = dict(L=3, D=64, n_seq=500, seed=0, n_annot=7)
STREAM_CFG = dict(K=8, Kr=4, rho_res=0.05, rho_sub=0.2, cap_frac=0.05, seed=7, stats_impl="v1", merge_impl="loop")
N_PILOT = 120

RESULT_KEYS = ["top_val", "top_tok", "res_tok", "res_val", "res_key", "sub_bin", "sub_sum", "sub_sq", "enr",
               "ann_tot", "gram", "res_seed_limited", "res_seed_key"]
SCALAR_KEYS = ["n_seen", "n_sub", "gram_rows", "res_seeded_bins", "res_seed_limited_bins", "top_seed_short_groups"]
STAT_KEYS = ["batches", "dense_layer_batches", "redo_layers", "compacted", "elements", "top_cand", "res_cand"]


def _np(x):
    import torch
    if torch.is_tensor(x):
        if x.dtype == torch.bfloat16:
            x = x.float()
        return x.detach().cpu().numpy().copy()
    return np.asarray(x)


def drive(atlas, stream, torch_dtype):
    """The reference's own driver loop (tests/test_exactness.py:54-86)."""
    import torch
    for b in stream.batches:
        ctx = atlas.make_ctx(b.T, torch.from_numpy(b.valid_rows), torch.from_numpy(b.tok), torch.from_numpy(b.ann))
        Hb = [torch.from_numpy(h).to(torch_dtype) for h in b.H]
        atlas.begin_batch(ctx)
        for l, h in enumerate(Hb):
            atlas.observe(l, h)
        redo = atlas.end_batch()
        if redo:
            atlas.begin_batch(ctx, redo_layers=redo)
            for l, h in enumerate(Hb):
                atlas.observe(l, h)
            assert atlas.end_batch() == []


def save_result(path, res, extra):
    out = dict(extra)
    for k in RESULT_KEYS:
        if k in res:
            out[k] = _np(res[k])
    for k in SCALAR_KEYS:
        if k in res:
            out[k] = np.int64(res[k])
    for k in STAT_KEYS:
        out["stat_" + k] = np.int64(res["stats"].get(k, 0))
    np.savez_compressed(path, **out)


def gen_streams():
    import torch
    from atlas.core import Atlas, AtlasConfig
    from atlas.reference import pilot_edges, pilot_seeds, reference
    for name, (skw, ckw, seeded, seed_c) in STREAM_CASES.items():
        t0 = time.time()
        st = make_stream(**STREAM_SHAPE, **skw)
        tdt = torch.bfloat16 if st.dtype == "bf16" else torch.float32
        Hp = [torch.from_numpy(np.concatenate([s[l] for s in st.seqs[:N_PILOT]])).to(tdt) for l in range(st.L)]
        E = pilot_edges(Hp)
        cfg = AtlasConfig(**STREAM_CFG, **ckw)
        atlas = Atlas(st.L, st.D, E, cfg, n_annot=STREAM_SHAPE["n_annot"], device="cpu")
        extra = {"digest": np.array(stream_digest(st)), "E": _np(E)}
        if seeded:
            ts, rk = pilot_seeds(Hp, E, cfg.K, cfg.Kr, n_total=int(st.lens.sum()), c=seed_c)
            atlas.seed(ts, rk)
            extra["top_seed"], extra["res_seed_key"] = _np(ts), _np(rk)
        drive(atlas, st, tdt)
        res = atlas.result()
        save_result(HERE / f"stream_{name}.npz", res, extra)
        if name == "bf16":
            Hall, toks, A = st.all_tokens()
            annf = np.zeros((toks.size, STREAM_SHAPE["n_annot"]), np.float32)
            r, c = np.nonzero(A >= 0)
            annf[r, A[r, c]] = 1
            ref = reference([torch.from_numpy(h).to(tdt) for h in Hall], torch.from_numpy(toks), E, cfg.K, cfg.Kr,
                            cfg.rho_sub, cfg.seed, ann=torch.from_numpy(annf), levels=cfg.enrich_levels)
            np.savez_compressed(HERE / "offline.npz", **{k: _np(v) for k, v in ref.items()})
        print(f"stream {name}: {time.time() - t0:.1f}s, stats {res['stats']}", flush=True)


def gen_keys():
    import torch
    from atlas.core import token_keys, top_key
    g = np.random.default_rng(11)
    toks = np.concatenate([np.array([0, 1, 2, 1023, 1024, 2**31 - 1, 2**31, 2**32 - 1], np.int64),
                           g.integers(0, 2**32, 2000, dtype=np.int64)])
    out = {"tok": toks}
    for seed in (0, 7, 0x1_0000_0005):
        out[f"keys_seed{seed}"] = _np(token_keys(torch.from_numpy(toks), seed))
    f32 = np.finfo(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, f32.max, -f32.max, f32.tiny, -f32.tiny, 1e-45, -1e-45,
                        1.0, -1.0, 0.5, -0.5], np.float32)
    s = np.concatenate([special, g.standard_normal(2000).astype(np.float32) * 10])
    t = g.integers(0, 2**32, s.size, dtype=np.int64)
    out.update(s=s, s_tok=t, top_key=_np(top_key(torch.from_numpy(s), torch.from_numpy(t))))
    np.savez_compressed(HERE / "keys.npz", **out)


def gen_grouped_merge():
    import torch
    from atlas.core import I64_MIN, grouped_merge
    g = np.random.default_rng(5)
    out = {}
    for case, (G, K, rounds, n) in enumerate([(50, 8, 4, 300), (7, 32, 3, 500), (200, 4, 5, 150)]):
        st = torch.full((G, K), I64_MIN, dtype=torch.long)
        pt = torch.full((G, K), -1, dtype=torch.long)
        pv = torch.full((G, K), float("-inf"))
        used = set()
        for r in range(rounds):
            gid = g.integers(0, G, n)
            sc = g.integers(-2**40, 2**40, n)
            keep = [i for i in range(n) if (int(gid[i]), int(sc[i])) not in used]
            for i in keep:
                used.add((int(gid[i]), int(sc[i])))
            gid, sc = gid[keep], sc[keep]
            tok = g.integers(0, 2**32, gid.size)
            val = g.standard_normal(gid.size).astype(np.float32)
            out[f"c{case}_r{r}_g"], out[f"c{case}_r{r}_s"] = gid, sc
            out[f"c{case}_r{r}_t"], out[f"c{case}_r{r}_v"] = tok, val
            grouped_merge(st, [pt, pv], torch.from_numpy(gid), torch.from_numpy(sc),
                          [torch.from_numpy(tok), torch.from_numpy(val)], K, pay_fill=[-1, float("-inf")])
        out[f"c{case}_meta"] = np.array([G, K, rounds])
        out[f"c{case}_state"], out[f"c{case}_tok"], out[f"c{case}_val"] = _np(st), _np(pt), _np(pv)
    np.savez_compressed(HERE / "grouped_merge.npz", **out)


def gen_merge_from():
    import torch
    from atlas.core import Atlas, AtlasConfig
    from atlas.reference import pilot_edges, pilot_seeds
    from tests.streams import Stream
    st = make_stream(L=2, D=48, n_seq=400, seed=3, dtype="bf16", n_annot=5)
    tdt = torch.bfloat16
    Hp = [torch.from_numpy(np.concatenate([s[l] for s in st.seqs[:N_PILOT]])).to(tdt) for l in range(st.L)]
    E = pilot_edges(Hp)
    cfg = AtlasConfig(K=8, Kr=4, rho_res=0.05, rho_sub=0.2, cap_frac=0.05, seed=11, stats_impl="v1", merge_impl="loop")
    ts, rk = pilot_seeds(Hp, E, cfg.K, cfg.Kr, n_total=int(st.lens.sum()))
    out = {"digest": np.array(stream_digest(st)), "E": _np(E), "top_seed": _np(ts), "res_seed_key": _np(rk)}
    shards = []
    for half in (0, 1):
        sub = Stream(st.L, st.D, st.dtype, st.lens, st.seqs, st.ann_full,
                     [b for i, b in enumerate(st.batches) if i % 2 == half], st.order)
        at = Atlas(st.L, st.D, E, cfg, n_annot=5, device="cpu")
        at.seed(ts, rk)
        drive(at, sub, tdt)
        sd = at.state_dict()
        for k in Atlas._STATE + ["enr", "ann_tot"]:
            out[f"s{half}_{k}"] = _np(sd[k])
        out[f"s{half}_n_seen"], out[f"s{half}_n_sub"] = np.int64(sd["n_seen"]), np.int64(sd["n_sub"])
        shards.append(at)
    shards[0].merge_from(shards[1])
    res = shards[0].result()
    for k in RESULT_KEYS:
        if k in res:
            out["m_" + k] = _np(res[k])
    for k in SCALAR_KEYS:
        out["m_" + k] = np.int64(res[k])
    np.savez_compressed(HERE / "merge_from.npz", **out)


def gen_pilot():
    import torch
    from atlas.reference import pilot_edges, pilot_seeds
    from tests.streams import pilot_inputs
    Hs, groups = pilot_inputs()
    Ht = [torch.from_numpy(h) for h in Hs]
    E = pilot_edges(Ht)
    ts, rk = pilot_seeds(Ht, E, 16, 8, n_total=10**6, groups=torch.from_numpy(groups))
    ts0, rk0 = pilot_seeds(Ht, E, 16, 8, n_total=10**6)
    np.savez_compressed(HERE / "pilot.npz", E=_np(E), top_seed=_np(ts), res_seed_key=_np(rk),
                        top_seed_nogroups=_np(ts0), res_seed_key_nogroups=_np(rk0))


def gen_kernels():
    """Reference Triton kernels under the interpreter (CPU)."""
    os.environ["TRITON_INTERPRET"] = "1"
    import torch
    from atlas.filter_triton import filter_candidates
    from atlas.stats_triton import sub_stats
    from tests.streams import FILTER_CASES, STATS_CASES, filter_inputs, stats_inputs
    out = {}
    for case in range(len(FILTER_CASES)):
        H, rowmap, tp, tn = (torch.from_numpy(x) for x in filter_inputs(case))
        H = H.to(torch.bfloat16)
        v, r, c, cnt = filter_candidates(H, rowmap, tp, tn, 1 << 16, BLOCK_T=32, BLOCK_D=128)
        n = int(cnt)
        o = np.lexsort((_np(c[:n]), _np(r[:n])))
        _, _, _, cnt64 = filter_candidates(H, rowmap, tp, tn, 64, BLOCK_T=32, BLOCK_D=128)
        out.update({f"f{case}_val": _np(v[:n])[o], f"f{case}_row": _np(r[:n])[o], f"f{case}_col": _np(c[:n])[o],
                    f"f{case}_count": np.int64(n), f"f{case}_count_cap64": np.int64(int(cnt64))})
    np.savez_compressed(HERE / "filter.npz", **out)
    out = {}
    for case in range(len(STATS_CASES)):
        X, E0, E1, levels = stats_inputs(case)
        s, sq, cnt, M = sub_stats(torch.from_numpy(X).to(torch.bfloat16), torch.from_numpy(E0),
                                  torch.from_numpy(E1), levels, BLOCK_N=8, BLOCK_D=32)
        out.update({f"s{case}_sum": _np(s), f"s{case}_sq": _np(sq), f"s{case}_cnt": _np(cnt), f"s{case}_M": _np(M)})
    np.savez_compressed(HERE / "sub_stats.npz", **out)


def gen_c1():
    """BASELINE config 0 on the reference: ESM-2 8M (random init, seed 0), fp32 CPU, 512 sequences."""
    import torch
    from atlas.core import Atlas, AtlasConfig
    from atlas.reference import pilot_edges, pilot_seeds
    from tests.c1 import C1, build_model, c1_batches, c1_sequences, forward_layers
    torch.set_num_threads(1)
    t0 = time.time()
    model = build_model()
    seqs = c1_sequences()
    pilot_seqs = list(range(C1["n_pilot"]))
    Hp, prot = [[] for _ in range(C1["L"])], []
    for b in c1_batches(seqs, pilot_seqs):
        Hs = forward_layers(model, b)
        for l in range(C1["L"]):
            Hp[l].append(torch.from_numpy(Hs[l][b.valid_rows]))
        prot.append(torch.from_numpy(b.tok // 1024))
    Hp = [torch.cat(h) for h in Hp]
    prot = torch.cat(prot)
    E = torch.cat([pilot_edges([h]) for h in Hp])
    n_total = int(sum(len(s) for s in seqs))
    cfg = AtlasConfig(K=C1["K"], Kr=C1["Kr"], stats_impl="v1", merge_impl="loop", seed=0)
    parts = [pilot_seeds([h], E[li:li + 1], cfg.K, cfg.Kr, n_total, groups=prot) for li, h in enumerate(Hp)]
    ts, rk = torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts])
    atlas = Atlas(C1["L"], C1["D"], E, cfg, n_annot=C1["n_annot"], device="cpu")
    atlas.seed(ts, rk)
    for b in c1_batches(seqs, list(range(len(seqs)))):
        Hs = forward_layers(model, b)
        ctx = atlas.make_ctx(b.T, torch.from_numpy(b.valid_rows), torch.from_numpy(b.tok), torch.from_numpy(b.ann))
        atlas.begin_batch(ctx)
        for l in range(C1["L"]):
            atlas.observe(l, torch.from_numpy(Hs[l]))
        redo = atlas.end_batch()
        if redo:
            atlas.begin_batch(ctx, redo_layers=redo)
            for l in range(C1["L"]):
                atlas.observe(l, torch.from_numpy(Hs[l]))
            assert atlas.end_batch() == []
    res = atlas.result()
    gram = _np(res.pop("gram"))
    idx = np.random.default_rng(0).integers(0, C1["D"], (4096, 2))
    extra = {"E": _np(E), "top_seed": _np(ts),
             "gram_diag": np.stack([np.diag(g_) for g_ in gram]), "gram_idx": idx,
             "gram_sample": gram[:, idx[:, 0], idx[:, 1]], "gram_fro": np.sqrt((gram ** 2).sum((1, 2)))}
    save_result(HERE / "c1_esm8m.npz", res, extra)
    compact_exact_fields(HERE / "c1_esm8m.npz")
    print(f"c1: {time.time() - t0:.1f}s, n_seen {res['n_seen']}, stats {res['stats']}", flush=True)


DATA_CASE = dict(n_seq=3000, seed=4, tokens_per_batch=8192, window=1000, pilot_tokens=20000, batches=(0, 3, -1))


DATA_X_GROUP = [7, 11, 2, 40]


def data_case() -> dict:
    """A dataset in the reference's on-disk format that exercises every rule of the batch plan and
    of the annotation fill: lengths from 5 to 1500 (truncation at 1022, equal lengths whose order a
    stable sort must keep), letters outside the standard 20 (X B U Z O and a lowercase one), and
    annotation intervals that run past the truncated end, are empty after truncation, or pile up
    more than max_ann deep."""
    import torch
    rng = np.random.default_rng(DATA_CASE["seed"])
    n = DATA_CASE["n_seq"]
    lens = np.clip(np.round(rng.lognormal(np.log(250), 0.8, n)), 5, 1500).astype(np.int32)
    lens[::97] = 300  # repeated lengths
    lens[40] = 1500  # truncated; one interval lies entirely past its truncated end
    letters = np.frombuffer(b"ACDEFGHIKLMNPQRSTVWYXBUZOa", np.uint8)
    p = np.r_[np.full(20, 0.049), np.full(6, 0.02 / 6)]
    seqs = [letters[rng.choice(26, int(m), p=p / p.sum())].tobytes().decode() for m in lens]
    iv = []
    for i in rng.choice(n, 1500, replace=False):
        m = int(lens[i])
        for _ in range(int(rng.integers(1, 5))):
            a0 = int(rng.integers(0, m))
            iv.append((i, a0, int(min(m + 5, a0 + rng.integers(1, 80))), int(rng.integers(21, 60))))
    for i in (7, 11):  # 12 intervals over one region: more than max_ann - 1 = 7 extra columns
        for k in range(12):
            iv.append((i, 1, 4 + k, 30 + k))
    iv.append((40, 1100, 1200, 50))  # entirely past the truncated end
    iv = np.array(iv, np.int32)[rng.permutation(len(iv))]
    return {"acc": [f"T{i:05d}" for i in range(n)], "seq": seqs, "len": torch.from_numpy(lens),
            "iv": torch.from_numpy(iv), "vocab": [f"a{k}" for k in range(60)]}


def gen_data():
    """The reference's SwissProt (atlas/data.py) on data_case(): plans, pilot plan, coverage, and
    the tensors of a few batches."""
    import io

    import torch
    from atlas.data import SwissProt, shuffled_order
    from tests.c1 import ESM_TOKENS
    c = DATA_CASE
    buf = io.BytesIO()
    torch.save(data_case(), buf)
    buf.seek(0)
    ds = SwissProt(buf)
    vocab = {t: i for i, t in enumerate(ESM_TOKENS)}
    order = shuffled_order(len(ds), c["seed"])
    out = {"order": _np(order)}
    plans = {"shuffled": ds.plan(order, c["tokens_per_batch"], c["window"], c["seed"]),
             "sorted": ds.plan(order, c["tokens_per_batch"], c["window"], c["seed"], shuffle_batches=False)}
    plans["pilot"] = ds.pilot_plan(plans["shuffled"], c["pilot_tokens"], c["tokens_per_batch"], c["seed"])
    for name, pl in plans.items():
        out[f"plan_{name}_flat"] = np.array([i for g in pl for i in g], np.int64)
        out[f"plan_{name}_sizes"] = np.array([len(g) for g in pl], np.int64)
    cov = ds.coverage(order[:500])
    out.update({f"cov_{k}": np.array(v) for k, v in cov.items()})
    aa = {ch: vocab.get(ch, vocab["<unk>"]) for ch in set("ACDEFGHIKLMNPQRSTVWY") | set("XBUZO")}
    groups = {bi: plans["shuffled"][bi] for bi in c["batches"]}
    groups["x"] = DATA_X_GROUP  # the sequences with the deep interval piles and the longest one
    for bi, grp in groups.items():
        b = ds._make(grp, aa, vocab["<cls>"], vocab["<eos>"], vocab["<pad>"])
        for k in ("input_ids", "attention_mask", "valid_rows", "tok", "ann", "seq_idx"):
            out[f"b{bi}_{k}"] = _np(getattr(b, k))
        out[f"b{bi}_n_rows"] = np.int64(b.n_rows)
    out["ann_dropped"] = np.int64(ds.ann_dropped)
    np.savez_compressed(HERE / "data_plan.npz", **out)


C1_DIGEST_FIELDS = ("top_val", "top_tok", "res_tok", "res_val", "res_key", "sub_bin", "enr", "ann_tot",
                    "res_seed_limited", "res_seed_key")


def digest(a) -> str:
    """sha256 of an array's bytes (bool as uint8): bit-exact comparison without storing the array."""
    import hashlib
    a = np.ascontiguousarray(a)
    if a.dtype == bool:
        a = a.astype(np.uint8)
    return hashlib.sha256(a.tobytes()).hexdigest()


def compact_exact_fields(path):
    """Replace the large exact fields of a fixture by their sha256 digests (keeps it small)."""
    z = dict(np.load(path))
    out = {}
    for k, v in z.items():
        if k in C1_DIGEST_FIELDS:
            out["sha_" + k] = np.array(digest(v))
            out["shape_" + k] = np.array(v.shape)
        else:
            out[k] = v
    np.savez_compressed(path, **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("PROTEUS_REF"), required=os.environ.get("PROTEUS_REF") is None,
                    help="checkout of the reference project (read-only)")
    ap.add_argument("--only", nargs="*", default=None)
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    jobs = {"streams": gen_streams, "keys": gen_keys, "grouped_merge": gen_grouped_merge,
            "merge_from": gen_merge_from, "pilot": gen_pilot, "kernels": gen_kernels, "c1": gen_c1,
            "data": gen_data}
    for name, fn in jobs.items():
        if a.only is None or name in a.only:
            t0 = time.time()
            fn()
            print(f"[golden] {name} done in {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    main()
