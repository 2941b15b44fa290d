"""The decomposition the dense kernels are built on (proteus_b200/csrc/dense.cu), restated in numpy
and checked against the oracle's dense pass (the reference's Atlas._dense, atlas/core.py:407-446):

* per column and pole, the admissible top-K candidates are the batch elements with s > seed and
  top_key(s, tok) above the state's K-th key; when there are at most K of them they are exactly the
  records to merge, otherwise the batch's top-K by top_key is selected first;
* per reservoir (pole, bin), the rows of the bin whose key lies under the bin's ceiling (the larger
  of the state's Kr-th key and the seed; the whole key range when neither is set) are admitted all
  at once when there are at most Kr of them, otherwise their first Kr in ascending key order.

Merged into the same state with the same grouped merge, both give the oracle's state bit for bit,
over a stream that starts from an empty state (every column needs its selections), a seeded state,
and batches with runs of identical values (ties on the value, broken by token id). CPU only: this
pins the algorithm; the GPU tests pin the kernels to the oracle."""
from __future__ import annotations

import copy

import numpy as np
import pytest

from oracle import atlas_np as O

I64_MIN = np.iinfo(np.int64).min


def _dense_rule(o: O.AtlasOracle, l: int, H: np.ndarray, used: dict) -> None:
    """Merges layer l's dense records into o's state by the decomposition; counts in `used` how
    often each branch ran (columns x poles for top-K, columns x bins for the reservoir)."""
    ctx = o.ctx
    Hv = H[ctx.valid_rows].astype(np.float32)
    n_v, D = Hv.shape
    K, Kr, B = o.cfg.K, o.cfg.Kr, o.B
    tok = ctx.tok
    cols = np.arange(D)
    for p in (0, 1):
        S = Hv if p == 0 else -Hv
        g = (l * 2 + p) * D + cols
        keys = O.top_key(S, tok[:, None])                          # [n_v, D]
        adm = (S > o.top_seed[g][None, :]) & (keys > o.top_k[g, K - 1][None, :])
        rr, cc = [], []
        for d in range(D):
            if adm[:, d].sum() <= K:                               # direct: the candidates themselves
                r = np.nonzero(adm[:, d])[0]
                used["top_direct"] += 1
            else:                                                  # hard: batch top-K first
                top = np.argsort(-keys[:, d], kind="stable")[:K]
                r = top[adm[top, d]]
                used["top_select"] += 1
            rr.append(r)
            cc.append(np.full(r.size, d))
        r, c = np.concatenate(rr), np.concatenate(cc)
        if r.size:
            O.grouped_merge(o.top_k, [o.top_t, o.top_s], g[c], keys[r, c], [tok[r], S[r, c]], K,
                            pay_fill=[-1, O.NEG_INF])
        if not o.cfg.reservoir:
            continue
        b_of = O.bin_of(S, o.E[l, p])                              # [n_v, D]
        gb = g * B
        for bb in range(B):
            th = np.maximum(o.res_s[gb + bb, Kr - 1], o.res_seed[gb + bb])
            ceil = np.where(th == I64_MIN, np.int64(1) << 32, O.neg_i64(th))
            inb = (b_of == bb) & (ctx.key[:, None] < ceil[None, :])
            rr, cc = [], []
            for d in range(D):
                r = np.nonzero(inb[:, d])[0]
                if r.size > Kr:                                    # ordered: first Kr by key
                    r = r[np.argsort(ctx.key[r], kind="stable")[:Kr]]
                    used["res_ordered"] += 1
                elif r.size:
                    used["res_direct"] += 1
                rr.append(r)
                cc.append(np.full(r.size, d))
            r, c = np.concatenate(rr), np.concatenate(cc)
            if r.size:
                O.grouped_merge(o.res_s, [o.res_t, o.res_v], gb[c] + bb, O.neg_i64(ctx.key[r]), [tok[r], Hv[r, c]], Kr)


def _batches(rng, n_batches, T, D, n_seq=6):
    """Padded batches of n_seq sequences; one sequence per batch is low-complexity (runs of the
    same value in every column), which makes ties on the value."""
    out = []
    L = T // n_seq
    for bi in range(n_batches):
        H = (rng.standard_t(3, size=(T, D)) * rng.uniform(0.5, 2.0, D) + rng.normal(0, 0.5, D)).astype(np.float32)
        lc = rng.integers(n_seq)
        rep = rng.choice(2, size=L) == 0
        H[lc * L:(lc + 1) * L][rep] = H[lc * L][None, :] * 2.5
        lens = rng.integers(L // 2, L - 1, n_seq)
        valid = np.concatenate([s * L + 1 + np.arange(n) for s, n in enumerate(lens)])
        tok = np.concatenate([O.pack_tok(np.full(n, bi * n_seq + s), np.arange(n)) for s, n in enumerate(lens)])
        out.append((H, valid, tok))
    return out


@pytest.mark.parametrize("seeded", [False, True])
def test_dense_decomposition_equals_reference_dense(seeded):
    rng = np.random.default_rng(11 + seeded)
    L, D, T, K, Kr = 1, 40, 360, 8, 4
    batches = _batches(rng, 6, T, D)
    pilot = np.concatenate([b[0][b[1]] for b in batches[:2]])
    E = O.pilot_edges([pilot])
    cfg = O.OracleConfig(K=K, Kr=Kr, subsample=False, gram=False, naive=True, rho_res=0.05)
    want = O.AtlasOracle(L, D, E, cfg)
    if seeded:
        ts, rk = O.pilot_seeds([pilot], E, K, Kr, n_total=20 * T)
        want.seed(ts, rk)
        want._dense_layers = {0}  # seeding clears the dense-first layers; every batch stays dense here
    got = copy.deepcopy(want)
    used = dict.fromkeys(("top_direct", "top_select", "res_direct", "res_ordered"), 0)
    for H, valid, tok in batches:
        ctx = want.make_ctx(T, valid, tok)
        want.begin_batch(ctx)
        want.observe(0, H)
        want.end_batch()
        got.ctx = got.make_ctx(T, valid, tok)
        _dense_rule(got, 0, H, used)
        for name in ("top_k", "top_t", "top_s", "res_s", "res_t"):
            np.testing.assert_array_equal(getattr(got, name), getattr(want, name), err_msg=name)
        np.testing.assert_array_equal(np.nan_to_num(got.res_v, nan=-7.0), np.nan_to_num(want.res_v, nan=-7.0))
    assert (want.top_t >= 0).any() and (want.res_t >= 0).any()
    assert all(v > 0 for v in used.values()), used  # every branch of the decomposition ran
