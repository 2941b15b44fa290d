"""TEST INFRASTRUCTURE ONLY — numpy restatement of the reference streaming atlas.

Restates, function by function, haelyons/proteus `atlas/core.py` (the `Atlas` engine with
`stats_impl="v1"`, `merge_impl="loop"`, `backend="torch"`, i.e. the reference's exactness path)
and the offline ground truth `atlas/reference.py:reference`. It is the checker for the CUDA
product (tests/) and the timed CPU baseline of bench.py (kind "port"); nothing in proteus_b200
imports it.

Everything runs in fp32 on the exact fp32 images of the streamed activations (bf16 -> fp32 is
exact, and the reference compares bf16 activations against fp32 thresholds in fp32 too:
`core.py:279`, `filter_triton.py:39-41`). Integer work (hash, keys, selections, counts) is exact.

Pinned against the reference's own outputs: tests/golden/make_golden.py runs the reference
package (imported read-only) on seeded streams and records every result field;
tests/test_oracle_golden.py requires this restatement to reproduce them bit for bit (sums and
Gram within the tolerances the reference's tests use).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import numpy as np

NEG_INF = np.float32(-np.inf)
POS_INF = np.float32(np.inf)
I64_MIN = np.iinfo(np.int64).min
I64_MAX = np.iinfo(np.int64).max
M32 = 0xFFFFFFFF
SEQ_STRIDE = 1024


# ----------------------------------------------------------------------------- hashing / keys
def token_keys(tok, seed: int = 0) -> np.ndarray:
    """Wellons lowbias32 of (tok ^ seed) & M32, as int64 in [0, 2^32) (core.py:46-55)."""
    x = ((np.asarray(tok, np.int64) ^ np.int64(seed & M32)) & M32).astype(np.uint32)
    x = x ^ (x >> np.uint32(16))
    x = x * np.uint32(0x7FEB352D)
    x = x ^ (x >> np.uint32(15))
    x = x * np.uint32(0x846CA68B)
    x = x ^ (x >> np.uint32(16))
    return x.astype(np.int64)


def pack_tok(seq_idx, pos) -> np.ndarray:
    """tok = seq * 1024 + pos (core.py:58-59)."""
    return np.asarray(seq_idx, np.int64) * SEQ_STRIDE + np.asarray(pos, np.int64)


def top_key(s, tok) -> np.ndarray:
    """int64 key ordering (s desc, tok asc); -0.0 canonicalised to +0.0 (core.py:66-71)."""
    s32 = np.asarray(s, np.float32) + np.float32(0.0)
    i = s32.view(np.int32).astype(np.int64)
    i = np.where(i < 0, i ^ 0x7FFFFFFF, i)
    return i * 4294967296 + (M32 - np.asarray(tok, np.int64))


def bin_of(s, E) -> np.ndarray:
    """#{b : s >= E_b} - 1 in {-1, 0..B-1} (core.py:107-109)."""
    return (np.asarray(s)[..., None] >= E).sum(-1) - 1


def nextdown(x) -> np.ndarray:
    """nextafter(x, -inf) in fp32 (the reference's torch.nextafter toward -inf)."""
    x = np.asarray(x, np.float32)
    return np.nextafter(x, np.float32(-np.inf)).astype(np.float32)


def neg_i64(x) -> np.ndarray:
    """Two's-complement negation of int64 (I64_MIN stays I64_MIN, as torch's `-t` does)."""
    return (~np.asarray(x, np.int64)) + np.int64(1)


def grouped_merge(state_score, state_pay, g, score, pay, K, pay_fill=None) -> int:
    """In-place exact merge of candidates into per-group top-K, descending (core.py:75-104).

    The reference sorts candidates by (group, score desc), keeps at most K per group, and takes
    topk over [state | candidates]. Real scores are unique within a group, so the result does not
    depend on tie order; fill entries all carry the same fill payload."""
    g = np.asarray(g, np.int64)
    if g.size == 0:
        return 0
    order = np.lexsort((score, g))                     # group asc, score asc
    gs, ss = g[order], score[order]
    ug, start, cnt = np.unique(gs, return_index=True, return_counts=True)
    seg = np.repeat(np.arange(ug.size), cnt)
    rank = (start + cnt)[seg] - 1 - np.arange(gs.size)  # 0 = largest in its group
    keep = rank < K
    nu = ug.size
    fill = NEG_INF if np.issubdtype(score.dtype, np.floating) else I64_MIN
    cs = np.full((nu, K), fill, dtype=score.dtype)
    cs[seg[keep], rank[keep]] = ss[keep]
    allv = np.concatenate((state_score[ug], cs), 1)
    idx = np.argsort(allv, axis=1, kind="stable")[:, ::-1][:, :K]
    state_score[ug] = np.take_along_axis(allv, idx, 1)
    for j, (sp, p) in enumerate(zip(state_pay, pay)):
        if pay_fill is not None:
            pf = pay_fill[j]
        else:
            pf = np.nan if np.issubdtype(p.dtype, np.floating) else -1
        cp = np.full((nu, K), pf, dtype=sp.dtype)
        cp[seg[keep], rank[keep]] = np.asarray(p)[order][keep]
        sp[ug] = np.take_along_axis(np.concatenate((sp[ug], cp), 1), idx, 1)
    return nu


def symmetrize_upper(U: np.ndarray) -> np.ndarray:
    """triu(U) + triu(U, 1)^T over the last two axes (core.py:756-759)."""
    up = np.triu(U)
    return up + np.swapaxes(np.triu(U, 1), -1, -2)


# ----------------------------------------------------------------------------- host threads
# numpy releases the GIL inside its array loops, so row / column chunks on a thread pool use every
# host core; results are concatenated in order and equal the single-threaded expressions exactly.
_POOL = None


def _threads() -> int:
    return max(1, int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1)))


def _pool():
    global _POOL
    if _POOL is None:
        from concurrent.futures import ThreadPoolExecutor
        _POOL = ThreadPoolExecutor(max_workers=_threads())
    return _POOL


def _par_filter(H, valid, tp, ntn):
    """nonzero(((H > tp) | (H < ntn)) & valid[:, None]) in row-major order, by row chunks."""
    T = H.shape[0]
    nt = _threads()
    if nt == 1 or H.size < (1 << 22):
        return np.nonzero(((H > tp[None, :]) | (H < ntn[None, :])) & valid[:, None])
    bounds = np.linspace(0, T, nt + 1).astype(np.int64)

    def part(i):
        a, b = bounds[i], bounds[i + 1]
        r, c = np.nonzero(((H[a:b] > tp[None, :]) | (H[a:b] < ntn[None, :])) & valid[a:b, None])
        return r + a, c
    res = list(_pool().map(part, range(nt)))
    return np.concatenate([r for r, _ in res]), np.concatenate([c for _, c in res])


def _par_ge(s, E):
    """s[:, :, None] >= E[None] ([n, D, B] booleans) by column chunks."""
    n, D = s.shape
    nt = _threads()
    if nt == 1 or s.size < (1 << 20):
        return s[:, :, None] >= E[None]
    out = np.empty((n, D, E.shape[-1]), bool)
    bounds = np.linspace(0, D, nt + 1).astype(np.int64)

    def part(i):
        a, b = bounds[i], bounds[i + 1]
        np.greater_equal(s[:, a:b, None], E[None, a:b], out=out[:, a:b])
    list(_pool().map(part, range(nt)))
    return out


# ----------------------------------------------------------------------------- config / ctx
@dataclass
class OracleConfig:
    """Field-for-field the reference's AtlasConfig (core.py:113-132)."""
    K: int = 64
    Kr: int = 16
    rho_res: float = 0.01
    rho_sub: float = 0.05
    enrich_levels: tuple = (2, 3, 4)
    gram: bool = True
    cap_frac: float = 0.005
    cap_frac_early: float = 0.0
    early_layers: int = 2
    backend: str = "torch"
    stats_impl: str = "v1"
    merge_impl: str = "loop"
    seed_c: float = 4.0
    seed_z: float = 2.0
    seed: int = 0
    reservoir: bool = True
    subsample: bool = True
    naive: bool = False


@dataclass
class OracleCtx:
    """The reference's BatchCtx (core.py:135-157) as host numpy arrays."""
    T: int
    valid_rows: np.ndarray
    tok: np.ndarray
    key: np.ndarray
    rowmap: np.ndarray
    sub_idx: np.ndarray
    res_in_sub: np.ndarray
    ann_sub: np.ndarray | None = None
    n_v: int = 0
    n_s: int = 0
    n_r: int = 0
    sub_rows: np.ndarray | None = None


class AtlasOracle:
    """Streaming atlas, reference semantics (core.py:160-704), numpy on the CPU."""

    def __init__(self, n_layers: int, D: int, edges: np.ndarray, cfg: OracleConfig, n_annot: int = 0):
        L, B = n_layers, edges.shape[-1]
        assert edges.shape == (L, 2, D, B), edges.shape
        self.L, self.D, self.B, self.cfg = L, D, B, cfg
        self.E = np.ascontiguousarray(edges, dtype=np.float32)
        self.U_res = int(cfg.rho_res * 2**32)
        self.U_sub = int(cfg.rho_sub * 2**32)
        assert self.U_sub >= self.U_res
        K, Kr = cfg.K, cfg.Kr
        G = L * 2 * D
        self.top_s = np.full((G, K), NEG_INF, np.float32)
        self.top_t = np.full((G, K), -1, np.int64)
        self.top_k = np.full((G, K), I64_MIN, np.int64)
        self.res_s = np.full((G * B, Kr), I64_MIN, np.int64)
        self.res_t = np.full((G * B, Kr), -1, np.int64)
        self.res_v = np.full((G * B, Kr), np.nan, np.float32)
        self.n_seen = 0
        self.n_sub = 0
        self.sub_sum = np.zeros((L, D), np.float64)
        self.sub_sq = np.zeros((L, D), np.float64)
        self.sub_bin = np.zeros((L, 2, D, B), np.int64)
        self.n_a = n_annot
        nl = len(cfg.enrich_levels)
        if n_annot:
            self.enr = np.zeros((L, 2, nl, D, n_annot), np.int64)
            self.ann_tot = np.zeros(n_annot, np.int64)
        self.gram = np.zeros((L, D, D), np.float32) if cfg.gram else None
        self.gram64 = np.zeros((L, D, D), np.float64) if cfg.gram else None
        self.gram_rows = 0
        self.top_seed = np.full(G, NEG_INF, np.float32)
        self.res_seed = np.full(G * B, I64_MIN, np.int64)
        self.enabled = True
        self.stats = {"batches": 0, "dense_layer_batches": 0, "redo_layers": 0,
                      "compacted": 0, "elements": 0, "top_cand": 0, "res_cand": 0}
        self.ctx: OracleCtx | None = None
        self._pending: dict = {}
        self._dense_layers = set(range(L))
        self._active = None
        self._sub_done: set = set()

    # -------------------------------------------------------------- batch setup (core.py:210-259)
    def make_ctx(self, T: int, valid_rows, tok, ann_ids=None) -> OracleCtx:
        valid_rows = np.asarray(valid_rows, np.int64)
        tok = np.asarray(tok, np.int64)
        assert tok.size == 0 or (tok.min() >= 0 and tok.max() < 2**32)
        key = token_keys(tok, self.cfg.seed)
        sub = np.nonzero(key < self.U_sub)[0]
        res_in_sub = np.nonzero(key[sub] < self.U_res)[0]
        rowmap = np.full(T, -1, np.int64)
        rowmap[valid_rows] = np.arange(valid_rows.size)
        ann_sub = None
        if self.n_a and ann_ids is not None:
            a = np.asarray(ann_ids, np.int64)[sub]
            ann_sub = np.zeros((sub.size, self.n_a), np.float32)
            r, c = np.nonzero(a >= 0)
            ann_sub[r, a[r, c]] = 1.0
        return OracleCtx(T=T, valid_rows=valid_rows, tok=tok, key=key, rowmap=rowmap, sub_idx=sub,
                         res_in_sub=res_in_sub, ann_sub=ann_sub, n_v=valid_rows.size, n_s=sub.size,
                         n_r=res_in_sub.size, sub_rows=valid_rows[sub])

    def begin_batch(self, ctx: OracleCtx, redo_layers=None):
        self.ctx = ctx
        self._pending = {}
        if redo_layers is None:
            self._active = set(range(self.L))
            self._sub_done = set()
            self.stats["elements"] += 2 * ctx.n_v * self.D * self.L
        else:
            self._active = set(redo_layers)
        L, D, B, Kr = self.L, self.D, self.B, self.cfg.Kr
        tau_top = np.maximum(nextdown(self.top_s[:, -1]), self.top_seed).reshape(L, 2, D)
        kth = np.maximum(self.res_s[:, Kr - 1], self.res_seed).reshape(L, 2, D, B)
        underfilled = kth < -self.U_res
        eps = np.where(underfilled, self.E, POS_INF).min(-1)
        eps = nextdown(eps)
        self.thr = np.minimum(tau_top, eps) if self.cfg.reservoir else tau_top.copy()

    # -------------------------------------------------------------- hook body (core.py:262-293)
    def observe(self, l: int, H: np.ndarray):
        """H: [T, D] fp32 image of the hook output (padding rows included)."""
        if not self.enabled or l not in self._active:
            return
        ctx = self.ctx
        H = np.asarray(H, np.float32)
        if l in self._dense_layers:
            self._dense(l, H)
            return
        rr, cc = _par_filter(H, ctx.rowmap >= 0, self.thr[l, 0], -self.thr[l, 1])
        cnt = rr.size
        vals = H[rr, cc].astype(np.float32)
        rows = ctx.rowmap[rr]
        R = None
        if self.cfg.subsample or self.cfg.reservoir:
            Hn = H[ctx.sub_rows]
            if self.cfg.subsample and l not in self._sub_done:
                self._stats_v1(l, Hn)
            R = Hn[ctx.res_in_sub] if self.cfg.reservoir else None
        self._pending[l] = (vals, rows, cc.astype(np.int64), cnt, R)

    def _cap(self, ctx, l=None) -> int:
        f = self.cfg.cap_frac
        if self.cfg.cap_frac_early > 0 and l is not None and l < self.cfg.early_layers:
            f = self.cfg.cap_frac_early
        return max(4096, int(f * ctx.n_v * self.D))

    def _stats_v1(self, l, Hs):
        """core.py:312-338: batch sums -> fp64; cumulative-threshold bin counts; exact enrichment
        counts; fp32 Gram."""
        self._sub_done.add(l)
        n = Hs.shape[0]
        if n == 0:
            return
        # the reference sums each batch in fp32 (torch's cascade sum) and widens; numpy's column
        # sums are sequential, so the restatement sums in fp64, which stays within the reference
        # test's own 1e-6 tolerance of both the fp64 truth and the reference's result
        H64 = Hs.astype(np.float64)
        self.sub_sum[l] += H64.sum(0)
        self.sub_sq[l] += (Hs * Hs).astype(np.float64).sum(0)
        levels = list(self.cfg.enrich_levels)
        for p, sgn in ((0, 1.0), (1, -1.0)):
            s = Hs * np.float32(sgn)
            ge = _par_ge(s, self.E[l, p])
            cnt_ge = ge.sum(0)
            nxt = np.concatenate((cnt_ge[:, 1:], np.zeros_like(cnt_ge[:, :1])), 1)
            self.sub_bin[l, p] += cnt_ge - nxt
            if self.n_a and self.ctx.ann_sub is not None:
                m = ge[:, :, levels].transpose(0, 2, 1).reshape(n, -1).astype(np.float32)
                c = m.T @ self.ctx.ann_sub
                self.enr[l, p] += np.rint(c.reshape(len(levels), self.D, -1)).astype(np.int64)
        if self.gram is not None:
            self.gram[l] += Hs.T @ Hs
            if l == 0:
                self.gram_rows += n

    # -------------------------------------------------------------- dense path (core.py:407-446)
    def _dense(self, l, H):
        ctx = self.ctx
        Hv = H[ctx.valid_rows]
        if self.cfg.subsample and l not in self._sub_done:
            self._stats_v1(l, Hv[ctx.sub_idx])
        D, B, K, Kr = self.D, self.B, self.cfg.K, self.cfg.Kr
        n_v = Hv.shape[0]
        cols = np.arange(D)
        for p, sgn in ((0, 1.0), (1, -1.0)):
            S = Hv if p == 0 else -Hv
            k = min(K, n_v)
            if k > 0:
                vk = np.partition(S, n_v - k, axis=0)[n_v - k]
                gD = (l * 2 + p) * D + cols
                r, c = np.nonzero(S >= vk[None, :])
                v = S[r, c]
                ok = v > self.top_seed[gD[c]]
                r, c, v = r[ok], c[ok], v[ok]
                t = ctx.tok[r]
                self.stats["top_cand"] += int(v.size)
                grouped_merge(self.top_k, [self.top_t, self.top_s], gD[c], top_key(v, t), [t, v], K,
                              pay_fill=[-1, NEG_INF])
            if not self.cfg.reservoir:
                continue
            b = bin_of(S, self.E[l, p])
            gb = ((l * 2 + p) * D + cols) * B
            kr = min(Kr, n_v)
            if kr == 0:
                continue
            for bb in range(B):
                seed = self.res_seed[gb + bb]
                unseeded = seed == I64_MIN
                seed_key = np.where(unseeded, I64_MAX, neg_i64(seed))
                inb = (b == bb) & (unseeded[None, :] | (ctx.key[:, None] < seed_key[None, :]))
                km = np.where(inb, ctx.key[:, None], I64_MAX)
                ki = np.argpartition(km, kr - 1, axis=0)[:kr]
                kv = np.take_along_axis(km, ki, 0)
                ok = kv < I64_MAX
                gg = np.broadcast_to((gb + bb)[None, :], (kr, D))[ok]
                cc = np.broadcast_to(cols[None, :], (kr, D))[ok]
                self.stats["res_cand"] += int(gg.size)
                grouped_merge(self.res_s, [self.res_t, self.res_v], gg, -kv[ok],
                              [ctx.tok[ki[ok]], Hv[ki[ok], cc]], Kr)
        self.stats["dense_layer_batches"] += 1
        self._pending[l] = None

    # -------------------------------------------------------------- after forward (core.py:450-545)
    def end_batch(self) -> list:
        ctx = self.ctx
        filt = [l for l, v in self._pending.items() if v is not None]
        redo = []
        if filt:
            cnts = [self._pending[l][3] for l in filt]
            redo = [l for l, c in zip(filt, cnts) if c > self._cap(ctx, l)]
            ok = [(l, c) for l, c in zip(filt, cnts) if c <= self._cap(ctx, l)]
            if ok:
                self._merge_filtered(ok)
        dense_done = [l for l, v in self._pending.items() if v is None]
        if not self.cfg.naive:
            self._dense_layers -= set(dense_done)
        if redo:
            self.stats["redo_layers"] += len(redo)
            self._dense_layers |= set(redo)
        else:
            self.n_seen += ctx.n_v
            self.n_sub += ctx.n_s
            if self.n_a and ctx.ann_sub is not None:
                self.ann_tot += np.rint(ctx.ann_sub.sum(0)).astype(np.int64)
            self.stats["batches"] += 1
        return redo

    def _merge_filtered(self, ok):
        ctx, D, B, K, Kr = self.ctx, self.D, self.B, self.cfg.K, self.cfg.Kr
        lay = np.concatenate([np.full(c, l, np.int64) for l, c in ok])
        vals = np.concatenate([self._pending[l][0][:c] for l, c in ok]).astype(np.float32)
        rows = np.concatenate([self._pending[l][1][:c] for l, c in ok])
        cols = np.concatenate([self._pending[l][2][:c] for l, c in ok])
        self.stats["compacted"] += int(lay.size)
        tok, key = ctx.tok[rows], ctx.key[rows]
        kth_key = self.top_k[:, K - 1]
        res_thr = np.maximum(self.res_s[:, Kr - 1], self.res_seed)
        top_g, top_v, top_t = [], [], []
        res_g, res_v, res_k, res_t = [], [], [], []
        for p, sgn in ((0, 1.0), (1, -1.0)):
            s = vals * np.float32(sgn)
            g = (lay * 2 + p) * D + cols
            m = (s > self.top_seed[g]) & (top_key(s, tok) > kth_key[g])
            top_g.append(g[m]); top_v.append(s[m]); top_t.append(tok[m])
            if not self.cfg.reservoir:
                continue
            b = bin_of(s, self.E[lay, p, cols])
            gr = g * B + np.maximum(b, 0)
            m = (b >= 0) & (key >= self.U_res) & (neg_i64(key) > res_thr[gr])
            res_g.append(gr[m]); res_k.append(key[m]); res_t.append(tok[m]); res_v.append(vals[m])
        if self.cfg.reservoir:  # bulk rows (key < U_res), per layer and pole (core.py:529-545)
            colsD = np.arange(D)
            for l, _ in ok:
                R = self._pending[l][4]
                if R is None or R.shape[0] == 0:
                    continue
                ridx = ctx.sub_idx[ctx.res_in_sub]
                rk, rt = ctx.key[ridx], ctx.tok[ridx]
                for p, sgn in ((0, 1.0), (1, -1.0)):
                    s = R * np.float32(sgn)
                    b = bin_of(s, self.E[l, p])
                    gr = (((l * 2 + p) * D + colsD) * B)[None, :] + np.maximum(b, 0)
                    m = (b >= 0) & (neg_i64(rk)[:, None] > res_thr[gr])
                    r_i, c_i = np.nonzero(m)
                    res_g.append(gr[r_i, c_i]); res_k.append(rk[r_i]); res_t.append(rt[r_i])
                    res_v.append(R[r_i, c_i])
        tg, tv, tt = np.concatenate(top_g), np.concatenate(top_v), np.concatenate(top_t)
        self.stats["top_cand"] += int(tg.size)
        grouped_merge(self.top_k, [self.top_t, self.top_s], tg, top_key(tv, tt), [tt, tv], K,
                      pay_fill=[-1, NEG_INF])
        if not self.cfg.reservoir:
            return
        rg = np.concatenate(res_g)
        self.stats["res_cand"] += int(rg.size)
        grouped_merge(self.res_s, [self.res_t, self.res_v], rg, neg_i64(np.concatenate(res_k)),
                      [np.concatenate(res_t), np.concatenate(res_v).astype(np.float32)], Kr)

    # -------------------------------------------------------------- outputs (core.py:593-704)
    def flush_gram(self):
        if self.gram is not None:
            self.gram64 += self.gram.astype(np.float64)
            self.gram[:] = 0

    _STATE = ["top_s", "top_t", "top_k", "res_s", "res_t", "res_v", "sub_sum", "sub_sq", "sub_bin", "E",
              "top_seed", "res_seed"]

    def state_dict(self) -> dict:
        st = {k: getattr(self, k).copy() for k in self._STATE}
        if self.n_a:
            st["enr"], st["ann_tot"] = self.enr.copy(), self.ann_tot.copy()
        st.update(n_seen=self.n_seen, n_sub=self.n_sub, stats=dict(self.stats),
                  dense_layers=sorted(self._dense_layers), cfg=dict(self.cfg.__dict__), n_a=self.n_a)
        return st

    def load_state_dict(self, st: dict):
        assert st["cfg"] == dict(self.cfg.__dict__)
        assert np.array_equal(np.asarray(st["E"]), self.E)
        for k in self._STATE:
            getattr(self, k)[...] = np.asarray(st[k])
        if self.n_a:
            self.enr[...] = np.asarray(st["enr"]); self.ann_tot[...] = np.asarray(st["ann_tot"])
        if self.gram is not None:
            self.gram64[:] = 0; self.gram[:] = 0; self.gram_rows = 0
        self.n_seen, self.n_sub, self.stats = st["n_seen"], st["n_sub"], dict(st["stats"])
        self._dense_layers = set(st["dense_layers"])

    def merge_from(self, other: "AtlasOracle"):
        """core.py:628-654: concat + top-K per group by the unique int64 keys; sums."""
        assert np.array_equal(other.E, self.E) and other.cfg.__dict__ == self.cfg.__dict__
        assert np.array_equal(other.top_seed, self.top_seed) and np.array_equal(other.res_seed, self.res_seed)
        K, Kr = self.cfg.K, self.cfg.Kr
        for sk, pays, k in (("top_k", ("top_t", "top_s"), K), ("res_s", ("res_t", "res_v"), Kr)):
            allv = np.concatenate((getattr(self, sk), getattr(other, sk)), 1)
            idx = np.argsort(allv, axis=1, kind="stable")[:, ::-1][:, :k]
            setattr(self, sk, np.take_along_axis(allv, idx, 1))
            for pk in pays:
                setattr(self, pk, np.take_along_axis(np.concatenate((getattr(self, pk), getattr(other, pk)), 1), idx, 1))
        for k in ["sub_sum", "sub_sq", "sub_bin"]:
            getattr(self, k)[...] += getattr(other, k)
        if self.n_a:
            self.enr += other.enr; self.ann_tot += other.ann_tot
        if self.gram is not None:
            self.flush_gram(); other.flush_gram(); self.gram64 += other.gram64
            self.gram_rows += other.gram_rows
        self.n_seen += other.n_seen
        self.n_sub += other.n_sub
        for k, x in other.stats.items():
            self.stats[k] = self.stats.get(k, 0) + x

    def result(self) -> dict:
        L, D, B, K, Kr = self.L, self.D, self.B, self.cfg.K, self.cfg.Kr
        self.flush_gram()
        sign = np.array([1.0, -1.0], np.float32).reshape(1, 2, 1, 1)
        out = {"top_val": self.top_s.reshape(L, 2, D, K) * sign, "top_tok": self.top_t.reshape(L, 2, D, K).copy(),
               "res_tok": self.res_t.reshape(L, 2, D, B, Kr).copy(), "res_val": self.res_v.reshape(L, 2, D, B, Kr).copy(),
               "res_key": neg_i64(self.res_s.reshape(L, 2, D, B, Kr)), "edges": self.E.copy(),
               "n_seen": self.n_seen, "n_sub": self.n_sub, "sub_sum": self.sub_sum.copy(),
               "sub_sq": self.sub_sq.copy(), "sub_bin": self.sub_bin.copy(), "stats": dict(self.stats),
               "cfg": dict(self.cfg.__dict__)}
        if self.n_a:
            out["enr"] = self.enr.copy()
            out["ann_tot"] = self.ann_tot.copy()
        if self.gram is not None:
            out["gram"] = symmetrize_upper(self.gram64)
            out["gram_rows"] = self.gram_rows
        out.update(self.verify_seeds())
        return out

    def seed(self, top_seed=None, res_seed_key=None):
        """core.py:680-692."""
        if top_seed is not None:
            self.top_seed[:] = np.asarray(top_seed, np.float32).reshape(-1)
            self._dense_layers = set()
        if res_seed_key is not None:
            k = np.asarray(res_seed_key, np.int64).reshape(-1)
            self.res_seed[:] = np.where(k >= 2**32, I64_MIN, -k)

    def verify_seeds(self) -> dict:
        """core.py:694-704."""
        n_kept = (self.res_t >= 0).sum(1)
        seeded = self.res_seed != I64_MIN
        bad = seeded & (n_kept < self.cfg.Kr)
        L, D, B = self.L, self.D, self.B
        seed_key = np.where(seeded, neg_i64(self.res_seed), np.int64(2**32))
        short = ((self.top_t >= 0).sum(1) < self.cfg.K) & (self.top_seed > NEG_INF)
        return {"res_seeded_bins": int(seeded.sum()), "res_seed_limited_bins": int(bad.sum()),
                "res_seed_limited": bad.reshape(L, 2, D, B), "res_seed_key": seed_key.reshape(L, 2, D, B),
                "top_seed_short_groups": int(short.sum())}


# ----------------------------------------------------------------------------- offline truth
def offline_reference(Hs, toks, edges, K, Kr, rho_sub, seed=0, ann=None, levels=(2, 3, 4)) -> dict:
    """Materialised ground truth for every streamed field (reference.py:9-52). Hs: per layer
    [N, D] fp32 valid-token activations; toks [N]; ann [N, A] 0/1 or None."""
    L = len(Hs)
    N, D = Hs[0].shape
    B = edges.shape[-1]
    toks = np.asarray(toks, np.int64)
    key = token_keys(toks, seed)
    sub = key < int(rho_sub * 2**32)
    out = {k: [] for k in ["top_val", "top_tok", "res_key", "res_tok", "res_val", "sub_sum", "sub_sq",
                           "sub_bin", "gram", "enr"]}
    cols = np.arange(D)
    for l in range(L):
        H = np.asarray(Hs[l], np.float32)
        tv, tt, rk, rt, rv, sb, en = [], [], [], [], [], [], []
        for p, sgn in ((0, 1.0), (1, -1.0)):
            S = H * np.float32(sgn)
            tk = top_key(S, np.broadcast_to(toks[:, None], S.shape))
            i = np.argsort(tk, axis=0, kind="stable")[::-1][:K]
            v = S[i, cols[None, :]]
            tv.append((v * np.float32(sgn)).T); tt.append(toks[i].T)
            b = bin_of(S, edges[l, p])
            kb, tb, vb = [], [], []
            for bb in range(B):
                km = np.where(b == bb, key[:, None], I64_MAX)
                ki = np.argsort(km, axis=0, kind="stable")[:Kr]
                kv = np.take_along_axis(km, ki, 0)
                empty = kv == I64_MAX
                kb.append(kv.T); tb.append(np.where(empty, -1, toks[ki]).T)
                vb.append(np.where(empty, np.float32(np.nan), H[ki, cols[None, :]]).T)
            rk.append(np.stack(kb, 1)); rt.append(np.stack(tb, 1)); rv.append(np.stack(vb, 1))
            bs = b[sub]
            sb.append(np.stack([(bs == bb).sum(0) for bb in range(B)], 1).astype(np.float64))
            if ann is not None:
                Ss = S[sub]
                en.append(np.stack([(Ss >= edges[l, p, :, lev]).astype(np.float64).T @ ann[sub] for lev in levels]))
        out["top_val"].append(np.stack(tv)); out["top_tok"].append(np.stack(tt))
        out["res_key"].append(np.stack(rk)); out["res_tok"].append(np.stack(rt)); out["res_val"].append(np.stack(rv))
        Hsub = H[sub].astype(np.float64)
        out["sub_sum"].append(Hsub.sum(0)); out["sub_sq"].append((Hsub ** 2).sum(0))
        out["sub_bin"].append(np.stack(sb))
        out["gram"].append(Hsub.T @ Hsub)
        if ann is not None:
            out["enr"].append(np.stack(en))
    res = {k: np.stack(v) for k, v in out.items() if v}
    res["n_sub"] = int(sub.sum())
    return res


# ----------------------------------------------------------------------------- pilot math
def pilot_edges(Hs, probs=(0.5, 0.9, 0.99, 0.999, 0.9999)) -> np.ndarray:
    """Quantile lower edges, strictly increasing along the bins (reference.py:55-75)."""
    out = []
    for H in Hs:
        n, D = H.shape
        idx = np.array([min(n - 1, int(round(q * (n - 1)))) for q in probs])
        s = np.sort(np.asarray(H, np.float32), axis=0)
        out.append(np.stack([s[idx].T, (-s[(n - 1) - idx]).T]))
    E = np.stack(out).astype(np.float32)
    for b in range(1, E.shape[-1]):
        E[..., b] = np.maximum(E[..., b], np.nextafter(E[..., b - 1], np.float32(np.inf)))
    return E


def pilot_seeds(Hs, E, K, Kr, n_total, c=4.0, z=2.0, groups=None):
    """Seeds (reference.py:78-122): top seed = nextafter(2K-th largest pilot s, -inf); reservoir key
    ceilings from a z-sigma lower bound of the pilot bin mass; with protein `groups` [n] the bound
    uses the effective count n_eff = (sum_g c_g)^2 / sum_g c_g^2 over the groups' bin counts."""
    tops, keys = [], []
    if groups is not None:
        g = np.asarray(groups, np.int64).reshape(-1)
        order = np.argsort(g, kind="stable")
        gs = g[order]
        run_starts = np.nonzero(np.r_[True, gs[1:] != gs[:-1]])[0]
    for li, H in enumerate(Hs):
        n, D = H.shape
        kk = min(2 * K, n)
        tp, kp = [], []
        for p, sgn in ((0, 1.0), (1, -1.0)):
            s = np.asarray(H, np.float32) * np.float32(sgn)
            t = -np.partition(-s, kk - 1, axis=0)[kk - 1]
            tp.append(nextdown(t))
            ge = s[..., None] >= E[li, p][None]
            in_bin = ge & ~np.concatenate((ge[..., 1:], np.zeros_like(ge[..., :1])), -1)
            cnt = in_bin.sum(0).astype(np.float64)
            if groups is None:
                m_lo = np.maximum(cnt - z * np.sqrt(cnt), 0) / n
            else:
                per = np.add.reduceat(in_bin[order].astype(np.int32), run_starts, axis=0).astype(np.int64)
                n_eff = cnt * cnt / np.maximum((per * per).sum(0).astype(np.float64), 1)  # per: [groups, D, B]
                m_lo = (cnt / n) * np.maximum(1 - z / np.sqrt(np.maximum(n_eff, 1e-9)), 0)
            with np.errstate(divide="ignore"):
                theta = np.where(m_lo > 0, c * Kr * 2.0**32 / (n_total * m_lo), 2.0**32)
            kp.append(np.floor(np.minimum(theta, 2.0**32)).astype(np.int64))
        tops.append(np.stack(tp))
        keys.append(np.stack(kp))
    return np.stack(tops), np.stack(keys)
