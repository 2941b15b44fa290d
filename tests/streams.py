"""Seeded synthetic activation streams shared by the golden-fixture script, the oracle tests and
the GPU parity tests.

`make_stream` follows the shape of the reference's own exactness stream
(haelyons/proteus tests/test_exactness.py:17-31, :54-86): per-sequence activations
Gaussian * scale + shift, rare x5 outlier spikes, a late distribution shift after 70% of the
sequences (forces candidate-buffer overflow and dense redo), optional grid rounding (tie-heavy),
variable batch sizes 4-40, BOS/EOS row layout r*Lmax+1+pos, garbage x50 on padding rows. It is
written with numpy's PCG64 so the same stream can be rebuilt anywhere; `stream_digest` fingerprints
it so a fixture can tell when a rebuild differs.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np

SEQ_STRIDE = 1024


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even), returned as fp32 (finite inputs)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def cast(x: np.ndarray, dtype: str) -> np.ndarray:
    return bf16_round(x) if dtype == "bf16" else np.asarray(x, np.float32)


@dataclass
class Batch:
    T: int
    H: list            # per layer [T, D] fp32 (exact images of the stream dtype)
    valid_rows: np.ndarray
    tok: np.ndarray
    ann: np.ndarray    # [n_v, 3] annotation ids, -1 padded


@dataclass
class Stream:
    L: int
    D: int
    dtype: str
    lens: np.ndarray
    seqs: list          # per sequence [L, n, D] fp32
    ann_full: list      # per sequence [n, 3]
    batches: list
    order: list

    def all_tokens(self):
        """Valid-token activations per layer in sequence order, with token ids and annotations."""
        Hall = [np.concatenate([s[l] for s in self.seqs]) for l in range(self.L)]
        toks = np.concatenate([np.int64(j) * SEQ_STRIDE + np.arange(int(n), dtype=np.int64)
                               for j, n in enumerate(self.lens)])
        return Hall, toks, np.concatenate(self.ann_full)


def make_stream(L=3, D=96, n_seq=600, seed=0, dtype="bf16", grid=0.0, shuffle_order=False,
                n_annot=7, bmin=4, bmax=40, lmin=5, lmax=120) -> Stream:
    g = np.random.default_rng(seed)
    lens = g.integers(lmin, lmax, n_seq)
    scale = (g.random((L, D)) * 3 + 0.1).astype(np.float32)
    shift = g.standard_normal((L, D)).astype(np.float32)
    seqs = []
    for i, n in enumerate(lens.tolist()):
        H = g.standard_normal((L, n, D)).astype(np.float32) * scale[:, None] + shift[:, None]
        H = H * (1 + 4 * (g.random((L, n, D)) < 0.002)).astype(np.float32)
        if i > 0.7 * n_seq:
            H = H + np.float32(2.5) * scale[:, None]
        if grid:
            H = np.round(H / grid) * np.float32(grid)
        seqs.append(cast(H, dtype))
    ann_full = [g.integers(-1, n_annot, (int(n), 3)) for n in lens]
    order = (g.permutation(n_seq).tolist() if shuffle_order else list(range(n_seq)))
    batches = []
    i = 0
    while i < n_seq:
        bsz = int(g.integers(bmin, bmax))
        idx = order[i:min(n_seq, i + bsz)]
        i += len(idx)
        Lmax = max(int(lens[j]) for j in idx) + 2
        T = len(idx) * Lmax
        Hb = [cast(g.standard_normal((T, D)).astype(np.float32) * 50, dtype) for _ in range(L)]
        vr, tk, an = [], [], []
        for r, j in enumerate(idx):
            n = int(lens[j])
            rows = r * Lmax + 1 + np.arange(n)
            for l in range(L):
                Hb[l][rows] = seqs[j][l]
            vr.append(rows)
            tk.append(np.int64(j) * SEQ_STRIDE + np.arange(n, dtype=np.int64))
            an.append(ann_full[j])
        batches.append(Batch(T, Hb, np.concatenate(vr).astype(np.int64), np.concatenate(tk),
                             np.concatenate(an).astype(np.int64)))
    return Stream(L, D, dtype, lens, seqs, ann_full, batches, order)


def stream_digest(st: Stream) -> str:
    h = hashlib.sha256()
    for b in st.batches:
        for x in b.H:
            h.update(np.ascontiguousarray(x).tobytes())
        h.update(b.valid_rows.tobytes()); h.update(b.tok.tobytes()); h.update(b.ann.tobytes())
    return h.hexdigest()


def pilot_edges_np(Hs, probs=(0.5, 0.9, 0.99, 0.999, 0.9999)) -> np.ndarray:
    """Quantile lower edges per (layer, pole, column), strictly increasing — the reference's
    pilot_edges rule (atlas/reference.py:55-75) in numpy, used to seed test streams."""
    out = []
    for H in Hs:
        n, D = H.shape
        idx = np.array([min(n - 1, int(round(q * (n - 1)))) for q in probs])
        per = []
        for sgn in (1.0, -1.0):
            s = np.sort(H.astype(np.float32) * np.float32(sgn), axis=0)
            per.append(s[idx].T)
        out.append(np.stack(per))
    E = np.stack(out).astype(np.float32)
    for b in range(1, E.shape[-1]):
        E[..., b] = np.maximum(E[..., b], np.nextafter(E[..., b - 1], np.float32(np.inf)))
    return E


# ----------------------------------------------------------------------------- kernel-level inputs
FILTER_CASES = [dict(T=777, D=300, thr_base=2.5, ninf=7), dict(T=500, D=256, thr_base=8.0, ninf=0),
                dict(T=1024, D=96, thr_base=1.0, ninf=3)]


def filter_inputs(case: int):
    """Filter-kernel case in the shape of the reference's tests/test_triton_kernel.py:13-46:
    bf16 H ~ N(0, 2^2), 15% padding rows, thresholds U(thr_base, thr_base+2), a few columns whose
    negative threshold is -inf (everything valid survives there)."""
    c = FILTER_CASES[case]
    g = np.random.default_rng(100 + case)
    H = bf16_round(g.standard_normal((c["T"], c["D"])).astype(np.float32) * 2)
    valid = g.random(c["T"]) > 0.15
    rowmap = np.full(c["T"], -1, np.int64)
    rowmap[valid] = np.arange(int(valid.sum()))
    tp = (g.random(c["D"]) * 2 + c["thr_base"]).astype(np.float32)
    tn = (g.random(c["D"]) * 2 + c["thr_base"]).astype(np.float32)
    tn[:c["ninf"]] = -np.inf
    return H, rowmap, tp, tn


STATS_CASES = [dict(n=203, D=150, B=5, levels=(2, 3, 4)), dict(n=5, D=33, B=5, levels=(2, 3, 4)),
               dict(n=37, D=40, B=5, levels=()), dict(n=1000, D=64, B=5, levels=(1, 3))]


def stats_inputs(case: int):
    """Subsample-statistics case in the shape of tests/test_stats_triton.py:18-49: per-column scaled
    Gaussian bf16 rows, edges taken from the data's own quantiles (exact ties on edges occur)."""
    c = STATS_CASES[case]
    g = np.random.default_rng(200 + case)
    n, D, B = c["n"], c["D"], c["B"]
    X = bf16_round(g.standard_normal((n, D)).astype(np.float32) * (g.random(D).astype(np.float32) * 2 + 0.2))
    q = np.array([0.5, 0.9, 0.99, 0.999, 0.9999][:B])
    k = (q * (n - 1)).astype(np.int64)
    E0 = np.ascontiguousarray(np.sort(X, 0)[k].T)
    E1 = np.ascontiguousarray(np.sort(-X, 0)[k].T)
    return X, E0, E1, c["levels"]


def pilot_inputs():
    """Heavy-tailed pilot activations for two layers (the second rounded to quarters: ties on
    edges), 100 proteins of 30 rows each."""
    g = np.random.default_rng(9)
    n, D = 3000, 40
    Hs = [(g.standard_t(3, (n, D)) * (g.random(D) + 0.5) + g.standard_normal(D) * 0.5).astype(np.float32)
          for _ in range(2)]
    Hs[1] = (np.round(Hs[1] * 4) / 4).astype(np.float32)
    groups = np.repeat(np.arange(n // 30), 30).astype(np.int64)
    return Hs, groups
