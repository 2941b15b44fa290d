"""Sequence datasets and batching — drop-in for haelyons/proteus atlas/data.py, plus a writer of
synthetic datasets in the same on-disk format.

Format (the reference's scripts/build_swissprot.py output): a torch-saved dict with
`acc` (list of str), `seq` (list of str), `len` (int32 [N]), `iv` (int32 [M, 4]: seq index, start,
end, annotation id) and `vocab` (list of annotation names; ids 0-20 are the residue classes).

Batching follows the reference's plan (data.py:50-97): sequences are length-bucketed within
windows of the (shuffled) order, greedily packed while max_len * count <= tokens_per_batch,
batches shuffled within each window; rows of a batch are r*Lmax + 1 + pos (BOS/EOS layout) and
token ids are seq*1024 + pos.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .core import pack_tok

AA = "ACDEFGHIKLMNPQRSTVWY"
# natural-like residue background (approximate UniProt composition, percent), order of AA
AA_BACKGROUND = np.array([8.25, 1.37, 5.45, 6.75, 3.86, 7.07, 2.27, 5.96, 5.84, 9.66, 2.42, 4.06, 4.70, 3.93, 5.53,
                          6.56, 5.34, 6.87, 1.08, 2.92])


@dataclass
class Batch:
    input_ids: torch.Tensor       # [B, Lmax] int64
    attention_mask: torch.Tensor  # [B, Lmax] int64
    valid_rows: torch.Tensor      # [n_v] positions in the flattened [B*Lmax] rows
    tok: torch.Tensor             # [n_v] packed (seq_idx, pos)
    ann: torch.Tensor             # [n_v, M_a] annotation ids, -1 padded
    seq_idx: torch.Tensor         # [B]
    n_rows: int                   # B * Lmax


class SwissProt:
    def __init__(self, path_or_dict, max_res: int = 1022, max_ann: int = 8):
        d = path_or_dict if isinstance(path_or_dict, dict) else torch.load(path_or_dict, weights_only=False)
        self.d = d
        self.seq = d["seq"]
        self.len = torch.as_tensor(d["len"]).long()
        self.vocab = d["vocab"]
        self.max_res, self.max_ann = max_res, max_ann
        iv = torch.as_tensor(d["iv"]).long().reshape(-1, 4)
        iv = iv[torch.argsort(iv[:, 0], stable=True)]
        self.iv = iv
        cnt = torch.bincount(iv[:, 0], minlength=len(self.seq))
        self.iv_ptr = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(cnt, 0)])
        self.ann_dropped = 0

    def __len__(self):
        return len(self.seq)

    def coverage(self, idx: torch.Tensor | None = None) -> dict:
        L = self.len if idx is None else self.len[idx]
        drop = (L - self.max_res).clamp(min=0)
        return {"n_seq": int(L.numel()), "n_res_full": int(L.sum()), "n_res_used": int(L.clamp(max=self.max_res).sum()),
                "n_truncated": int((drop > 0).sum()), "frac_seq_truncated": float((drop > 0).float().mean()),
                "frac_res_dropped": float(drop.sum() / max(1, int(L.sum())))}

    def plan(self, order: torch.Tensor, tokens_per_batch: int, window: int = 8192, seed: int = 0,
             shuffle_batches: bool = True) -> list[list[int]]:
        g = torch.Generator().manual_seed(seed)
        out = []
        for c0 in range(0, len(order), window):
            ch = order[c0:c0 + window]
            Lc = self.len[ch].clamp(max=self.max_res)
            ch = ch[torch.argsort(Lc, stable=True)]
            groups, cur, cur_max = [], [], 0
            for i in ch.tolist():
                n = min(int(self.len[i]), self.max_res) + 2
                m = max(cur_max, n)
                if cur and m * (len(cur) + 1) > tokens_per_batch:
                    groups.append(cur)
                    cur, m = [], n
                cur.append(i)
                cur_max = m
            if cur:
                groups.append(cur)
            perm = torch.randperm(len(groups), generator=g).tolist() if shuffle_batches else range(len(groups))
            out.extend(groups[gi] for gi in perm)
        return out

    def batches(self, tokenizer_vocab: dict, order: torch.Tensor, tokens_per_batch: int, chunk: int = 8192,
                seed: int = 0, start: int = 0, plan: list | None = None, shuffle_batches: bool = True):
        plan = plan if plan is not None else self.plan(order, tokens_per_batch, chunk, seed, shuffle_batches)
        aa_tok = {c: tokenizer_vocab.get(c, tokenizer_vocab["<unk>"]) for c in set(AA) | set("XBUZO")}
        cls_, eos, pad = tokenizer_vocab["<cls>"], tokenizer_vocab["<eos>"], tokenizer_vocab["<pad>"]
        for grp in plan[start:]:
            yield self._make(grp, aa_tok, cls_, eos, pad)

    def pilot_plan(self, plan: list[list[int]], pilot_tokens: int, tokens_per_batch: int, seed: int = 0):
        """Pilot batches of sequences drawn uniformly from the whole plan (every pilot sequence is
        also streamed, which keeps the top-K seed exact)."""
        seqs = [i for grp in plan for i in grp]
        perm = torch.randperm(len(seqs), generator=torch.Generator().manual_seed(seed + 7)).tolist()
        pick, n = [], 0
        for j in perm:
            i = seqs[j]
            pick.append(i)
            n += min(int(self.len[i]), self.max_res)
            if n >= pilot_tokens:
                break
        return self.plan(torch.tensor(pick), tokens_per_batch, window=len(pick), seed=seed)

    def _make(self, idx, aa_tok, cls_, eos, pad) -> Batch:
        B = len(idx)
        lens = [min(int(self.len[i]), self.max_res) for i in idx]
        Lmax = max(lens) + 2
        ids = torch.full((B, Lmax), pad, dtype=torch.long)
        am = torch.zeros((B, Lmax), dtype=torch.long)
        lut = np.full(128, aa_tok["X"], np.int64)
        for c, t in aa_tok.items():
            lut[ord(c)] = t
        rows, toks, anns = [], [], []
        for r, (i, n) in enumerate(zip(idx, lens)):
            s = self.seq[i][:n]
            codes = np.frombuffer(s.encode("ascii"), np.uint8)
            ids[r, 0] = cls_
            ids[r, 1:n + 1] = torch.from_numpy(lut[codes])
            ids[r, n + 1] = eos
            am[r, :n + 2] = 1
            rows.append(r * Lmax + 1 + torch.arange(n))
            toks.append(pack_tok(torch.full((n,), i), torch.arange(n)))
            anns.append(self._ann(i, codes, n))
        return Batch(ids, am, torch.cat(rows), torch.cat(toks), torch.cat(anns), torch.tensor(idx), B * Lmax)

    _AA_IDX = None

    def _ann(self, i, codes, n) -> torch.Tensor:
        if SwissProt._AA_IDX is None:
            t = np.full(128, 20, np.int64)
            for k, c in enumerate(AA):
                t[ord(c)] = k
            SwissProt._AA_IDX = t
        A = torch.full((n, self.max_ann), -1, dtype=torch.long)
        A[:, 0] = torch.from_numpy(SwissProt._AA_IDX[codes])
        iv = self.iv[self.iv_ptr[i]:self.iv_ptr[i + 1]]
        if iv.numel():
            fill = torch.ones(n, dtype=torch.long)
            for _, a0, a1, k in iv.tolist():
                a1 = min(a1, n)
                if a0 >= a1:
                    continue
                pos = torch.arange(a0, a1)
                ok = fill[pos] < self.max_ann
                self.ann_dropped += int((~ok).sum())
                pos = pos[ok]
                A[pos, fill[pos]] = k
                fill[pos] += 1
        return A


def shuffled_order(n: int, seed: int = 0) -> torch.Tensor:
    return torch.randperm(n, generator=torch.Generator().manual_seed(seed))


def synthetic_dataset(n_seq: int, seed: int = 0, median_len: float = 300.0, sigma: float = 0.6, max_len: int = 1022,
                      low_complexity: float = 0.005) -> dict:
    """Synthetic proteins in the on-disk format: log-normal lengths (median, sigma) truncated at
    max_len, residues from a natural-like background, a fraction of low-complexity sequences
    (80% Ser or 80% Gly) that trigger dense-path bursts. No annotation intervals: the annotation
    classes are the 21 residue classes."""
    rng = np.random.default_rng(seed)
    lens = np.clip(np.round(rng.lognormal(np.log(median_len), sigma, n_seq)), 8, max_len).astype(np.int32)
    p = AA_BACKGROUND / AA_BACKGROUND.sum()
    letters = np.frombuffer(AA.encode(), np.uint8)
    lowc = rng.random(n_seq) < low_complexity
    seqs = []
    for i, n in enumerate(lens.tolist()):
        codes = letters[rng.choice(20, n, p=p)]
        if lowc[i]:
            mark = rng.random(n) < 0.8
            codes = codes.copy()
            codes[mark] = ord("S") if rng.random() < 0.5 else ord("G")
        seqs.append(codes.tobytes().decode())
    return {"acc": [f"SYN{i:07d}" for i in range(n_seq)], "seq": seqs, "len": torch.from_numpy(lens),
            "iv": torch.zeros((0, 4), dtype=torch.int32), "vocab": list(AA) + ["X"],
            "low_complexity": torch.from_numpy(lowc)}
