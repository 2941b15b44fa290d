"""Protein datasets, the deterministic batch plan and batch tensors — drop-in for haelyons/proteus
atlas/data.py (same names: `SwissProt`, `Batch`, `shuffled_order`), plus `synthetic_dataset`, a
writer of synthetic proteins in the same on-disk format.

On-disk format (the output of the reference's scripts/build_swissprot.py:3-10): a torch-saved dict
  acc   list[str]        accession per sequence
  seq   list[str]        residues (one letter per residue)
  len   int32 [N]        sequence lengths
  iv    int32 [M, 4]     annotation intervals (sequence index, start, end exclusive, annotation id)
  vocab list[str]        annotation names; ids 0-19 are the standard residues, 20 the others

The batch plan has to be the reference's, batch for batch: a checkpoint records the index of the
next batch of the plan, and a run resumed by either build must continue with the same sequences.
The rule (atlas/data.py:50-74):
  1. the sequence order is cut into consecutive windows of `window` sequences;
  2. inside a window the sequences are sorted by truncated length, min(len, max_res), stably;
  3. the lengths then never decrease along the window, so a batch of `m` sequences whose longest
     (= last) one has truncated length n occupies m * (n + 2) padded rows (BOS and EOS); a
     sequence joins the open batch while that product stays <= tokens_per_batch and otherwise
     opens the next batch;
  4. the batches of each window are permuted by torch.randperm on ONE torch.Generator seeded with
     `seed` and carried across windows (no permutation with shuffle_batches=False).
The pilot plan (atlas/data.py:86-97) draws sequences of the whole plan in the order of
torch.randperm(n, generator seeded with seed + 7) until their truncated lengths reach pilot_tokens,
and plans them as one window.

Batch layout (atlas/data.py:99-116): row r of a batch holds <cls>, the residues, <eos>, then
padding up to the batch's longest sequence + 2; the flattened row of residue p of row r is
r * Lmax + 1 + p; token id = sequence index * 1024 + p (core.pack_tok). Per-residue annotation ids
(atlas/data.py:118-135): column 0 is the residue class; the intervals of the sequence, in file
order, fill columns 1, 2, ... of every position they cover, and an interval that finds a position's
max_ann columns full is dropped there (counted in `ann_dropped`).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .core import pack_tok

AA = "ACDEFGHIKLMNPQRSTVWY"
_TOKEN_LETTERS = AA + "XBUZO"  # letters with their own ESM token; anything else is read as X
# natural-like residue background (approximate UniProt composition, percent), order of AA
AA_BACKGROUND = np.array([8.25, 1.37, 5.45, 6.75, 3.86, 7.07, 2.27, 5.96, 5.84, 9.66, 2.42, 4.06, 4.70, 3.93, 5.53,
                          6.56, 5.34, 6.87, 1.08, 2.92])

_CLASS_OF_ASCII = np.full(256, 20, np.int64)  # residue class per ASCII code: 0-19 standard, 20 other
for _k, _c in enumerate(AA):
    _CLASS_OF_ASCII[ord(_c)] = _k


@dataclass
class Batch:
    input_ids: torch.Tensor       # [B, Lmax] int64
    attention_mask: torch.Tensor  # [B, Lmax] int64
    valid_rows: torch.Tensor      # [n_v] positions in the flattened [B*Lmax] rows
    tok: torch.Tensor             # [n_v] packed (seq_idx, pos)
    ann: torch.Tensor             # [n_v, max_ann] annotation ids, -1 padded
    seq_idx: torch.Tensor         # [B]
    n_rows: int                   # B * Lmax (rows the hooks see, padding included)


def _ascii(s: str) -> np.ndarray:
    return np.frombuffer(s.encode("ascii", "replace"), np.uint8)


def pack_window(lengths: np.ndarray, tokens_per_batch: int) -> list[tuple[int, int]]:
    """[start, stop) ranges of the batches of one window whose truncated lengths are sorted
    ascending (rule 3 of the module docstring)."""
    out, start = [], 0
    for j, n in enumerate(lengths.tolist()):
        if j > start and (n + 2) * (j - start + 1) > tokens_per_batch:
            out.append((start, j))
            start = j
    if len(lengths):
        out.append((start, len(lengths)))
    return out


class SwissProt:
    """A protein dataset in the on-disk format (a path, or the dict itself)."""

    def __init__(self, path_or_dict, max_res: int = 1022, max_ann: int = 8):
        d = path_or_dict if isinstance(path_or_dict, dict) else torch.load(path_or_dict, weights_only=False)
        self.d = d
        self.seq = d["seq"]
        self.len = torch.as_tensor(d["len"]).long()
        self.vocab = d["vocab"]
        self.max_res, self.max_ann = max_res, max_ann
        self._trunc = self.len.clamp(max=max_res).numpy()
        iv = np.asarray(torch.as_tensor(d["iv"]).long().reshape(-1, 4).numpy())
        # intervals grouped by sequence, file order kept within a sequence
        iv = iv[np.argsort(iv[:, 0], kind="stable")]
        self._iv = iv
        self._iv_start = np.searchsorted(iv[:, 0], np.arange(len(self.seq) + 1), side="left")
        self.ann_dropped = 0

    def __len__(self):
        return len(self.seq)

    def coverage(self, idx: torch.Tensor | None = None) -> dict:
        """Sequence / residue counts of the (selected) sequences and what truncation drops."""
        n = self.len if idx is None else self.len[idx]
        cut = (n - self.max_res).clamp(min=0)
        total = int(n.sum())
        return {"n_seq": int(n.numel()), "n_res_full": total, "n_res_used": total - int(cut.sum()),
                "n_truncated": int((cut > 0).sum()), "frac_seq_truncated": float((cut > 0).float().mean()),
                "frac_res_dropped": float(cut.sum() / max(1, total))}  # float32, as the reference reports it

    # ------------------------------------------------------------------ plans
    def plan(self, order: torch.Tensor, tokens_per_batch: int, window: int = 8192, seed: int = 0,
             shuffle_batches: bool = True) -> list[list[int]]:
        """The deterministic batch plan (lists of sequence indices) of the module docstring."""
        order = np.asarray(torch.as_tensor(order).long().numpy())
        gen = torch.Generator().manual_seed(seed)
        plan = []
        for w0 in range(0, order.size, window):
            win = order[w0:w0 + window]
            win = win[np.argsort(self._trunc[win], kind="stable")]
            batches = [win[a:b].tolist() for a, b in pack_window(self._trunc[win], tokens_per_batch)]
            if shuffle_batches:
                batches = [batches[k] for k in torch.randperm(len(batches), generator=gen).tolist()]
            plan += batches
        return plan

    def pilot_plan(self, plan: list[list[int]], pilot_tokens: int, tokens_per_batch: int, seed: int = 0):
        """Pilot batches from sequences drawn uniformly from the whole plan (all lengths). Every
        pilot sequence is streamed as well, which keeps the top-K seed exact."""
        pool = [i for batch in plan for i in batch]
        perm = torch.randperm(len(pool), generator=torch.Generator().manual_seed(seed + 7)).numpy()
        drawn = np.asarray(pool, np.int64)[perm] if pool else np.zeros(0, np.int64)
        reach = np.cumsum(self._trunc[drawn]) if drawn.size else drawn
        k = int(np.searchsorted(reach, pilot_tokens, side="left")) + 1  # first prefix that reaches the target
        pick = drawn[:min(k, drawn.size)]
        return self.plan(torch.from_numpy(pick.copy()), tokens_per_batch, window=max(1, pick.size), seed=seed)

    # ------------------------------------------------------------------ batches
    def batches(self, tokenizer_vocab: dict, order: torch.Tensor, tokens_per_batch: int, chunk: int = 8192,
                seed: int = 0, start: int = 0, plan: list | None = None, shuffle_batches: bool = True):
        """Batch objects of the plan from batch index `start` (the plan is built when not given)."""
        plan = plan if plan is not None else self.plan(order, tokens_per_batch, chunk, seed, shuffle_batches)
        for group in plan[start:]:
            yield self.make_batch(group, tokenizer_vocab)

    def make_batch(self, group: list[int], tokenizer_vocab: dict) -> Batch:
        """Padded input ids, attention mask, valid rows, token ids and annotations of one batch."""
        v = tokenizer_vocab
        unk = v["<unk>"]
        lut = np.full(256, v.get("X", unk), np.int64)
        for c in _TOKEN_LETTERS:
            lut[ord(c)] = v.get(c, unk)
        lens = [int(self._trunc[i]) for i in group]
        B, Lmax = len(group), max(lens) + 2
        ids = np.full((B, Lmax), v["<pad>"], np.int64)
        am = np.zeros((B, Lmax), np.int64)
        rows, toks, anns = [], [], []
        for r, (i, n) in enumerate(zip(group, lens)):
            codes = _ascii(self.seq[i][:n])
            ids[r, 0], ids[r, n + 1] = v["<cls>"], v["<eos>"]
            ids[r, 1:n + 1] = lut[codes]
            am[r, :n + 2] = 1
            rows.append(r * Lmax + 1 + np.arange(n))
            toks.append(pack_tok(torch.full((n,), i), torch.arange(n)))
            anns.append(self.annotations(i, codes))
        return Batch(torch.from_numpy(ids), torch.from_numpy(am), torch.from_numpy(np.concatenate(rows)),
                     torch.cat(toks), torch.from_numpy(np.concatenate(anns)), torch.tensor(group), B * Lmax)

    def annotations(self, i: int, codes: np.ndarray) -> np.ndarray:
        """[n, max_ann] annotation ids of sequence i's first n residues (module docstring)."""
        n = codes.size
        A = np.full((n, self.max_ann), -1, np.int64)
        A[:, 0] = _CLASS_OF_ASCII[codes]
        iv = self._iv[self._iv_start[i]:self._iv_start[i + 1]]
        if iv.size == 0 or self.max_ann < 2:
            return A
        pos, cls = [], []
        for _, a0, a1, k in iv.tolist():
            a1 = min(a1, n)
            if a0 < a1:
                pos.append(np.arange(a0, a1))
                cls.append(np.full(a1 - a0, k, np.int64))
        if not pos:
            return A
        pos, cls = np.concatenate(pos), np.concatenate(cls)
        o = np.argsort(pos, kind="stable")  # per position, the covering intervals in file order
        pos, cls = pos[o], cls[o]
        first = np.searchsorted(pos, pos, side="left")
        col = 1 + np.arange(pos.size) - first
        keep = col < self.max_ann
        A[pos[keep], col[keep]] = cls[keep]
        self.ann_dropped += int((~keep).sum())
        return A


def shuffled_order(n: int, seed: int = 0) -> torch.Tensor:
    """The seeded sequence order of a run (torch.randperm on a generator seeded with `seed`)."""
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
