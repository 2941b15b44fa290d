"""Pilot-pass math: bin edges and exact-preserving seeds — drop-in for haelyons/proteus
atlas/reference.py:pilot_edges / pilot_seeds (reference.py:55-122).

Runs once per run on the device holding the pilot activations (PyTorch ops; not on the per-batch
hot path). One column-chunk sort serves both poles: the pole-1 order statistics are the negated
pole-0 ones read from the other end.
"""
from __future__ import annotations

import torch


def _quantile_rows(n: int, probs) -> list[int]:
    return [min(n - 1, int(round(q * (n - 1)))) for q in probs]


def pilot_edges(Hs: list, probs=(0.5, 0.9, 0.99, 0.999, 0.9999), chunk: int = 512) -> torch.Tensor:
    """E[l, p, d, b] = probs[b]-quantile (row round(q*(n-1)) of the sorted column) of s = +h / -h,
    forced strictly increasing along b. Returns [L, 2, D, B] fp32 on the input's device."""
    out = []
    for H in Hs:
        n, D = H.shape
        idx = torch.tensor(_quantile_rows(n, probs), device=H.device)
        ridx = (n - 1) - idx
        p0, p1 = [], []
        for c0 in range(0, D, chunk):
            s, _ = torch.sort(H[:, c0:c0 + chunk].float(), dim=0)
            p0.append(s.index_select(0, idx).T)
            p1.append((-s.index_select(0, ridx)).T)  # sort(-h)[i] == -sort(h)[n-1-i]
            del s
        out.append(torch.stack([torch.cat(p0), torch.cat(p1)]))
    E = torch.stack(out)
    for b in range(1, E.shape[-1]):
        E[..., b] = torch.maximum(E[..., b], torch.nextafter(E[..., b - 1], torch.full_like(E[..., b - 1], float("inf"))))
    return E


def pilot_seeds(Hs: list, E: torch.Tensor, K: int, Kr: int, n_total: int, c: float = 4.0, z: float = 2.0,
                chunk: int = 512, groups: torch.Tensor | None = None):
    """Seeds from pilot activations of tokens that are also streamed (reference.py:78-122):
    top_seed [L,2,D] = nextafter(2K-th largest pilot s, -inf); res_seed_key [L,2,D,B] = floor of
    c*Kr*2^32 / (n_total * m_lo) clamped to 2^32, m_lo a z-sigma lower bound of the pilot bin mass
    (with protein groups: effective count n_eff = (sum c_i)^2 / sum c_i^2). Returns CPU tensors."""
    if groups is not None:
        _, gidx = torch.unique(groups, return_inverse=True)
        n_g = int(gidx.max()) + 1
        chunk = min(chunk, 128)
    tops, keys = [], []
    for li, H in enumerate(Hs):
        n, D = H.shape
        kk = min(2 * K, n)
        tp, kp = [], []
        for p, sgn in ((0, 1.0), (1, -1.0)):
            t_cols, k_cols = [], []
            Ep = E[li, p].to(H.device)
            for c0 in range(0, D, chunk):
                s = H[:, c0:c0 + chunk].float() * sgn
                t = torch.topk(s, kk, dim=0).values[kk - 1]
                t_cols.append(torch.nextafter(t, torch.full_like(t, float("-inf"))))
                ge = s.unsqueeze(-1) >= Ep[c0:c0 + chunk]
                in_bin = ge & ~torch.cat((ge[..., 1:], torch.zeros_like(ge[..., :1])), -1)
                cnt = in_bin.sum(0).double()
                if groups is None:
                    m_lo = (cnt - z * cnt.sqrt()).clamp(min=0) / n
                else:
                    per = torch.zeros((n_g,) + tuple(cnt.shape), dtype=torch.float32, device=s.device)
                    per.index_add_(0, gidx.to(s.device), in_bin.float())
                    n_eff = cnt ** 2 / (per.double() ** 2).sum(0).clamp(min=1)
                    m_lo = (cnt / n) * (1 - z / n_eff.clamp(min=1e-9).sqrt()).clamp(min=0)
                    del per
                theta = torch.where(m_lo > 0, c * Kr * 2.0**32 / (n_total * m_lo), torch.full_like(m_lo, 2.0**32))
                k_cols.append(theta.clamp(max=2.0**32).floor().to(torch.int64))
                del s, ge, in_bin
            tp.append(torch.cat(t_cols))
            kp.append(torch.cat(k_cols))
        tops.append(torch.stack(tp))
        keys.append(torch.stack(kp))
    return torch.stack(tops).cpu(), torch.stack(keys).cpu()
