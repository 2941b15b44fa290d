"""Pilot pass on the device: bin edges and exact-preserving seeds — drop-in for haelyons/proteus
atlas/reference.py:pilot_edges / pilot_seeds (reference.py:55-122), same arguments and results.

The reference sorts every column (torch.sort) for the edges and takes a top-k per column for the top
seed. Both only need a few order statistics per column, so here they are exact radix selections on
the device (atlas_column_select over the transposed pilot activations), and the bin masses and
per-protein counts behind the reservoir seeds are integer counts (atlas_pilot_counts), finished by
the reference's fp64 arithmetic in atlas_pilot_seeds. Activations must be on a CUDA device (bf16,
fp16 or fp32); there is no CPU path.

  edges  E[l, 0, d, b] = value at rank round(q_b (n-1)) of column d;  E[l, 1, d, b] = the same for
         s = -h; forced strictly increasing along b with nextafter(., +inf)
  seeds  top_seed[l, p, d] = nextafter(2K-th largest s, -inf); res_seed_key[l, p, d, b] = key
         ceiling with c*Kr expected keys below it over the stream, from a z-sigma lower bound of the
         bin's pilot mass (with protein groups: effective count n_eff = (sum c_i)^2 / sum c_i^2)
"""
from __future__ import annotations

import torch

from ._lib import AtlasKernelError, call, dtype_code, ptr, stream_ptr

ROWS_PER_CHUNK = 4096  # pilot rows per CTA column-strip in the count kernel


def _device_input(H: torch.Tensor) -> torch.Tensor:
    if not H.is_cuda:
        raise AtlasKernelError("pilot activations must be on a CUDA device: the pilot runs on the sm_100a kernels")
    if H.dim() != 2 or H.shape[0] < 1:
        raise ValueError(f"pilot activations must be [n >= 1, D], got {tuple(H.shape)}")
    return H if H.stride(1) == 1 else H.contiguous()


def _transposed(H: torch.Tensor) -> torch.Tensor:
    """XT [D, ldx] (ldx = n rounded up to 8) holding H transposed (atlas_gather_transpose)."""
    n, D = H.shape
    ldx = -(-n // 8) * 8
    XT = torch.empty(D, ldx, dtype=H.dtype, device=H.device)
    rows = torch.arange(n, dtype=torch.int32, device=H.device)
    call("atlas_gather_transpose", ptr(H), dtype_code(H.dtype), n, D, H.stride(0), ptr(rows), n, ptr(XT), ldx, 0,
         stream_ptr(H.device))
    return XT


def column_values_at_ranks(H: torch.Tensor, ranks: list[int]) -> torch.Tensor:
    """[D, len(ranks)] fp32: per column of H [n, D], the values at the given ascending ranks."""
    import ctypes
    H = _device_input(H)
    n, D = H.shape
    XT = _transposed(H)
    out = torch.empty(D, len(ranks), dtype=torch.float32, device=H.device)
    rk = (ctypes.c_int64 * len(ranks))(*ranks)
    call("atlas_column_select", ptr(XT), dtype_code(H.dtype), XT.stride(0), n, D, ctypes.cast(rk, ctypes.c_void_p),
         len(ranks), ptr(out), stream_ptr(H.device))
    return out


def _quantile_ranks(n: int, probs) -> list[int]:
    return [min(n - 1, int(round(q * (n - 1)))) for q in probs]


def pilot_edges(Hs: list, probs=(0.5, 0.9, 0.99, 0.999, 0.9999), chunk: int = 512) -> torch.Tensor:
    """E [L, 2, D, B] fp32 on the activations' device (`chunk`, the reference's column chunk of its
    sort, is accepted and unused)."""
    out = []
    for H in Hs:
        H = _device_input(H)
        n, D = H.shape
        r = _quantile_ranks(n, probs)
        B = len(r)
        sel = column_values_at_ranks(H, r + [(n - 1) - x for x in r])
        E = torch.empty(2, D, B, dtype=torch.float32, device=H.device)
        call("atlas_pilot_edges", ptr(sel), D, B, ptr(E), stream_ptr(H.device))
        out.append(E)
    return torch.stack(out)


def _visiting_order(groups: torch.Tensor | None, n: int, dev):
    """(order int32 | None, run_last uint8 | None, chunk_start int64): rows grouped by protein
    (stable), the end of each protein's run, and chunk starts at run starts."""
    if groups is None:
        starts = torch.arange(0, n, ROWS_PER_CHUNK, dtype=torch.int64, device=dev)
        return None, None, torch.cat([starts, torch.tensor([n], dtype=torch.int64, device=dev)])
    g = groups.reshape(-1).to(dev, torch.int64)
    if g.numel() != n:
        raise ValueError(f"groups has {g.numel()} entries for {n} pilot rows")
    order = torch.argsort(g, stable=True)
    gs = g[order]
    change = torch.ones(n, dtype=torch.bool, device=dev)
    change[1:] = gs[1:] != gs[:-1]                       # first row of each run
    run_last = torch.ones(n, dtype=torch.uint8, device=dev)
    run_last[:-1] = change[1:].to(torch.uint8)           # last row of each run
    run_starts = torch.nonzero(change).squeeze(1)
    n_chunks = max(1, min(65535, -(-n // ROWS_PER_CHUNK)))
    want = torch.arange(n_chunks, dtype=torch.int64, device=dev) * n // n_chunks
    pos = torch.searchsorted(run_starts, want).clamp(max=run_starts.numel() - 1)
    starts = torch.unique(run_starts[pos])
    return order.to(torch.int32), run_last, torch.cat([starts, torch.tensor([n], dtype=torch.int64, device=dev)])


def pilot_seeds(Hs: list, E: torch.Tensor, K: int, Kr: int, n_total: int, c: float = 4.0, z: float = 2.0,
                chunk: int = 512, groups: torch.Tensor | None = None):
    """(top_seed [L, 2, D] fp32, res_seed_key [L, 2, D, B] int64), CPU tensors, from pilot activations
    of tokens that are also streamed; `groups` [n] gives each pilot row's protein (`chunk` is
    accepted and unused)."""
    tops, keys = [], []
    for li, H in enumerate(Hs):
        H = _device_input(H)
        n, D = H.shape
        dev = H.device
        El = E[li].to(dev, torch.float32).contiguous()
        B = El.shape[-1]
        kk = min(2 * K, n)
        sel2 = column_values_at_ranks(H, [n - kk, kk - 1])
        order, run_last, cstart = _visiting_order(groups, n, dev)
        cnt = torch.zeros(2, D, B, dtype=torch.int64, device=dev)
        sq = torch.zeros(2, D, B, dtype=torch.int64, device=dev)
        st = stream_ptr(dev)
        call("atlas_pilot_counts", ptr(H), dtype_code(H.dtype), H.stride(0), n, D, ptr(order), ptr(run_last),
             ptr(cstart), cstart.numel() - 1, ptr(El), B, ptr(cnt), ptr(sq), st)
        top = torch.empty(2, D, dtype=torch.float32, device=dev)
        key = torch.empty(2, D, B, dtype=torch.int64, device=dev)
        call("atlas_pilot_seeds", ptr(cnt), ptr(sq), ptr(sel2), D, B, n, Kr, int(n_total), float(c), float(z),
             int(groups is not None), ptr(top), ptr(key), st)
        tops.append(top)
        keys.append(key)
    return torch.stack(tops).cpu(), torch.stack(keys).cpu()


@torch.no_grad()
def pilot_pass(model, batches: list, device, n_layers: int, d_ff: int, probs=(0.5, 0.9, 0.99, 0.999, 0.9999),
               seeds: tuple | None = None, edges: torch.Tensor | None = None, mem_frac: float = 0.45):
    """Edges (and, with seeds=(K, Kr, n_total), the seeds) of a pilot over `batches`, with the pilot
    activations kept on the device a group of layers at a time: the pilot forward runs once per
    group, each group as large as `mem_frac` of the free device memory allows, so a large pilot
    (C4: 660k tokens x 33 layers x 5120 units, 222 GB in bf16) never has to sit in host memory.
    `edges` [L, 2, D, B] given: no edges are computed, only the seeds. Seeds use protein groups (the
    sequence of each pilot row), as the reference's run_atlas does. Returns (E cpu, (top_seed,
    res_seed_key) on the device or None, pilot token count)."""
    from .esm import pilot
    n_tok = sum(int(b.valid_rows.numel()) for b in batches)
    per_layer = n_tok * d_ff * 2
    free = torch.cuda.mem_get_info(device)[0]
    group = max(1, min(n_layers, int(mem_frac * free // max(per_layer, 1))))
    E_parts, ts_parts, rk_parts = [None] * n_layers, [None] * n_layers, [None] * n_layers
    prot = None
    for l0 in range(0, n_layers, group):
        layers = range(l0, min(n_layers, l0 + group))
        Hs, _ = pilot(model, iter(batches), device, 1 << 62, store_device=device, layers=layers)
        if prot is None:
            prot = (pilot.last_tok // 1024).to(device)
        for l in layers:
            El = pilot_edges([Hs[l]], probs=probs) if edges is None else edges[l:l + 1].to(device)
            E_parts[l] = El.cpu()
            if seeds is not None:
                K, Kr, n_total = seeds
                ts_parts[l], rk_parts[l] = pilot_seeds([Hs[l]], El, K, Kr, n_total, groups=prot)
            Hs[l] = None
        del Hs
        torch.cuda.empty_cache()
    E = torch.cat(E_parts)
    sd = (torch.cat(ts_parts), torch.cat(rk_parts)) if seeds is not None else None
    return E, sd, n_tok
