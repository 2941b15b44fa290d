"""Tensor-level wrappers over the C ABI, one per kernel, plus the reference's kernel-level functions
(`filter_candidates`, `sub_stats`, `gram_accumulate`, `grouped_merge`) with the same arguments,
results and error behaviour as haelyons/proteus atlas/filter_triton.py, atlas/stats_triton.py and
atlas/core.py:75-104 — backed only by the sm_100a library (no fallback).
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import call, dtype_code, ptr, require_cuda, stream_ptr

I64_MIN = torch.iinfo(torch.int64).min


def _i32(t):
    return t if t.dtype == torch.int32 else t.to(torch.int32)


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


# ----------------------------------------------------------------------------- K1 filter
def filter_compact(H, rowmap32, thr_pos, thr_neg, out_val, out_row, out_col, count, cap):
    """atlas_filter_compact on preallocated buffers (count must be zero on entry)."""
    T, D = H.shape
    call("atlas_filter_compact", ptr(H), dtype_code(H.dtype), T, D, H.stride(0), ptr(rowmap32), ptr(thr_pos),
         ptr(thr_neg), ptr(out_val), ptr(out_row), ptr(out_col), ptr(count), int(cap), stream_ptr(H.device))


def filter_candidates(H, rowmap, thr_pos, thr_neg, max_out, **_tile):
    """Drop-in for filter_triton.filter_candidates (filter_triton.py:65-86): returns
    (vals fp32 [max_out], rows int64, cols int64, count 0-d device tensor); count > max_out means
    overflow. Tile arguments of the Triton version are accepted and ignored."""
    require_cuda(H, "H")
    assert H.stride(1) == 1
    dev = H.device
    out_val = torch.empty(max_out, device=dev, dtype=torch.float32)
    out_row = torch.empty(max_out, device=dev, dtype=torch.int32)
    out_col = torch.empty(max_out, device=dev, dtype=torch.int32)
    counter = torch.zeros(1, device=dev, dtype=torch.int32)
    filter_compact(H, _i32(rowmap), thr_pos.contiguous().float(), thr_neg.contiguous().float(), out_val, out_row,
                   out_col, counter, max_out)
    return out_val, out_row.long(), out_col.long(), counter[0]


# ----------------------------------------------------------------------------- gathers / stats
def gather_transpose(H, rows32, XT, col0: int):
    T, D = H.shape
    call("atlas_gather_transpose", ptr(H), dtype_code(H.dtype), T, D, H.stride(0), ptr(rows32), rows32.numel(),
         ptr(XT), XT.stride(0), int(col0), stream_ptr(H.device))


def gather_rows(H, rows32, R):
    T, D = H.shape
    call("atlas_gather_rows", ptr(H), dtype_code(H.dtype), T, D, H.stride(0), ptr(rows32), rows32.numel(), ptr(R),
         stream_ptr(H.device))


def sub_stats_into(XT, col0, n, E0, E1, levels, sum_, sq, bins, masks, n_pad):
    """Accumulate subsample statistics of XT[:, col0:col0+n] into (sum_, sq, bins) and write masks."""
    import ctypes
    D = XT.shape[0]
    B = E0.shape[1]
    NL = len(levels)
    lev = (ctypes.c_int32 * max(NL, 1))(*levels) if NL else None
    call("atlas_sub_stats", ptr(XT), dtype_code(XT.dtype), XT.stride(0), int(col0), int(n), D, ptr(E0), ptr(E1), B,
         ctypes.cast(lev, ctypes.c_void_p) if lev is not None else None, NL, ptr(sum_), ptr(sq), ptr(bins),
         ptr(masks) if NL else None, int(n_pad), stream_ptr(XT.device))


def stats_enrich_supported(dtype, B: int, NL: int, A_pad: int) -> bool:
    return bool(_lib.load().atlas_stats_enrich_supported(dtype_code(dtype), B, NL, A_pad))


class StatsEnrichWorkspace:
    """Zero-filled device workspace of atlas_sub_stats_enrich (range partials of the column sums and
    per-column-tile tickets), grown on demand."""

    def __init__(self, device):
        self.device = device
        self.buf = None

    def get(self, D: int, n: int) -> torch.Tensor:
        need = int(_lib.load().atlas_stats_enrich_ws_bytes(D, n))
        if self.buf is None or self.buf.numel() < need:
            self.buf = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self.buf


def sub_stats_enrich_into(XT, col0, n, E0, E1, levels, sum_, sq, bins, annT, enr, A, ws: StatsEnrichWorkspace):
    """Fused atlas_sub_stats_enrich over XT[:, col0:col0+n]: moments and bin masses of the columns
    and the enrichment contingencies enr [2*NL*D, A] += masks . annT^T, masks never materialised."""
    import ctypes
    D = XT.shape[0]
    B = E0.shape[1]
    NL = len(levels)
    lev = (ctypes.c_int32 * NL)(*levels)
    w = ws.get(D, n)
    call("atlas_sub_stats_enrich", ptr(XT), dtype_code(XT.dtype), XT.stride(0), int(col0), int(n), D, ptr(E0), ptr(E1),
         B, ctypes.cast(lev, ctypes.c_void_p), NL, ptr(sum_), ptr(sq), ptr(bins), ptr(annT), annT.shape[0],
         annT.shape[1], ptr(enr), int(A), ptr(w), w.numel(), stream_ptr(XT.device))


def sub_stats(X, E0, E1, levels, **_tile):
    """Drop-in for stats_triton.sub_stats (stats_triton.py:77-117): X [n, D] (unit column stride);
    returns (sum fp64 [D], sumsq fp64 [D], counts int32 [2, D, B], masks int8 [2, NL, D, n8])."""
    require_cuda(X, "X")
    assert X.stride(1) == 1
    n, D = X.shape
    B = E0.shape[1]
    NL = len(levels)
    n8 = round_up(n, 8)
    dev = X.device
    XT = torch.empty(D, max(n8, 8), device=dev, dtype=X.dtype)
    if n:
        gather_transpose(X, torch.arange(n, device=dev, dtype=torch.int32), XT, 0)
    s = torch.zeros(D, device=dev, dtype=torch.float64)
    sq = torch.zeros(D, device=dev, dtype=torch.float64)
    bins = torch.zeros(2, D, B, device=dev, dtype=torch.int64)
    masks = torch.zeros(2, max(NL, 1), D, max(n8, 8), device=dev, dtype=torch.int8)
    if n:
        sub_stats_into(XT, 0, n, E0.contiguous().float(), E1.contiguous().float(), list(levels), s, sq, bins, masks,
                       masks.shape[-1])
    return s, sq, bins.to(torch.int32), masks[:, :NL, :, :n8]


def count_gemm_i8(masks2d, annT, out, A: int):
    """out[M, A] (int64) += masks2d[M, n_pad] @ annT[A_pad, n_pad]^T, exact."""
    M, n_pad = masks2d.shape
    call("atlas_count_gemm_i8", ptr(masks2d), M, n_pad, ptr(annT), annT.shape[0], ptr(out), int(A),
         stream_ptr(masks2d.device))


def gram_upper(XT, n: int, C):
    """C[D, D] += XT[:, :n] XT[:, :n]^T on the upper 128-block triangle."""
    D = XT.shape[0]
    call("atlas_gram_upper", ptr(XT), dtype_code(XT.dtype), XT.stride(0), int(n), D, ptr(C), stream_ptr(XT.device))


def gram_accumulate(X, C, **_tile):
    """Drop-in for stats_triton.gram_accumulate (stats_triton.py:148-169): C [D, D] fp32 contiguous
    += X^T X on the upper block triangle (blocks of 128), in place; returns C."""
    require_cuda(X, "X")
    assert X.stride(1) == 1 and C.is_contiguous() and C.dtype == torch.float32
    n, D = X.shape
    if n == 0:
        return C
    n8 = round_up(n, 8)
    XT = torch.empty(D, n8, device=X.device, dtype=X.dtype)
    gather_transpose(X, torch.arange(n, device=X.device, dtype=torch.int32), XT, 0)
    gram_upper(XT, n, C)
    return C


# ----------------------------------------------------------------------------- merges
class MergeWorkspace:
    """Device scratch of atlas_grouped_merge, grown on demand and reused."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.G = self.n = -1
        self.i32 = None
        self.bytes = None

    def get(self, G: int, n_max: int):
        lib = _lib.load()
        need_i = lib.atlas_merge_ws_i32(G, n_max)
        need_b = lib.atlas_merge_ws_bytes(n_max)
        if self.i32 is None or self.i32.numel() < need_i:
            self.i32 = torch.empty(int(need_i * 1.25) + 64, device=self.device, dtype=torch.int32)
        if self.bytes is None or self.bytes.numel() < need_b:
            self.bytes = torch.empty(int(need_b * 1.25) + 256, device=self.device, dtype=torch.uint8)
        return self.i32, self.bytes


_WS: dict = {}


def grouped_merge_records(state_sc, state_tok, state_val, K, g, sc, tok, val, n_dev, n_max, ws: MergeWorkspace = None):
    G = state_sc.shape[0]
    if ws is None:
        ws = _WS.setdefault(state_sc.device, MergeWorkspace(state_sc.device))
    wi, wb = ws.get(G, n_max)
    call("atlas_grouped_merge", ptr(state_sc), ptr(state_tok), ptr(state_val), G, int(K), ptr(g), ptr(sc), ptr(tok),
         ptr(val), ptr(n_dev), int(n_max), ptr(wi), ptr(wb), stream_ptr(state_sc.device))


def grouped_merge(state_score, state_pay, g, score, pay, K, pay_fill=None):
    """Drop-in for core.grouped_merge (core.py:75-104) for int64 scores with payloads
    (int64, fp32): merges candidates into the per-group top-K in place. Returns the number of
    candidates (the reference returns the number of touched groups, which needs a host sync)."""
    require_cuda(state_score, "state_score")
    assert state_score.dtype == torch.int64 and len(state_pay) == 2
    n = g.numel()
    if n == 0:
        return 0
    dev = state_score.device
    n_dev = torch.tensor([n], device=dev, dtype=torch.int32)
    grouped_merge_records(state_score, state_pay[0], state_pay[1], K, _i32(g).contiguous(), score.contiguous(),
                          pay[0].to(torch.int64).contiguous(), pay[1].to(torch.float32).contiguous(), n_dev, n)
    return n


def merge_rows(sc, tok, val, osc, otok, oval):
    G, K = sc.shape
    call("atlas_merge_rows", ptr(sc), ptr(tok), ptr(val), ptr(osc), ptr(otok), ptr(oval), G, K, stream_ptr(sc.device))
