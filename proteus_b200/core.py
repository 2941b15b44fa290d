"""Streaming per-neuron atlas on B200 — drop-in for haelyons/proteus `atlas/core.py`.

Same public surface: `AtlasConfig` (every field, same defaults), `BatchCtx`, `Atlas` with
`make_ctx / begin_batch / observe / end_batch / seed / verify_seeds / flush_gram / state_dict /
load_state_dict / merge_from / result`, the state tensors under their reference names, dtypes and
shapes (so checkpoints are interchangeable), and the helpers `token_keys, pack_tok, unpack_tok,
top_key, bin_of, symmetrize_upper`.

What runs where (all compute is the sm_100a library; there is no CPU path):
  begin_batch  atlas_thresholds                      (core.py:250-259)
  observe      atlas_filter_compact                  (K1, filter_triton.py)
               atlas_gather_transpose / _rows        (subsample rows -> transposed staging / bulk rows)
               atlas_sub_stats_enrich                (moments, bin masses, enrichment in one pass;
                                                     or atlas_sub_stats + atlas_count_gemm_i8; core.py:312-404)
               atlas_gram_upper                      (upper-block Gram over staged subsample rows)
               atlas_dense_select                    (_dense, core.py:407-446), run on the device only
                                                     when the layer is dense or its buffer overflowed
  end_batch    atlas_admit + atlas_grouped_merge x2  (core.py:450-590)
  merge_from   atlas_merge_rows                      (core.py:628-654)

Differences a caller can observe: end_batch never asks for a forward re-run (an overflowed layer
takes the dense path inside the hook, on the same activations, with the same result), and the
per-batch host synchronisation of the reference (count readback) is gone; `stats` is read from
device counters when accessed. The Gram of the subsample is accumulated over staged rows of
several batches (fp32 accumulation order differs; result within the 1e-3 Frobenius contract).
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from . import kernels as KN
from ._lib import AtlasKernelError, call, dtype_code, load, ptr, stream_ptr


class _rf:
    """Trace range around a hot-path region: always an NVTX range (nsys / ncu `--nvtx`), plus a
    torch.profiler range while a profiler records. The names are the reference's record_function
    ranges (atlas.compact, atlas.subsample, atlas.sub.*, atlas.merge.*, atlas.dense; core.py:726-727),
    so traces of the two builds line up."""

    __slots__ = ("name", "_p")

    def __init__(self, name: str):
        self.name = name
        self._p = None

    def __enter__(self):
        torch.cuda.nvtx.range_push(self.name)
        if torch.autograd.profiler._is_profiler_enabled:
            self._p = torch.profiler.record_function(self.name)
            self._p.__enter__()
        return self

    def __exit__(self, *exc):
        if self._p is not None:
            self._p.__exit__(*exc)
            self._p = None
        torch.cuda.nvtx.range_pop()
        return False

NEG_INF = float("-inf")
I64_MIN = torch.iinfo(torch.int64).min
M32 = 0xFFFFFFFF
SEQ_STRIDE = 1024  # tok id = seq_idx * 1024 + residue position (< 1022)


# ----------------------------------------------------------------------------- host helpers
def _mul32(x: torch.Tensor, c: int) -> torch.Tensor:
    """(x * c) mod 2^32 for 0 <= x < 2^32 in int64 without overflow (split c in 16-bit halves)."""
    lo, hi = c & 0xFFFF, c >> 16
    return (x * lo + (((x * hi) & 0xFFFF) << 16)) & M32


def token_keys(tok: torch.Tensor, seed: int = 0) -> torch.Tensor:
    """Bijective 32-bit lowbias32 mix of token ids (core.py:46-55) -> int64 in [0, 2^32)."""
    x = (tok.to(torch.int64) ^ (seed & M32)) & M32
    x = x ^ (x >> 16)
    x = _mul32(x, 0x7FEB352D)
    x = x ^ (x >> 15)
    x = _mul32(x, 0x846CA68B)
    return x ^ (x >> 16)


def pack_tok(seq_idx: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    return seq_idx.to(torch.int64) * SEQ_STRIDE + pos.to(torch.int64)


def unpack_tok(tok: torch.Tensor):
    return tok // SEQ_STRIDE, tok % SEQ_STRIDE


def top_key(s: torch.Tensor, tok: torch.Tensor) -> torch.Tensor:
    """int64 key ordering (s desc, tok asc), -0.0 canonicalised (core.py:66-71)."""
    i = (s.float() + 0.0).view(torch.int32).to(torch.int64)
    i = torch.where(i < 0, i ^ 0x7FFFFFFF, i)
    return i * 4294967296 + (M32 - tok.to(torch.int64))


def bin_of(s: torch.Tensor, E: torch.Tensor) -> torch.Tensor:
    return (s.unsqueeze(-1) >= E).sum(-1) - 1


def symmetrize_upper(U: torch.Tensor) -> torch.Tensor:
    """Full symmetric matrix from its upper triangle (core.py:756-759)."""
    return torch.triu(U) + torch.triu(U, 1).transpose(-1, -2)


# ----------------------------------------------------------------------------- config
@dataclass
class AtlasConfig:
    """Field for field the reference's AtlasConfig (core.py:113-132). `backend`, `stats_impl` and
    `merge_impl` are accepted and kept (they are part of checkpoint/merge equality) but every
    value runs the same sm_100a kernels."""
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
    stats_impl: str = "v3"
    merge_impl: str = "stacked"
    seed_c: float = 4.0
    seed_z: float = 2.0
    seed: int = 0
    reservoir: bool = True
    subsample: bool = True
    naive: bool = False


@dataclass
class BatchCtx:
    """Per-batch row information decided on the host (core.py:135-157), plus the int32 index
    arrays and the transposed annotation one-hots the kernels read."""
    T: int
    valid_rows: torch.Tensor
    tok: torch.Tensor
    key: torch.Tensor
    rowmap: torch.Tensor
    sub_idx: torch.Tensor
    res_in_sub: torch.Tensor
    ann_sub: torch.Tensor | None = None
    ann_sub_i8: torch.Tensor | None = None
    n_v: int = 0
    n_s: int = 0
    n_r: int = 0
    sub_rows: torch.Tensor | None = None
    # kernel-side arrays
    rowmap32: torch.Tensor | None = None     # [T] valid index or -1
    valid32: torch.Tensor | None = None      # [n_v] rows of H
    sub_rows32: torch.Tensor | None = None   # [n_s] rows of H in the hashed subsample
    res_rows32: torch.Tensor | None = None   # [n_r] rows of H with key < U_res
    res_vidx32: torch.Tensor | None = None   # [n_r] their valid indices
    key_order32: torch.Tensor | None = None  # [n_v] valid indices by ascending key
    annT: torch.Tensor | None = None         # [A_pad, n_pad] int8 one-hots, transposed
    ann_counts: torch.Tensor | None = None   # [n_a] int64 column sums of ann_sub
    ready: object = None                     # CUDA event: the context's tensors are complete (device make_ctx)

    def to(self, device, non_blocking: bool = False) -> "BatchCtx":
        mv = lambda t: None if t is None else t.to(device, non_blocking=non_blocking)  # noqa: E731
        kw = {k: (mv(v) if torch.is_tensor(v) else v) for k, v in self.__dict__.items()}
        return BatchCtx(**kw)


def _ceil(x: int, m: int) -> int:
    return (x + m - 1) // m * m


# ----------------------------------------------------------------------------- the atlas
class Atlas:
    GRAM_STAGE_ROWS = int(os.environ.get("PROTEUS_GRAM_STAGE_ROWS", "16384"))

    def __init__(self, n_layers: int, D: int, edges: torch.Tensor, cfg: AtlasConfig, n_annot: int = 0, device="cuda"):
        L, B = n_layers, edges.shape[-1]
        assert edges.shape == (L, 2, D, B), edges.shape
        self.dev = torch.device(device)
        if self.dev.type != "cuda":
            raise AtlasKernelError("proteus_b200.Atlas runs on the sm_100a kernels only: device must be CUDA")
        if self.dev.index is None:
            self.dev = torch.device("cuda", torch.cuda.current_device())
        load()
        if B > 8:
            raise ValueError("at most 8 bins per (layer, pole, unit)")
        if L > 64:
            raise ValueError("at most 64 layers")
        self.L, self.D, self.B, self.cfg = L, D, B, cfg
        dev = self.dev
        self.E = edges.to(dev, torch.float32).contiguous()
        self.U_res = int(cfg.rho_res * 2**32)
        self.U_sub = int(cfg.rho_sub * 2**32)
        assert self.U_sub >= self.U_res
        K, Kr = cfg.K, cfg.Kr
        if not (1 <= K <= 256 and 1 <= Kr <= 256):
            raise ValueError("K and Kr must be in 1..256")
        G = L * 2 * D
        self.top_s = torch.full((G, K), NEG_INF, device=dev)
        self.top_t = torch.full((G, K), -1, dtype=torch.long, device=dev)
        self.top_k = torch.full((G, K), I64_MIN, dtype=torch.long, device=dev)
        self.res_s = torch.full((G * B, Kr), I64_MIN, dtype=torch.long, device=dev)
        self.res_t = torch.full((G * B, Kr), -1, dtype=torch.long, device=dev)
        self.res_v = torch.full((G * B, Kr), float("nan"), device=dev)
        self.n_seen = 0
        self.n_sub = 0
        self.sub_sum = torch.zeros(L, D, dtype=torch.float64, device=dev)
        self.sub_sq = torch.zeros(L, D, dtype=torch.float64, device=dev)
        self.sub_bin = torch.zeros(L, 2, D, B, dtype=torch.int64, device=dev)
        self.n_a = n_annot
        nl = len(cfg.enrich_levels)
        if n_annot:
            self.enr = torch.zeros(L, 2, nl, D, n_annot, dtype=torch.int64, device=dev)
            self.ann_tot = torch.zeros(n_annot, dtype=torch.int64, device=dev)
        self.gram = torch.zeros(L, D, D, dtype=torch.float32, device=dev) if cfg.gram else None
        # fp64 Gram accumulator: on the device by default (a flush is then one device add instead of a
        # 4 B/element copy to the host and a host add; 2x the fp32 Gram in HBM, e.g. 6.9 GB for
        # 33 x 5120^2); PROTEUS_GRAM64_HOST=1 keeps it in host memory as the reference does.
        g64_dev = "cpu" if os.environ.get("PROTEUS_GRAM64_HOST", "0") == "1" else dev
        self.gram64 = torch.zeros(L, D, D, dtype=torch.float64, device=g64_dev) if cfg.gram else None
        self.gram_rows = 0
        self.top_seed = torch.full((G,), NEG_INF, device=dev)
        self.res_seed = torch.full((G * B,), I64_MIN, dtype=torch.long, device=dev)
        self.enabled = True
        self._stats = {"batches": 0, "dense_layer_batches": 0, "redo_layers": 0,
                       "compacted": 0, "elements": 0, "top_cand": 0, "res_cand": 0}
        # device counters folded into stats on access: compacted, top_cand, res_cand, overflowed layers
        self._dev_stats = torch.zeros(4, dtype=torch.int64, device=dev)
        self.ctx: BatchCtx | None = None
        self._pending: dict[int, str] = {}
        self._dense_layers: set[int] = set(range(L))
        self._active: set[int] | None = None
        self._sub_done: set[int] = set()
        # per-batch device scratch (grown on demand)
        self.thr = torch.empty(L, 2, D, device=dev)
        # the batch's admission thresholds, written by begin_batch: K-th top key per group, reservoir
        # ceiling per bin (compact copies of top_k[:, K-1] and max(res_s[:, Kr-1], res_seed))
        self._top_kth = torch.empty(G, dtype=torch.long, device=dev)
        self._res_thr = torch.empty(G * B, dtype=torch.long, device=dev)
        self._counts = torch.zeros(L, dtype=torch.int32, device=dev)
        self._flags = torch.zeros(L + 4, dtype=torch.int32, device=dev)  # [0,L) dense ran; L: n_top; L+1: n_res; L+2: err
        self._cand = None
        self._cand_cap = 0
        self._R = None
        self._R_used = False
        self._lists = None
        self._list_caps = (0, 0)
        self._dense_scratch = None
        self._masks = None
        self._xt_batch = None
        self._stage = None
        self._stage_fill = [0] * L
        self._act_dtype = None
        self._ws_top = KN.MergeWorkspace(dev)
        self._ws_res = KN.MergeWorkspace(dev)
        self._ws_se = KN.StatsEnrichWorkspace(dev)
        self._cap_cache = None
        self.kernel_timer = None  # optional object with start(name) / stop(name) around kernel launches

    # ------------------------------------------------------------------ stats
    @property
    def stats(self) -> dict:
        """Counters of the reference (core.py:198-199); device counters are read here (one sync)."""
        d = self._dev_stats.tolist()
        s = dict(self._stats)
        s["compacted"] += d[0]
        s["top_cand"] += d[1]
        s["res_cand"] += d[2]
        s["redo_layers"] += d[3]
        s["dense_layer_batches"] += d[3]
        return s

    @stats.setter
    def stats(self, value: dict):
        self._stats = dict(value)
        self._dev_stats.zero_()

    # ------------------------------------------------------------------ batch setup
    def make_ctx(self, T: int, valid_rows: torch.Tensor, tok: torch.Tensor, ann_ids: torch.Tensor | None = None,
                 device=None) -> BatchCtx:
        """Host tensors in; every row-level decision is made here (core.py:210-237). device="cpu"
        builds a host-side context (e.g. on a prefetch thread) to be moved with ctx.to(dev)."""
        valid_rows = torch.as_tensor(valid_rows).to("cpu", torch.int64)
        tok = torch.as_tensor(tok).to("cpu", torch.int64)
        assert tok.numel() == 0 or (int(tok.min()) >= 0 and int(tok.max()) < 2**32), "token ids must be in [0, 2^32)"
        key = token_keys(tok, self.cfg.seed)
        sub = torch.nonzero(key < self.U_sub).squeeze(1)
        res_in_sub = torch.nonzero(key[sub] < self.U_res).squeeze(1)
        rowmap = torch.full((T,), -1, dtype=torch.long)
        rowmap[valid_rows] = torch.arange(valid_rows.numel())
        ann_sub = ann_i8 = annT = ann_counts = None
        n_s = sub.numel()
        if self.n_a and ann_ids is not None:
            a = torch.as_tensor(ann_ids).to("cpu", torch.int64)[sub]
            ann_sub = torch.zeros(n_s, self.n_a)
            r, c = torch.nonzero(a >= 0, as_tuple=True)
            ann_sub[r, a[r, c]] = 1.0
            r8, c8 = -(-n_s // 8) * 8, -(-self.n_a // 8) * 8
            ann_i8 = torch.zeros(r8, c8, dtype=torch.int8)
            ann_i8[:n_s, :self.n_a] = ann_sub.to(torch.int8)
            annT = torch.zeros(max(16, _ceil(self.n_a, 16)), max(128, _ceil(n_s, 128)), dtype=torch.int8)
            annT[:self.n_a, :n_s] = ann_sub.T.to(torch.int8)
            ann_counts = ann_sub.sum(0).round().to(torch.int64)
        d = self.dev if device is None else torch.device(device)
        sub_rows = valid_rows[sub]
        ctx = BatchCtx(T=T, valid_rows=valid_rows, tok=tok, key=key, rowmap=rowmap, sub_idx=sub, res_in_sub=res_in_sub,
                       ann_sub=ann_sub, ann_sub_i8=ann_i8, n_v=valid_rows.numel(), n_s=n_s, n_r=res_in_sub.numel(),
                       sub_rows=sub_rows, rowmap32=rowmap.to(torch.int32), valid32=valid_rows.to(torch.int32),
                       sub_rows32=sub_rows.to(torch.int32), res_rows32=sub_rows[res_in_sub].to(torch.int32),
                       res_vidx32=sub[res_in_sub].to(torch.int32),
                       key_order32=torch.argsort(key).to(torch.int32), annT=annT, ann_counts=ann_counts)
        return ctx if d.type == "cpu" else ctx.to(d)

    @torch.no_grad()
    def make_ctx_device(self, T: int, valid_rows, tok, ann_ids=None, stream=None) -> BatchCtx:
        """make_ctx on the device (atlas_ctx_rows / atlas_ctx_annotations): the same row-level
        decisions as make_ctx (core.py:210-237) from the batch's raw valid rows, token ids and
        annotation ids (host tensors, pinned for an asynchronous copy, or device tensors). Runs on
        `stream` (default: the current stream); only that stream is waited on, for the two counts
        (n_s, n_r) the host needs to size the batch's launches, so a prefetch thread can build the
        next context on a side stream while the main stream works. The context's `ready` event is
        waited on by begin_batch."""
        dev = self.dev
        st = stream if stream is not None else torch.cuda.current_stream(dev)
        with torch.cuda.device(dev), torch.cuda.stream(st):
            vr = torch.as_tensor(valid_rows).to(dev, torch.int64, non_blocking=True)
            tk = torch.as_tensor(tok).to(dev, torch.int64, non_blocking=True)
            n_v = vr.numel()
            i64 = dict(dtype=torch.int64, device=dev)
            i32 = dict(dtype=torch.int32, device=dev)
            key, sub_idx, res_in_sub = torch.empty(n_v, **i64), torch.empty(n_v, **i64), torch.empty(n_v, **i64)
            rowmap32 = torch.empty(T, **i32)
            sub_rows32, res_rows32, res_vidx32 = torch.empty(n_v, **i32), torch.empty(n_v, **i32), torch.empty(n_v, **i32)
            key_order32 = torch.empty(n_v, **i32)
            counts = torch.zeros(2, **i64)
            err = torch.zeros(1, **i32)
            ws = torch.empty(int(load().atlas_ctx_ws_bytes(n_v)), dtype=torch.uint8, device=dev)
            call("atlas_ctx_rows", ptr(vr), ptr(tk), n_v, T, self.cfg.seed, self.U_sub, self.U_res, ptr(key),
                 ptr(rowmap32), ptr(sub_idx), ptr(res_in_sub), ptr(sub_rows32), ptr(res_rows32), ptr(res_vidx32),
                 ptr(key_order32), ptr(counts), ptr(err), ptr(ws), ws.numel(), st.cuda_stream)
            host = torch.empty(3, dtype=torch.int64, pin_memory=True)
            host[:2].copy_(counts, non_blocking=True)
            host[2:].copy_(err, non_blocking=True)
            done = torch.cuda.Event()
            done.record(st)
            done.synchronize()  # this stream only: the counts size the views below
            n_s, n_r, bad = (int(x) for x in host.tolist())
            if bad:
                raise ValueError("token ids must be in [0, 2^32) and valid rows inside the batch")
            annT = ann_counts = None
            if self.n_a and ann_ids is not None:
                ann = torch.as_tensor(ann_ids).to(dev, torch.int64, non_blocking=True)
                ann = ann.view(n_v, -1).contiguous()
                A_pad, n_pad = max(16, _ceil(self.n_a, 16)), max(128, _ceil(n_s, 128))
                annT = torch.empty(A_pad, n_pad, dtype=torch.int8, device=dev)
                ann_counts = torch.empty(self.n_a, **i64)
                call("atlas_ctx_annotations", ptr(sub_idx), ptr(counts), ptr(ann), n_v, ann.shape[1], self.n_a,
                     ptr(annT), A_pad, n_pad, ptr(ann_counts), st.cuda_stream)
            valid32 = vr.to(torch.int32)
            ready = torch.cuda.Event()
            ready.record(st)
        return BatchCtx(T=T, valid_rows=vr, tok=tk, key=key, rowmap=rowmap32, sub_idx=sub_idx[:n_s],
                        res_in_sub=res_in_sub[:n_r], n_v=n_v, n_s=n_s, n_r=n_r, sub_rows=sub_rows32[:n_s],
                        rowmap32=rowmap32, valid32=valid32, sub_rows32=sub_rows32[:n_s], res_rows32=res_rows32[:n_r],
                        res_vidx32=res_vidx32[:n_r], key_order32=key_order32, annT=annT, ann_counts=ann_counts,
                        ready=ready)

    def _cap(self, ctx, l=None) -> int:
        f = self.cfg.cap_frac
        if self.cfg.cap_frac_early > 0 and l is not None and l < self.cfg.early_layers:
            f = self.cfg.cap_frac_early
        return max(4096, int(f * ctx.n_v * self.D))

    def _ensure_buffers(self, ctx: BatchCtx):
        L, D, B, K, Kr = self.L, self.D, self.B, self.cfg.K, self.cfg.Kr
        dev = self.dev
        cap_main = self._cap(ctx, self.L)
        cap_early = self._cap(ctx, 0)
        cap = max(cap_main, cap_early)
        if cap > self._cand_cap:
            c = int(cap * 1.25)
            self._cand = (torch.empty(L, c, device=dev), torch.empty(L, c, dtype=torch.int32, device=dev),
                          torch.empty(L, c, dtype=torch.int32, device=dev))
            self._cand_cap = c
        n_r = ctx.n_r
        caps = [self._cap(ctx, l) for l in range(L)]
        top_need = sum(max(2 * c, 2 * D * min(K, ctx.n_v)) for c in caps)
        res_need = sum(max(2 * c + 2 * n_r * D, 2 * D * B * min(Kr, ctx.n_v)) for c in caps) if self.cfg.reservoir else 1
        tcap, rcap = self._list_caps
        if top_need > tcap or res_need > rcap:
            tcap, rcap = max(tcap, int(top_need * 1.25)), max(rcap, int(res_need * 1.25))
            mk = lambda n: (torch.empty(n, dtype=torch.int32, device=dev), torch.empty(n, dtype=torch.int64, device=dev),  # noqa: E731
                            torch.empty(n, dtype=torch.int64, device=dev), torch.empty(n, dtype=torch.float32, device=dev))
            self._lists = (mk(tcap), mk(rcap))
            self._list_caps = (tcap, rcap)
        if self._act_dtype is not None and self.cfg.reservoir and ctx.n_r and (
                self._R is None or self._R.shape[1] < ctx.n_r or self._R.dtype != self._act_dtype):
            self._R = torch.empty(L, int(ctx.n_r * 1.25) + 1, D, dtype=self._act_dtype, device=dev)
        self._R_used = False
        sb = load().atlas_dense_scratch_bytes(ctx.n_v, D, B, dtype_code(self._act_dtype or torch.float32))
        if self._dense_scratch is None or self._dense_scratch.numel() < sb:
            # zero-filled: the dense kernels count strip arrivals in it and leave those words at zero
            self._dense_scratch = torch.zeros(int(sb * 1.25) + 256, dtype=torch.uint8, device=dev)

    def begin_batch(self, ctx: BatchCtx, redo_layers: list[int] | None = None):
        """Thresholds for this batch from the state at batch start (device only, no sync)."""
        if ctx.valid_rows.device != self.dev:
            ctx = ctx.to(self.dev)
        if ctx.ready is not None:  # built on another stream (make_ctx_device): order and keep its memory
            cur = torch.cuda.current_stream(self.dev)
            cur.wait_event(ctx.ready)
            for t in ctx.__dict__.values():
                if torch.is_tensor(t) and t.is_cuda:
                    t.record_stream(cur)
        if redo_layers is not None:
            if redo_layers:
                raise ValueError("end_batch never requests a redo: overflowed layers take the dense path in the hook")
            return
        self.ctx = ctx
        self._pending = {}
        self._active = set(range(self.L))
        self._sub_done = set()
        self._stats["elements"] += 2 * ctx.n_v * self.D * self.L
        self._ensure_buffers(ctx)
        self._counts.zero_()
        self._flags[:self.L + 2].zero_()  # the list-overflow flag (slot L + 2) stays set once raised
        c = self.cfg
        call("atlas_thresholds", ptr(self.top_s), c.K, ptr(self.res_s), c.Kr, ptr(self.top_seed), ptr(self.res_seed),
             ptr(self.E), self.L * 2 * self.D, self.B, self.U_res, int(bool(c.reservoir)), ptr(self.thr),
             ptr(self.top_k), ptr(self._top_kth), ptr(self._res_thr), stream_ptr(self.dev))

    # ------------------------------------------------------------------ hook body
    @torch.no_grad()
    def observe(self, l: int, H: torch.Tensor):
        """H: [T, D] hook output for layer l (bf16 / fp16 / fp32, rows include padding)."""
        if not self.enabled or self._active is None or l not in self._active:
            return
        ctx = self.ctx
        if H.device != self.dev:
            raise AtlasKernelError(f"activations on {H.device}, atlas on {self.dev}")
        if H.stride(1) != 1:
            H = H.contiguous()
        T, D = H.shape
        assert T == ctx.T and D == self.D, (H.shape, ctx.T, self.D)
        if self._act_dtype is None:
            self._act_dtype = H.dtype
        elif H.dtype != self._act_dtype:
            raise TypeError(f"activation dtype changed from {self._act_dtype} to {H.dtype}")
        dense = l in self._dense_layers
        cap = self._cap(ctx, l)
        st = stream_ptr(self.dev)
        dt = dtype_code(H.dtype)
        kt = self.kernel_timer
        if not dense:
            cv, cr, cc = self._cand
            with _rf("atlas.compact"):
                if kt is not None:
                    kt.start("filter")
                call("atlas_filter_compact", ptr(H), dt, T, D, H.stride(0), ptr(ctx.rowmap32), ptr(self.thr[l, 0]),
                     ptr(self.thr[l, 1]), ptr(cv[l]), ptr(cr[l]), ptr(cc[l]), ptr(self._counts[l:l + 1]), cap, st)
                if kt is not None:
                    kt.stop("filter")
        if self.cfg.subsample and l not in self._sub_done:
            with _rf("atlas.subsample"):
                self._subsample(l, H)
        if self.cfg.reservoir and not dense and ctx.n_r:
            if self._R is None or self._R.shape[1] < ctx.n_r or self._R.dtype != H.dtype:
                # sized in begin_batch once the activation dtype is known; only the first batch
                # allocates here, before any layer of the batch has written bulk rows
                assert not self._R_used, "bulk-row buffer resized mid-batch"
                self._R = torch.empty(self.L, int(ctx.n_r * 1.25) + 1, D, dtype=H.dtype, device=self.dev)
            self._R_used = True
            with _rf("atlas.merge.bulk"):
                KN.gather_rows(H, ctx.res_rows32, self._R[l])
        # dense path: forced for dense layers, predicated on count > cap for filtered ones
        (tg, tsc, tt, tv), (rg, rsc, rt, rv) = self._lists
        tcap, rcap = self._list_caps
        c = self.cfg
        fl = self._flags
        with _rf("atlas.dense"):
            if kt is not None:
                kt.start("dense")
            self._dense_call(H, dt, T, D, l, ctx, c, cap, dense, tg, tsc, tt, tv, tcap, rg, rsc, rt, rv, rcap, fl, st)
            if kt is not None:
                kt.stop("dense", work=ctx.n_v if dense else 0)
        self._pending[l] = "dense" if dense else "filtered"

    def _dense_call(self, H, dt, T, D, l, ctx, c, cap, dense, tg, tsc, tt, tv, tcap, rg, rsc, rt, rv, rcap, fl, st):
        call("atlas_dense_select", ptr(H), dt, T, D, H.stride(0), l, ptr(ctx.valid32), ctx.n_v, ptr(ctx.tok),
             ptr(ctx.key), ptr(ctx.key_order32), self.B, c.K, c.Kr, int(bool(c.reservoir)), ptr(self.top_seed),
             ptr(self.top_k), ptr(self.res_s), ptr(self.res_seed), ptr(self.E), ptr(self._counts[l:l + 1]), cap,
             int(dense), ptr(tg), ptr(tsc), ptr(tt), ptr(tv), ptr(fl[self.L:self.L + 1]), tcap, ptr(rg), ptr(rsc),
             ptr(rt), ptr(rv), ptr(fl[self.L + 1:self.L + 2]), rcap, ptr(self._dense_scratch),
             self._dense_scratch.numel(), ptr(fl[l:l + 1]), ptr(fl[self.L + 2:self.L + 3]), st)

    def _subsample(self, l: int, H: torch.Tensor):
        """Gather the hashed-subsample rows (transposed) and accumulate bin masses, moments,
        enrichment counts; stage the rows for the Gram."""
        ctx = self.ctx
        self._sub_done.add(l)
        n = ctx.n_s
        if n == 0:
            return
        D = self.D
        n8 = _ceil(n, 8)
        if self.gram is not None:
            cap_rows = max(_ceil(self.GRAM_STAGE_ROWS, 64), _ceil(n8, 64))
            if self._stage is None or self._stage.shape[2] < n8 or self._stage.dtype != H.dtype:
                self._drain_gram()
                self._stage = torch.empty(self.L, D, cap_rows, dtype=H.dtype, device=self.dev)
                self._stage_fill = [0] * self.L
            if self._stage_fill[l] + n8 > self._stage.shape[2]:
                self._gram_layer(l)
            XT = self._stage[l]
            col0 = self._stage_fill[l]
        else:
            if self._xt_batch is None or self._xt_batch.shape[1] < n8 or self._xt_batch.dtype != H.dtype:
                self._xt_batch = torch.empty(D, _ceil(n8, 64), dtype=H.dtype, device=self.dev)
            XT, col0 = self._xt_batch, 0
        KN.gather_transpose(H, ctx.sub_rows32, XT, col0)
        levels = list(self.cfg.enrich_levels)
        ann = bool(self.n_a) and ctx.annT is not None and len(levels) > 0
        if ann and KN.stats_enrich_supported(XT.dtype, self.B, len(levels), ctx.annT.shape[0]):
            # one pass over the staged rows: moments, bin masses and the enrichment contingencies,
            # the 0/1 masks built in shared memory for the int8 tensor-core contraction
            kt = self.kernel_timer
            if kt is not None:
                kt.start("stats")
            with _rf("atlas.sub.kernel"):
                KN.sub_stats_enrich_into(XT, col0, n, self.E[l, 0], self.E[l, 1], levels, self.sub_sum[l],
                                         self.sub_sq[l], self.sub_bin[l], ctx.annT,
                                         self.enr[l].view(2 * len(levels) * D, self.n_a), self.n_a, self._ws_se)
            if kt is not None:
                kt.stop("stats", work=n)
            if self.gram is not None:
                self._stage_fill[l] += n8
                if l == 0:
                    self.gram_rows += n
            return
        n_pad = ctx.annT.shape[1] if ann else _ceil(n, 8)
        masks = None
        if ann:
            need = 2 * len(levels) * D * n_pad
            if self._masks is None or self._masks.numel() < need:
                self._masks = torch.empty(int(need * 1.25), dtype=torch.int8, device=self.dev)
            masks = self._masks[:need]
        with _rf("atlas.sub.kernel"):
            KN.sub_stats_into(XT, col0, n, self.E[l, 0], self.E[l, 1], levels if ann else [], self.sub_sum[l],
                              self.sub_sq[l], self.sub_bin[l], masks, n_pad)
        if ann:
            with _rf("atlas.sub.enrich"):
                KN.count_gemm_i8(masks.view(2 * len(levels) * D, n_pad), ctx.annT,
                                 self.enr[l].view(2 * len(levels) * D, self.n_a), self.n_a)
        if self.gram is not None:
            self._stage_fill[l] += n8
            if l == 0:
                self.gram_rows += n

    def _gram_layer(self, l: int):
        f = self._stage_fill[l]
        if f > 0:
            kt = self.kernel_timer
            if kt is not None:
                kt.start("gram")
            with _rf("atlas.sub.gram"):
                KN.gram_upper(self._stage[l], f, self.gram[l])
            if kt is not None:
                kt.stop("gram", work=f)
            self._stage_fill[l] = 0

    def _drain_gram(self):
        if self._stage is None:
            return
        for l in range(self.L):
            self._gram_layer(l)

    # ------------------------------------------------------------------ after forward
    @torch.no_grad()
    def end_batch(self) -> list[int]:
        """Admit and merge every pending candidate; no host sync. Always returns [] (layers whose
        buffer overflowed already took the exact dense path in the hook)."""
        ctx = self.ctx
        if ctx is None:
            return []
        L, D, B, c = self.L, self.D, self.B, self.cfg
        filt = [l for l, m in self._pending.items() if m == "filtered"]
        dense_done = [l for l, m in self._pending.items() if m == "dense"]
        (tg, tsc, tt, tv), (rg, rsc, rt, rv) = self._lists
        tcap, rcap = self._list_caps
        fl = self._flags
        st = stream_ptr(self.dev)
        cap_main, cap_early = self._cap(ctx, L), self._cap(ctx, 0)
        with _rf("atlas.merge"):
            self._merge_batch(ctx, L, c, filt, tg, tsc, tt, tv, rg, rsc, rt, rv, tcap, rcap, fl, st, cap_main,
                              cap_early)
        # device-side counters (no sync): compacted survivors of non-overflowed layers, candidates,
        # overflowed layers (each took one dense pass)
        self._count_batch(L, c, filt, fl, cap_main, cap_early)
        self._stats["dense_layer_batches"] += len(dense_done)
        if not c.naive:
            self._dense_layers -= set(dense_done)
        self.n_seen += ctx.n_v
        self.n_sub += ctx.n_s
        if self.n_a and ctx.ann_counts is not None:
            self.ann_tot += ctx.ann_counts
        self._stats["batches"] += 1
        self._pending = {}
        self._active = None
        return []

    def _merge_batch(self, ctx, L, c, filt, tg, tsc, tt, tv, rg, rsc, rt, rv, tcap, rcap, fl, st, cap_main, cap_early):
        D, B = self.D, self.B
        if filt:
            mode = (torch.zeros(L, dtype=torch.int8))
            mode[filt] = 1
            cv, cr, cc = self._cand
            R = self._R if (c.reservoir and ctx.n_r) else None
            kt = self.kernel_timer
            if kt is not None:
                kt.start("admit")
            with _rf("atlas.merge.cand"):
                call("atlas_admit", L, D, B, c.K, c.Kr, self.U_res, int(bool(c.reservoir)), mode.data_ptr(),
                     ptr(self._counts), cap_main, cap_early if c.cap_frac_early > 0 else cap_main,
                     c.early_layers if c.cap_frac_early > 0 else 0, ptr(cv), ptr(cr), ptr(cc), self._cand_cap,
                     ptr(ctx.tok), ptr(ctx.key), ptr(R), dtype_code(self._act_dtype), ctx.n_r if R is not None else 0,
                     R.shape[1] if R is not None else 0, ptr(ctx.res_vidx32), ptr(self.top_seed), ptr(self._top_kth),
                     ptr(self._res_thr), ptr(self.E), ptr(tg), ptr(tsc), ptr(tt), ptr(tv),
                     ptr(fl[L:L + 1]), tcap, ptr(rg), ptr(rsc), ptr(rt), ptr(rv), ptr(fl[L + 1:L + 2]), rcap,
                     ptr(fl[L + 2:L + 3]), st)
            if kt is not None:
                kt.stop("admit")
        kt = self.kernel_timer
        if kt is not None:
            kt.start("merge")
        with _rf("atlas.merge.top"):
            KN.grouped_merge_records(self.top_k, self.top_t, self.top_s, c.K, tg, tsc, tt, tv, fl[L:L + 1], tcap,
                                     self._ws_top)
        if c.reservoir:
            with _rf("atlas.merge.res"):
                KN.grouped_merge_records(self.res_s, self.res_t, self.res_v, c.Kr, rg, rsc, rt, rv, fl[L + 1:L + 2],
                                         rcap, self._ws_res)
        if kt is not None:
            kt.stop("merge")

    def _count_batch(self, L, c, filt, fl, cap_main, cap_early):
        """Survivors of the non-overflowed filtered layers, records admitted, overflowed layers (each
        took the dense path): added to the device counters by one kernel, no host read."""
        fmask = torch.zeros(L, dtype=torch.int8)
        if filt:
            fmask[filt] = 1
        early = c.early_layers if c.cap_frac_early > 0 else 0
        call("atlas_batch_counters", ptr(self._counts), L, fmask.data_ptr(), cap_main, cap_early, early,
             ptr(fl[L:L + 1]), ptr(fl[L + 1:L + 2]), ptr(self._dev_stats), stream_ptr(self.dev))

    def device_status(self) -> int:
        """Status word of the bounded device waits on this atlas's GPU: 0, or the code of the first
        wait (tcgen05 / TMA mbarrier) that gave up; that launch's output is then incomplete."""
        import ctypes
        v = ctypes.c_int(0)
        with torch.cuda.device(self.dev):
            call("atlas_device_status", ctypes.byref(v), 0)
        return int(v.value)

    def check_errors(self):
        """Raise if the device recorded anything that invalidates the state: a record list that ran
        out of capacity (the flag is sticky from the batch that overflowed it; never expected, the
        lists are sized for each batch's worst case), or a bounded wait that gave up. One
        synchronisation. state_dict() and result() call it, so a flagged state is never written to
        a checkpoint or returned."""
        if int(self._flags[self.L + 2]):
            raise AtlasKernelError("a candidate record list overflowed its capacity: this atlas state is incomplete")
        st = self.device_status()
        if st:
            raise AtlasKernelError(f"device status {st}: a bounded wait of a tensor-core or TMA kernel gave up, "
                                   "so its output is incomplete: this atlas state is invalid")

    # ------------------------------------------------------------------ outputs
    def flush_gram(self):
        """fp32 device Gram (after draining staged rows) -> fp64 accumulator (core.py:593-599)."""
        if self.gram is not None:
            self._drain_gram()
            self.gram64 += self.gram.to(self.gram64.device).double()
            self.gram.zero_()

    _STATE = ["top_s", "top_t", "top_k", "res_s", "res_t", "res_v", "sub_sum", "sub_sq", "sub_bin", "E",
              "top_seed", "res_seed"]

    def state_dict(self) -> dict:
        """Checkpoint dict in the reference's format (core.py:605-614); CPU tensors, no Gram.
        Raises (check_errors) instead of returning a state the device flagged as incomplete."""
        self.check_errors()
        st = {k: getattr(self, k).cpu() for k in self._STATE}
        if self.n_a:
            st["enr"], st["ann_tot"] = self.enr.cpu(), self.ann_tot.cpu()
        st.update(n_seen=self.n_seen, n_sub=self.n_sub, stats=dict(self.stats),
                  dense_layers=sorted(self._dense_layers), cfg=dict(self.cfg.__dict__), n_a=self.n_a)
        return st

    def load_state_dict(self, st: dict):
        assert st["cfg"] == dict(self.cfg.__dict__), "config mismatch on resume"
        assert torch.equal(st["E"].to(self.E.device), self.E), "bin edges differ: resume must reuse the checkpointed pilot"
        for k in self._STATE:
            getattr(self, k).copy_(st[k].to(self.dev))
        if self.n_a:
            self.enr.copy_(st["enr"].to(self.dev))
            self.ann_tot.copy_(st["ann_tot"].to(self.dev))
        if self.gram is not None:
            self.gram64.zero_()
            self.gram.zero_()
            self.gram_rows = 0
            self._stage_fill = [0] * self.L
        self.n_seen, self.n_sub = st["n_seen"], st["n_sub"]
        self.stats = dict(st["stats"])
        self._dense_layers = set(st["dense_layers"])

    @torch.no_grad()
    def merge_from(self, other):
        """Fold in an atlas of a DISJOINT token set (same edges, cfg, seeds) — core.py:628-654. The
        other atlas may be this class or the reference's (any device)."""
        assert torch.equal(other.E.to(self.dev), self.E) and other.cfg.__dict__ == self.cfg.__dict__
        assert torch.equal(other.top_seed.to(self.dev), self.top_seed) and \
            torch.equal(other.res_seed.to(self.dev), self.res_seed), \
            "shards must share seeds (derive them from the GLOBAL stream size)"
        o = lambda t: t.to(self.dev).contiguous()  # noqa: E731
        KN.merge_rows(self.top_k, self.top_t, self.top_s, o(other.top_k), o(other.top_t), o(other.top_s))
        KN.merge_rows(self.res_s, self.res_t, self.res_v, o(other.res_s), o(other.res_t), o(other.res_v))
        for k in ["sub_sum", "sub_sq", "sub_bin"]:
            getattr(self, k).add_(getattr(other, k).to(self.dev))
        if self.n_a:
            self.enr += other.enr.to(self.dev)
            self.ann_tot += other.ann_tot.to(self.dev)
        if self.gram is not None:
            self.flush_gram()
            other.flush_gram()
            self.gram64 += other.gram64.to(self.gram64.device)
            self.gram_rows += other.gram_rows
        self.n_seen += other.n_seen
        self.n_sub += other.n_sub
        merged = self.stats
        for k, x in other.stats.items():
            merged[k] = merged.get(k, 0) + x
        self.stats = merged

    def result(self) -> dict:
        """Final views and checks (core.py:656-676)."""
        L, D, B, K, Kr = self.L, self.D, self.B, self.cfg.K, self.cfg.Kr
        self.flush_gram()
        self.check_errors()
        top_s = self.top_s.view(L, 2, D, K).cpu()
        sign = torch.tensor([1.0, -1.0]).view(1, 2, 1, 1)
        out = {
            "top_val": top_s * sign, "top_tok": self.top_t.view(L, 2, D, K).cpu(),
            "res_tok": self.res_t.view(L, 2, D, B, Kr).cpu(), "res_val": self.res_v.view(L, 2, D, B, Kr).cpu(),
            "res_key": -self.res_s.view(L, 2, D, B, Kr).cpu(),
            "edges": self.E.cpu(), "n_seen": self.n_seen, "n_sub": self.n_sub,
            "sub_sum": self.sub_sum.cpu(), "sub_sq": self.sub_sq.cpu(), "sub_bin": self.sub_bin.cpu(),
            "stats": dict(self.stats), "cfg": self.cfg.__dict__,
        }
        if self.n_a:
            out["enr"] = self.enr.cpu()
            out["ann_tot"] = self.ann_tot.cpu()
        if self.gram is not None:
            out["gram"] = symmetrize_upper(self.gram64.cpu())
            out["gram_rows"] = self.gram_rows
        out.update(self.verify_seeds())
        return out

    # ------------------------------------------------------------------ seeds
    @torch.no_grad()
    def seed(self, top_seed: torch.Tensor | None = None, res_seed_key: torch.Tensor | None = None):
        """Exact-preserving start thresholds (core.py:680-692)."""
        if top_seed is not None:
            self.top_seed.copy_(top_seed.reshape(-1).to(self.dev, torch.float32))
            self._dense_layers = set()
        if res_seed_key is not None:
            k = res_seed_key.reshape(-1).to(self.dev, torch.long)
            self.res_seed.copy_(torch.where(k >= 2**32, torch.full_like(k, I64_MIN), -k))

    def verify_seeds(self) -> dict:
        """Bins whose reservoir is short although seeded (core.py:694-704)."""
        n_kept = (self.res_t >= 0).sum(1)
        seeded = self.res_seed != I64_MIN
        bad = seeded & (n_kept < self.cfg.Kr)
        L, D, B = self.L, self.D, self.B
        seed_key = torch.where(seeded, -self.res_seed, torch.full_like(self.res_seed, 2**32))
        return {"res_seeded_bins": int(seeded.sum()), "res_seed_limited_bins": int(bad.sum()),
                "res_seed_limited": bad.view(L, 2, D, B).cpu(), "res_seed_key": seed_key.view(L, 2, D, B).cpu(),
                "top_seed_short_groups": int(((self.top_t >= 0).sum(1) < self.cfg.K).logical_and(self.top_seed > NEG_INF).sum())}
