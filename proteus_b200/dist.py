"""Data-parallel atlas over the GPUs of one node: one process per GPU, disjoint sequence shards,
an exact combine of the shard states at the end.

The stream shards with no communication: every rank runs the full forward + atlas on the batches
`plan[rank::world]`, with edges and seeds computed from the GLOBAL stream (the reference's merge
contract, tests/test_resume_merge.py:56-60; Atlas.merge_from asserts it, atlas/core.py:632-634).

`merge_states` is merge_from (atlas/core.py:628-654) across ranks:
  top-K / reservoirs: the G group rows are cut into `world` slices; an all-to-all sends slice r of
    every rank to rank r, which merges the `world` sorted copies of its slice (the GPU row merge:
    keys are unique across shards, so the result is the exact top-K / bottom-Kr of the union) and
    an all-gather returns the merged rows to every rank (each row crosses NVLink twice, instead of
    every rank receiving every rank's whole state);
  counts (sub_bin, enr, ann_tot, n_seen, n_sub): all-reduce SUM in int64 (exact);
  moments (sub_sum, sub_sq, fp64): all-gathered and summed in rank order (deterministic);
  Gram: each rank flushes to fp64; layer by layer, an all-to-all sends slice r of every rank's
    matrix to rank r, which sums the `world` copies in rank order (deterministic, and each rank
    receives one slice per peer instead of every peer's whole matrix), and an all-gather returns
    the summed slices to every rank.
The shards must share edges, config and both seeds: a SHA-256 of their bytes is compared first.
"""
from __future__ import annotations

import hashlib

import torch
import torch.distributed as dist

I64_MIN = torch.iinfo(torch.int64).min


def shard_plan(plan: list, world: int, rank: int) -> list:
    """Batches of this rank: plan[rank::world] (disjoint, covering, deterministic)."""
    return plan[rank::world]


class Lockstep:
    """Per-batch agreement of the ranks of a sharded stream on how to go on. Each rank proposes a
    code (0 = continue, larger = stop, e.g. 1 = simulated cap, 2 = deadline: checkpoint and exit)
    and says whether it has batches left; after `agree` every rank holds the same largest code and
    knows whether any rank still has work. Ranks whose shard is exhausted keep calling `agree`
    (without a batch) until every shard is, so all ranks leave the loop at the same step and enter
    the combine together, and a stop taken by one rank is taken by all. One all-reduce of two ints
    per batch; given a host (gloo) group and no device, it never waits for a GPU stream."""

    def __init__(self, group=None, device=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.buf = torch.zeros(2, dtype=torch.int64, device=device if device is not None else "cpu")

    def agree(self, code: int, more: bool) -> tuple[int, bool]:
        if self.world == 1:
            return int(code), bool(more)
        self.buf[0] = int(code)
        self.buf[1] = int(bool(more))
        dist.all_reduce(self.buf, op=dist.ReduceOp.MAX, group=self.group)
        c, m = self.buf.tolist()
        return int(c), bool(m)


def _row_merge_cuda(sc, tok, val, osc, otok, oval):
    from .kernels import merge_rows
    merge_rows(sc, tok, val, osc, otok, oval)


def _exchange_rows(sc, tok, val, fills, world, group, row_merge):
    """All-to-all of row slices, merge of the `world` copies, all-gather of the merged slices."""
    G, K = sc.shape
    per = -(-G // world)
    Gp = per * world
    dev = sc.device

    def pad(t, fill):
        if Gp == G:
            return t.contiguous()
        p = torch.full((Gp - G, K), fill, dtype=t.dtype, device=dev)
        return torch.cat([t, p]).contiguous()

    parts = [pad(sc, I64_MIN), pad(tok, fills[0]), pad(val, fills[1])]
    recv = [torch.empty_like(p) for p in parts]
    for src, dst in zip(parts, recv):
        dist.all_to_all_single(dst, src, group=group)
    # recv[i] holds, for every source rank s, rows [s*per, (s+1)*per) = this rank's slice from rank s
    mine = [r.view(world, per, K) for r in recv]
    acc = [mine[i][0].clone() for i in range(3)]
    for s in range(1, world):
        row_merge(acc[0], acc[1], acc[2], mine[0][s].contiguous(), mine[1][s].contiguous(), mine[2][s].contiguous())
    out = [torch.empty_like(p) for p in parts]
    for o, a in zip(out, acc):
        dist.all_gather_into_tensor(o, a.contiguous(), group=group)
    return [o[:G] for o in out]


def _sum_in_rank_order(t: torch.Tensor, world, group) -> torch.Tensor:
    bufs = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(bufs, t.contiguous(), group=group)
    acc = bufs[0].clone()
    for b in bufs[1:]:
        acc += b
    return acc


def _reduce_slices_in_rank_order(t: torch.Tensor, world, group) -> torch.Tensor:
    """Sum of `t` over the ranks, in rank order, returned on every rank: all-to-all of `world`
    slices of the flattened tensor, a rank-ordered sum of the copies of the own slice, all-gather
    of the sums. Per rank it receives about 2x the tensor, against world x for an all-gather of
    whole tensors, with the same summation order."""
    n = t.numel()
    per = -(-n // world)
    flat = t.reshape(-1)
    src = flat if per * world == n else torch.cat([flat, flat.new_zeros(per * world - n)])
    recv = torch.empty_like(src)
    dist.all_to_all_single(recv, src.contiguous(), group=group)
    parts = recv.view(world, per)
    acc = parts[0].clone()
    for r in range(1, world):
        acc += parts[r]
    out = torch.empty_like(src)
    dist.all_gather_into_tensor(out, acc, group=group)
    return out[:n].view_as(t)


def shard_signature(atlas) -> str:
    """SHA-256 of the bytes of the edges, both seeds and the config: two shards may be combined only
    when these are identical (atlas/core.py:632-634)."""
    h = hashlib.sha256()
    for t in (atlas.E, atlas.top_seed, atlas.res_seed):
        h.update(str(tuple(t.shape)).encode())
        h.update(t.detach().contiguous().cpu().numpy().tobytes())
    h.update(repr(sorted(atlas.cfg.__dict__.items())).encode())
    return h.hexdigest()


def warm_up(group=None, device=None):
    """Run each collective of merge_states once on a few bytes. The backend sets up its peer
    connections (NCCL: one channel per peer for the all-to-all) on first use; doing it here keeps
    that one-time cost out of a timed combine. Every rank must call it."""
    world = dist.get_world_size(group)
    if world == 1:
        return
    dev = device if device is not None else torch.device("cpu")
    w = torch.zeros(world * 8, dtype=torch.int64, device=dev)
    dist.all_to_all_single(torch.empty_like(w), w, group=group)
    dist.all_gather_into_tensor(torch.empty_like(w), w[:8].contiguous(), group=group)
    bufs = [torch.empty(8, dtype=torch.int64, device=dev) for _ in range(world)]
    dist.all_gather(bufs, w[:8].contiguous(), group=group)
    dist.all_reduce(w[:1], op=dist.ReduceOp.SUM, group=group)
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)


class _Sections:
    """CUDA-event (or, on CPU, wall-clock) times of the combine's sections, in ms."""

    def __init__(self, out: dict | None, device):
        self.out, self.cuda = out, out is not None and device.type == "cuda"
        self.t = None

    def mark(self, name: str | None):
        if self.out is None:
            return
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
        else:
            import time
            e = time.perf_counter()
        if self.t is not None:
            prev_name, prev = self.t
            if self.cuda:
                e.synchronize()
                self.out[prev_name] = prev.elapsed_time(e)
            else:
                self.out[prev_name] = (e - prev) * 1e3
        self.t = (name, e) if name is not None else None


@torch.no_grad()
def merge_states(atlas, group=None, row_merge=None, gram: bool = True, timings: dict | None = None):
    """Combine the shard atlases of all ranks in place; afterwards every rank holds the merged
    atlas (equal to merge_from applied over all shards). `atlas` needs the reference's state
    attributes (top_k/top_t/top_s, res_s/res_t/res_v, sub_*, enr/ann_tot, n_seen/n_sub, stats,
    E, top_seed, res_seed, cfg). `row_merge` defaults to the GPU row merge (atlas_merge_rows)."""
    world = dist.get_world_size(group)
    if world == 1:
        return atlas
    row_merge = row_merge or _row_merge_cuda
    sec = _Sections(timings, atlas.top_k.device)
    sec.mark("signature_ms")
    # the shards must share edges, config and both seeds (atlas/core.py:632-634)
    sigs = [None] * world
    dist.all_gather_object(sigs, shard_signature(atlas), group=group)
    if len(set(sigs)) != 1:
        raise ValueError("shards must share edges, config and seeds (derive them from the GLOBAL stream)")
    sec.mark("rows_ms")
    atlas.top_k, atlas.top_t, atlas.top_s = _exchange_rows(atlas.top_k, atlas.top_t, atlas.top_s, (-1, float("-inf")),
                                                           world, group, row_merge)
    atlas.res_s, atlas.res_t, atlas.res_v = _exchange_rows(atlas.res_s, atlas.res_t, atlas.res_v, (-1, float("nan")),
                                                           world, group, row_merge)
    sec.mark("sums_ms")
    for k in ("sub_bin",) + (("enr", "ann_tot") if getattr(atlas, "n_a", 0) else ()):
        t = getattr(atlas, k)
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    for k in ("sub_sum", "sub_sq"):
        getattr(atlas, k).copy_(_sum_in_rank_order(getattr(atlas, k), world, group))
    dev = atlas.top_k.device
    cnt = torch.tensor([atlas.n_seen, atlas.n_sub, getattr(atlas, "gram_rows", 0)], dtype=torch.int64, device=dev)
    dist.all_reduce(cnt, op=dist.ReduceOp.SUM, group=group)
    atlas.n_seen, atlas.n_sub = int(cnt[0]), int(cnt[1])
    sec.mark("gram_ms")
    if gram and getattr(atlas, "gram", None) is not None:
        atlas.flush_gram()
        for l in range(atlas.gram64.shape[0]):
            g = atlas.gram64[l].to(dev)
            atlas.gram64[l].copy_(_reduce_slices_in_rank_order(g, world, group).to(atlas.gram64.device))
        atlas.gram_rows = int(cnt[2])
    sec.mark("stats_ms")
    stats = [None] * world
    dist.all_gather_object(stats, dict(atlas.stats), group=group)
    merged = {}
    for st in stats:
        for k, v in st.items():
            merged[k] = merged.get(k, 0) + v
    atlas.stats = merged
    sec.mark(None)
    return atlas
