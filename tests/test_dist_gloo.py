"""Multi-rank protocol on CPU (gloo, world size 2): sharding of the batch plan, and the exact
cross-rank state combine of proteus_b200.dist.merge_states against the reference's merged result
(tests/golden/merge_from.npz, two shards merged by the reference's Atlas.merge_from). The row merge
of the GPU path is replaced by a CPU restatement (the oracle's semantics) so no GPU is needed; a
rank that fails before the combine makes the other rank's collective end with an error, not hang."""
from __future__ import annotations

import os
import socket
import traceback
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.harness import golden


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def cpu_row_merge(sc, tok, val, osc, otok, oval):
    """Row-wise top-K of two sorted states (atlas/core.py:636-643 semantics), CPU."""
    K = sc.shape[1]
    allv = torch.cat([sc, osc], 1)
    idx = torch.argsort(allv, dim=1, descending=True, stable=True)[:, :K]
    sc.copy_(torch.gather(allv, 1, idx))
    tok.copy_(torch.gather(torch.cat([tok, otok], 1), 1, idx))
    val.copy_(torch.gather(torch.cat([val, oval], 1), 1, idx))


class _Stats(SimpleNamespace):
    pass


def _shard(z, h):
    t = lambda k: torch.from_numpy(np.array(z[f"s{h}_{k}"]))  # noqa: E731
    cfg = SimpleNamespace(K=8, Kr=4, rho_res=0.05, rho_sub=0.2, cap_frac=0.05, seed=11)
    a = _Stats(top_k=t("top_k"), top_t=t("top_t"), top_s=t("top_s"), res_s=t("res_s"), res_t=t("res_t"),
               res_v=t("res_v"), sub_sum=t("sub_sum"), sub_sq=t("sub_sq"), sub_bin=t("sub_bin"), E=t("E"),
               top_seed=t("top_seed"), res_seed=t("res_seed"), enr=t("enr"), ann_tot=t("ann_tot"), n_a=5,
               n_seen=int(z[f"s{h}_n_seen"]), n_sub=int(z[f"s{h}_n_sub"]), gram=None, cfg=cfg,
               stats={"batches": 1})
    return a


def _empty_shard(z):
    """A rank that streamed nothing: the same edges, seeds and config, empty state."""
    a = _shard(z, 0)
    a.top_k.fill_(torch.iinfo(torch.int64).min)
    a.top_t.fill_(-1)
    a.top_s.fill_(float("-inf"))
    a.res_s.fill_(torch.iinfo(torch.int64).min)
    a.res_t.fill_(-1)
    a.res_v.fill_(float("nan"))
    for k in ("sub_sum", "sub_sq", "sub_bin", "enr", "ann_tot"):
        getattr(a, k).zero_()
    a.n_seen = a.n_sub = 0
    a.stats = {"batches": 0}
    return a


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime
        torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                             timeout=datetime.timedelta(seconds=20))
        from proteus_b200.dist import merge_states, shard_plan, warm_up
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure before the combine")
        if mode == "gram":  # the Gram's sliced all-to-all reduction against a plain rank-order sum
            from proteus_b200.dist import _reduce_slices_in_rank_order
            ts = [torch.from_numpy(np.random.default_rng(r).standard_normal((37, 53))) for r in range(world)]
            want = ts[0].clone()
            for t in ts[1:]:
                want += t
            got = _reduce_slices_in_rank_order(ts[rank].clone(), world, None)
            q.put((rank, {"equal": bool(torch.equal(got, want))}))
            torch.distributed.destroy_process_group()
            return
        z = golden("merge_from")
        a = _shard(z, rank) if rank < 2 else _empty_shard(z)
        if mode == "badsig" and rank == 1:
            a.res_seed = a.res_seed.clone()
            a.res_seed.view(-1)[7] += 1  # one seed differs: the shards were not seeded alike
        warm_up()
        merge_states(a, row_merge=cpu_row_merge, gram=False)
        want = {k[2:]: v for k, v in z.items() if k.startswith("m_")}
        L, D, K, B, Kr = 2, 48, 8, 5, 4
        ok = {
            "top_tok": np.array_equal(a.top_t.view(L, 2, D, K).numpy(), want["top_tok"]),
            "top_val": np.array_equal((a.top_s.view(L, 2, D, K) * torch.tensor([1., -1.]).view(1, 2, 1, 1)).numpy(),
                                      want["top_val"]),
            "res_tok": np.array_equal(a.res_t.view(L, 2, D, B, Kr).numpy(), want["res_tok"]),
            "res_key": np.array_equal((-a.res_s).view(L, 2, D, B, Kr).numpy(), want["res_key"]),
            "sub_bin": np.array_equal(a.sub_bin.numpy(), want["sub_bin"]),
            "enr": np.array_equal(a.enr.numpy(), want["enr"]),
            "ann_tot": np.array_equal(a.ann_tot.numpy(), want["ann_tot"]),
            "n": (a.n_seen, a.n_sub) == (int(want["n_seen"]), int(want["n_sub"])),
            "sums": np.allclose(a.sub_sum.numpy(), want["sub_sum"], rtol=1e-12, atol=1e-9),
            "shard": sorted(sum((shard_plan(list(range(11)), world, r) for r in range(world)), [])) == list(range(11)),
        }
        q.put((rank, ok))
        torch.distributed.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-400:]}"))


def _run(mode, timeout=120, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in ps:
        r, v = q.get(timeout=timeout)
        out[r] = v
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_merge_states_two_ranks_matches_reference():
    out = _run("ok")
    for r in (0, 1):
        assert isinstance(out[r], dict), out[r]
        assert all(out[r].values()), out[r]


def test_merge_states_five_ranks_uneven_slices_matches_reference():
    """World size 5: the 2*2*48 = 192 group rows do not divide by 5, so the all-to-all slices are
    padded; ranks 2-4 streamed nothing. Every rank must still end with the reference's merged state."""
    out = _run("ok", world=5, timeout=180)
    for r in range(5):
        assert isinstance(out[r], dict), out[r]
        assert all(out[r].values()), (r, out[r])


def test_failed_rank_ends_combine_with_error_not_hang():
    out = _run("fail")
    assert isinstance(out[1], str) and "injected failure" in out[1]
    assert isinstance(out[0], str), "rank 0 must see an error (timeout or peer loss), not a result"


def _lockstep_worker(rank, world, port, plan_lens, stop_at, q):
    """The run_atlas loop's control flow over a plan of plan_lens[rank] batches: rank r proposes a
    deadline stop once it has streamed stop_at[r] batches (and has more left)."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime
        torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                             timeout=datetime.timedelta(seconds=20))
        from proteus_b200.dist import Lockstep
        lock = Lockstep()
        done, steps = 0, 0
        while True:
            want = 0
            if done < plan_lens[rank]:
                done += 1
                if stop_at[rank] is not None and done >= stop_at[rank] and done < plan_lens[rank]:
                    want = 2
            code, more = lock.agree(want, done < plan_lens[rank])
            steps += 1
            if code or not more:
                break
        q.put((rank, (code, done, steps)))
        torch.distributed.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-400:]}"))


def _run_lockstep(plan_lens, stop_at, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = len(plan_lens)
    ps = [ctx.Process(target=_lockstep_worker, args=(r, world, port, plan_lens, stop_at, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in ps:
        r, v = q.get(timeout=timeout)
        out[r] = v
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_lockstep_one_rank_at_deadline_stops_every_rank_at_the_same_step():
    """plan[rank::world] gives the ranks plans of different lengths; rank 1 reaches its deadline
    after 3 batches. Both ranks must stop at that step (rank 0 with 3 of its 7 batches done), not
    rank 1 alone while rank 0 streams on towards the combine."""
    out = _run_lockstep([7, 6], [None, 3])
    assert out[0] == (2, 3, 3) and out[1] == (2, 3, 3), out


def test_lockstep_uneven_shards_leave_the_loop_together():
    """No stop: the rank with the shorter shard keeps agreeing until the longer one is done, so both
    leave the loop at the same step and enter the combine together."""
    out = _run_lockstep([7, 4], [None, None])
    assert out[0] == (0, 7, 7) and out[1] == (0, 4, 7), out


def test_gram_slices_reduce_in_rank_order():
    """The Gram's combine (all-to-all of slices, rank-ordered sum, all-gather) equals the plain sum
    of the ranks' matrices in rank order, bit for bit, with a size that does not divide by 3."""
    out = _run("gram", world=3)
    for r in range(3):
        assert out[r] == {"equal": True}, out[r]


def test_shards_with_different_seeds_are_refused():
    out = _run("badsig")
    for r in (0, 1):
        assert isinstance(out[r], str) and "must share edges, config and seeds" in out[r], out[r]
