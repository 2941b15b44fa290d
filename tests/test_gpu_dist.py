"""The cross-GPU combine on real GPUs: two ranks over NCCL, each holding one of the reference's two
shard states (tests/golden/merge_from.npz) on its own GPU, combined by proteus_b200.dist.merge_states
with the GPU row merge (atlas_merge_rows); every rank must end with the reference's merged result
(Atlas.merge_from, atlas/core.py:628-654), bit for bit. Needs two GPUs (skipped otherwise); NVLS is
off and the process group has a short timeout, so a rank that fails ends the other's collective
with an error instead of a hang."""
from __future__ import annotations

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import datetime
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                             timeout=datetime.timedelta(seconds=60), device_id=dev)
        from proteus_b200.dist import merge_states
        from tests.harness import golden
        from tests.test_dist_gloo import _shard
        z = golden("merge_from")
        a = _shard(z, rank)
        for k, v in list(vars(a).items()):
            if torch.is_tensor(v):
                setattr(a, k, v.to(dev))
        merge_states(a, gram=False)
        torch.cuda.synchronize()
        want = {k[2:]: v for k, v in z.items() if k.startswith("m_")}
        L, D, K, B, Kr = 2, 48, 8, 5, 4
        sign = torch.tensor([1., -1.], device=dev).view(1, 2, 1, 1)
        ok = {
            "top_tok": np.array_equal(a.top_t.view(L, 2, D, K).cpu().numpy(), want["top_tok"]),
            "top_val": np.array_equal((a.top_s.view(L, 2, D, K) * sign).cpu().numpy(), want["top_val"]),
            "res_tok": np.array_equal(a.res_t.view(L, 2, D, B, Kr).cpu().numpy(), want["res_tok"]),
            "res_key": np.array_equal((-a.res_s).view(L, 2, D, B, Kr).cpu().numpy(), want["res_key"]),
            "sub_bin": np.array_equal(a.sub_bin.cpu().numpy(), want["sub_bin"]),
            "enr": np.array_equal(a.enr.cpu().numpy(), want["enr"]),
            "ann_tot": np.array_equal(a.ann_tot.cpu().numpy(), want["ann_tot"]),
            "n": (a.n_seen, a.n_sub) == (int(want["n_seen"]), int(want["n_sub"])),
            "sums": np.allclose(a.sub_sum.cpu().numpy(), want["sub_sum"], rtol=1e-12, atol=1e-9),
        }
        q.put((rank, ok))
        torch.distributed.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-600:]}"))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_merge_states_two_gpus_nccl_matches_reference():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = {}
    for _ in ps:
        r, v = q.get(timeout=300)
        out[r] = v
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in (0, 1):
        assert isinstance(out[r], dict), out[r]
        assert all(out[r].values()), out[r]
