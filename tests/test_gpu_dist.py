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
        # a Gram per rank (fp64 accumulator, already flushed): the combine must return the rank-order sum
        grams = [torch.from_numpy(np.random.default_rng(r).standard_normal((2, 48, 48))) for r in range(world)]
        a.gram = torch.zeros(2, 48, 48, device=dev)
        a.gram64 = grams[rank].to(dev)
        a.gram_rows = 100 + rank
        a.flush_gram = lambda: None
        merge_states(a, gram=True)
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
            "gram": np.array_equal(a.gram64.cpu().numpy(), (grams[0] + grams[1]).numpy()),
            "gram_rows": a.gram_rows == 201,
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


def _run_atlas(args, nproc, cwd, env_extra=None):
    import subprocess
    import sys
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", **(env_extra or {}))
    if nproc == 1:
        cmd = [sys.executable, "-m", "proteus_b200.run_atlas", *args]
    else:
        cmd = ["timeout", "-k", "30", "840", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}", "-m",
               "proteus_b200.run_atlas", *args]
    r = subprocess.run(cmd, cwd=cwd, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return r.stdout


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_run_atlas_two_ranks_equals_one_rank(tmp_path):
    """run_atlas under torchrun on two GPUs (each rank streams plan[rank::2], seeds from the global
    stream, exact NCCL combine) gives the single-GPU run's atlas bit for bit; a two-rank run stopped
    by --stop-after and resumed gives it too (both ranks stop at the same step)."""
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    base = ["--model", "8M", "--data", "synthetic:600:4", "--dtype", "bf16", "--tokens-per-batch", "8192",
            "--pilot-tokens", "8192", "--K", "16", "--Kr", "8", "--seed-thresholds", "--ckpt-every", "3"]
    one, two, part = tmp_path / "one", tmp_path / "two", tmp_path / "part"
    _run_atlas(base + ["--device", "cuda:0", "--out", str(one)], 1, root)
    _run_atlas(base + ["--out", str(two)], 2, root)
    out = _run_atlas(base + ["--out", str(part), "--stop-after", "4"], 2, root)
    assert "stopping after 4" in out
    assert {p.name for p in (part / "ckpt").iterdir()} == {"rank0", "rank1"}
    _run_atlas(base + ["--out", str(part), "--resume"], 2, root)
    A = torch.load(one / "atlas.pt", weights_only=False)
    for other in (two, part):
        Bm = torch.load(other / "atlas.pt", weights_only=False)
        for k in ("top_val", "top_tok", "res_tok", "res_key", "sub_bin", "enr", "ann_tot", "edges"):
            assert torch.equal(A[k], Bm[k]), (other.name, k)
        assert torch.equal(torch.nan_to_num(A["res_val"], nan=-7.0), torch.nan_to_num(Bm["res_val"], nan=-7.0))
        assert A["n_seen"] == Bm["n_seen"] and A["n_sub"] == Bm["n_sub"]
        assert torch.allclose(A["sub_sum"], Bm["sub_sum"], rtol=1e-9, atol=1e-9)
