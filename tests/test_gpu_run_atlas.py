"""End-to-end driver on the GPU (python -m proteus_b200.run_atlas, the drop-in for the reference's
scripts/run_atlas.py): a full run equals a run stopped between checkpoints and resumed — the
reference's resume contract (tests/test_resume_merge.py:104-132): every exact field bitwise equal,
n_seen equal; the Gram is not checkpointed (gram_rows says how many rows it covers)."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _run(args, cwd):
    r = subprocess.run([sys.executable, "-m", "proteus_b200.run_atlas", *args], cwd=cwd, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    return r.stdout


@pytest.mark.parametrize("seeded", [False, True])
def test_full_run_equals_stop_and_resume(tmp_path, seeded):
    base = ["--model", "8M", "--data", "synthetic:400:3", "--device", "cuda:0", "--dtype", "bf16",
            "--tokens-per-batch", "8192", "--pilot-tokens", "8192", "--K", "16", "--Kr", "8", "--ckpt-every", "5"]
    if seeded:
        base.append("--seed-thresholds")
    full, part = tmp_path / "full", tmp_path / "part"
    _run(base + ["--out", str(full)], ROOT)
    out1 = _run(base + ["--out", str(part), "--stop-after", "7"], ROOT)
    assert "stopping after 7" in out1
    out2 = _run(base + ["--out", str(part), "--resume"], ROOT)
    assert "resumed from ckpt_5.pt" in out2
    A = torch.load(full / "atlas.pt", weights_only=False)
    B = torch.load(part / "atlas.pt", weights_only=False)
    for k in ("top_val", "top_tok", "res_tok", "res_key", "sub_bin", "enr", "ann_tot"):
        assert torch.equal(A[k], B[k]), k
    assert torch.allclose(A["res_val"], B["res_val"], equal_nan=True, rtol=0, atol=0)
    assert torch.allclose(A["sub_sum"], B["sub_sum"], rtol=1e-9, atol=1e-9)
    assert A["n_seen"] == B["n_seen"] and A["n_sub"] == B["n_sub"]
    assert B["gram_rows"] < A["gram_rows"]  # the resumed run's Gram covers the batches after the resume


def test_profile_at_writes_kernel_table_and_range_attribution(tmp_path):
    """--profile-at (run_atlas.py:240-266 of the reference): the profiled batch gets a kernel table,
    a per-range attribution in which the atlas ranges own the atlas kernels, and the trace."""
    out = tmp_path / "prof"
    _run(["--model", "8M", "--data", "synthetic:200:3", "--device", "cuda:0", "--dtype", "bf16",
          "--tokens-per-batch", "8192", "--pilot-tokens", "8192", "--K", "16", "--Kr", "8", "--seed-thresholds",
          "--profile-at", "2", "--out", str(out)], ROOT)
    assert (out / "profile_batch_2.txt").stat().st_size > 0
    assert (out / "profile_batch_2.trace.json.gz").exists()
    import json
    res = json.loads((out / "profile_batch_2_ranges.json").read_text())
    assert "filter_bulk_kernel" in " ".join(res["atlas.compact"]["kernels"])
    assert res["atlas.merge.top"]["busy_us"] > 0
