"""A device-side failure cannot pass unnoticed.

Two things invalidate an atlas state without any exception at launch time: a bounded device wait
(tcgen05 / TMA mbarrier) that gave up, which leaves that launch's output incomplete, and a record
list that ran out of capacity, which drops records. Both are recorded on the device. These tests
plant the failure from the host (the status word is written through a test hook; the list flag is
set directly), never by making a wait run out, and check that the state is then refused: by
check_errors, by result(), and by state_dict(), which every checkpoint goes through, so run_atlas
writes no checkpoint over a flagged state.
"""
from __future__ import annotations

import ctypes
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from tests.golden.make_golden import STREAM_CFG, STREAM_SHAPE
from tests.harness import drive, golden
from tests.streams import Stream, make_stream

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = Path(__file__).resolve().parents[1]


def _atlas_over(batches):
    from proteus_b200.core import Atlas, AtlasConfig
    z = golden("stream_bf16_seeded")
    st = make_stream(**STREAM_SHAPE)
    at = Atlas(st.L, st.D, torch.from_numpy(z["E"]), AtlasConfig(**STREAM_CFG), n_annot=STREAM_SHAPE["n_annot"],
               device=DEV)
    at.seed(torch.from_numpy(z["top_seed"]), torch.from_numpy(z["res_seed_key"]))
    sub = Stream(st.L, st.D, st.dtype, st.lens, st.seqs, st.ann_full, st.batches[:batches], st.order)
    drive(at, sub, to_input=lambda h: torch.from_numpy(h).to(DEV).to(torch.bfloat16))
    return at, st


def _reset_status():
    from proteus_b200 import _lib
    v = ctypes.c_int(0)
    assert _lib.load().atlas_device_status(ctypes.byref(v), 1) == 0
    return v.value


def test_device_status_blocks_result_and_checkpoint():
    from proteus_b200 import _lib
    from proteus_b200._lib import AtlasKernelError
    assert _reset_status() == 0
    at, _ = _atlas_over(3)
    at.check_errors()
    assert at.device_status() == 0
    assert _lib.load().atlas_device_status_set(7) == 0
    try:
        assert at.device_status() == 7
        with pytest.raises(AtlasKernelError, match="device status 7"):
            at.check_errors()
        with pytest.raises(AtlasKernelError, match="device status 7"):
            at.state_dict()
        with pytest.raises(AtlasKernelError, match="device status 7"):
            at.result()
    finally:
        assert _reset_status() == 7
    at.check_errors()
    assert at.state_dict()["n_seen"] == at.n_seen


def test_list_overflow_flag_survives_later_batches():
    """The overflow flag is raised by the batch whose lists overflowed and stays raised through the
    batches after it (begin_batch clears the per-batch slots only)."""
    from proteus_b200._lib import AtlasKernelError
    at, st = _atlas_over(2)
    at._flags[at.L + 2] = 1
    more = Stream(st.L, st.D, st.dtype, st.lens, st.seqs, st.ann_full, st.batches[2:4], st.order)
    drive(at, more, to_input=lambda h: torch.from_numpy(h).to(DEV).to(torch.bfloat16))
    with pytest.raises(AtlasKernelError, match="overflowed"):
        at.check_errors()
    with pytest.raises(AtlasKernelError, match="overflowed"):
        at.state_dict()


def test_run_atlas_writes_no_checkpoint_over_flagged_state(tmp_path):
    """run_atlas with the status word already set: the first checkpoint attempt raises and nothing
    is written."""
    code = (
        "import sys, ctypes\n"
        "from proteus_b200 import _lib\n"
        "assert _lib.load().atlas_device_status_set(5) == 0\n"
        "from proteus_b200 import run_atlas\n"
        "try:\n"
        "    run_atlas.main(sys.argv[1:])\n"
        "except _lib.AtlasKernelError as e:\n"
        "    print('REFUSED:', e)\n"
        "    sys.exit(3)\n"
    )
    out = tmp_path / "run"
    r = subprocess.run([sys.executable, "-c", code, "--model", "8M", "--data", "synthetic:120:3", "--device", "cuda:0",
                        "--dtype", "bf16", "--tokens-per-batch", "8192", "--pilot-tokens", "8192", "--K", "16",
                        "--Kr", "8", "--ckpt-every", "2", "--out", str(out)],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 3, r.stdout[-2000:] + r.stderr[-2000:]
    assert "REFUSED: device status 5" in r.stdout
    assert not list((out / "ckpt").glob("ckpt_*.pt"))
    assert not (out / "atlas.pt").exists()
