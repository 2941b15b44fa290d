"""Host-side pieces of the run_atlas driver (no GPU): checkpoint writing and resume selection (the
reference writes atomically and keeps the last two, scripts/run_atlas.py:39-44,211-212; a damaged
newest checkpoint falls back to the one before it), and the --profile-at range attribution of a
Chrome trace (the report of atlas/proftrace.py:32-81)."""
from __future__ import annotations

import json

import pytest

import torch

from proteus_b200.proftrace import attribute, table
from proteus_b200.run_atlas import atomic_save, load_latest_ckpt


def _ckpt(nb):
    return {"atlas": {"top_s": torch.arange(6.0), "n_seen": nb}, "next_batch": nb, "args_key": "k"}


def test_atomic_save_leaves_no_temporary(tmp_path):
    atomic_save(_ckpt(5), tmp_path / "ckpt_5.pt")
    assert sorted(p.name for p in tmp_path.iterdir()) == ["ckpt_5.pt"]
    p, st = load_latest_ckpt(tmp_path)
    assert p.name == "ckpt_5.pt" and st["next_batch"] == 5


def test_resume_skips_truncated_or_foreign_newest_checkpoint(tmp_path, capsys):
    atomic_save(_ckpt(5), tmp_path / "ckpt_5.pt")
    atomic_save(_ckpt(10), tmp_path / "ckpt_10.pt")
    raw = (tmp_path / "ckpt_10.pt").read_bytes()
    (tmp_path / "ckpt_10.pt").write_bytes(raw[: len(raw) // 3])  # a copy cut short
    p, st = load_latest_ckpt(tmp_path)
    assert p.name == "ckpt_5.pt" and st["next_batch"] == 5
    assert "skipping unreadable checkpoint ckpt_10.pt" in capsys.readouterr().out
    torch.save({"unrelated": 1}, tmp_path / "ckpt_20.pt")  # readable, but not an atlas checkpoint
    p, st = load_latest_ckpt(tmp_path)
    assert p.name == "ckpt_5.pt"


def test_resume_with_no_readable_checkpoint_starts_fresh(tmp_path):
    assert load_latest_ckpt(tmp_path) == (None, None)
    (tmp_path / "ckpt_3.pt").write_bytes(b"\x00garbage")
    assert load_latest_ckpt(tmp_path) == (None, None)


def test_range_attribution_of_a_trace(tmp_path):
    ev = [
        {"ph": "X", "cat": "gpu_user_annotation", "name": "atlas.merge", "ts": 100, "dur": 50},
        {"ph": "X", "cat": "gpu_user_annotation", "name": "atlas.merge.top", "ts": 110, "dur": 20},
        {"ph": "X", "cat": "gpu_user_annotation", "name": "atlas.compact", "ts": 0, "dur": 30},
        {"ph": "X", "cat": "kernel", "name": "filter_bulk_kernel", "ts": 5, "dur": 20},
        {"ph": "X", "cat": "kernel", "name": "admit_kernel", "ts": 101, "dur": 8},
        {"ph": "X", "cat": "kernel", "name": "merge_groups_kernel", "ts": 112, "dur": 15},
        {"ph": "X", "cat": "kernel", "name": "elementwise", "ts": 60, "dur": 10},
        {"ph": "X", "cat": "user_annotation", "name": "atlas.merge", "ts": 90, "dur": 70},
    ]
    path = tmp_path / "t.json"
    path.write_text(json.dumps({"traceEvents": ev}))
    res = attribute(path)
    assert res["atlas.compact"] == {"count": 1, "span_us": 30.0, "busy_us": 20.0, "idle_us": 10.0,
                                    "kernels": {"filter_bulk_kernel": 20.0}}
    assert res["atlas.merge"]["busy_us"] == 8.0 and res["atlas.merge"]["kernels"] == {"admit_kernel": 8.0}
    assert res["atlas.merge.top"]["kernels"] == {"merge_groups_kernel": 15.0}  # innermost range wins
    assert res["_total"]["busy_us"] == 53.0 and res["_total"]["count"] == 4
    txt = table(res)
    assert "atlas.merge.top" in txt and "filter_bulk_kernel" in txt


def test_checkpoint_writer_background_keeps_last_two_and_runs_follow_up(tmp_path):
    from proteus_b200.run_atlas import CheckpointWriter
    w = CheckpointWriter(tmp_path, keep=2)
    done = []
    for nb in (5, 10, 15):
        w.save(_ckpt(nb), tmp_path / f"ckpt_{nb}.pt", after=lambda nb=nb: done.append(nb))
    w.wait()
    assert sorted(p.name for p in tmp_path.iterdir()) == ["ckpt_10.pt", "ckpt_15.pt"]
    assert done == [5, 10, 15]  # one write at a time, in order, each follow-up after its file
    p, st = load_latest_ckpt(tmp_path)
    assert p.name == "ckpt_15.pt" and torch.equal(st["atlas"]["top_s"], torch.arange(6.0))


def test_checkpoint_writer_reports_a_failed_write(tmp_path):
    import pytest
    from proteus_b200.run_atlas import CheckpointWriter
    w = CheckpointWriter(tmp_path / "missing_dir")
    w.save(_ckpt(5), tmp_path / "missing_dir" / "ckpt_5.pt")
    with pytest.raises((FileNotFoundError, RuntimeError), match="does not exist|No such file"):
        w.wait()
    w.wait()  # the error is reported once


def test_prefetch_close_joins_a_blocked_producer():
    """The stream loop may stop with the producer blocked on a full queue or busy on the next item:
    close() must stop and join it (a producer left inside a torch op at interpreter exit aborts the
    process)."""
    import threading
    import time

    from proteus_b200.run_atlas import Prefetch
    made = []

    def gen():
        for i in range(100):
            made.append(i)
            yield torch.full((4,), i)

    p = Prefetch(gen(), 2)
    assert int(next(p)[0]) == 0 and int(next(p)[0]) == 1
    time.sleep(0.3)  # the producer fills the queue and blocks
    t0 = time.time()
    p.close()
    assert time.time() - t0 < 5 and not any(t.name == "prefetch" and t.is_alive() for t in threading.enumerate())
    assert len(made) < 10


def test_prefetch_reraises_producer_errors_and_ends():
    from proteus_b200.run_atlas import Prefetch

    def bad():
        yield 1
        raise ValueError("broken batch")

    p = Prefetch(bad(), 2)
    assert next(p) == 1
    with pytest.raises(ValueError, match="broken batch"):
        next(p)
    p.close()
    q = Prefetch(iter([1, 2]), 1)
    assert list(q) == [1, 2]
    q.close()


def test_overhead_summary_windows():
    from proteus_b200.run_atlas import overhead_summary
    paired = [(i, 10.0 if i < 60 else 0.2 + (i % 7) * 0.001) for i in range(5000)]
    s = overhead_summary(paired)
    assert s["paired_batches"] == 5000
    assert s["prefix_0_59"]["n"] == 60 and s["prefix_0_59"]["median"] == 10.0
    assert s["steady"]["n"] == 1600 and s["steady_from_batch"] == 3400 and abs(s["steady"]["median"] - 0.203) < 1e-9
    assert set(s["windows"]) == {"0-100", "100-1000", "1000-3000", "3000-5000"}
    assert overhead_summary([]) == {"paired_batches": 0}
