"""End-to-end atlas run, resumable — drop-in for haelyons/proteus scripts/run_atlas.py (same flags).

  python -m proteus_b200.run_atlas --model 650M --data data.pt --out runs/x [--resume] ...
  torchrun --nproc-per-node 8 -m proteus_b200.run_atlas ...   (one shard of the batch plan per GPU)

Outputs in --out (as the reference, run_atlas.py:3-8): ckpt/ckpt_<batch>.pt (atomic, last 2 kept),
batches.jsonl (one record per batch; its GPU times come from CUDA events read a few batches later,
so the loop never drains the GPU to time a batch), run.json (summary), atlas.pt (final result +
sha256 digests of the exact fields). With several ranks each rank checkpoints its own shard under ckpt/rank<r>/ and
the shard states are combined exactly (proteus_b200.dist.merge_states) before rank 0 writes atlas.pt.

--data accepts the reference's Swiss-Prot .pt format or `synthetic:<n_seq>[:<seed>]` (C4-like
synthetic proteins). Models are built from their published architecture with a seeded random init
(no network), or loaded from a local HuggingFace directory.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import queue
import sys
import threading
import time
from pathlib import Path

import torch

from .core import Atlas, AtlasConfig
from .data import SwissProt, shuffled_order, synthetic_dataset
from .esm import attach, flops_per_batch, load
from .pilot import pilot_pass


def sync(dev):
    if torch.device(dev).type == "cuda":
        torch.cuda.synchronize()


def atomic_save(obj, path: Path):
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save(obj, tmp)
    with open(tmp, "rb") as f:
        os.fsync(f.fileno())
    os.replace(tmp, path)


def write_profile(prof, path: Path, dev):
    """Kernel table (key_averages, by device time) plus the per-range attribution of the Chrome
    trace (span / busy / idle per atlas.* range with its top kernels) and the gzipped trace, as
    the reference's --profile-at output (run_atlas.py:341-365)."""
    import gzip
    import shutil
    from .proftrace import attribute, table
    try:
        tp = path.with_suffix(".trace.json")
        prof.export_chrome_trace(str(tp))
        res = attribute(tp)
        path.with_name(path.stem + "_ranges.txt").write_text(table(res, top=10))
        path.with_name(path.stem + "_ranges.json").write_text(json.dumps(res))
        with open(tp, "rb") as fi, gzip.open(str(tp) + ".gz", "wb") as fo:
            shutil.copyfileobj(fi, fo)
        tp.unlink()
    except Exception as e:  # noqa: BLE001  the attribution is a diagnostic; the run goes on
        print(f"[atlas] trace attribution failed: {e!r}", flush=True)
    ka = prof.key_averages()
    keys = ("self_device_time_total", "self_cuda_time_total") if torch.device(dev).type == "cuda" else ("self_cpu_time_total",)
    for key in keys:
        try:
            path.write_text(ka.table(sort_by=key, row_limit=60))
            return
        except Exception:  # noqa: BLE001  key names differ between torch versions
            continue
    path.write_text(ka.table(row_limit=60))


class CheckpointWriter:
    """Checkpoints written behind the stream. `save` takes a host copy of the state on the calling
    thread (a consistent snapshot between two batches; the device keeps working on the next batch
    afterwards) and hands the disk write (tmp + fsync + rename), the pruning to the newest `keep`
    files and an optional follow-up (the run summary) to a background thread, so a multi-GB
    checkpoint no longer stalls the batch loop. One write is in flight at a time: a new checkpoint
    first waits for the previous one. `wait` joins the write and re-raises its error, if any."""

    def __init__(self, ck_dir: Path, keep: int = 2):
        self.ck_dir, self.keep = ck_dir, keep
        self._t = None
        self._err = None

    def _write(self, obj, path: Path, after):
        try:
            atomic_save(obj, path)
            for old in sorted(self.ck_dir.glob("ckpt_*.pt"), key=lambda q: int(q.stem.split("_")[1]))[:-self.keep]:
                old.unlink()
            if after is not None:
                after()
        except BaseException as e:  # noqa: BLE001  re-raised on the caller's thread by wait()
            self._err = e

    def save(self, obj, path: Path, after=None):
        self.wait()
        self._t = threading.Thread(target=self._write, args=(obj, path, after), name="ckpt-writer")
        self._t.start()

    def wait(self):
        if self._t is not None:
            self._t.join()
            self._t = None
        if self._err is not None:
            e, self._err = self._err, None
            raise e


def load_latest_ckpt(d: Path):
    """(path, checkpoint dict) of the newest readable checkpoint in d, or (None, None). A newest file
    that cannot be read (truncated by a kill during a copy, or damaged) is reported and skipped in
    favour of the one before it: the writer keeps the last two (atomic tmp + fsync + rename)."""
    c = sorted(d.glob("ckpt_*.pt"), key=lambda p: int(p.stem.split("_")[1]))
    for p in reversed(c):
        try:
            st = torch.load(p, weights_only=False, map_location="cpu")
            if not isinstance(st, dict) or "atlas" not in st or "next_batch" not in st:
                raise ValueError("not an atlas checkpoint")
            return p, st
        except Exception as e:  # noqa: BLE001  any unreadable file: fall back to the previous one
            print(f"[atlas] skipping unreadable checkpoint {p.name}: {type(e).__name__}: {e}", flush=True)
    return None, None


def parser():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="8M")
    ap.add_argument("--control", default="none", choices=["none", "shuffled", "random"])
    ap.add_argument("--control-seed", type=int, default=None)
    ap.add_argument("--data", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--dtype", default="bf16")
    ap.add_argument("--max-seqs", type=int, default=0)
    ap.add_argument("--tokens-per-batch", type=int, default=32768)
    ap.add_argument("--window", type=int, default=8192)
    ap.add_argument("--sorted-batches", action="store_true")
    ap.add_argument("--pilot-tokens", type=int, default=32768)
    ap.add_argument("--K", type=int, default=64)
    ap.add_argument("--Kr", type=int, default=16)
    ap.add_argument("--backend", default="torch")
    ap.add_argument("--cap-frac-early", type=float, default=0.0)
    ap.add_argument("--stats-impl", default="v3", choices=["v3", "v2", "v1"])
    ap.add_argument("--merge-impl", default="stacked", choices=["stacked", "loop"])
    ap.add_argument("--no-reservoir", action="store_true")
    ap.add_argument("--no-subsample", action="store_true")
    ap.add_argument("--no-gram", action="store_true")
    ap.add_argument("--naive", action="store_true")
    ap.add_argument("--count-ties", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--ckpt-every", type=int, default=500)
    ap.add_argument("--gram-flush-every", type=int, default=500)
    ap.add_argument("--resume", action="store_true")
    ap.add_argument("--stop-after", type=int, default=0)
    ap.add_argument("--seed-thresholds", action="store_true")
    ap.add_argument("--pair-forward", action="store_true")
    ap.add_argument("--pair-every", type=int, default=0)
    ap.add_argument("--plan-offset", type=int, default=0)
    ap.add_argument("--prefetch", type=int, default=2)
    ap.add_argument("--only-acc", default=None)
    ap.add_argument("--edges-from", default=None)
    ap.add_argument("--exclude-acc", default=None)
    ap.add_argument("--edge-q", type=float, nargs="+", default=[0.5, 0.9, 0.99, 0.999, 0.9999])
    ap.add_argument("--profile-at", type=int, nargs="*", default=[])
    ap.add_argument("--max-batches", type=int, default=0)
    ap.add_argument("--deadline", type=float, default=0.0)
    ap.add_argument("--host-ctx", action="store_true",
                    help="build batch contexts with the host make_ctx (as the reference) instead of on the device")
    return ap


def _args_key(a) -> dict:
    keep = ["model", "control", "data", "dtype", "max_seqs", "tokens_per_batch", "window", "sorted_batches",
            "pilot_tokens", "K", "Kr", "no_reservoir", "no_subsample", "no_gram", "naive", "seed",
            "seed_thresholds", "max_batches", "exclude_acc", "edge_q", "only_acc", "edges_from"]
    key = {k: getattr(a, k) for k in keep}
    if getattr(a, "control_seed", None) is not None:
        key["control_seed"] = a.control_seed
    return key


def _dataset(spec: str):
    if spec.startswith("synthetic:"):
        parts = spec.split(":")
        return SwissProt(synthetic_dataset(int(parts[1]), seed=int(parts[2]) if len(parts) > 2 else 0))
    return SwissProt(spec)


def overhead_summary(paired: list) -> dict:
    """Atlas overhead vs the hook-free forward of the same batch (atlas pass / forward - 1) over the
    paired batches, as the reference reports it (results/README.md:205-208): whole run, the prefix
    (batches 0-59), the steady state (the last 1,600 paired batches, or the last half of a shorter
    run) and windows of the plan, each as median / mean. `paired`: (global batch index, overhead)."""
    import statistics
    if not paired:
        return {"paired_batches": 0}
    paired = sorted(paired)

    def mm(xs):
        xs = [x for _, x in xs]
        return {"n": len(xs), "median": statistics.median(xs), "mean": statistics.fmean(xs)} if xs else None

    n = len(paired)
    steady = paired[-1600:] if n >= 3200 else paired[n // 2:]
    out = {"paired_batches": n, "whole": mm(paired), "prefix_0_59": mm([x for x in paired if x[0] < 60]),
           "steady": mm(steady), "steady_from_batch": steady[0][0]}
    last = paired[-1][0] + 1
    edges = [0, 100, 1000, 3000, max(3000, last)]
    out["windows"] = {f"{a}-{b}": mm([x for x in paired if a <= x[0] < b]) for a, b in zip(edges[:-1], edges[1:])
                      if any(a <= x[0] < b for x in paired)}
    return out


class Prefetch:
    """Items of `it` produced `n` ahead on a background thread (the batch and its host-side context,
    as the reference's prefetch thread builds them). `close()` stops the producer and joins it: the
    producer checks the stop flag between items, and close() drains the queue so a producer blocked
    on a full queue wakes up. Every exit path of the stream loop closes it, so no producer is still
    inside a torch op when the interpreter shuts down."""

    _END = object()

    def __init__(self, it, n):
        self._q = queue.Queue(maxsize=max(1, n))
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._work, args=(it,), name="prefetch", daemon=True)
        self._t.start()

    def _work(self, it):
        try:
            for x in it:
                while not self._stop.is_set():
                    try:
                        self._q.put(x, timeout=0.1)
                        break
                    except queue.Full:
                        continue
                if self._stop.is_set():
                    return
        except BaseException as e:  # noqa: BLE001  re-raised on the consumer's thread
            self._put_final(e)
            return
        self._put_final(self._END)

    def _put_final(self, x):
        while not self._stop.is_set():
            try:
                self._q.put(x, timeout=0.1)
                return
            except queue.Full:
                continue

    def __iter__(self):
        return self

    def __next__(self):
        x = self._q.get()
        if x is self._END:
            raise StopIteration
        if isinstance(x, BaseException):
            raise x
        return x

    def close(self):
        self._stop.set()
        while self._t.is_alive():
            try:
                while True:
                    self._q.get_nowait()
            except queue.Empty:
                pass
            self._t.join(timeout=0.1)


def main(argv=None):
    a = parser().parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=1800),
                                             device_id=torch.device("cuda", local))
        # the per-batch stop agreement runs on the host (gloo), so it never waits for the GPU stream
        ctl_group = torch.distributed.new_group(backend="gloo", timeout=datetime.timedelta(seconds=1800))
        dev = f"cuda:{local}"
    else:
        dev = a.device
        ctl_group = None
    out = Path(a.out)
    ck_dir = out / "ckpt" if world == 1 else out / "ckpt" / f"rank{rank}"
    ck_dir.mkdir(parents=True, exist_ok=True)
    dtype = {"bf16": torch.bfloat16, "fp32": torch.float32, "fp16": torch.float16}[a.dtype]
    log = (lambda *x: print(*x, flush=True)) if rank == 0 else (lambda *x: None)

    t0 = time.time()
    ds = _dataset(a.data)
    order = shuffled_order(len(ds), a.seed)
    n_excluded = 0

    def acc_set(path):
        return {ln.split("\t")[0].split(",")[0].strip() for ln in open(path) if ln.strip() and not ln.startswith("Entry")}
    if a.only_acc:
        inc = acc_set(a.only_acc)
        order = order[torch.tensor([ds.d["acc"][i] in inc for i in order.tolist()], dtype=torch.bool)]
    if a.exclude_acc:
        ex = acc_set(a.exclude_acc)
        drop = torch.tensor([acc in ex for acc in ds.d["acc"]], dtype=torch.bool)
        keep = ~drop[order]
        n_excluded = int((~keep).sum())
        order = order[keep]
    if a.max_seqs:
        order = order[: a.max_seqs]
    ctl_seed = a.seed if a.control_seed is None else a.control_seed
    model, tok, info = load(a.model, a.control, dtype=dtype, device=dev, seed=ctl_seed)
    info["control_seed"] = ctl_seed
    vocab = tok.get_vocab()
    L, D = info["n_layers"], info["d_ff"]
    plan = ds.plan(order, a.tokens_per_batch, a.window, a.seed, shuffle_batches=not a.sorted_batches)
    if a.max_batches:
        plan = plan[: a.max_batches]
    n_total = int(sum(min(int(ds.len[i]), ds.max_res) for grp in plan for i in grp))
    t_load = time.time() - t0

    cfg = AtlasConfig(K=a.K, Kr=a.Kr, backend=a.backend, seed=a.seed, reservoir=not a.no_reservoir,
                      subsample=not a.no_subsample, gram=not a.no_gram and not a.no_subsample, naive=a.naive,
                      stats_impl=a.stats_impl, merge_impl=a.merge_impl, cap_frac_early=a.cap_frac_early)
    ck, st = load_latest_ckpt(ck_dir) if a.resume else (None, None)
    t1 = time.time()
    seeds = None
    if ck is not None:
        assert st["args_key"] == _args_key(a), "resume with different run arguments"
        E = st["atlas"]["E"]
        start = st["next_batch"]
    else:
        given = None
        if a.edges_from:
            src = torch.load(a.edges_from, map_location="cpu", weights_only=False)
            given = src["edges"] if "edges" in src else src["atlas"]["E"]
        if given is not None and not a.seed_thresholds:
            E = given
        else:
            # the pilot on the device, a group of layers at a time (its activations never sit in host
            # memory), edges and seeds from the device pilot kernels
            pplan = ds.pilot_plan(plan, a.pilot_tokens, a.tokens_per_batch, a.seed)
            pbatches = list(ds.batches(vocab, order, a.tokens_per_batch, plan=pplan))
            E, seeds, _ = pilot_pass(model, pbatches, torch.device(dev), L, D, probs=tuple(a.edge_q),
                                     seeds=(a.K, a.Kr, n_total) if a.seed_thresholds else None, edges=given)
        start = a.plan_offset
    t_pilot = time.time() - t1
    atlas = Atlas(L, D, E, cfg, n_annot=len(ds.vocab) if cfg.subsample else 0, device=dev)
    if ck is not None:
        atlas.load_state_dict(st["atlas"])
        log(f"[atlas] resumed from {ck.name}: batch {start}/{len(plan)}, n_seen {atlas.n_seen}")
    elif seeds is not None:
        atlas.seed(*seeds)
        log(f"[atlas] seeded thresholds for n_total={n_total}: reservoir bins seeded "
            f"{int((atlas.res_seed != torch.iinfo(torch.int64).min).sum())}/{atlas.res_seed.numel()}")
    attach(model, atlas.observe)
    my_plan = plan if world == 1 else plan[rank::world]

    def summary(done: bool, bi: int):
        return {"args": vars(a), "model": info, "coverage": ds.coverage(order), "n_excluded": n_excluded,
                "n_batches_plan": len(plan), "next_batch": bi, "complete": done, "world": world,
                "seconds": {"load": t_load, "pilot": t_pilot, "stream_this_process": time.time() - t2},
                "n_seen": atlas.n_seen, "stats": atlas.stats}

    logf = open(out / ("batches.jsonl" if world == 1 else f"batches.rank{rank}.jsonl"), "a")
    ckpt_s, batch_s, last_ckpt_s = 0.0, 0.0, None

    writer = CheckpointWriter(ck_dir, keep=2)

    def save_ckpt(next_batch):
        """Snapshot now, write in the background; the time on the batch loop's path is the host copy
        (plus any wait for the previous write)."""
        nonlocal ckpt_s, last_ckpt_s
        t = time.time()
        obj = {"atlas": atlas.state_dict(), "next_batch": next_batch, "args_key": _args_key(a), "model": info}
        after = None
        if rank == 0:
            sm = summary(False, next_batch)
            after = lambda: (out / "run.json").write_text(json.dumps(sm, indent=1))  # noqa: E731
        writer.save(obj, ck_dir / f"ckpt_{next_batch}.pt", after)
        last_ckpt_s = time.time() - t
        ckpt_s = max(ckpt_s, last_ckpt_s)
        log(f"[atlas] checkpoint at batch {next_batch}/{len(my_plan)} ({last_ckpt_s:.1f}s on the loop, written in the background)")

    t2 = time.time()
    n_done = 0
    paired = []  # (global batch index, atlas overhead vs the paired hook-free forward)
    # with several ranks every stop is collective (Lockstep): a rank that reaches its deadline or
    # cap stops all ranks at the same step, and ranks whose shard is exhausted wait for the others,
    # so no rank enters the combine's collectives while another still streams or has returned
    from .dist import Lockstep
    lock = Lockstep(group=ctl_group)
    STOP_CAP, STOP_DEADLINE = 1, 2

    def finish_process_group():
        if world > 1:
            torch.distributed.destroy_process_group()

    # Per-batch records are timed by CUDA events on the loop's stream and written once the events
    # have completed (a lag of up to `lag` batches), so the loop never drains the GPU to time a
    # batch; the host stays ahead and the GPU stays busy. The paired hook-free forward is timed the
    # same way.
    pending = []  # [rec, start event, atlas-pass start, atlas-pass end, paired-forward events or None]
    lag = 2

    def ev():
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def drain(keep: int):
        """Write the records of completed batches; wait for all but the last `keep`."""
        nonlocal batch_s
        while pending:
            rec, e0, ea, eb, fe = pending[0]
            if len(pending) > keep:
                eb.synchronize()
            elif not eb.query():
                break
            pending.pop(0)
            atlas_s = ea.elapsed_time(eb) / 1e3
            fwd_s = fe[0].elapsed_time(fe[1]) / 1e3 if fe is not None else None
            rec.update({"seconds": e0.elapsed_time(eb) / 1e3, "fwd_only_s": fwd_s, "atlas_pass_s": atlas_s,
                        "overhead_vs_fwd": (atlas_s / fwd_s - 1) if fwd_s else None})
            if fwd_s:
                paired.append((rec["batch"] * world + rank, atlas_s / fwd_s - 1))
            if rec["n_done"] > 2:
                batch_s = max(batch_s, rec["seconds"])
            del rec["n_done"]
            logf.write(json.dumps(rec) + "\n")
        logf.flush()

    def _stream(src_iter):
        """The batch loop; returns the agreed stop code (None after the whole plan)."""
        nonlocal n_done, batch_s, last_ckpt_s
        item = next(src_iter, None)
        bi = start
        while True:
            want = 0
            if item is not None:
                b, ctx_host = item
                tb = time.time()
                e0 = ev()
                ids, am = b.input_ids.to(dev, non_blocking=True), b.attention_mask.to(dev, non_blocking=True)
                fe = None
                if a.pair_forward or (a.pair_every and bi % a.pair_every == 0):
                    atlas.enabled = False
                    # an untimed forward first: a batch shape met for the first time makes the host
                    # plan its attention kernels, and that time belongs to neither measured pass
                    model(input_ids=ids, attention_mask=am)
                    f0 = ev()
                    model(input_ids=ids, attention_mask=am)
                    fe = (f0, ev())
                    atlas.enabled = True
                prof = None
                if bi in a.profile_at:
                    acts = [torch.profiler.ProfilerActivity.CPU]
                    if torch.device(dev).type == "cuda":
                        acts.append(torch.profiler.ProfilerActivity.CUDA)
                    prof = torch.profiler.profile(activities=acts)
                    prof.__enter__()
                if prof is not None:
                    sync(dev)
                ea = ev()
                if ctx_host is not None:
                    ctx = ctx_host.to(dev)
                elif a.host_ctx:
                    ctx = atlas.make_ctx(b.n_rows, b.valid_rows, b.tok, b.ann)
                else:
                    ctx = atlas.make_ctx_device(b.n_rows, b.valid_rows, b.tok, b.ann)
                n_before = atlas.n_seen
                atlas.begin_batch(ctx)
                model(input_ids=ids, attention_mask=am)
                redo = atlas.end_batch()
                assert redo == []
                gram_flushed = bi % a.gram_flush_every == a.gram_flush_every - 1
                if gram_flushed:
                    atlas.flush_gram()
                eb = ev()
                if prof is not None:
                    sync(dev)
                    prof.__exit__(None, None, None)
                    write_profile(prof, out / f"profile_batch_{bi}.txt", dev)
                    log(f"[atlas] profiled batch {bi} -> profile_batch_{bi}.txt")
                # seconds (start of the batch to the end of its atlas pass), fwd_only_s, atlas_pass_s
                # and overhead_vs_fwd are filled from the events by drain()
                rec = {"batch": bi, "n_seen_before": n_before, "n_valid": ctx.n_v, "rows": b.n_rows,
                       "Lmax": int(b.input_ids.shape[1]), "t_enqueue_start": tb, "t_enqueue_end": time.time(),
                       "gram_flushed": gram_flushed, "flops": flops_per_batch(info, b.n_rows, b.input_ids.shape[1]),
                       "redo_layers": [], "n_done": n_done}
                n_done += 1
                bi += 1
                last_ckpt_s = None
                if bi % a.ckpt_every == 0:
                    drain(0)
                    save_ckpt(bi)
                rec["ckpt_s"] = last_ckpt_s
                pending.append([rec, e0, ea, eb, fe])
                drain(lag)
                item = next(src_iter, None)
                if a.deadline and item is not None and \
                        time.time() > a.deadline - 2 * (batch_s + max(ckpt_s, 30.0)):
                    want = STOP_DEADLINE
                elif a.stop_after and n_done >= a.stop_after:
                    want = STOP_CAP
            code, more = lock.agree(want, item is not None)
            if code or not more:
                drain(0)
            if code == STOP_DEADLINE:
                if bi % a.ckpt_every:
                    save_ckpt(bi)
                writer.wait()
                log(f"[atlas] deadline approaching: stopped cleanly at batch {bi}; rerun with --resume")
                return code
            if code == STOP_CAP:
                log(f"[atlas] stopping after {n_done} batches (simulated cap)")
                writer.wait()
                if rank == 0:
                    (out / "run.json").write_text(json.dumps(summary(False, bi), indent=1))
                return code
            if not more:
                return None

    prefetch = None
    side = torch.cuda.Stream(device=torch.device(dev)) if not a.host_ctx else None

    def with_ctx(b):
        """The batch with its context: on the device (a side stream; the prefetch thread waits only
        for it) or, with --host-ctx, built on the host as the reference does."""
        b.input_ids = b.input_ids.pin_memory()  # the loop's copies of the batch are then asynchronous
        b.attention_mask = b.attention_mask.pin_memory()
        if a.host_ctx:
            return b, atlas.make_ctx(b.n_rows, b.valid_rows, b.tok, b.ann, device="cpu")
        return b, atlas.make_ctx_device(b.n_rows, b.valid_rows.pin_memory(), b.tok.pin_memory(),
                                        b.ann.pin_memory() if b.ann is not None else None, stream=side)

    with torch.no_grad():
        src_iter = ds.batches(vocab, order, a.tokens_per_batch, plan=my_plan, start=start)
        if a.prefetch > 0:
            prefetch = Prefetch((with_ctx(b) for b in src_iter), a.prefetch)
            src_iter = prefetch
        else:
            src_iter = iter((b, None) for b in src_iter)
        try:
            code = _stream(src_iter)
        finally:
            if prefetch is not None:
                prefetch.close()
    if code is not None:
        finish_process_group()
        return
    writer.wait()
    logf.close()
    atlas.check_errors()
    combine_s = None
    if world > 1:
        from .dist import merge_states, warm_up
        parts = [None] * world
        torch.distributed.all_gather_object(parts, paired)
        paired = [x for part in parts for x in part]
        warm_up(device=torch.device(dev))
        sync(dev)
        tc0 = time.time()
        merge_states(atlas)
        sync(dev)
        combine_s = time.time() - tc0
        log(f"[atlas] shard states of {world} ranks combined in {combine_s:.2f}s")
    if rank != 0:
        torch.distributed.destroy_process_group()
        return
    res = atlas.result()
    res.update({"model": info, "coverage": ds.coverage(order), "vocab": ds.vocab, "order_seed": a.seed,
                "n_total_plan": n_total, "n_batches": len(plan)})
    tf = time.time()
    atomic_save(res, out / "atlas.pt")
    final_s = time.time() - tf
    digests = {k: hashlib.sha256(res[k].contiguous().numpy().tobytes()).hexdigest()
               for k in ("top_val", "top_tok", "res_tok", "res_val", "res_key", "sub_bin", "enr", "ann_tot", "edges")
               if k in res}
    sm = summary(True, len(plan))
    sm.update({"overhead": overhead_summary(paired), "combine_s": combine_s,
               "dense_layer_batches": res["stats"].get("dense_layer_batches"),
               "digests": digests, "final_save_s": final_s, "gram_rows": res.get("gram_rows"),
               "res_seeded_bins": res["res_seeded_bins"], "res_seed_limited_bins": res["res_seed_limited_bins"],
               "top_seed_short_groups": res["top_seed_short_groups"]})
    (out / "run.json").write_text(json.dumps(sm, indent=1))
    log(f"[atlas] done: final save {final_s:.1f}s; seed verification: {res['res_seed_limited_bins']} of "
        f"{res['res_seeded_bins']} seeded bins short, top-K groups short {res['top_seed_short_groups']}")
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
