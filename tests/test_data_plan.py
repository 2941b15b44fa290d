"""The batch plan, pilot plan, coverage report and batch tensors of proteus_b200.data equal the
reference's own (tests/golden/data_plan.npz, made by the reference's atlas/data.py SwissProt on
tests/golden/make_golden.py:data_case()): a checkpoint's next-batch index must name the same batch
in both builds, and the hooks must see the same rows, token ids and annotations."""
from __future__ import annotations

import io

import numpy as np
import torch

from tests.c1 import ESM_TOKENS
from tests.golden.make_golden import DATA_CASE, DATA_X_GROUP, data_case
from tests.harness import golden


def _dataset(from_bytes: bool):
    from proteus_b200.data import SwissProt
    d = data_case()
    if not from_bytes:
        return SwissProt(d)
    buf = io.BytesIO()
    torch.save(d, buf)
    buf.seek(0)
    return SwissProt(buf)


def _plan_arrays(plan):
    return np.array([i for g in plan for i in g], np.int64), np.array([len(g) for g in plan], np.int64)


def test_plans_and_batches_equal_the_reference():
    from proteus_b200.data import shuffled_order
    z = golden("data_plan")
    c = DATA_CASE
    ds = _dataset(from_bytes=True)
    order = shuffled_order(len(ds), c["seed"])
    assert np.array_equal(order.numpy(), z["order"])
    plans = {"shuffled": ds.plan(order, c["tokens_per_batch"], c["window"], c["seed"]),
             "sorted": ds.plan(order, c["tokens_per_batch"], c["window"], c["seed"], shuffle_batches=False)}
    plans["pilot"] = ds.pilot_plan(plans["shuffled"], c["pilot_tokens"], c["tokens_per_batch"], c["seed"])
    for name, pl in plans.items():
        flat, sizes = _plan_arrays(pl)
        assert np.array_equal(flat, z[f"plan_{name}_flat"]), name
        assert np.array_equal(sizes, z[f"plan_{name}_sizes"]), name
    cov = ds.coverage(order[:500])
    for k, v in cov.items():
        assert np.array_equal(np.array(v), z[f"cov_{k}"]), k
    vocab = {t: i for i, t in enumerate(ESM_TOKENS)}
    groups = {bi: plans["shuffled"][bi] for bi in c["batches"]}
    groups["x"] = DATA_X_GROUP
    for bi, grp in groups.items():
        b = ds.make_batch(grp, vocab)
        for k in ("input_ids", "attention_mask", "valid_rows", "tok", "ann", "seq_idx"):
            got = getattr(b, k).numpy()
            assert got.dtype == np.int64 and np.array_equal(got, z[f"b{bi}_{k}"]), (bi, k)
        assert b.n_rows == int(z[f"b{bi}_n_rows"])
    assert ds.ann_dropped == int(z["ann_dropped"]) > 0


def test_batches_generator_and_dict_input():
    """batches() yields make_batch of the plan from `start`; a dict loads like a file."""
    from proteus_b200.data import shuffled_order
    c = DATA_CASE
    a, b = _dataset(False), _dataset(True)
    order = shuffled_order(len(a), c["seed"])
    vocab = {t: i for i, t in enumerate(ESM_TOKENS)}
    plan = a.plan(order, c["tokens_per_batch"], c["window"], c["seed"])
    got = list(a.batches(vocab, order, c["tokens_per_batch"], chunk=c["window"], seed=c["seed"], start=len(plan) - 2))
    assert len(got) == 2
    want = b.make_batch(plan[-1], vocab)
    assert torch.equal(got[-1].input_ids, want.input_ids) and torch.equal(got[-1].ann, want.ann)
