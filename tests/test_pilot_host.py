"""Host-side pieces that need no GPU: the oracle's pilot edges / seeds against the reference's
outputs, the dataset batcher, token keys, and the ESM hook plumbing on a tiny CPU model."""
from __future__ import annotations

import numpy as np
import torch

from tests.harness import golden
from tests.streams import pilot_inputs


def test_oracle_pilot_edges_and_seeds_match_reference():
    """The oracle's pilot math (the checker of the device pilot) against the reference's own
    pilot_edges / pilot_seeds outputs, with and without protein groups."""
    from oracle import atlas_np as O
    Hs, groups = pilot_inputs()
    z = golden("pilot")
    E = O.pilot_edges(Hs)
    assert np.array_equal(E, z["E"])
    ts, rk = O.pilot_seeds(Hs, E, 16, 8, n_total=10**6, groups=groups)
    assert np.array_equal(ts, z["top_seed"]) and np.array_equal(rk, z["res_seed_key"])
    ts0, rk0 = O.pilot_seeds(Hs, E, 16, 8, n_total=10**6)
    assert np.array_equal(ts0, z["top_seed_nogroups"]) and np.array_equal(rk0, z["res_seed_key_nogroups"])


def test_token_keys_and_top_key_match_reference():
    from proteus_b200.core import token_keys, top_key
    z = golden("keys")
    for seed in (0, 7, 0x1_0000_0005):
        assert np.array_equal(token_keys(torch.from_numpy(z["tok"]), seed).numpy(), z[f"keys_seed{seed}"])
    assert np.array_equal(top_key(torch.from_numpy(z["s"]), torch.from_numpy(z["s_tok"])).numpy(), z["top_key"])


def test_synthetic_dataset_and_plan():
    from proteus_b200.data import SwissProt, shuffled_order, synthetic_dataset
    from proteus_b200.esm import Vocab
    d = synthetic_dataset(3000, seed=1)
    L = d["len"].numpy()
    assert L.max() <= 1022 and abs(np.median(L) - 300) < 25
    assert 0 < int(d["low_complexity"].sum()) < 60
    ds = SwissProt(d)
    order = shuffled_order(len(ds), 0)
    plan = ds.plan(order, 32768)
    assert sorted(i for g in plan for i in g) == list(range(3000))
    b = next(ds.batches(Vocab().get_vocab(), order, 32768, plan=plan))
    assert b.n_rows <= 32768 and b.valid_rows.numel() == b.tok.numel() == b.ann.shape[0]
    Lmax = b.input_ids.shape[1]
    assert bool((b.attention_mask.view(-1)[b.valid_rows] == 1).all())
    assert bool(((b.valid_rows % Lmax) >= 1).all())
    assert int(b.ann[:, 0].max()) <= 20


def test_hooks_feed_ffn_preactivation():
    from proteus_b200.esm import attach, load
    model, _, info = load("8M", dtype=torch.float32, device="cpu")
    seen = {}
    hs = attach(model, lambda l, H: seen.__setitem__(l, H.shape))
    ids = torch.randint(4, 24, (2, 10))
    model(input_ids=ids, attention_mask=torch.ones_like(ids))
    for h in hs:
        h.remove()
    assert len(seen) == info["n_layers"] == 6 and all(s == (20, 1280) for s in seen.values())
