"""BASELINE config 0 (the exactness case): ESM-2 8M architecture, random init seed 0, 512 synthetic
sequences (residues i.i.d. uniform over the 20 standard amino acids, lengths uniform 30-400),
pilot = the first 64 of them, K=16, Kr=8, 5 bins at pilot quantiles, reference rho defaults,
tok = seq*1024 + pos.

Shared by tests/golden/make_golden.py (which feeds the reference's Atlas) and the tests (which feed
the oracle on CPU and the CUDA product on the GPU from the same forward). The model is built from a
hand-written config because no pretrained weights are reachable offline; only consistency between
the arms matters.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

C1 = dict(L=6, D=1280, K=16, Kr=8, n_seq=512, n_pilot=64, lmin=30, lmax=400, n_annot=21,
          tokens_per_batch=8192, seed=0)

# ESM-2 alphabet (33 tokens): specials, then residues in the model's own order
ESM_TOKENS = ["<cls>", "<pad>", "<eos>", "<unk>", "L", "A", "G", "V", "S", "E", "R", "T", "I", "D", "P", "K", "Q",
              "N", "F", "Y", "M", "H", "W", "C", "X", "B", "U", "Z", "O", ".", "-", "<null_1>", "<mask>"]
ESM_ID = {t: i for i, t in enumerate(ESM_TOKENS)}
AA = "ACDEFGHIKLMNPQRSTVWY"


@dataclass
class C1Batch:
    input_ids: torch.Tensor
    attention_mask: torch.Tensor
    T: int
    valid_rows: np.ndarray
    tok: np.ndarray
    ann: np.ndarray


def c1_sequences() -> list:
    rng = np.random.default_rng(C1["seed"])
    lens = rng.integers(C1["lmin"], C1["lmax"] + 1, C1["n_seq"])
    return ["".join(AA[i] for i in rng.integers(0, 20, int(n))) for n in lens]


def esm_config(L=6, d=320, ff=1280, heads=20):
    from transformers import EsmConfig
    return EsmConfig(vocab_size=33, hidden_size=d, num_hidden_layers=L, num_attention_heads=heads,
                     intermediate_size=ff, max_position_embeddings=1026, position_embedding_type="rotary",
                     pad_token_id=1, mask_token_id=32, token_dropout=True, emb_layer_norm_before=False,
                     layer_norm_eps=1e-5, hidden_act="gelu", hidden_dropout_prob=0.0,
                     attention_probs_dropout_prob=0.0)


def build_model(device="cpu", dtype=torch.float32):
    from transformers import EsmModel
    torch.manual_seed(C1["seed"])
    m = EsmModel(esm_config(), add_pooling_layer=False)
    return m.to(device=device, dtype=dtype).eval()


def c1_batches(seqs: list, idx: list):
    """Greedy padded batches in the given order: rows r*Lmax + 1 + pos, <= tokens_per_batch rows."""
    cur = []
    groups = []
    for i in idx:
        n = len(seqs[i]) + 2
        m = max([len(seqs[j]) + 2 for j in cur] + [n])
        if cur and m * (len(cur) + 1) > C1["tokens_per_batch"]:
            groups.append(cur)
            cur = []
        cur.append(i)
    if cur:
        groups.append(cur)
    for grp in groups:
        Lmax = max(len(seqs[i]) for i in grp) + 2
        B = len(grp)
        ids = torch.full((B, Lmax), ESM_ID["<pad>"], dtype=torch.long)
        am = torch.zeros((B, Lmax), dtype=torch.long)
        rows, toks, anns = [], [], []
        for r, i in enumerate(grp):
            s = seqs[i]
            n = len(s)
            ids[r, 0] = ESM_ID["<cls>"]
            ids[r, 1:n + 1] = torch.tensor([ESM_ID[c] for c in s])
            ids[r, n + 1] = ESM_ID["<eos>"]
            am[r, :n + 2] = 1
            rows.append(r * Lmax + 1 + np.arange(n))
            toks.append(np.int64(i) * 1024 + np.arange(n, dtype=np.int64))
            anns.append(np.array([AA.index(c) for c in s], np.int64)[:, None])
        yield C1Batch(ids, am, B * Lmax, np.concatenate(rows).astype(np.int64), np.concatenate(toks),
                      np.concatenate(anns))


@torch.no_grad()
def forward_layers(model, b: C1Batch, device="cpu", keep_device=False):
    """Run the forward and return every layer's pre-GELU FFN output [B*Lmax, d_ff] (fp32 numpy,
    or device tensors in the model dtype with keep_device=True)."""
    outs = []
    hs = [layer.intermediate.dense.register_forward_hook(
        lambda _m, _i, o: outs.append(o.reshape(-1, o.shape[-1]) if keep_device else
                                      o.reshape(-1, o.shape[-1]).float().cpu().numpy()))
        for layer in model.encoder.layer]
    try:
        model(input_ids=b.input_ids.to(device), attention_mask=b.attention_mask.to(device))
    finally:
        for h in hs:
            h.remove()
    return outs
