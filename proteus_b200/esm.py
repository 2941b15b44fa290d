"""ESM-2 models and the forward hooks that feed the atlas — drop-in for haelyons/proteus
atlas/esm.py.

Hook point (esm.py:52-63 of the reference): encoder.layer[i].intermediate.dense output, the
pre-GELU FFN activation [B, L, d_ff], handed to the sink flattened to [B*L, d_ff] — a view of
the live activation, consumed by the sink's kernels on the current stream before the forward
moves on.

Weights: this build has no network, so `load` builds the architecture from its published
configuration with a seeded random init (the reference's `control="random"`), unless a local
HuggingFace checkpoint directory is given.
"""
from __future__ import annotations

import os

import torch

# name -> (layers, d_model, d_ff, heads)
ARCH = {
    "8M": (6, 320, 1280, 20),
    "35M": (12, 480, 1920, 20),
    "150M": (30, 640, 2560, 20),
    "650M": (33, 1280, 5120, 20),
    "3B": (36, 2560, 10240, 40),
}
MODELS = {"8M": "facebook/esm2_t6_8M_UR50D", "35M": "facebook/esm2_t12_35M_UR50D",
          "150M": "facebook/esm2_t30_150M_UR50D", "650M": "facebook/esm2_t33_650M_UR50D",
          "3B": "facebook/esm2_t36_3B_UR50D"}

# ESM-2 alphabet: specials, residues in the model's order, then the rest (33 tokens)
ESM_TOKENS = ["<cls>", "<pad>", "<eos>", "<unk>", "L", "A", "G", "V", "S", "E", "R", "T", "I", "D", "P", "K", "Q",
              "N", "F", "Y", "M", "H", "W", "C", "X", "B", "U", "Z", "O", ".", "-", "<null_1>", "<mask>"]


class Vocab:
    """The tokenizer surface the batcher needs (get_vocab)."""

    def __init__(self):
        self._v = {t: i for i, t in enumerate(ESM_TOKENS)}

    def get_vocab(self) -> dict:
        return dict(self._v)


def esm_config(name: str):
    from transformers import EsmConfig
    L, d, ff, heads = ARCH[name]
    return EsmConfig(vocab_size=33, hidden_size=d, num_hidden_layers=L, num_attention_heads=heads,
                     intermediate_size=ff, max_position_embeddings=1026, position_embedding_type="rotary",
                     pad_token_id=1, mask_token_id=32, token_dropout=True, emb_layer_norm_before=False,
                     layer_norm_eps=1e-5, hidden_act="gelu", hidden_dropout_prob=0.0,
                     attention_probs_dropout_prob=0.0)


def load(name: str, control: str = "none", dtype=torch.bfloat16, device="cpu", seed: int = 0):
    """Returns (model, tokenizer-like vocab, info) as the reference's load() (esm.py:21-49)."""
    from transformers import EsmModel
    local = name if os.path.isdir(str(name)) else None
    if local:
        model = EsmModel.from_pretrained(local, add_pooling_layer=False, attn_implementation="sdpa")
        arch = os.path.basename(local)
    else:
        if name not in ARCH:
            raise ValueError(f"unknown model {name!r} (known: {sorted(ARCH)})")
        torch.manual_seed(seed)
        cfg = esm_config(name)
        cfg._attn_implementation = "sdpa"
        dev = torch.device(device)
        with torch.device(dev):  # initialise on the target device (seconds instead of minutes for 650M+)
            model = EsmModel(cfg, add_pooling_layer=False)
        arch = MODELS.get(name, name)
    if control == "shuffled":
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for _, p in model.named_parameters():
                flat = p.data.view(-1)
                flat.copy_(flat[torch.randperm(flat.numel(), generator=g).to(flat.device)])
    elif control not in ("none", "random"):
        raise ValueError(control)
    model = model.to(device=device, dtype=dtype).eval()
    info = {"hf": arch, "control": control if local else "random",
            "attn": getattr(model.config, "_attn_implementation", "eager"),
            "n_layers": model.config.num_hidden_layers, "d_model": model.config.hidden_size,
            "d_ff": model.config.intermediate_size, "n_params": sum(p.numel() for p in model.parameters())}
    return model, Vocab(), info


def ffn_modules(model):
    return [layer.intermediate.dense for layer in model.encoder.layer]


def attach(model, sink):
    """sink(l, H[B*L, d_ff]) from each FFN pre-activation hook; returns the hook handles."""
    handles = []
    for i, mod in enumerate(ffn_modules(model)):
        def hook(_m, _inp, out, i=i):
            sink(i, out.reshape(-1, out.shape[-1]))
        handles.append(mod.register_forward_hook(hook))
    return handles


def flops_per_batch(info: dict, n_rows: int, Lmax: int) -> float:
    """Dense matmul FLOPs of one forward over n_rows padded positions (esm.py:66-70 convention)."""
    d, f, L = info["d_model"], info["d_ff"], info["n_layers"]
    return n_rows * L * (2 * (4 * d * d + 2 * d * f) + 4 * Lmax * d)


@torch.no_grad()
def pilot(model, batches, device, max_tokens: int, store_device="cpu", layers=None):
    """Valid-token FFN activations per layer from the first batches -> list[[N, d_ff]] (esm.py:73-98).
    `layers` restricts the capture to a subset (the others are returned as None), which bounds the
    memory of large pilots."""
    L = model.config.num_hidden_layers
    keep = set(range(L)) if layers is None else set(layers)
    bufs = [[] for _ in range(L)]
    cur = {}

    def sink(l, H):
        if l in keep:
            bufs[l].append(H.index_select(0, cur["rows"]).to(store_device))

    hs = attach(model, sink)
    n = 0
    toks = []
    try:
        for b in batches:
            cur["rows"] = b.valid_rows.to(device)
            model(input_ids=b.input_ids.to(device), attention_mask=b.attention_mask.to(device))
            n += b.valid_rows.numel()
            toks.append(b.tok)
            if n >= max_tokens:
                break
    finally:
        for h in hs:
            h.remove()
    pilot.last_tok = torch.cat(toks) if toks else torch.zeros(0, dtype=torch.long)
    return [torch.cat(x) if x else None for x in bufs], n
