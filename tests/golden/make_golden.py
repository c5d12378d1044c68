"""Generate golden logits for the oracle from an independent FP32 implementation.

The reference julia1-rs reports its FP32 CPU path matching the upstream Python
runtime (README.md:158), which runs HF transformers' ModernBertModel as the
encoder, `nn.TransformerEncoderLayer(norm_first=True, activation="relu")` layers
as the decision head (src/model.rs:16-30) and `Sequential(LayerNorm, Linear, GELU,
Linear)` as the scorer (src/model.rs:32-40). This script rebuilds that model in
PyTorch FP32 on CPU, loads a tiny seeded synthetic checkpoint written in the
reference's layout, and stores inputs + logits (+ encoder hidden states) as
fixtures. The checkpoint itself is regenerated from its seed by the tests.

Run: python tests/golden/make_golden.py   (CPU only, a few seconds)
"""
import os
import sys
import tempfile

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "julia1-rs_b200"))
from julia1 import synthetic  # noqa: E402

CASES = {
    # name: (checkpoint shape, seed, sequence lengths, markers per sequence, qtypes)
    "tiny": (dict(hidden=128, heads=2, layers=4, intermediate=256, vocab=1000, max_positions=512, head_layers=2),
             7, [150, 37, 300, 1, 2], 4, [0, 1, 2, 0, 1]),
    "j384": (dict(hidden=384, heads=6, layers=5, intermediate=1152, vocab=2000, max_positions=1024, head_layers=1),
             11, [260, 129, 64], 3, [2, 0, 1]),
}


def build_model(shape, tensors):
    from transformers import ModernBertConfig, ModernBertModel
    H = shape["hidden"]
    cfg = ModernBertConfig(vocab_size=shape["vocab"], hidden_size=H, intermediate_size=shape["intermediate"],
                           num_hidden_layers=shape["layers"], num_attention_heads=shape["heads"],
                           global_attn_every_n_layers=3, local_attention=128, global_rope_theta=160000.0,
                           local_rope_theta=10000.0, max_position_embeddings=shape["max_positions"], norm_eps=1e-5,
                           norm_bias=False, attention_bias=False, mlp_bias=False, hidden_activation="gelu",
                           embedding_dropout=0.0, attention_dropout=0.0, mlp_dropout=0.0,
                           attn_implementation="eager", pad_token_id=0)
    enc = ModernBertModel(cfg).eval()
    sd = {k[len("encoder."):]: torch.tensor(np.array(v)) for k, v in tensors.items() if k.startswith("encoder.")}
    missing, unexpected = enc.load_state_dict(sd, strict=False)
    assert not unexpected and all("attn_norm" in m or "rotary" in m for m in missing), (missing, unexpected)
    head = torch.nn.ModuleList([torch.nn.TransformerEncoderLayer(H, H // 64, 4 * H, dropout=0.0, activation="relu",
                                                                 norm_first=True, batch_first=True)
                                for _ in range(shape["head_layers"])]).eval()
    head.load_state_dict({k[len("head.layers."):]: torch.tensor(np.array(v)) for k, v in tensors.items()
                          if k.startswith("head.layers.")})
    scorer = torch.nn.Sequential(torch.nn.LayerNorm(H), torch.nn.Linear(H, H), torch.nn.GELU(),
                                 torch.nn.Linear(H, 1)).eval()
    scorer.load_state_dict({k[len("scorer."):]: torch.tensor(np.array(v)) for k, v in tensors.items()
                            if k.startswith("scorer.")})
    type_emb = torch.tensor(np.array(tensors["type_emb.weight"]))
    return enc, head, scorer, type_emb


@torch.no_grad()
def run(shape, tensors, rows):
    enc, head, scorer, type_emb = build_model(shape, tensors)
    logits, hidden = [], []
    for ids, markers, qtype in rows:
        ii = torch.tensor(ids.astype(np.int64))[None]
        h = enc(input_ids=ii, attention_mask=torch.ones_like(ii)).last_hidden_state  # final_norm applied
        hidden.append(h[0].numpy())
        x = h + type_emb[qtype]
        for layer in head:
            x = layer(x)
        y = x[0, torch.tensor(markers.astype(np.int64))]
        logits.append(scorer(y)[:, 0].numpy())
    return logits, hidden


def main():
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    out_dir = os.path.dirname(os.path.abspath(__file__))
    for name, (shape, seed, lens, nmk, qtypes) in CASES.items():
        with tempfile.TemporaryDirectory() as td:
            root = synthetic.write_checkpoint(td, seed=seed, perturb=True, **shape)
            tensors = synthetic.read_safetensors(os.path.join(root, "model.safetensors"))
            rows = synthetic.synthetic_batch(lens, vocab=shape["vocab"], markers_per_seq=nmk, seed=seed + 1,
                                              mask_markers=False)
            rows = [(ids, mk, q) for (ids, mk, _), q in zip(rows, qtypes)]
            logits, hidden = run(shape, tensors, rows)
        np.savez_compressed(os.path.join(out_dir, "%s_fp32.npz" % name),
                            seed=seed, lens=np.array(lens), qtypes=np.array(qtypes), markers_per_seq=nmk,
                            shape=np.array([shape[k] for k in sorted(shape)]), shape_keys=np.array(sorted(shape)),
                            ids=np.concatenate([r[0] for r in rows]),
                            markers=np.concatenate([r[1] for r in rows]),
                            row_markers=np.array([len(r[1]) for r in rows]),
                            logits=np.concatenate(logits).astype(np.float32),
                            hidden=np.concatenate(hidden).astype(np.float32)[::7])  # every 7th row, keeps it small
        print(name, "ok", [l.round(4).tolist() for l in logits][:2])


if __name__ == "__main__":
    main()
