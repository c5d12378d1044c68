"""Seeded synthetic Julia-1 checkpoints in the reference's on-disk layout.

There is no real Julia-1 checkpoint on this machine, so tests and benchmarks
run on random weights written exactly where the reference reads them:
`julia_config.json`, `encoder/config.json` (keys required by ModelConfig::from_values,
src/config.rs:43-96) and an F32 `model.safetensors` with the tensor names and
shapes of HostWeights::load (src/model.rs:55-110).

Linear and embedding weights are N(0, std) (std 0.02). LayerNorm weights are 1
and biases 0, as the benchmark configuration asks; `perturb=True` instead draws
LayerNorm weights 1 + N(0, 0.1) and biases N(0, 0.02), so parity tests exercise
every bias and gain path.
"""
import hashlib
import json
import os
import struct

import numpy as np

# ModernBERT-base shape used by every benchmark configuration.
BASE = dict(hidden=768, heads=12, layers=22, intermediate=1152, vocab=50368, max_positions=8192, head_layers=2,
            local_attention=128, global_every=3, global_theta=160000.0, local_theta=10000.0)


def tensor_specs(hidden, layers, intermediate, vocab, head_layers):
    """(name, shape, kind) in the order HostWeights::load reads them. kind: w (linear/emb), g (LN gain), b (bias)."""
    H, I, FF = hidden, intermediate, 4 * hidden
    out = [("encoder.embeddings.tok_embeddings.weight", (vocab, H), "w"), ("encoder.embeddings.norm.weight", (H,), "g")]
    for l in range(layers):
        p = "encoder.layers.%d." % l
        if l > 0:
            out.append((p + "attn_norm.weight", (H,), "g"))
        out += [(p + "attn.Wqkv.weight", (3 * H, H), "w"), (p + "attn.Wo.weight", (H, H), "w"),
                (p + "mlp_norm.weight", (H,), "g"), (p + "mlp.Wi.weight", (2 * I, H), "w"),
                (p + "mlp.Wo.weight", (H, I), "w")]
    out += [("encoder.final_norm.weight", (H,), "g"), ("type_emb.weight", (3, H), "w")]
    for j in range(head_layers):
        p = "head.layers.%d." % j
        out += [(p + "norm1.weight", (H,), "g"), (p + "norm1.bias", (H,), "b"),
                (p + "self_attn.in_proj_weight", (3 * H, H), "w"), (p + "self_attn.in_proj_bias", (3 * H,), "b"),
                (p + "self_attn.out_proj.weight", (H, H), "w"), (p + "self_attn.out_proj.bias", (H,), "b"),
                (p + "norm2.weight", (H,), "g"), (p + "norm2.bias", (H,), "b"),
                (p + "linear1.weight", (FF, H), "w"), (p + "linear1.bias", (FF,), "b"),
                (p + "linear2.weight", (H, FF), "w"), (p + "linear2.bias", (H,), "b")]
    out += [("scorer.0.weight", (H,), "g"), ("scorer.0.bias", (H,), "b"), ("scorer.1.weight", (H, H), "w"),
            ("scorer.1.bias", (H,), "b"), ("scorer.3.weight", (1, H), "w"), ("scorer.3.bias", (1,), "b")]
    return out


def configs(hidden, heads, layers, intermediate, vocab, max_positions, head_layers, local_attention, global_every,
            global_theta, local_theta):
    julia = {"format_version": 1, "weight_dtype": "float32", "head_layers": head_layers}
    enc = {"model_type": "modernbert", "hidden_size": hidden, "num_attention_heads": heads,
           "num_hidden_layers": layers, "intermediate_size": intermediate,
           "global_attn_every_n_layers": global_every, "local_attention": local_attention,
           "global_rope_theta": global_theta, "local_rope_theta": local_theta, "attention_bias": False,
           "mlp_bias": False, "norm_bias": False, "hidden_activation": "gelu", "vocab_size": vocab,
           "max_position_embeddings": max_positions, "norm_eps": 1e-5}
    return julia, enc


def write_checkpoint(root, seed=0, std=0.02, perturb=False, **shape):
    """Write a checkpoint directory; returns its path. Deterministic in (shape, seed, std, perturb)."""
    p = dict(BASE)
    p.update(shape)
    os.makedirs(os.path.join(root, "encoder"), exist_ok=True)
    julia, enc = configs(**p)
    with open(os.path.join(root, "julia_config.json"), "w") as f:
        json.dump(julia, f)
    with open(os.path.join(root, "encoder", "config.json"), "w") as f:
        json.dump(enc, f)
    specs = tensor_specs(p["hidden"], p["layers"], p["intermediate"], p["vocab"], p["head_layers"])
    header, off = {}, 0
    for name, shp, _ in specs:
        n = int(np.prod(shp)) * 4
        header[name] = {"dtype": "F32", "shape": list(shp), "data_offsets": [off, off + n]}
        off += n
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    rng = np.random.default_rng(seed)
    tmp = os.path.join(root, "model.safetensors.part")
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name, shp, kind in specs:
            if kind == "w":
                a = rng.standard_normal(shp, dtype=np.float32) * np.float32(std)
            elif kind == "g":
                a = (np.float32(1.0) + rng.standard_normal(shp, dtype=np.float32) * np.float32(0.1)) if perturb \
                    else np.ones(shp, np.float32)
            else:
                a = rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02) if perturb \
                    else np.zeros(shp, np.float32)
            f.write(np.ascontiguousarray(a, dtype="<f4").tobytes())
    os.replace(tmp, os.path.join(root, "model.safetensors"))
    return root


def cached_checkpoint(seed=0, std=0.02, perturb=False, base_dir=None, **shape):
    """write_checkpoint into a directory keyed by its parameters (reused when complete)."""
    p = dict(BASE)
    p.update(shape)
    key = json.dumps([sorted(p.items()), seed, std, perturb]).encode()
    tag = hashlib.sha1(key).hexdigest()[:12]
    base = base_dir or os.environ.get("J1_CKPT_CACHE", "/tmp/j1_ckpt")
    root = os.path.join(base, tag)
    if not os.path.exists(os.path.join(root, "model.safetensors")):
        write_checkpoint(root, seed=seed, std=std, perturb=perturb, **p)
    return root


def read_safetensors(path):
    """Minimal F32 safetensors reader -> {name: np.ndarray} (memory-mapped, read-only)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        assert info["dtype"] == "F32", name
        a, b = info["data_offsets"]
        out[name] = mm[8 + n + a: 8 + n + b].view("<f4").reshape(info["shape"])
    return out


def synthetic_batch(lens, vocab=50368, markers_per_seq=4, seed=1, cls_id=1, sep_id=2, mask_id=4, qtype=0,
                    option_block=None, mask_markers=True):
    """Encoded rows (ids, marker positions, qtype) with ids ~ U[5, vocab).

    Position 0 is CLS and the last position SEP. With option_block=None each row
    carries `markers_per_seq` MASK markers at early positions 1, 3, 5, ...;
    option_block=(n_options, tokens_per_option, head_tokens) instead lays the row out as
    [CLS] head [SEP] n x ([MASK] + option tokens) [SEP] state ... [SEP]
    (the marker serialization of the reference's Encoder::sequence).
    With mask_markers=False the marker positions keep their random ids: with random
    weights, MASK markers give nearly tied logits, random ids spread them apart.
    """
    rng = np.random.default_rng(seed)
    rows = []
    for L in lens:
        ids = rng.integers(5, vocab, size=L, dtype=np.int64).astype(np.uint32)
        ids[0] = cls_id
        ids[-1] = sep_id
        if option_block is None:
            k = min(markers_per_seq, max(0, (L - 2 + 1) // 2))
            mk = np.array([1 + 2 * i for i in range(k)], dtype=np.uint32)
        else:
            nopt, per, head = option_block
            ids[1 + head] = sep_id
            pos = 2 + head
            mk = []
            for _ in range(nopt):
                if pos >= L - 1:
                    break
                mk.append(pos)
                pos += 1 + per
            mk = np.array(mk, dtype=np.uint32)
            if pos < L - 1:
                ids[pos] = sep_id
        if mask_markers:
            ids[mk] = mask_id
        rows.append((ids, mk, qtype))
    return rows
