"""TEST INFRASTRUCTURE ONLY: Python front of the CPU oracle (j1_oracle.cpp).

Loads a checkpoint directory the way the reference does -- ModelConfig::from_values
(src/config.rs:43-96) and HostWeights::load (src/model.rs:55-110) over an F32
safetensors file -- and runs the oracle's two restatements of the forward:

  mode "fp32": the reference CPU path (src/cpu/mod.rs:201-340)
  mode "bf16": the reference CUDA path's precision chain (src/cuda/mod.rs:446-511)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this.
"""
import ctypes as C
import json
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _lib():
    from oracle import build as ob  # noqa: local build recipe
    path = ob.LIB
    if not os.path.exists(path):
        path = ob.build_oracle()
    L = C.CDLL(path)
    u32p, f32p, u8p = C.POINTER(C.c_uint32), C.POINTER(C.c_float), C.POINTER(C.c_uint8)
    L.oracle_create.argtypes = [C.c_void_p, C.POINTER(C.c_void_p), C.c_int]
    L.oracle_create.restype = C.c_void_p
    L.oracle_destroy.argtypes = [C.c_void_p]
    L.oracle_forward.argtypes = [C.c_void_p, C.c_int, u32p, C.c_size_t, u32p, u32p, u8p, C.c_size_t, u32p, u32p,
                                 C.c_size_t, f32p, C.c_void_p, C.c_int]
    L.oracle_forward.restype = C.c_int
    L.oracle_linear.argtypes = [f32p, C.c_size_t, f32p, C.c_size_t, C.c_size_t, f32p, C.c_size_t, C.c_size_t, C.c_int,
                                C.c_void_p, C.c_int]
    L.oracle_linear_geglu.argtypes = [f32p, C.c_size_t, f32p, C.c_size_t, C.c_size_t, f32p, C.c_int]
    for fn in ("oracle_exp", "oracle_erf", "oracle_gelu", "oracle_bf16"):
        getattr(L, fn).argtypes = [C.c_float]
        getattr(L, fn).restype = C.c_float
    L.oracle_has_avx512.restype = C.c_int
    return L


_L = None


def lib():
    global _L
    if _L is None:
        _L = _lib()
    return _L


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "heads", "intermediate", "layers", "half_window", "vocab",
                                       "max_positions", "head_layers")] + \
               [("norm_eps", C.c_float), ("global_", C.POINTER(C.c_int)), ("rope_theta", C.POINTER(C.c_float))]


def load_config(root):
    """ModelConfig::from_values (src/config.rs:43-96)."""
    julia = json.load(open(os.path.join(root, "julia_config.json")))
    enc = json.load(open(os.path.join(root, "encoder", "config.json")))
    assert julia["format_version"] == 1 and julia.get("weight_dtype", "float32") == "float32"
    assert enc["model_type"] == "modernbert" and enc["hidden_activation"] == "gelu"
    H, heads, L = enc["hidden_size"], enc["num_attention_heads"], enc["num_hidden_layers"]
    every, local = enc["global_attn_every_n_layers"], enc["local_attention"]
    assert H % heads == 0 and H // heads == 64
    types = enc.get("layer_types") or ["full_attention" if i % every == 0 else "sliding_attention" for i in range(L)]

    def theta(kind):
        rp = enc.get("rope_parameters", {}).get(kind)
        if rp is not None:
            return float(rp["rope_theta"])
        return float(enc["global_rope_theta" if kind == "full_attention" else "local_rope_theta"])

    return dict(hidden=H, heads=heads, intermediate=enc["intermediate_size"], layers=L,
                glob=[i % every == 0 for i in range(L)], half_window=local // 2,
                rope_theta=[theta(t) for t in types], norm_eps=float(enc.get("norm_eps", 1e-5)),
                vocab=enc["vocab_size"], max_positions=enc["max_position_embeddings"],
                head_layers=julia["head_layers"])


def read_safetensors(path):
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
        out[name] = np.ascontiguousarray(mm[8 + n + a: 8 + n + b].view("<f4").reshape(info["shape"]))
    return out


def weight_names(cfg):
    """Tensor names in HostWeights::load order (src/model.rs:55-110)."""
    names = ["encoder.embeddings.tok_embeddings.weight", "encoder.embeddings.norm.weight"]
    for l in range(cfg["layers"]):
        p = "encoder.layers.%d." % l
        if l > 0:
            names.append(p + "attn_norm.weight")
        names += [p + "attn.Wqkv.weight", p + "attn.Wo.weight", p + "mlp_norm.weight", p + "mlp.Wi.weight",
                  p + "mlp.Wo.weight"]
    names += ["encoder.final_norm.weight", "type_emb.weight"]
    for j in range(cfg["head_layers"]):
        p = "head.layers.%d." % j
        names += [p + s for s in ("norm1.weight", "norm1.bias", "self_attn.in_proj_weight", "self_attn.in_proj_bias",
                                  "self_attn.out_proj.weight", "self_attn.out_proj.bias", "norm2.weight",
                                  "norm2.bias", "linear1.weight", "linear1.bias", "linear2.weight", "linear2.bias")]
    names += ["scorer.0.weight", "scorer.0.bias", "scorer.1.weight", "scorer.1.bias", "scorer.3.weight",
              "scorer.3.bias"]
    return names


class Oracle:
    def __init__(self, root):
        self.cfg = load_config(root)
        self.tensors = read_safetensors(os.path.join(root, "model.safetensors"))
        c = self.cfg
        self._glob = (C.c_int * c["layers"])(*[1 if g else 0 for g in c["glob"]])
        self._theta = (C.c_float * c["layers"])(*c["rope_theta"])
        cfg = _Cfg(c["hidden"], c["heads"], c["intermediate"], c["layers"], c["half_window"], c["vocab"],
                   c["max_positions"], c["head_layers"], c["norm_eps"], self._glob, self._theta)
        self._arrays = [self.tensors[n] for n in weight_names(c)]
        ptrs = (C.c_void_p * len(self._arrays))(*[a.ctypes.data for a in self._arrays])
        self._h = lib().oracle_create(C.byref(cfg), ptrs, len(self._arrays))
        if not self._h:
            raise RuntimeError("oracle_create failed")

    def close(self):
        if getattr(self, "_h", None):
            lib().oracle_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward_flat(self, batch, mode="fp32", threads=0, hidden=False):
        """batch: object with ids, starts, lens, qtypes, marker_rows, marker_starts (numpy)."""
        arrs = [np.ascontiguousarray(getattr(batch, k), dtype=dt) for k, dt in
                (("ids", np.uint32), ("starts", np.uint32), ("lens", np.uint32), ("qtypes", np.uint8),
                 ("marker_rows", np.uint32), ("marker_starts", np.uint32))]
        ids, starts, lens, qt, mr, ms = arrs
        scores = np.zeros(mr.size, np.float32)
        hid = np.zeros((ids.size, self.cfg["hidden"]), np.float32) if hidden else None
        P = lambda a, t: a.ctypes.data_as(C.POINTER(t))  # noqa: E731
        rc = lib().oracle_forward(self._h, 0 if mode == "fp32" else 1, P(ids, C.c_uint32), ids.size,
                                  P(starts, C.c_uint32), P(lens, C.c_uint32), P(qt, C.c_uint8), lens.size,
                                  P(mr, C.c_uint32), P(ms, C.c_uint32), mr.size, P(scores, C.c_float),
                                  hid.ctypes.data if hidden else None, int(threads))
        assert rc == 0
        return (scores, hid) if hidden else scores


def linear(x, w, epi=0, bias=None, out=None, col=0, threads=0):
    """gemm.rs `linear` (epilogue 0..4 = Store, Add, Bias, BiasRelu, AddBias)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    rows, k = x.shape
    n = w.shape[0]
    if out is None:
        out = np.zeros((rows, n), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    P = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
    lib().oracle_linear(P(x), rows, P(w), n, k, P(out), out.shape[1], col, epi,
                        None if b is None else b.ctypes.data, threads)
    return out


def linear_geglu(x, w, threads=0):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    rows, k = x.shape
    g = np.zeros((rows, w.shape[0] // 2), np.float32)
    P = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
    lib().oracle_linear_geglu(P(x), rows, P(w), w.shape[0], k, P(g), threads)
    return g
