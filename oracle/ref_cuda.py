"""TEST INFRASTRUCTURE ONLY: the reference's own CUDA BF16 path, run on this GPU.

Loads oracle/_ref/kernels.cubin -- src/cuda/kernels.cu of julia1-rs compiled
unmodified for sm_100a by oracle/build.py -- and replays CudaModel::forward
(src/cuda/mod.rs:400-520) launch for launch. The reference's GEMMs are cuBLAS
`cublasGemmEx` calls with BF16 operands and COMPUTE_32F (src/cuda/mod.rs:347-375);
here the same cuBLAS library is reached through torch: `a @ w.T` on bf16 tensors
(BF16 out) and `torch.mm(..., out_dtype=torch.float32)` (FP32 out).

The reference kernels are specialized for hidden 384 (kernels.cu:8), so this
driver refuses other widths, as CudaModel::new does (src/cuda/mod.rs:175).
"""
import ctypes as C
import os

import numpy as np

from oracle import build as ob
from oracle import oracle as orc

_cuda = None


def _driver():
    global _cuda
    if _cuda is None:
        _cuda = C.CDLL("libcuda.so.1")
        _cuda.cuModuleLoadData.argtypes = [C.POINTER(C.c_void_p), C.c_void_p]
        _cuda.cuModuleGetFunction.argtypes = [C.POINTER(C.c_void_p), C.c_void_p, C.c_char_p]
        _cuda.cuLaunchKernel.argtypes = [C.c_void_p] + [C.c_uint] * 7 + [C.c_void_p, C.POINTER(C.c_void_p),
                                                                           C.c_void_p]
    return _cuda


def _check(r, what):
    if r != 0:
        raise RuntimeError("%s failed: CUresult %d" % (what, r))


class RefCudaModel:
    """CudaModel of the reference, driven from Python over its own compiled kernels."""

    NAMES = ("embed_ln", "ln_bf16", "final_norm", "geglu", "bias_act", "gather_rows", "scorer", "attention_rope",
             "attention_plain")

    def __init__(self, root, torch):
        self.torch = torch
        cubin = ob.CUBIN
        if not os.path.exists(cubin):
            raise FileNotFoundError("reference kernels not built: " + cubin)
        cfg = orc.load_config(root)
        if cfg["hidden"] != 384:
            raise ValueError("CUDA kernels are specialized for hidden 384 / head_dim 64")
        self.cfg = cfg
        torch.cuda.init()
        torch.zeros(1, device="cuda")  # primary context current on this thread
        D = _driver()
        data = open(cubin, "rb").read()
        self._image = C.create_string_buffer(data, len(data))
        mod = C.c_void_p()
        _check(D.cuModuleLoadData(C.byref(mod), C.cast(self._image, C.c_void_p)), "cuModuleLoadData")
        self._mod = mod
        self.fn = {}
        for n in self.NAMES:
            f = C.c_void_p()
            _check(D.cuModuleGetFunction(C.byref(f), mod, n.encode()), "cuModuleGetFunction " + n)
            self.fn[n] = f
        T = orc.read_safetensors(os.path.join(root, "model.safetensors"))
        dev = lambda a, dt: torch.tensor(np.array(a), device="cuda").to(dt).contiguous()  # noqa: E731
        f32, b16 = torch.float32, torch.bfloat16
        H, L = cfg["hidden"], cfg["layers"]
        self.emb = dev(T["encoder.embeddings.tok_embeddings.weight"], f32)
        self.emb_norm = dev(T["encoder.embeddings.norm.weight"], f32)
        self.layers = []
        ropes = {}
        for l in range(L):
            p = "encoder.layers.%d." % l
            theta = cfg["rope_theta"][l]
            if theta not in ropes:
                inv = (1.0 / np.power(np.float32(theta), np.arange(0, 64, 2, dtype=np.float32) / np.float32(64)))
                inv = inv.astype(np.float32)
                f = np.arange(cfg["max_positions"], dtype=np.float32)[:, None] * inv[None, :]
                ropes[theta] = (dev(np.cos(f), f32), dev(np.sin(f), f32))
            self.layers.append(dict(
                attn_norm=dev(T[p + "attn_norm.weight"], f32) if l > 0 else None,
                wqkv=dev(T[p + "attn.Wqkv.weight"], b16), wo=dev(T[p + "attn.Wo.weight"], b16),
                mlp_norm=dev(T[p + "mlp_norm.weight"], f32), wi=dev(T[p + "mlp.Wi.weight"], b16),
                wo2=dev(T[p + "mlp.Wo.weight"], b16), rope=ropes[theta], glob=cfg["glob"][l]))
        self.final_norm = dev(T["encoder.final_norm.weight"], f32)
        self.type_emb = dev(T["type_emb.weight"], f32)
        self.head = []
        for j in range(cfg["head_layers"]):
            p = "head.layers.%d." % j
            g = lambda s, dt=f32: dev(T[p + s], dt)  # noqa: E731
            self.head.append(dict(n1w=g("norm1.weight"), n1b=g("norm1.bias"),
                                  in_w=g("self_attn.in_proj_weight", b16), in_b=g("self_attn.in_proj_bias"),
                                  out_w=g("self_attn.out_proj.weight", b16), out_b=g("self_attn.out_proj.bias"),
                                  n2w=g("norm2.weight"), n2b=g("norm2.bias"), l1w=g("linear1.weight", b16),
                                  l1b=g("linear1.bias"), l2w=g("linear2.weight", b16), l2b=g("linear2.bias")))
        self.s_nw, self.s_nb = dev(T["scorer.0.weight"], f32), dev(T["scorer.0.bias"], f32)
        self.s_w1, self.s_b1 = dev(T["scorer.1.weight"], b16), dev(T["scorer.1.bias"], f32)
        self.s_w2 = dev(T["scorer.3.weight"], f32).reshape(-1)
        self.s_b2 = float(np.array(T["scorer.3.bias"])[0])

    # ------------------------------------------------------------ launch helpers
    def _launch(self, name, grid, block, args):
        vals = []
        for a in args:
            if a is None:
                vals.append(C.c_void_p(0))
            elif hasattr(a, "data_ptr"):
                vals.append(C.c_void_p(a.data_ptr()))
            elif isinstance(a, float):
                vals.append(C.c_float(a))
            else:
                vals.append(C.c_int(int(a)))
        params = (C.c_void_p * len(vals))(*[C.cast(C.pointer(v), C.c_void_p) for v in vals])
        stream = self.torch.cuda.current_stream().cuda_stream
        g = grid if isinstance(grid, tuple) else (grid, 1, 1)
        _check(_driver().cuLaunchKernel(self.fn[name], g[0], g[1], g[2], block, 1, 1, 0, C.c_void_p(stream), params,
                                        None), "cuLaunchKernel " + name)

    def _ln(self, x, delta, pending, w, b, out, rows, eps):
        self._launch("ln_bf16", (rows + 7) // 8, 256, [x, delta, pending, w, b, out, rows, float(eps)])

    def _attention(self, rope, qkv, out, tiles, ntiles, window):
        H = self.cfg["hidden"]
        cos, sin = rope if rope is not None else (None, None)
        scale = float(np.float32(0.125) * np.float32(1.4426950408889634))
        self._launch("attention_rope" if rope is not None else "attention_plain", (ntiles, self.cfg["heads"], 1), 128,
                     [qkv, 3 * H, out, H, tiles, cos, sin, window, scale])

    # ------------------------------------------------------------ forward (src/cuda/mod.rs:400-520)
    def forward_flat(self, batch):
        torch = self.torch
        cfg = self.cfg
        H, I, FF, eps = cfg["hidden"], cfg["intermediate"], 4 * cfg["hidden"], cfg["norm_eps"]
        t, m = int(batch.ids.size), int(batch.marker_rows.size)
        tiles = []
        for s, n in zip(batch.starts.tolist(), batch.lens.tolist()):
            for q0 in range(0, n, 64):
                tiles += [s, n, q0]
        ntiles = len(tiles) // 3
        qtok = np.repeat(batch.qtypes.astype(np.int32), batch.lens.astype(np.int64))
        d = lambda a: torch.tensor(np.asarray(a), device="cuda")  # noqa: E731
        ids = d(batch.ids.astype(np.int32))
        qtype_t = d(qtok)
        tiles_t = d(np.array(tiles, np.int32))
        markers = d(batch.marker_rows.astype(np.int32))
        f32, b16 = torch.float32, torch.bfloat16
        x = torch.empty((t, H), device="cuda", dtype=f32)
        xn = torch.empty((t, H), device="cuda", dtype=b16)
        ctx = torch.empty((t, H), device="cuda", dtype=b16)
        g = torch.empty((t, I), device="cuda", dtype=b16)
        self._launch("embed_ln", (t + 7) // 8, 256, [ids, self.emb, self.emb_norm, x, xn, t, float(eps)])
        delta = None
        for ly in self.layers:
            if ly["attn_norm"] is not None:
                self._ln(x, delta, None, ly["attn_norm"], None, xn, t, eps)
            qkv = (xn @ ly["wqkv"].t()).contiguous()
            window = -1 if ly["glob"] else cfg["half_window"]
            self._attention(ly["rope"], qkv, ctx, tiles_t, ntiles, window)
            delta = (ctx @ ly["wo"].t()).contiguous()
            self._ln(x, delta, None, ly["mlp_norm"], None, xn, t, eps)
            h = (xn @ ly["wi"].t()).contiguous()
            n8 = (t * I + 7) // 8
            self._launch("geglu", (n8 + 255) // 256, 256, [h, g, t, I])
            delta = (g @ ly["wo2"].t()).contiguous()
        h0 = self.head[0]
        self._launch("final_norm", (t + 7) // 8, 256,
                     [x, delta, self.final_norm, self.type_emb, qtype_t, h0["n1w"], h0["n1b"], xn, t, float(eps)])

        def bias_act(inp, bias, out, rows, cols, relu):
            n4 = (rows * cols + 3) // 4
            self._launch("bias_act", (n4 + 255) // 256, 256, [inp, bias, out, rows, cols, relu])

        def mm32(a, w):
            return torch.mm(a, w.t(), out_dtype=torch.float32)

        qkv = torch.empty((t, 3 * H), device="cuda", dtype=b16)
        hbuf = torch.empty((t, FF), device="cuda", dtype=b16)
        ym = torch.empty((max(m, 1), H), device="cuda", dtype=f32)
        ymb = torch.empty((max(m, 1), H), device="cuda", dtype=b16)
        cm = torch.empty((max(m, 1), H), device="cuda", dtype=b16)
        hm = torch.empty((max(m, 1), FF), device="cuda", dtype=b16)
        delta, pending = None, None
        nh = len(self.head)
        for j, hl in enumerate(self.head):
            if j > 0:
                self._ln(x, delta, pending, hl["n1w"], hl["n1b"], xn, t, 1e-5)
            bias_act(mm32(xn, hl["in_w"]).contiguous(), hl["in_b"], qkv, t, 3 * H, 0)
            self._attention(None, qkv, ctx, tiles_t, ntiles, -1)
            if j + 1 < nh:
                delta = (ctx @ hl["out_w"].t()).contiguous()
                self._ln(x, delta, hl["out_b"], hl["n2w"], hl["n2b"], xn, t, 1e-5)
                bias_act(mm32(xn, hl["l1w"]).contiguous(), hl["l1b"], hbuf, t, FF, 1)
                delta = (hbuf @ hl["l2w"].t()).contiguous()
                pending = hl["l2b"]
            else:
                self._launch("gather_rows", (m + 7) // 8, 256, [ctx, markers, cm, m, 2])
                self._launch("gather_rows", (m + 7) // 8, 256, [x, markers, ym, m, 4])
                dm = (cm[:m] @ hl["out_w"].t()).contiguous()
                self._ln(ym, dm, hl["out_b"], hl["n2w"], hl["n2b"], ymb, m, 1e-5)
                bias_act(mm32(ymb[:m], hl["l1w"]).contiguous(), hl["l1b"], hm, m, FF, 1)
                delta = (hm[:m] @ hl["l2w"].t()).contiguous()
                pending = hl["l2b"]
        self._ln(ym, delta, pending, self.s_nw, self.s_nb, ymb, m, 1e-5)
        z = mm32(ymb[:m], self.s_w1).contiguous()
        scores = torch.empty((max(m, 1),), device="cuda", dtype=f32)
        self._launch("scorer", (m + 7) // 8, 256, [z, self.s_b1, self.s_w2, float(self.s_b2), scores, m])
        torch.cuda.synchronize()
        return scores[:m].cpu().numpy()
