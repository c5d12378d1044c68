"""Kernel-level parity of the tcgen05 GEMM epilogues and the attention kernel.

Each op is called through the C ABI (j1_op_*) on torch CUDA tensors and compared
with a plain PyTorch fp32 restatement of the same op. Tolerances are written per
test; BF16 outputs are compared to the fp32 reference rounded once to BF16, so
the bound is about one BF16 ulp plus fp32 summation-order noise.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import julia1 as j1  # noqa: E402


def _rand(torch, shape, std, seed, dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda", dtype=torch.float32) * std).to(dtype)


def _close_bf16(out, ref, rtol=1.6e-2, atol=2e-3):
    diff = (out.float() - ref.float()).abs()
    bound = atol + rtol * ref.float().abs()
    bad = (diff > bound).sum().item()
    assert bad == 0, "max diff %g, %d elements out of tolerance" % (diff.max().item(), bad)


def _resid_check(torch, x, x0, src, W, b=None):
    """x == x0 + bf16(src . W^T) (+ b): the GEMM output is rounded to BF16 before the residual
    add, as the reference's GEMM writes BF16 (src/cuda/mod.rs:456,461) and ln_bf16 adds it.
    fp32 summation order may move an output across a BF16 rounding boundary: such elements
    (at most 0.1%) may differ by one BF16 ulp of the product. Returns the reference x.
    LayerNorm outputs are then checked against the LayerNorm of the kernel's own x, so that
    such a flip (already bounded here) is not counted twice."""
    acc = src.float() @ W.float().t()
    xr = x0 + acc.to(torch.bfloat16).float() + (b if b is not None else 0)
    diff = (x - xr).abs()
    ulp = acc.abs().clamp_min(1e-30) * 2.0 ** -7
    off = diff > 1e-4 + 1e-5 * xr.abs()
    assert (diff[off] <= ulp[off] * 1.01 + 1e-4).all(), diff.max().item()
    assert off.float().mean().item() <= 1e-3, off.float().mean().item()
    return xr


GEMM_SHAPES = [(1, 768, 768), (100, 2304, 768), (128, 768, 1152), (300, 3072, 768), (1024, 2304, 768),
               (4096, 768, 768), (257, 1152, 384)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_bf16_store(torch_cuda, M, N, K):
    torch = torch_cuda
    A = _rand(torch, (M, K), 1.0, 1, torch.bfloat16)
    W = _rand(torch, (N, K), 0.02, 2, torch.bfloat16)
    out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    j1.op_gemm(j1.EPI_BF16, A, W, out=out)
    ref = A.float() @ W.float().t()
    _close_bf16(out, ref.to(torch.bfloat16).float())


@pytest.mark.parametrize("relu", [False, True])
def test_gemm_bias_relu(torch_cuda, relu):
    torch = torch_cuda
    M, N, K = 333, 3072, 768
    A = _rand(torch, (M, K), 1.0, 3, torch.bfloat16)
    W = _rand(torch, (N, K), 0.02, 4, torch.bfloat16)
    b = _rand(torch, (N,), 0.5, 5, torch.float32)
    out = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    j1.op_gemm(j1.EPI_BF16, A, W, out=out, bias=b, relu=relu)
    ref = A.float() @ W.float().t() + b
    if relu:
        ref = ref.clamp_min(0)
    _close_bf16(out, ref.to(torch.bfloat16).float())


def _close_bf16_flips(out, ref, scale, frac=2e-3):
    """_close_bf16, except that an input rounded to BF16 before the fused math (as the
    reference rounds its GEMM outputs) may round the other way when fp32 summation order
    moves it across a rounding boundary: such elements (at most `frac`) may differ by up to
    2^-6 of `scale`, the magnitude of the inputs they were computed from."""
    diff = (out.float() - ref.float()).abs()
    bad = diff > 2e-3 + 1.6e-2 * ref.float().abs()
    assert (diff[bad] <= 2.0 ** -6 * scale[bad] + 2e-3).all(), diff.max().item()
    assert bad.float().mean().item() <= frac, bad.float().mean().item()


def _qkv_ref(torch, acc, cos, sin, pos, H):
    """EPI_QKV_ROPE restated: qkv = bf16(acc) (the reference's GEMM output), q and k rotated
    in fp32 (rotate-half on d, d + 32 within each head) and rounded again. Returns (ref, scale)."""
    M = acc.shape[0]
    r = acc.to(torch.bfloat16).float()
    c, s_ = cos[pos.long()], sin[pos.long()]
    qk = r[:, :2 * H].reshape(M, 2 * H // 64, 64)
    lo, hi = qk[..., :32], qk[..., 32:]
    rot = torch.cat([lo * c[:, None] - hi * s_[:, None], hi * c[:, None] + lo * s_[:, None]], dim=-1)
    ref = torch.cat([rot.reshape(M, 2 * H), r[:, 2 * H:]], dim=1).to(torch.bfloat16).float()
    mag = torch.maximum(lo.abs(), hi.abs())
    scale = torch.cat([torch.cat([mag, mag], dim=-1).reshape(M, 2 * H), r[:, 2 * H:].abs()], dim=1)
    return ref, scale


def _geglu_ref(torch, acc, I):
    """EPI_GEGLU restated: h = bf16(acc) (the reference's GEMM output), g = gelu(h_a) * h_b."""
    h = acc.to(torch.bfloat16).float()
    ref = (torch.nn.functional.gelu(h[:, :I]) * h[:, I:]).to(torch.bfloat16).float()
    scale = (h[:, :I].abs() + 1.0) * h[:, I:].abs()
    return ref, scale


def _rope_tables(torch, theta, positions):
    # rope_table (src/config.rs:99-112): f32 inv_freq, f32 products
    inv = 1.0 / np.power(np.float32(theta), (np.arange(32, dtype=np.float32) * 2) / np.float32(64)).astype(np.float32)
    f = np.arange(positions, dtype=np.float32)[:, None] * inv[None, :].astype(np.float32)
    return (torch.tensor(np.cos(f), device="cuda"), torch.tensor(np.sin(f), device="cuda"))


@pytest.mark.parametrize("H,theta", [(768, 10000.0), (768, 160000.0), (384, 10000.0)])
def test_gemm_qkv_rope(torch_cuda, H, theta):
    torch = torch_cuda
    lens = [200, 77, 512, 3]
    M = sum(lens)
    pos = torch.tensor(np.concatenate([np.arange(n) for n in lens]).astype(np.int32), device="cuda")
    A = _rand(torch, (M, H), 1.0, 6, torch.bfloat16)
    W = _rand(torch, (3 * H, H), 0.02, 7, torch.bfloat16)
    cos, sin = _rope_tables(torch, theta, 1024)
    out = torch.empty((M, 3 * H), device="cuda", dtype=torch.bfloat16)
    j1.op_gemm(j1.EPI_QKV_ROPE, A, W, out=out, pos=pos, rope_cos=cos, rope_sin=sin, rope_cols=2 * H)
    acc = A.float() @ W.float().t()
    ref, scale = _qkv_ref(torch, acc, cos, sin, pos, H)
    _close_bf16_flips(out, ref, scale)


@pytest.mark.parametrize("M,I,K", [(500, 1152, 768), (64, 1152, 384), (4096, 1152, 768)])
def test_gemm_geglu(torch_cuda, M, I, K):
    torch = torch_cuda
    A = _rand(torch, (M, K), 1.0, 8, torch.bfloat16)
    Wf = _rand(torch, (2 * I, K), 0.02, 9, torch.bfloat16).float()
    Wi = torch.empty((2 * I, K), device="cuda", dtype=torch.bfloat16)
    j1.op_geglu_interleave(Wf.contiguous(), Wi, I, K)
    out = torch.empty((M, I), device="cuda", dtype=torch.bfloat16)
    j1.op_gemm(j1.EPI_GEGLU, A, Wi, out=out)
    acc = A.float() @ Wf.t()
    ref, scale = _geglu_ref(torch, acc, I)
    _close_bf16_flips(out, ref, scale)


@pytest.mark.parametrize("M,H,K,bias,ln_bias", [(300, 768, 768, False, False), (1000, 768, 1152, True, True),
                                                (129, 384, 384, False, False), (4096, 768, 3072, True, True)])
def test_gemm_resid_ln(torch_cuda, M, H, K, bias, ln_bias):
    torch = torch_cuda
    A = _rand(torch, (M, K), 1.0, 10, torch.bfloat16)
    W = _rand(torch, (H, K), 0.02, 11, torch.bfloat16)
    x0 = _rand(torch, (M, H), 1.0, 12, torch.float32)
    b = _rand(torch, (H,), 0.1, 13, torch.float32) if bias else None
    g = 1.0 + _rand(torch, (H,), 0.1, 14, torch.float32)
    bb = _rand(torch, (H,), 0.1, 15, torch.float32) if ln_bias else None
    x = x0.clone()
    xn = torch.empty((M, H), device="cuda", dtype=torch.bfloat16)
    j1.op_gemm(j1.EPI_RESID_LN, A, W, x=x, bias=b, ln_w=g, ln_b=bb, ln_eps=1e-5, xn=xn)
    _resid_check(torch, x, x0, A, W, b)
    ref = torch.nn.functional.layer_norm(x, (H,), g, bb, 1e-5)
    _close_bf16(xn, ref.to(torch.bfloat16).float())


@pytest.mark.parametrize("K,bias", [(768, False), (1152, True)])
def test_gemm_resid_ln_epilogue_widths_same_bits(torch_cuda, K, bias):
    """The residual kernel runs eight epilogue warps when each cluster has at most two 256-row
    units (8,192 rows here) and four otherwise (32,768 rows): a row's updated x and its
    normalised xn must not depend on which, so the first 8,192 rows of the large launch equal
    the small launch to the last bit (tolerance 0)."""
    torch = torch_cuda
    M_small, M_big, H = 8192, 32768, 768
    A = _rand(torch, (M_big, K), 1.0, 80, torch.bfloat16)
    W = _rand(torch, (H, K), 0.02, 81, torch.bfloat16)
    x0 = _rand(torch, (M_big, H), 1.0, 82, torch.float32)
    b = _rand(torch, (H,), 0.1, 83, torch.float32) if bias else None
    g = 1.0 + _rand(torch, (H,), 0.1, 84, torch.float32)
    bb = _rand(torch, (H,), 0.1, 85, torch.float32)
    xa, xb = x0.clone(), x0[:M_small].clone()
    xna = torch.empty((M_big, H), device="cuda", dtype=torch.bfloat16)
    xnb = torch.empty((M_small, H), device="cuda", dtype=torch.bfloat16)
    j1.op_gemm(j1.EPI_RESID_LN, A, W, x=xa, bias=b, ln_w=g, ln_b=bb, xn=xna)
    j1.op_gemm(j1.EPI_RESID_LN, A[:M_small].contiguous(), W, x=xb, bias=b, ln_w=g, ln_b=bb, xn=xnb)
    assert torch.equal(xa[:M_small], xb)
    assert torch.equal(xna[:M_small], xnb)


@pytest.mark.parametrize("M", [32768, 131072])
def test_c2_gemm_sweep_full_size(torch_cuda, M):
    """The GEMM-sweep configuration's large sizes (M = 32,768 and 131,072 rows, hidden 768):
    every fused GEMM of an encoder layer against its fp32 restatement, with the tolerances
    of the small-size tests above."""
    torch = torch_cuda
    H, I = 768, 1152
    pos = torch.arange(M, device="cuda", dtype=torch.int32) % 512
    cos, sin = _rope_tables(torch, 160000.0, 512)
    A = _rand(torch, (M, H), 1.0, 40, torch.bfloat16)
    # QKV 768 -> 2304 + RoPE on q and k
    W = _rand(torch, (3 * H, H), 0.02, 41, torch.bfloat16)
    out = torch.empty((M, 3 * H), device="cuda", dtype=torch.bfloat16)
    j1.op_gemm(j1.EPI_QKV_ROPE, A, W, out=out, pos=pos, rope_cos=cos, rope_sin=sin, rope_cols=2 * H)
    acc = A.float() @ W.float().t()
    ref, scale = _qkv_ref(torch, acc, cos, sin, pos, H)
    _close_bf16_flips(out, ref, scale)
    del out, acc, ref, scale
    # Wi 768 -> 2304 + GEGLU -> 1152
    Wf = _rand(torch, (2 * I, H), 0.02, 42, torch.bfloat16).float()
    Wi = torch.empty((2 * I, H), device="cuda", dtype=torch.bfloat16)
    j1.op_geglu_interleave(Wf.contiguous(), Wi, I, H)
    g = torch.empty((M, I), device="cuda", dtype=torch.bfloat16)
    j1.op_gemm(j1.EPI_GEGLU, A, Wi, out=g)
    acc = A.float() @ Wf.t()
    ref, scale = _geglu_ref(torch, acc, I)
    _close_bf16_flips(g, ref, scale)
    del acc, ref, scale
    # Wo 768 -> 768 and Wo2 1152 -> 768, each + FP32 residual + LayerNorm
    lw = 1.0 + _rand(torch, (H,), 0.1, 43, torch.float32)
    for K, src, seed in [(H, A, 44), (I, g, 46)]:
        W = _rand(torch, (H, K), 0.02, seed, torch.bfloat16)
        x0 = _rand(torch, (M, H), 1.0, seed + 1, torch.float32)
        x = x0.clone()
        xn = torch.empty((M, H), device="cuda", dtype=torch.bfloat16)
        j1.op_gemm(j1.EPI_RESID_LN, src, W, x=x, ln_w=lw, ln_eps=1e-5, xn=xn)
        _resid_check(torch, x, x0, src, W)
        _close_bf16(xn, torch.nn.functional.layer_norm(x, (H,), lw, None, 1e-5).to(torch.bfloat16).float())


@pytest.mark.parametrize("H,K", [(256, 256), (512, 1024), (1024, 1024), (384, 1152)])
def test_gemm_resid_ln_widths(torch_cuda, H, K):
    """The other hidden widths of the row-split residual kernel: clusters of 1 (H 256), 2 (H 512),
    4 (H 1024) CTAs of 256 columns each, and 2 CTAs of 192 columns (H 384)."""
    torch = torch_cuda
    M = 1000
    A = _rand(torch, (M, K), 1.0, 60, torch.bfloat16)
    W = _rand(torch, (H, K), 0.02, 61, torch.bfloat16)
    x0 = _rand(torch, (M, H), 1.0, 62, torch.float32)
    g = 1.0 + _rand(torch, (H,), 0.1, 63, torch.float32)
    bb = _rand(torch, (H,), 0.1, 64, torch.float32)
    x = x0.clone()
    xn = torch.empty((M, H), device="cuda", dtype=torch.bfloat16)
    j1.op_gemm(j1.EPI_RESID_LN, A, W, x=x, ln_w=g, ln_b=bb, ln_eps=1e-5, xn=xn)
    _resid_check(torch, x, x0, A, W)
    _close_bf16(xn, torch.nn.functional.layer_norm(x, (H,), g, bb, 1e-5).to(torch.bfloat16).float())


@pytest.mark.parametrize("grid", [3, 6, 9, 148])
def test_gemm_resid_ln_grid_limits(torch_cuda, grid):
    """Fewer clusters than 128-row units: each cluster walks many units through both TMEM
    buffers and both statistics slots."""
    torch = torch_cuda
    M, H, K = 5000, 768, 1152
    A = _rand(torch, (M, K), 1.0, 70, torch.bfloat16)
    W = _rand(torch, (H, K), 0.02, 71, torch.bfloat16)
    x0 = _rand(torch, (M, H), 1.0, 72, torch.float32)
    g = 1.0 + _rand(torch, (H,), 0.1, 73, torch.float32)
    x = x0.clone()
    xn = torch.empty((M, H), device="cuda", dtype=torch.bfloat16)
    j1.op_gemm(j1.EPI_RESID_LN, A, W, x=x, ln_w=g, ln_eps=1e-5, xn=xn, grid_limit=grid)
    _resid_check(torch, x, x0, A, W)
    _close_bf16(xn, torch.nn.functional.layer_norm(x, (H,), g, None, 1e-5).to(torch.bfloat16).float())


def test_gemm_resid_only(torch_cuda):
    torch = torch_cuda
    M, H, K = 777, 768, 1152
    A = _rand(torch, (M, K), 1.0, 16, torch.bfloat16)
    W = _rand(torch, (H, K), 0.02, 17, torch.bfloat16)
    x0 = _rand(torch, (M, H), 1.0, 18, torch.float32)
    x = x0.clone()
    j1.op_gemm(j1.EPI_RESID, A, W, x=x)
    _resid_check(torch, x, x0, A, W)


@pytest.mark.parametrize("M,H", [(5, 768), (300, 768), (50, 384)])
def test_gemm_scorer(torch_cuda, M, H):
    torch = torch_cuda
    A = _rand(torch, (M, H), 1.0, 19, torch.bfloat16)
    W = _rand(torch, (H, H), 0.02, 20, torch.bfloat16)
    b1 = _rand(torch, (H,), 0.1, 21, torch.float32)
    w2 = _rand(torch, (H,), 0.05, 22, torch.float32)
    scores = torch.empty((M,), device="cuda", dtype=torch.float32)
    j1.op_gemm(j1.EPI_SCORER, A, W, bias=b1, w2=w2, b2=0.25, scores=scores)
    z = A.float() @ W.float().t() + b1
    ref = (torch.nn.functional.gelu(z) * w2).sum(1) + 0.25
    torch.testing.assert_close(scores, ref, rtol=1e-4, atol=1e-4)


def test_gemm_persistent_grid_limits(torch_cuda):
    """Fewer CTAs than tiles: every CTA walks several tiles through both TMEM buffers."""
    torch = torch_cuda
    M, N, K = 2048, 2304, 768
    A = _rand(torch, (M, K), 1.0, 23, torch.bfloat16)
    W = _rand(torch, (N, K), 0.02, 24, torch.bfloat16)
    ref = (A.float() @ W.float().t()).to(torch.bfloat16).float()
    for grid in (1, 3, 7, 148):
        out = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
        j1.op_gemm(j1.EPI_BF16, A, W, out=out, grid_limit=grid)
        _close_bf16(out, ref)


def _attention_ref(torch, qkv, H, starts, lens, window):
    t = qkv.shape[0]
    q = qkv[:, :H].float().reshape(t, H // 64, 64)
    k = qkv[:, H:2 * H].float().reshape(t, H // 64, 64)
    v = qkv[:, 2 * H:].float().reshape(t, H // 64, 64)
    out = torch.zeros((t, H), device="cuda", dtype=torch.float32)
    for s0, n in zip(starts, lens):
        qs, ks, vs = q[s0:s0 + n].transpose(0, 1), k[s0:s0 + n].transpose(0, 1), v[s0:s0 + n].transpose(0, 1)
        sc = (qs @ ks.transpose(1, 2)) * 0.125
        if window >= 0:
            i = torch.arange(n, device="cuda")
            sc = sc.masked_fill((i[:, None] - i[None, :]).abs() > window, float("-inf"))
        p = torch.softmax(sc, dim=-1)
        out[s0:s0 + n] = (p @ vs).transpose(0, 1).reshape(n, H)
    return out


@pytest.mark.parametrize("lens,window,H", [([512, 512], -1, 768), ([512, 300, 77], 64, 768),
                                           ([1, 2, 129, 1000], 64, 768), ([1000, 16, 640], -1, 768),
                                           ([2048], 64, 384), ([700], -1, 384)])
def test_attention(torch_cuda, lens, window, H):
    torch = torch_cuda
    t = sum(lens)
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.uint32)
    qkv = _rand(torch, (t, 3 * H), 1.0, 25, torch.bfloat16)
    ctx = torch.full((t, H), float("nan"), device="cuda", dtype=torch.bfloat16)
    j1.op_attention(qkv, H, starts, np.array(lens, np.uint32), window, ctx)
    ref = _attention_ref(torch, qkv, H, starts.tolist(), lens, window)
    # P is rounded to bf16 before P.V (as the reference kernel does): ~0.5% relative noise
    diff = (ctx.float() - ref).abs()
    assert torch.isfinite(ctx.float()).all()
    assert diff.max().item() < 2.5e-2, diff.max().item()
    assert diff.mean().item() < 2.5e-3, diff.mean().item()
