"""GPU against GPU: the reference's own CUDA path and libj1 timed on the same B200.

The reference's CUDA backend is cuBLAS BF16 GEMMs (cublasGemmEx, COMPUTE_32F,
src/cuda/mod.rs:347-375) plus its own kernels.cu (row kernels and the mma.sync
attention, kernels.cu:66-391). oracle/ref_cuda.py replays CudaModel::forward over
kernels.cu compiled unmodified and cuBLAS reached through torch; those kernels only
support hidden 384 (kernels.cu:8), the width of the Julia-1 checkpoint, so the forward
is compared there: one micro-batch of 64 router-scale rows (32,768 tokens) through both,
host clock around each forward (H2D of the batch, all kernels, D2H of the logits).

Per GEMM (the GEMM-sweep configuration's shapes, hidden 768): cuBLAS BF16 through torch,
followed where the reference follows it by its own row kernel (geglu after Wi), against
j1_op_gemm with the fused epilogue; and at hidden 384, where the reference's residual +
LayerNorm kernel (ln_bf16, kernels.cu:97-109) runs, Wo and Wo2 with it. CUDA events,
back-to-back launches after warm-up. One JSON line ("ref-gpu-timing") carries the figures.
"""
import json
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import julia1 as j1  # noqa: E402
from julia1 import synthetic  # noqa: E402


def _events_ms(torch, fn, iters=10, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def _host_ms(torch, fn, iters=5, warm=2):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        torch.cuda.synchronize()
        best = min(best, (time.perf_counter() - t0) * 1e3)
    return best


@pytest.fixture(scope="module")
def ref384(torch_cuda):
    from oracle import ref_cuda
    ck = synthetic.cached_checkpoint(seed=0, hidden=384, heads=6, intermediate=1152)  # the Julia-1 shape
    return ck, ref_cuda.RefCudaModel(ck, torch_cuda)


def test_reference_cuda_path_vs_libj1(torch_cuda, ref384):
    torch = torch_cuda
    import bench
    ck, ref = ref384
    out = {}
    # ------------------------------------------------ whole forward at hidden 384
    rows = bench.make_rows(seed=1000, n=64)
    b = j1.Batch.new([j1.Encoded(*r) for r in rows])
    model = j1.CudaModel(ck, 0)
    try:
        z_ref = ref.forward_flat(b)
        z_lib = model.forward_flat(b)
        err = float(np.abs(z_ref - z_lib).max())
        ms_ref = _host_ms(torch, lambda: ref.forward_flat(b))
        ms_lib = _host_ms(torch, lambda: model.forward_flat(b))
    finally:
        model.close()
    t = b.tokens()
    out["forward_h384_64x512"] = {"tokens": t, "reference_ms": round(ms_ref, 3), "libj1_ms": round(ms_lib, 3),
                                  "reference_tokens_per_s": round(t / ms_ref * 1e3), "libj1_tokens_per_s":
                                  round(t / ms_lib * 1e3), "speedup": round(ms_ref / ms_lib, 2),
                                  "max_abs_logit_diff": err}
    # ------------------------------------------------ GEMMs, hidden 768 (cuBLAS [+ reference row kernel])
    H, I = 768, 1152
    g = torch.Generator(device="cuda").manual_seed(0)
    cos = torch.rand((8192, 32), generator=g, device="cuda")
    sin = torch.rand((8192, 32), generator=g, device="cuda")
    gemms = {}
    for M in (4096, 131072):
        for name, N, K in (("qkv", 3 * H, H), ("wo", H, H), ("wi_geglu", 2 * I, H), ("wo2", H, I)):
            A = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
            W = (torch.randn((N, K), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
            Wt = W.t()
            if name == "wi_geglu":
                h = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
                gg = torch.empty((M, I), device="cuda", dtype=torch.bfloat16)
                n8 = (M * I + 7) // 8

                def ref_fn():
                    torch.matmul(A, Wt, out=h)
                    ref._launch("geglu", (n8 + 255) // 256, 256, [h, gg, M, I])
                Wl = torch.empty_like(W)
                j1.op_geglu_interleave(W.float().contiguous(), Wl, I, K)
                outg = torch.empty((M, I), device="cuda", dtype=torch.bfloat16)
                lib_fn = lambda: j1.op_gemm(j1.EPI_GEGLU, A, Wl, out=outg, sync=False)  # noqa: E731
                note = "cuBLAS + reference geglu kernel"
            else:
                o = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
                ref_fn = lambda: torch.matmul(A, Wt, out=o)  # noqa: E731
                if name == "qkv":
                    lib_fn = lambda: j1.op_gemm(j1.EPI_QKV_ROPE, A, W, out=o, pos=torch.zeros(M, device="cuda", dtype=torch.int32), rope_cos=cos, rope_sin=sin, rope_cols=2 * H, sync=False)  # noqa: E731,E501
                    note = "cuBLAS (the reference rotates q, k inside its attention)"
                else:
                    x = torch.randn((M, N), generator=g, device="cuda")
                    xn = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
                    lw = torch.ones(N, device="cuda")
                    lib_fn = lambda: j1.op_gemm(j1.EPI_RESID_LN, A, W, x=x, ln_w=lw, xn=xn, sync=False)  # noqa: E731
                    note = "cuBLAS only: the reference's residual + LayerNorm kernel supports hidden 384 alone"
            ms_r = _events_ms(torch, ref_fn)
            ms_l = _events_ms(torch, lib_fn)
            gemms["%s_M%d" % (name, M)] = {"reference_ms": round(ms_r, 4), "libj1_ms": round(ms_l, 4),
                                           "speedup": round(ms_r / ms_l, 2), "reference": note,
                                           "libj1_tflops": round(2.0 * M * N * K / ms_l / 1e9, 1),
                                           "reference_tflops": round(2.0 * M * N * K / ms_r / 1e9, 1)}
            del A, W, Wt
    # ------------------------------------------------ residual + LayerNorm GEMMs at hidden 384 (the reference's width)
    H3 = 384
    for M in (4096, 131072):
        for name, N, K in (("wo_resid_ln_h384", H3, H3), ("wo2_resid_ln_h384", H3, I)):
            A = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
            W = (torch.randn((N, K), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
            Wt = W.t()
            x = torch.randn((M, N), generator=g, device="cuda")
            xn = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
            lw = torch.ones(N, device="cuda")
            d = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)

            def ref_fn():
                torch.matmul(A, Wt, out=d)
                ref._ln(x, d, None, lw, None, xn, M, 1e-5)
            lib_fn = lambda: j1.op_gemm(j1.EPI_RESID_LN, A, W, x=x, ln_w=lw, xn=xn, sync=False)  # noqa: E731
            ms_r = _events_ms(torch, ref_fn)
            ms_l = _events_ms(torch, lib_fn)
            nbytes = M * K * 2 + N * K * 2 + M * N * 8 + M * N * 2
            gemms["%s_M%d" % (name, M)] = {"reference_ms": round(ms_r, 4), "libj1_ms": round(ms_l, 4),
                                           "speedup": round(ms_r / ms_l, 2),
                                           "reference": "cuBLAS + reference ln_bf16 kernel",
                                           "libj1_gbs": round(nbytes / ms_l / 1e6, 1),
                                           "reference_gbs": round(nbytes / ms_r / 1e6, 1)}
            del A, W, Wt, x, xn, d
    out["gemms"] = gemms
    print("ref-gpu-timing " + json.dumps(out))
    assert err <= 3e-2
    # the B200 path must beat the reference's own CUDA path on the same GPU
    assert ms_lib < ms_ref
