"""Isolated fused-epilogue GEMM sweep (the BASELINE GEMM-sweep configuration).

  python -m julia1.gemm_sweep [--m 512,4096,32768,131072] [--iters 20]

Shapes at hidden 768 (ModernBERT-base): QKV 768->2304 (+RoPE), Wo 768->768 with the
FP32 residual + LayerNorm epilogue, Wi 768->2304 with the GEGLU epilogue (1152
outputs), Wo2 1152->768 with residual + LayerNorm. A ~ N(0,1) BF16, W ~ N(0,0.02).
Each shape is launched through j1_op_gemm on one stream and timed with CUDA events
over `iters` back-to-back launches after 3 warm-up launches; the SM clock is read
through NVML while the timed launches run. Prints one JSON line per (shape, M).
"""
import argparse
import json
import os
import sys
import threading

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if HERE not in sys.path:
    sys.path.insert(0, HERE)

import julia1 as j1  # noqa: E402

H, I = 768, 1152


class SmClock:
    """Median SM clock (MHz) seen by NVML while the block runs (None without NVML)."""

    def __init__(self, index):
        self.samples, self._stop = [], threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self._nv = pynvml
        except Exception:
            self._nv = None

    def __enter__(self):
        if self._nv:
            def run():
                while not self._stop.is_set():
                    self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                    self._stop.wait(0.01)
            self._t = threading.Thread(target=run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self._nv:
            self._stop.set()
            self._t.join()

    def median(self):
        s = sorted(self.samples)
        return s[len(s) // 2] if s else None


def shapes():
    return [("qkv_rope", j1.EPI_QKV_ROPE, 3 * H, H), ("wo_resid_ln", j1.EPI_RESID_LN, H, H),
            ("wi_geglu", j1.EPI_GEGLU, 2 * I, H), ("wo2_resid_ln", j1.EPI_RESID_LN, H, I)]


def main():
    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", default="512,4096,32768,131072")
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    dev = torch.cuda.current_device()
    g = torch.Generator(device="cuda").manual_seed(0)
    cos = torch.rand((8192, 32), generator=g, device="cuda")
    sin = torch.rand((8192, 32), generator=g, device="cuda")
    for M in [int(x) for x in a.m.split(",")]:
        for name, epi, N, K in shapes():
            A = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
            W = (torch.randn((N, K), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
            kw = {}
            if epi == j1.EPI_QKV_ROPE:
                kw = dict(out=torch.empty((M, N), device="cuda", dtype=torch.bfloat16),
                          pos=torch.arange(M, device="cuda", dtype=torch.int32) % 512, rope_cos=cos, rope_sin=sin,
                          rope_cols=2 * H)
            elif epi == j1.EPI_GEGLU:
                kw = dict(out=torch.empty((M, N // 2), device="cuda", dtype=torch.bfloat16))
            else:
                kw = dict(x=torch.randn((M, N), generator=g, device="cuda"),
                          ln_w=torch.ones(N, device="cuda"), xn=torch.empty((M, N), device="cuda", dtype=torch.bfloat16))
            for _ in range(3):
                j1.op_gemm(epi, A, W, sync=False, **kw)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with SmClock(dev) as clk:
                e0.record()
                for _ in range(a.iters):
                    j1.op_gemm(epi, A, W, sync=False, **kw)
                e1.record()
                torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / a.iters
            flops = 2.0 * M * N * K
            out_cols = N // 2 if epi == j1.EPI_GEGLU else N
            if epi == j1.EPI_RESID_LN:
                nbytes = M * K * 2 + N * K * 2 + M * N * 8 + M * N * 2
            else:
                nbytes = M * K * 2 + N * K * 2 + M * out_cols * 2
            print(json.dumps({"gemm": name, "M": M, "N": N, "K": K, "ms": round(ms, 4),
                              "tflops": round(flops / ms / 1e9, 1), "gbs": round(nbytes / ms / 1e6, 1),
                              "sm_mhz": clk.median()}), flush=True)
            del A, W, kw


if __name__ == "__main__":
    main()
