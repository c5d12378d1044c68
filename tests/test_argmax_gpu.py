"""Argmax agreement at the north star's bar, on the bench's own checkpoint and rows.

The benchmark runs the unperturbed seed-0 checkpoint (LayerNorm gamma = 1, beta = 0, weights
N(0, 0.02)) on router-scale rows (12-token question head, 20 x [MASK] + 11-token options,
state). This test scores J1_ARGMAX_ROWS of those rows (default 256) through the C ABI and
through the CPU restatements of the reference's BF16 CUDA chain (src/cuda/mod.rs:446-511)
and of its FP32 CPU path (src/cpu/mod.rs:201-340), and reports max-abs and max-relative
differences, the spread of each row's logits, the distribution of the reference's top-2
gaps and the argmax agreement over all rows and over rows whose gap exceeds twice the
tolerance (the north star's bar: identical argmax on >= 99.9% of rows vs the BF16 path;
the reference itself reports 1984/2000 for its CUDA path against FP32, README.md:159).

With random weights the option logits of a row are nearly tied (top-2 gaps of 1e-3 .. 1e-2),
so the 2 x 3e-2 cut keeps few or no rows. The assertions therefore also pin the rows outside
it: a row may choose differently only when the reference's top-2 gap is within twice the
largest difference measured on that row (a tie within the measured error), and the all-row
agreement against the BF16 chain must stay at or above ALL_ROWS_MIN.
"""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import julia1 as j1  # noqa: E402
from julia1 import synthetic  # noqa: E402
from oracle import oracle as orc  # noqa: E402

TOL_BF16, TOL_FP32 = 3e-2, 5e-2
ALL_ROWS_MIN = 0.90
N_ROWS = int(os.environ.get("J1_ARGMAX_ROWS", "256"))


def agreement_stats(gpu, ref, n_rows, n_opt, tol):
    """Max-abs / max-rel differences, spread, top-2 gap quantiles and argmax agreement."""
    g = gpu.reshape(n_rows, n_opt)
    r = ref.reshape(n_rows, n_opt)
    d = np.abs(g - r)
    srt = np.sort(r, axis=1)
    gap = srt[:, -1] - srt[:, -2]
    spread = srt[:, -1] - srt[:, 0]
    same = np.argmax(g, axis=1) == np.argmax(r, axis=1)
    resolvable = gap > 2 * tol
    row_err = d.max(axis=1)
    flips = np.nonzero(~same)[0]
    q = lambda a, p: float(np.quantile(a, p))  # noqa: E731
    return {
        "rows": n_rows, "max_abs": float(d.max()), "mean_abs": float(d.mean()),
        "max_rel": float((d / np.maximum(np.abs(r), 1e-3)).max()),
        "max_abs_over_row_spread": float((row_err / np.maximum(spread, 1e-9)).max()),
        "spread": {"min": q(spread, 0), "median": q(spread, 0.5), "max": q(spread, 1)},
        "top2_gap": {"min": q(gap, 0), "p01": q(gap, 0.01), "p10": q(gap, 0.1), "median": q(gap, 0.5),
                     "max": q(gap, 1)},
        "agree_all": int(same.sum()), "agree_all_rate": float(same.mean()),
        "resolvable_rows": int(resolvable.sum()), "agree_resolvable": int(same[resolvable].sum()),
        "flips": [{"row": int(i), "ref_gap": float(gap[i]), "row_max_abs": float(row_err[i])} for i in flips[:20]],
        "flips_within_error": bool(np.all(gap[flips] <= 2 * row_err[flips])),
    }


@pytest.fixture(scope="module")
def bench_case(torch_cuda):
    import bench
    ck = synthetic.cached_checkpoint(seed=0)  # the bench's checkpoint: gamma 1, beta 0
    rows = bench.make_rows(seed=1000, n=N_ROWS)  # the bench job's first rows
    b = j1.Batch.new([j1.Encoded(*r) for r in rows])
    m = j1.CudaModel(ck, 0)
    try:
        gpu = m.forward_flat(b)
    finally:
        m.close()
    o = orc.Oracle(ck)
    return b, gpu, o.forward_flat(b, mode="bf16"), o.forward_flat(b, mode="fp32")


def test_argmax_agreement_bench_checkpoint(bench_case):
    b, gpu, ref16, ref32 = bench_case
    n_opt = 20
    assert gpu.size == N_ROWS * n_opt and np.isfinite(gpu).all()
    s16 = agreement_stats(gpu, ref16, N_ROWS, n_opt, TOL_BF16)
    s32 = agreement_stats(gpu, ref32, N_ROWS, n_opt, TOL_FP32)
    chain = agreement_stats(ref16, ref32, N_ROWS, n_opt, TOL_FP32)  # the reference's own BF16 vs FP32
    print("argmax-stats " + json.dumps({"vs_bf16_chain": s16, "vs_fp32": s32, "bf16_chain_vs_fp32": chain}))
    assert s16["max_abs"] <= TOL_BF16 and s32["max_abs"] <= TOL_FP32
    # the north star's bar on the rows it can decide
    if s16["resolvable_rows"]:
        assert s16["agree_resolvable"] >= 0.999 * s16["resolvable_rows"]
    # every other choice: a different argmax only where the reference's top-2 gap is a tie
    # within the difference measured on that row
    assert s16["flips_within_error"], s16["flips"]
    assert s16["agree_all_rate"] >= ALL_ROWS_MIN
