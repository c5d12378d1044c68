"""The CPU oracle, pinned before it is trusted (no GPU needed).

1. The reference's own unit tests, restated against the oracle's GEMM and fast math:
   src/cpu/gemm.rs:377-406 (linear, 5 epilogues, strided output, ragged M; 1e-4 vs naive f64),
   src/cpu/gemm.rs:408-426 (fused GEGLU vs naive f64 with exact erf; 1e-4),
   src/cpu/fastmath.rs:51-77 (exp relative error < 3e-7 on [-87, 88); erf abs error < 1e-6 on [-6, 6)).
2. The whole FP32 forward against golden logits and encoder hidden states produced by an
   independent FP32 implementation of the same model (tests/golden/make_golden.py:
   transformers ModernBertModel + nn.TransformerEncoderLayer head + scorer).
3. The batching-invariance property of tests/checkpoint.rs:91-105 (|delta| < 1e-4).
"""
import math
import os

import numpy as np
import pytest

from oracle import oracle as orc
from julia1 import synthetic

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rnd_stream(seed):
    """The LCG `rnd` of src/cpu/gemm.rs:362-365: uniform in [-0.5, 0.5)."""
    s = seed

    def nxt():
        nonlocal s
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        return (s >> 8) / float(1 << 24) - 0.5
    return nxt


def lcg_array(nxt, n):
    return np.array([nxt() for _ in range(n)], dtype=np.float32)


@pytest.mark.parametrize("rows,n,k", [(1, 32, 7), (13, 96, 384), (70, 40, 300), (129, 1152, 384)])
def test_linear_matches_naive(rows, n, k):
    nxt = rnd_stream(1 + rows)
    x = lcg_array(nxt, rows * k).reshape(rows, k)
    w = lcg_array(nxt, n * k).reshape(n, k)
    bias = lcg_array(nxt, n)
    ldo = n + 5
    base = lcg_array(nxt, rows * ldo).reshape(rows, ldo)
    prod = x.astype(np.float64) @ w.astype(np.float64).T
    for mode in range(5):
        out = base.copy()
        orc.linear(x, w, epi=mode, bias=bias if mode >= 2 else None, out=out, col=3)
        v, b, old = prod, bias.astype(np.float64), base[:, 3:3 + n].astype(np.float64)
        expect = [v, old + v, v + b, np.maximum(v + b, 0.0), old + v + b][mode]
        assert np.abs(out[:, 3:3 + n] - expect).max() < 1e-4, mode
        assert np.array_equal(out[:, :3], base[:, :3]) and np.array_equal(out[:, 3 + n:], base[:, 3 + n:])


@pytest.mark.parametrize("rows,inter,k", [(1, 64, 384), (21, 128, 100), (300, 1152, 384)])
def test_geglu_matches_naive(rows, inter, k):
    nxt = rnd_stream(7 + rows)
    x = lcg_array(nxt, rows * k).reshape(rows, k)
    w = lcg_array(nxt, 2 * inter * k).reshape(2 * inter, k)
    prod = x.astype(np.float64) @ w.astype(np.float64).T
    u, v = prod[:, :inter], prod[:, inter:]
    erf = np.vectorize(math.erf)
    expect = 0.5 * u * (1.0 + erf(u / math.sqrt(2.0))) * v
    g = orc.linear_geglu(x, w)
    assert np.abs(g - expect).max() < 1e-4


def test_exp_close_to_libm():
    L = orc.lib()
    worst = 0.0
    x = np.float32(-87.0)
    step = np.float32(0.0013)
    while x < 88.0:
        a = L.oracle_exp(float(x))
        b = float(np.float32(math.exp(float(x))))
        worst = max(worst, abs((a - b) / b))
        x = np.float32(x + step)
    assert worst < 3e-7, worst
    assert L.oracle_exp(float("-inf")) < 1e-37


def test_erf_close_to_libm():
    L = orc.lib()
    worst = 0.0
    x = np.float32(-6.0)
    step = np.float32(0.0007)
    while x < 6.0:
        worst = max(worst, abs(L.oracle_erf(float(x)) - math.erf(float(x))))
        x = np.float32(x + step)
    assert worst < 1e-6, worst


def test_bf16_rounding_is_nearest_even():
    L = orc.lib()
    assert L.oracle_bf16(1.0) == 1.0
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: rounds to even (1.0)
    assert L.oracle_bf16(1.0 + 2.0 ** -8) == 1.0
    assert L.oracle_bf16(1.0 + 3 * 2.0 ** -8) == 1.0 + 2.0 ** -6


class _B:
    def __init__(self, rows):
        ids, starts, lens, qt, mr, ms = [], [], [], [], [], [0]
        off = 0
        for r_ids, r_mk, r_qt in rows:
            starts.append(off)
            lens.append(len(r_ids))
            qt.append(r_qt)
            ids.append(np.asarray(r_ids, np.uint32))
            mr.extend(off + int(m) for m in r_mk)
            ms.append(len(mr))
            off += len(r_ids)
        self.ids = np.concatenate(ids)
        self.starts, self.lens = np.array(starts, np.uint32), np.array(lens, np.uint32)
        self.qtypes, self.marker_rows = np.array(qt, np.uint8), np.array(mr, np.uint32)
        self.marker_starts = np.array(ms, np.uint32)


def _golden_case(name, tmp_path_factory):
    z = np.load(os.path.join(GOLDEN, "%s_fp32.npz" % name))
    shape = {str(k): int(v) for k, v in zip(z["shape_keys"], z["shape"])}
    root = synthetic.write_checkpoint(str(tmp_path_factory.mktemp(name)), seed=int(z["seed"]), perturb=True, **shape)
    rows, o, om = [], 0, 0
    for L, q, nm in zip(z["lens"], z["qtypes"], z["row_markers"]):
        rows.append((z["ids"][o:o + L], z["markers"][om:om + nm], int(q)))
        o += L
        om += nm
    return z, root, rows


@pytest.mark.parametrize("name", ["tiny", "j384"])
def test_oracle_fp32_matches_golden(name, tmp_path_factory):
    z, root, rows = _golden_case(name, tmp_path_factory)
    o = orc.Oracle(root)
    scores, hidden = o.forward_flat(_B(rows), mode="fp32", hidden=True)
    assert np.abs(hidden[::7] - z["hidden"]).max() < 2e-4
    err = np.abs(scores - z["logits"])
    assert err.max() < 1e-4, err.max()
    assert np.argmax(scores) == np.argmax(z["logits"])


@pytest.mark.parametrize("name", ["tiny", "j384"])
def test_oracle_bf16_chain_close_to_fp32(name, tmp_path_factory):
    """The BF16-emulating restatement stays within the north star's FP32-vs-CUDA bound (5e-2)."""
    z, root, rows = _golden_case(name, tmp_path_factory)
    o = orc.Oracle(root)
    s16 = o.forward_flat(_B(rows), mode="bf16")
    assert np.abs(s16 - z["logits"]).max() < 5e-2
    assert np.abs(s16 - z["logits"]).max() > 0  # it does round


def test_oracle_batching_invariance(tmp_path_factory):
    """tests/checkpoint.rs:91-105: a row scored alone equals the row scored inside a batch."""
    _, root, rows = _golden_case("tiny", tmp_path_factory)
    o = orc.Oracle(root)
    together = o.forward_flat(_B(rows), mode="fp32")
    off = 0
    for r in rows:
        alone = o.forward_flat(_B([r]), mode="fp32")
        assert alone.size == len(r[1])
        if alone.size:
            assert np.abs(alone - together[off:off + alone.size]).max() < 1e-4
        off += alone.size
    assert off == together.size
