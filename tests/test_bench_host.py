"""Host-side arithmetic of bench.py: the algorithmic FLOP/byte model behind `roofline`
and `gemm_tensor_peak` (no GPU)."""
import os
import sys

import pytest

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_local_pairs_matches_band_count():
    # pairs (i, j) with |i - j| <= 64 inside a sequence of S tokens: 129 S - 4160 for S >= 129
    for S in (129, 512, 1000):
        assert bench.local_pairs(S) == 129 * S - 4160
    assert bench.local_pairs(10) == 100  # short sequence: every pair


def test_family_model_flops():
    t, seqs = 2 * 512, [512, 512]
    f = bench.family_model(t, seqs, m=40)
    assert f["gemm_qkv_rope"]["flops"] == 2.0 * t * 2304 * 768
    assert f["gemm_wi_geglu"]["flops"] == 2.0 * t * 2304 * 768
    assert f["gemm_wo_resid_ln"]["flops"] == 2.0 * t * 768 * 768
    assert f["gemm_wo2_resid_ln"]["flops"] == 2.0 * t * 768 * 1152
    assert f["attn_global"]["flops"] == 4.0 * 768 * 2 * 512 * 512
    assert f["attn_local"]["flops"] == 4.0 * 768 * 2 * bench.local_pairs(512)
    # residual + LayerNorm bytes per token: A + x read + x write + xn write
    per_tok = (f["gemm_wo_resid_ln"]["bytes"] - 768 * 768 * 2) / t
    assert per_tok == 768 * 2 + 768 * 8 + 768 * 2


def test_encoder_flops_per_token():
    # 220.59 MFLOP of GEMMs per token plus attention: 238.37 MFLOP at S = 512
    assert bench.encoder_flops_per_token(512) == pytest.approx(238.37e6, rel=1e-3)


def test_gemm_peak_share():
    model_f = {f: {"flops": 1e12} for f in ("gemm_qkv_rope", "gemm_wo_resid_ln", "gemm_wi_geglu",
                                             "gemm_wo2_resid_ln")}
    timed = {f: (2.0, 2) for f in model_f}  # 2 launches in 2 ms per family -> 1 PF/s
    g = bench.gemm_peak_share(timed, model_f, 1638.8)
    assert g["tflops"] == pytest.approx(1000.0)
    assert g["frac_of_measured_burst"] == pytest.approx(1000.0 / 1638.8, abs=1e-4)
    assert g["frac_of_nominal"] == pytest.approx(1000.0 / 2250.0, abs=1e-4)
    assert bench.gemm_peak_share({}, model_f, 1362.0) is None


def test_encoder_flops_of_ragged_lengths():
    # one forward over several sequences is the sum of the per-sequence FLOPs
    lens = [16, 200, 1024]
    assert bench.encoder_flops(lens) == pytest.approx(sum(bench.encoder_flops([s]) for s in lens))
    assert bench.encoder_flops([8192]) / 8192 == pytest.approx(427.45e6, rel=1e-3)


def test_roofline_entry_fractions():
    fm = {"flops": 4.0e11, "bytes": 1.0e9, "bound": "tensor"}
    r = bench.roofline_entry("gemm_wi_geglu", fm, 0.4, 0.2, 6551.0, 1638.8, 1387.9, "measured")
    assert r["achieved"] == pytest.approx(1000.0) and r["frac"] == pytest.approx(1000.0 / 1638.8, abs=1e-4)
    assert r["frac_of_sustained"] == pytest.approx(1000.0 / 1387.9, abs=1e-4)
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s" and r["peak"] == 1638.8
    fm = {"flops": 1.0, "bytes": 1.3e9, "bound": "hbm"}
    r = bench.roofline_entry("gemm_wo2_resid_ln", fm, 0.26, 0.2, 6551.0, 1638.8, 1387.9, "measured")
    assert r["achieved"] == pytest.approx(5000.0) and r["frac"] == pytest.approx(5000.0 / 6551.0, abs=1e-4)


def test_job_split_covers_every_row_once():
    """The strong-scaling job: 4096 rows in 16 micro-batches of 256, dealt to 1/2/4/8 ranks."""
    from julia1.replicas import rank_share
    lens = [bench.SEQ] * bench.JOB_ROWS
    for world in (1, 2, 4, 8):
        shares = [rank_share(lens, bench.BATCH_ROWS, bench.MAX_BATCH_TOKENS, r, world) for r in range(world)]
        assert all(len(s) == 16 // world for s in shares)
        rows = sorted(i for s in shares for b in s for i in b)
        assert rows == list(range(bench.JOB_ROWS))


def test_traffic_table_parses_committed_profile():
    t = bench.traffic_table()
    if os.path.exists(os.path.join(ROOT, "profiles", "dram_traffic_per_launch.txt")):
        assert t["gemm_qkv_rope"] > 0 and t["gemm_wo_resid_ln"] > t["gemm_qkv_rope"]
