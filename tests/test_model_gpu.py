"""End-to-end parity of the B200 forward (libj1 through the C ABI) on seeded inputs.

Bars: option logits within max-abs 3e-2 of the
reference's CUDA BF16 path, within 5e-2 of its FP32 CPU path, identical argmax
on rows whose top-2 gap exceeds twice the tolerance.

References used here:
  * oracle "bf16" -- CPU restatement of the reference CUDA path (src/cuda/mod.rs:446-511)
  * oracle "fp32" -- CPU restatement of the reference CPU path (src/cpu/mod.rs:201-340)
  * RefCudaModel  -- the reference's own kernels.cu (compiled unmodified, hidden 384) + cuBLAS
  * golden        -- transformers ModernBertModel + torch head, tests/golden/*.npz
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import julia1 as j1  # noqa: E402
from julia1 import synthetic  # noqa: E402
from oracle import oracle as orc  # noqa: E402

TOL_BF16 = 3e-2
TOL_FP32 = 5e-2
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rows_to_batch(rows):
    return j1.Batch.new([j1.Encoded(ids, mk, q) for ids, mk, q in rows])


def argmax_agreement(a, b, marker_starts, tol):
    agree = total = 0
    for s, e in zip(marker_starts[:-1], marker_starts[1:]):
        if e - s < 2:
            continue
        ref = np.sort(b[s:e])
        if ref[-1] - ref[-2] <= 2 * tol:
            continue
        total += 1
        agree += int(np.argmax(a[s:e]) == np.argmax(b[s:e]))
    return agree, total


@pytest.fixture(scope="module")
def ckpt768():
    return synthetic.cached_checkpoint(seed=0, perturb=True)


@pytest.fixture(scope="module")
def model768(torch_cuda, ckpt768):
    m = j1.CudaModel(ckpt768, 0)
    yield m
    m.close()


@pytest.fixture(scope="module")
def oracle768(ckpt768):
    return orc.Oracle(ckpt768)


def test_model_name_and_config(model768):
    assert model768.name().startswith("cuda:0 (")
    c = model768.config()
    assert (c.hidden, c.heads, c.layers, c.intermediate, c.half_window, c.n_global) == (768, 12, 22, 1152, 64, 8)


def test_c1_parity_4x512(model768, oracle768):
    """Config 1: 4 x 512 tokens, 22 layers; random-id markers so the logits are spread."""
    rows = synthetic.synthetic_batch([512] * 4, markers_per_seq=8, seed=101, mask_markers=False)
    b = rows_to_batch(rows)
    gpu = model768.forward_flat(b)
    ref16 = oracle768.forward_flat(b, mode="bf16")
    ref32 = oracle768.forward_flat(b, mode="fp32")
    d16, d32 = np.abs(gpu - ref16).max(), np.abs(gpu - ref32).max()
    print("C1 spread %.4f  max|gpu-bf16| %.5f  max|gpu-fp32| %.5f  max|bf16-fp32| %.5f" %
          (ref32.max() - ref32.min(), d16, d32, np.abs(ref16 - ref32).max()))
    assert d16 <= TOL_BF16
    assert d32 <= TOL_FP32
    agree, total = argmax_agreement(gpu, ref16, b.marker_starts, TOL_BF16)
    assert agree == total


def test_ragged_parity(model768, oracle768):
    """Config 3 shape family: ragged lengths U[16, 1024] packed varlen (16 sequences here)."""
    rng = np.random.default_rng(3)
    lens = rng.integers(16, 1025, size=16).tolist()
    rows = synthetic.synthetic_batch(lens, markers_per_seq=6, seed=103, mask_markers=False)
    b = rows_to_batch(rows)
    gpu = model768.forward_flat(b)
    ref16 = oracle768.forward_flat(b, mode="bf16")
    assert np.abs(gpu - ref16).max() <= TOL_BF16
    agree, total = argmax_agreement(gpu, ref16, b.marker_starts, TOL_BF16)
    assert agree == total


def test_long_sequence_2048_parity(model768, oracle768):
    """Many key blocks per query tile on the global layers (online softmax across 16 blocks)."""
    rows = synthetic.synthetic_batch([2048], markers_per_seq=12, seed=105, mask_markers=False)
    b = rows_to_batch(rows)
    gpu = model768.forward_flat(b)
    ref32 = oracle768.forward_flat(b, mode="fp32")
    assert np.abs(gpu - ref32).max() <= TOL_FP32


def test_c3_ragged_64_full_size(model768, oracle768):
    """Config 3 at full size: 64 sequences, lengths U[16, 1024], packed varlen (~33K tokens),
    against the BF16-chain oracle; every row's argmax where the top-2 gap is resolvable."""
    rng = np.random.default_rng(2024)
    lens = rng.integers(16, 1025, size=64).tolist()
    rows = synthetic.synthetic_batch(lens, markers_per_seq=4, seed=140, mask_markers=False)
    b = rows_to_batch(rows)
    gpu = model768.forward_flat(b)
    ref16 = oracle768.forward_flat(b, mode="bf16")
    d = np.abs(gpu - ref16)
    print("C3 t=%d max|gpu-bf16| %.5f mean %.6f" % (b.tokens(), d.max(), d.mean()))
    assert d.max() <= TOL_BF16
    assert np.abs(gpu - ref16).max() <= 2e-2 * max(1.0, np.abs(ref16).max())
    agree, total = argmax_agreement(gpu, ref16, b.marker_starts, TOL_BF16)
    assert agree == total


def test_c4_8192_parity(model768, oracle768):
    """Config 4 sequence length (8192 = max_position_embeddings): global layers attend over
    all 8192 keys (128 key blocks of 64 per query tile); against the BF16-chain oracle."""
    rows = synthetic.synthetic_batch([8192], markers_per_seq=24, seed=141, mask_markers=False)
    b = rows_to_batch(rows)
    gpu = model768.forward_flat(b)
    ref16 = oracle768.forward_flat(b, mode="bf16")
    d = np.abs(gpu - ref16)
    print("C4 max|gpu-bf16| %.5f mean %.6f" % (d.max(), d.mean()))
    assert d.max() <= TOL_BF16


def test_c5_router_scale_256x512_full_size(model768, oracle768):
    """Config 5's per-forward batch at full size, the bench workload: 256 rows x 512 tokens
    (131,072 tokens), 20 option markers per row in Encoder::sequence's layout
    (src/encode.rs:167-187), m = 5,120. Over the whole batch: finite, deterministic, and
    sampled rows score bit for bit as they do alone; a slice of rows against the BF16-chain
    oracle. Because a row's scores do not depend on the rest of its batch (exactly), the
    slice's parity carries to every row of the full-size batch."""
    rows = synthetic.synthetic_batch([512] * 256, markers_per_seq=0, seed=1, option_block=(20, 11, 12),
                                     mask_markers=False)
    b = rows_to_batch(rows)
    a = model768.forward_flat(b)
    assert b.tokens() == 131072 and a.size == 256 * 20 and np.isfinite(a).all()
    assert np.array_equal(a, model768.forward_flat(b))
    for i in (0, 131, 255):
        alone = model768.forward_flat(rows_to_batch([rows[i]]))
        assert np.array_equal(alone, a[b.marker_starts[i]:b.marker_starts[i + 1]])
    part = rows_to_batch(rows[:6])
    ref16 = oracle768.forward_flat(part, mode="bf16")
    d = np.abs(a[:ref16.size] - ref16)
    print("C5 slice max|gpu-bf16| %.5f mean %.6f" % (d.max(), d.mean()))
    assert d.max() <= TOL_BF16
    agree, total = argmax_agreement(a[:ref16.size], ref16, part.marker_starts, TOL_BF16)
    assert agree == total


def test_batching_invariance_exact(model768):
    """tests/checkpoint.rs:91-105 property; here the per-row math is independent of the batch: exact."""
    rows = synthetic.synthetic_batch([300, 17, 129, 512, 1000, 64], markers_per_seq=5, seed=107, mask_markers=False)
    together = model768.forward(rows_to_batch(rows))
    for r, exp in zip(rows, together):
        alone = model768.forward(rows_to_batch([r]))[0]
        assert alone == exp


def test_long_context_2x8192_properties(model768):
    """Config 4 (2 x 8192): finite, deterministic, and each sequence scores as it does alone."""
    rows = synthetic.synthetic_batch([8192, 8192], markers_per_seq=20, seed=109, mask_markers=False)
    b = rows_to_batch(rows)
    a = model768.forward_flat(b)
    assert np.isfinite(a).all()
    assert np.array_equal(a, model768.forward_flat(b))
    first = model768.forward_flat(rows_to_batch(rows[:1]))
    assert np.array_equal(first, a[:first.size])


def test_engine_micro_batching_matches_model(torch_cuda, ckpt768, model768):
    rows = synthetic.synthetic_batch([40, 700, 33, 512, 90, 1, 260], markers_per_seq=3, seed=111, mask_markers=False)
    eng = j1.Engine.load(ckpt768, j1.EngineOptions(device="cuda:0", batch_size=3, max_batch_tokens=8192))
    try:
        got = eng.logits_encoded([j1.Encoded(*r) for r in rows])
        assert eng.device_name().startswith("cuda:0")
    finally:
        eng.close()
    for r, g in zip(rows, got):
        assert g == model768.forward(rows_to_batch([r]))[0]
    assert got[5] == []  # a 1-token row has no markers


def test_engine_pool_matches_model(torch_cuda, ckpt768, model768):
    """A pool engine (one replica + host worker per device) gives the single-model
    logits bit for bit; with one visible GPU the pool holds two replicas on it."""
    n = torch_cuda.cuda.device_count()
    devices = list(range(min(n, 4))) if n >= 2 else [0, 0]
    lens = np.random.default_rng(5).integers(1, 900, size=23).tolist()
    rows = synthetic.synthetic_batch(lens, markers_per_seq=2, seed=112, mask_markers=False)
    eng = j1.Engine.load(ckpt768, j1.EngineOptions(batch_size=2, max_batch_tokens=4096, max_length=1024),
                      devices=devices)
    try:
        got = eng.logits_encoded([j1.Encoded(*r) for r in rows])
    finally:
        eng.close()
    want = model768.forward(rows_to_batch(rows))
    assert got == [list(w) for w in want]


def test_forward_many_matches_single_forwards(model768):
    """j1_model_forward_many (staging of batch k+1 overlapped with forward k) gives each
    batch's single-forward scores bit for bit, for batches of different sizes."""
    rng = np.random.default_rng(7)
    batches = []
    for i in range(5):
        lens = rng.integers(1, 700, size=int(rng.integers(1, 9))).tolist()
        batches.append(rows_to_batch(synthetic.synthetic_batch(lens, markers_per_seq=3, seed=120 + i,
                                                               mask_markers=False)))
    got = model768.forward_many(batches)
    for b, g in zip(batches, got):
        assert np.array_equal(g, model768.forward_flat(b))
    assert model768.forward_many([]) == []


def test_forward_many_validates_every_batch_first(model768):
    good = rows_to_batch(synthetic.synthetic_batch([64, 64], markers_per_seq=2, seed=131))
    ids = good.ids.copy()
    ids[0] = 50368  # out of vocabulary
    bad = j1.Batch(ids, good.starts, good.lens, good.qtypes, good.marker_rows, good.marker_starts)
    with pytest.raises(j1.J1Error) as e:
        model768.forward_many([good, bad, good])
    assert e.value.status == j1.INVALID_ARG and "batch 1" in str(e.value)
    assert np.array_equal(model768.forward_many([good])[0], model768.forward_flat(good))


def test_forward_rejects_bad_batches(model768):
    rows = synthetic.synthetic_batch([64, 64], markers_per_seq=2, seed=113)
    b = rows_to_batch(rows)
    bad = j1.Batch(b.ids, b.starts, b.lens, b.qtypes, b.marker_rows.copy(), b.marker_starts)
    bad.marker_rows[-1] = 10  # belongs to sequence 0, listed under sequence 1
    with pytest.raises(j1.J1Error) as e:
        model768.forward_flat(bad)
    assert e.value.status == j1.INVALID_ARG
    ids = b.ids.copy()
    ids[3] = 50368
    with pytest.raises(j1.J1Error) as e:
        model768.forward_flat(j1.Batch(ids, b.starts, b.lens, b.qtypes, b.marker_rows, b.marker_starts))
    assert e.value.status == j1.INVALID_ARG
    # the model stays usable after rejected calls
    assert np.isfinite(model768.forward_flat(b)).all()
    assert model768.forward_flat(j1.Batch.new([])).size == 0


# ------------------------------------------------------------------ hidden 384 (the reference kernels' width)
@pytest.fixture(scope="module")
def j384(tmp_path_factory):
    z = np.load(os.path.join(GOLDEN, "j384_fp32.npz"))
    shape = {str(k): int(v) for k, v in zip(z["shape_keys"], z["shape"])}
    root = synthetic.write_checkpoint(str(tmp_path_factory.mktemp("j384")), seed=int(z["seed"]), perturb=True,
                                      **shape)
    rows, o, om = [], 0, 0
    for L, q, nm in zip(z["lens"], z["qtypes"], z["row_markers"]):
        rows.append((z["ids"][o:o + L], z["markers"][om:om + nm], int(q)))
        o += L
        om += nm
    return z, root, rows


def test_h384_against_golden(torch_cuda, j384):
    z, root, rows = j384
    m = j1.CudaModel(root, 0)
    try:
        gpu = m.forward_flat(rows_to_batch(rows))
    finally:
        m.close()
    assert np.abs(gpu - z["logits"]).max() <= TOL_FP32


def test_h384_against_reference_cuda_kernels(torch_cuda, j384):
    """The reference's own kernels.cu + cuBLAS vs (a) the BF16 oracle and (b) libj1."""
    from oracle import ref_cuda
    z, root, rows = j384
    # a bigger ragged batch on the same checkpoint as well
    more = synthetic.synthetic_batch([300, 129, 64, 513, 2], markers_per_seq=4, seed=115, vocab=2000,
                                     mask_markers=False)
    for rr in (rows, more):
        b = rows_to_batch(rr)
        ref = ref_cuda.RefCudaModel(root, torch_cuda).forward_flat(b)
        o16 = orc.Oracle(root).forward_flat(b, mode="bf16")
        m = j1.CudaModel(root, 0)
        try:
            gpu = m.forward_flat(b)
        finally:
            m.close()
        print("h384: max|ref-oracle16| %.2e  max|ref-libj1| %.2e" % (np.abs(ref - o16).max(), np.abs(ref - gpu).max()))
        assert np.abs(ref - o16).max() <= 5e-3  # the restatement follows the reference chain closely
        assert np.abs(ref - gpu).max() <= TOL_BF16
