"""Thread safety of the boundary (B200): a model handle and an engine handle are shared by
several host threads (the reference's `unsafe impl Send + Sync` with the forward under a
mutex, src/cuda/mod.rs:165-167,414-415; Engine::lock, src/engine.rs:78,226). Concurrent calls
from Python threads (ctypes releases the GIL, so the C calls overlap) give exactly the
results of the same calls made one after another."""
import threading

import numpy as np
import pytest

import julia1 as j1
from julia1 import synthetic

pytestmark = pytest.mark.gpu


def run_threads(fns):
    out, errs = [None] * len(fns), []

    def wrap(i, f):
        try:
            out[i] = f()
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    ts = [threading.Thread(target=wrap, args=(i, f)) for i, f in enumerate(fns)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs, errs
    return out


def test_model_and_engine_shared_by_threads(torch_cuda):
    ck = synthetic.cached_checkpoint(seed=0, perturb=True)
    batches = [j1.Batch.new([j1.Encoded(*r) for r in synthetic.synthetic_batch(
        [int(n) for n in np.random.default_rng(s).integers(64, 700, size=6)], seed=s, option_block=(4, 6, 8))])
        for s in range(4)]
    m = j1.CudaModel(ck, 0)
    want = [m.forward_flat(b) for b in batches]
    got = run_threads([lambda b=b: m.forward_flat(b) for b in batches] * 2)
    for i, g in enumerate(got):
        assert np.array_equal(g, want[i % 4])
    m.close()

    eng = j1.Engine.load(ck, j1.EngineOptions(device="cuda", batch_size=8, max_length=1024))
    rows = [[j1.Encoded(*r) for r in synthetic.synthetic_batch(
        [int(n) for n in np.random.default_rng(10 + s).integers(32, 900, size=12)], seed=10 + s,
        option_block=(3, 5, 6))] for s in range(3)]
    want = [eng.logits_encoded(r) for r in rows]
    got = run_threads([lambda r=r: eng.logits_encoded(r) for r in rows] * 2)
    for i, g in enumerate(got):
        assert g == want[i % 3]
    eng.close()
