"""Failure detection without a GPU fault (B200). Every failure is made on the host or by a
bounded device wait that runs out, never by faulting or hanging the GPU:
* injected allocation / launch failures, nonfinite scores and a failing host worker thread
  (j1_inject_fault) come back as J1_ERR_OOM / J1_ERR_CUDA / J1_ERR_NONFINITE / J1_ERR_INTERNAL ("Inference returned nonfinite logits",
  src/engine.rs:219-221) through the model, the engine and the router, and the same handle
  then computes the right logits again;
* a device wait on a barrier nothing arrives at times out after its limit, is reported as
  J1_ERR_DEVICE_TIMEOUT, and the context stays usable.
"""
import numpy as np
import pytest

import julia1 as j1
from julia1 import synthetic

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ckpt():
    return synthetic.cached_checkpoint(seed=0, perturb=True)


@pytest.fixture(scope="module")
def batch():
    return j1.Batch.new([j1.Encoded(*r) for r in synthetic.synthetic_batch([300, 512, 77], seed=3,
                                                                            option_block=(4, 6, 8))])


@pytest.fixture(scope="module")
def clean(torch_cuda, ckpt, batch):
    m = j1.CudaModel(ckpt, 0)
    want = m.forward_flat(batch)
    m.close()
    return want


def test_injected_faults_on_a_model(torch_cuda, ckpt, batch, clean):
    m = j1.CudaModel(ckpt, 0)
    try:
        for kind, status, text in [(j1.FAULT_ALLOC, j1.OOM, "out of device memory"),
                                   (j1.FAULT_LAUNCH, j1.CUDA, "injected launch failure"),
                                   (j1.FAULT_NAN, j1.NONFINITE, "Inference returned nonfinite logits")]:
            j1.inject_fault(kind, 1)
            with pytest.raises(j1.J1Error, match=text) as e:
                m.forward_flat(batch)
            assert e.value.status == status
            assert np.array_equal(m.forward_flat(batch), clean)  # the same handle recovers
    finally:
        for k in (j1.FAULT_ALLOC, j1.FAULT_LAUNCH, j1.FAULT_NAN):
            j1.inject_fault(k, 0)
        m.close()


def test_injected_faults_through_engine_and_router(torch_cuda, ckpt):
    eng = j1.Engine.load(ckpt, j1.EngineOptions(device="cuda", batch_size=4, max_length=1024))
    rows = [j1.Encoded(*r) for r in synthetic.synthetic_batch([200, 350, 90, 512, 64], seed=8,
                                                              option_block=(3, 5, 6))]
    want = eng.logits_encoded(rows)
    j1.inject_fault(j1.FAULT_LAUNCH, 1)
    with pytest.raises(j1.J1Error, match="injected launch failure"):
        eng.logits_encoded(rows)
    assert eng.logits_encoded(rows) == want
    j1.inject_fault(j1.FAULT_WORKER, 1)  # the engine's device worker throws on the host
    with pytest.raises(j1.J1Error, match="injected worker failure") as e:
        eng.logits_encoded(rows)
    assert e.value.status == j1.INTERNAL
    assert eng.logits_encoded(rows) == want
    enc = j1.EncoderOptions(cls_id=1, sep_id=2, mask_id=4, max_length=512)
    router = j1.Router(engine=eng, encoder=enc)
    rng = np.random.default_rng(2)
    req = j1.TokenizedRequest(rng.integers(5, 50000, 12).tolist(),
                              [rng.integers(5, 50000, 4).tolist() for _ in range(30)], rng.integers(5, 50000, 80).tolist())
    good = router.route(req)
    j1.inject_fault(j1.FAULT_NAN, 1)
    with pytest.raises(j1.J1Error) as e:
        router.route(req)
    assert e.value.status == j1.NONFINITE
    assert router.route(req).index == good.index
    router.close()
    eng.close()


def test_device_wait_timeout_is_reported(torch_cuda, ckpt, batch, clean):
    st = j1.selftest_device_timeout(0, 2_000_000)  # about a millisecond
    assert st == j1.DEVICE_TIMEOUT
    assert "site 99" in j1.last_error()
    m = j1.CudaModel(ckpt, 0)  # the context is still usable
    assert np.array_equal(m.forward_flat(batch), clean)
    m.close()
