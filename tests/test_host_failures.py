"""Host-side failures inside the library come back as statuses (CPU only, no GPU fault).

The C ABI must never let a C++ exception unwind into its caller (a C, Rust or ctypes
frame cannot survive one) nor let a host worker thread end the process. The failures are
injected on the host: J1_FAULT_HOST makes an entry point's body throw std::bad_alloc
(-> J1_ERR_OOM), J1_FAULT_WORKER makes a host worker thread of the tokenizer / text encoder
pools throw (-> J1_ERR_INTERNAL). After each failure the same call succeeds with the same
answer as before.
"""
import json
import math
import os
import threading

import pytest

import julia1 as j1

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(autouse=True)
def disarm():
    yield
    for k in (j1.FAULT_HOST, j1.FAULT_WORKER, j1.FAULT_THREAD):
        j1.inject_fault(k, 0)


@pytest.fixture(scope="module")
def tok():
    return j1.Tokenizer.from_file(os.path.join(GOLDEN, "tokenizer_nfc.json"))


@pytest.fixture(scope="module")
def enc(tmp_path_factory):
    d = tmp_path_factory.mktemp("enc_fail")
    with open(os.path.join(GOLDEN, "tokenizer_nfc.json"), encoding="utf-8") as f:
        (d / "tokenizer.json").write_text(f.read(), encoding="utf-8")
    (d / "tokenizer_config.json").write_text(json.dumps(
        {"mask_token": "[MASK]", "cls_token": "[CLS]", "sep_token": "[SEP]", "pad_token": "[PAD]"}))
    return j1.TextEncoder.load(str(d), max_length=128, head_length=48)


def test_internal_status_name():
    assert j1.lib().j1_status_name(j1.INTERNAL) == b"J1_ERR_INTERNAL"


def test_entry_point_exception_becomes_oom():
    want = j1.plan_batches([5, 700, 9, 33], batch_size=2)
    j1.inject_fault(j1.FAULT_HOST, 1)
    with pytest.raises(j1.J1Error, match="j1_plan_batches: host memory exhausted") as e:
        j1.plan_batches([5, 700, 9, 33], batch_size=2)
    assert e.value.status == j1.OOM
    assert j1.plan_batches([5, 700, 9, 33], batch_size=2) == want


def test_value_entry_points_survive_host_faults(tok):
    probs = j1.display_probabilities([0.5, 0.3, 0.2])
    tid = tok.token_to_id("[MASK]")
    j1.inject_fault(j1.FAULT_HOST, 1)
    assert all(math.isnan(p) for p in j1.display_probabilities([0.5, 0.3, 0.2]))
    assert "host memory exhausted" in j1.last_error()
    j1.inject_fault(j1.FAULT_HOST, 1)
    assert j1.Router.confident_winner([5.0, -3.0], 0) is False  # no answer rather than a crash
    j1.inject_fault(j1.FAULT_HOST, 1)
    assert tok.token_to_id("[MASK]") is None
    assert j1.display_probabilities([0.5, 0.3, 0.2]) == probs
    assert j1.Router.confident_winner([5.0, -3.0], 0) is True
    assert tok.token_to_id("[MASK]") == tid


def test_tokenizer_worker_exception_becomes_internal(tok):
    texts = ["the game state %d: café, naïve, 日本語 — move %d" % (i, i * 7) for i in range(300)]
    want = tok.encode_batch(texts, threads=1)
    for threads in (1, 4):
        j1.inject_fault(j1.FAULT_WORKER, 1)
        with pytest.raises(j1.J1Error, match="injected worker failure") as e:
            tok.encode_batch(texts, threads=threads)
        assert e.value.status == j1.INTERNAL
        assert tok.encode_batch(texts, threads=threads) == want


def test_text_encoder_worker_exception_becomes_internal(enc):
    rows = [j1.Request("state %d with [MASK] text" % i, "which move %d?" % i, ["win", "lose %d" % i, "draw"])
            for i in range(64)]
    want = enc.encode_batch(rows, threads=1)
    j1.inject_fault(j1.FAULT_WORKER, 1)
    with pytest.raises(j1.J1Error, match="injected worker failure") as e:
        enc.encode_batch(rows, threads=4)
    assert e.value.status == j1.INTERNAL
    got = enc.encode_batch(rows, threads=4)
    assert [(r.ids.tolist(), r.markers.tolist(), t) for r, t in got] == \
        [(r.ids.tolist(), r.markers.tolist(), t) for r, t in want]


def test_concurrent_calls_with_faults_armed(tok):
    """Many host threads call guarded entry points while faults fire: each call either
    succeeds with the right answer or reports OOM/INTERNAL; none takes the process down."""
    texts = ["row %d of the batch" % i for i in range(64)]
    want_ids = tok.encode_batch(texts, threads=1)
    want_plan = j1.plan_batches([5, 700, 9, 33], batch_size=2)
    j1.inject_fault(j1.FAULT_HOST, 40)
    j1.inject_fault(j1.FAULT_WORKER, 10)
    outcomes = []
    lock = threading.Lock()

    def worker(k):
        for _ in range(20):
            try:
                ok = (tok.encode_batch(texts, threads=2) == want_ids) if k % 2 else \
                    (j1.plan_batches([5, 700, 9, 33], batch_size=2) == want_plan)
                res = "ok" if ok else "wrong"
            except j1.J1Error as e:
                res = e.status
            with lock:
                outcomes.append(res)

    ths = [threading.Thread(target=worker, args=(k,)) for k in range(8)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    assert "wrong" not in outcomes
    assert set(outcomes) <= {"ok", j1.OOM, j1.INTERNAL}
    assert outcomes.count(j1.OOM) == 40 and outcomes.count(j1.INTERNAL) >= 1


def test_threads_that_cannot_start_are_done_without(tok, enc):
    """When worker threads cannot be started, the pool finishes the work on the threads it
    has (the calling thread at least): same results, no error."""
    texts = ["text %d: café 日本語 — %d" % (i, i * 3) for i in range(200)]
    want = tok.encode_batch(texts, threads=1)
    j1.inject_fault(j1.FAULT_THREAD, 1000)
    assert tok.encode_batch(texts, threads=8) == want
    rows = [j1.Request("state %d" % i, "which?", ["a", "b %d" % i]) for i in range(50)]
    got = enc.encode_batch(rows, threads=8)
    j1.inject_fault(j1.FAULT_THREAD, 0)
    ref = enc.encode_batch(rows, threads=1)
    assert [(e.ids.tolist(), t) for e, t in got] == [(e.ids.tolist(), t) for e, t in ref]
