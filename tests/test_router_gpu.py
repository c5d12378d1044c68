"""Tokenized requests and the router over the CUDA engine (B200).

* Engine::logits on tokenized requests (j1_engine_logits_tokenized) gives exactly the
  logits of j1_engine_logits_encoded on the rows the reference encoder builds
  (oracle/router_ref.py restating src/encode.rs:138-195).
* The router over the engine (j1_router_create) routes exactly like the restated
  Router::route_many (src/router.rs:143-210) whose model is the same engine called 16
  rows at a time (the reference's default batch_size), with the library router at
  batch_size 16 and at 4096 (a whole round per engine call): a row's forward does not
  depend on the other rows of its batch, so the logits and the routes are the same.
"""
import numpy as np
import pytest

import julia1 as j1
from julia1 import synthetic
from oracle import router_ref as R

pytestmark = pytest.mark.gpu

CLS, SEP, MASK = 1, 2, 4
ENC = j1.EncoderOptions(cls_id=CLS, sep_id=SEP, mask_id=MASK, max_length=512, head_length=256)
REF_ENC = R.EncOpts(CLS, SEP, MASK, 512, 256)


def rand_request(rng, n_opt, head=(8, 24), opt=(4, 14), state=(50, 400), qtype=0):
    tok = lambda n: rng.integers(5, 50000, size=int(n)).tolist()  # noqa: E731
    return j1.TokenizedRequest(tok(rng.integers(*head)), [tok(rng.integers(*opt)) for _ in range(n_opt)],
                               tok(rng.integers(*state)), qtype)


def to_ref(r):
    return R.Req(list(map(int, r.head)), [list(map(int, x)) for x in r.options], list(map(int, r.state)),
                 int(r.qtype))


@pytest.fixture(scope="module")
def engine(torch_cuda):
    ck = synthetic.cached_checkpoint(seed=0, perturb=True)
    e = j1.Engine.load(ck, j1.EngineOptions(device="cuda", batch_size=64, max_batch_tokens=65536, max_length=512))
    yield e
    e.close()


def test_logits_tokenized_equal_encoded(engine):
    rng = np.random.default_rng(21)
    rows = [rand_request(rng, int(rng.integers(2, 21)), qtype=int(rng.integers(0, 2))) for _ in range(40)]
    rows.append(rand_request(rng, 2, qtype=2))
    got = engine.logits_tokenized(rows, ENC)
    enc = []
    for r in rows:
        ids, mk, _ = R.encode_sequence(REF_ENC, to_ref(r))
        enc.append(j1.Encoded(np.array(ids, np.uint32), np.array(mk, np.uint32), int(r.qtype)))
    want = engine.logits_encoded(enc)
    assert got == want  # bitwise
    with pytest.raises(j1.J1Error, match="JSONL line 1: options must contain 2–20"):
        engine.logits_tokenized([rand_request(rng, 21)], ENC)


def test_router_over_engine_matches_reference(engine):
    rng = np.random.default_rng(22)
    rows = [rand_request(rng, int(n)) for n in rng.choice([2, 7, 20, 21, 45, 100], size=24)]
    rows.append(rows[5])

    def model(reqs):  # the reference's Engine::logits on one chunk of batch_size jobs
        enc = []
        for q in reqs:
            ids, mk, _ = R.encode_sequence(REF_ENC, q)
            enc.append(j1.Encoded(np.array(ids, np.uint32), np.array(mk, np.uint32), int(q.qtype)))
        return engine.logits_encoded(enc)

    want, want_rows, want_hits = R.Router(model, width=20, survivors=2, batch_size=16).route_many(
        [to_ref(r) for r in rows])
    for bs in (16, 4096):
        router = j1.Router(engine=engine, encoder=ENC, width=20, survivors=2, batch_size=bs)
        got = router.route_many(rows)
        router.close()
        for g, w in zip(got, want):
            assert (g.index, g.candidates, g.rounds, g.hierarchical) == \
                (w.index, w.candidates, w.rounds, w.hierarchical)
            np.testing.assert_allclose(g.probabilities, w.probabilities, rtol=0, atol=1e-12)
            assert (g.model_rows, g.cache_hits) == (want_rows, want_hits)
        assert any(g.hierarchical for g in got) and any(not g.hierarchical for g in got)


def test_engine_logits_on_text(engine, tmp_path):
    """Engine::logits on text requests (text encoder + tokenized path) equals logits_encoded
    on the rows the text encoder builds (Encoder::encode), bitwise."""
    import json
    import os
    golden = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    with open(os.path.join(golden, "tokenizer_nfc.json"), encoding="utf-8") as f:
        (tmp_path / "tokenizer.json").write_text(f.read(), encoding="utf-8")
    (tmp_path / "tokenizer_config.json").write_text(json.dumps(
        {"mask_token": "[MASK]", "cls_token": "[CLS]", "sep_token": "[SEP]", "pad_token": "[PAD]"}))
    tenc = j1.TextEncoder.load(str(tmp_path), max_length=512)
    rng = np.random.default_rng(4)
    words = ["north", "south", "gold", "wood", "attack", "defend", "trade", "café", "Ελλάδα", "日本語", "[MASK]"]
    reqs = [j1.Request(" ".join(rng.choice(words, size=int(rng.integers(10, 200)))), "which move?",
                       [" ".join(rng.choice(words, size=int(rng.integers(1, 4)))) for _ in range(int(n))],
                       qtype=("score" if i % 3 == 1 else "choice"))
            for i, n in enumerate(rng.integers(2, 21, size=30))]
    got = engine.logits(reqs, tenc)
    rows = [tenc.encode(r.state, r.question, r.options, r.qtype)[0] for r in reqs]
    assert got == engine.logits_encoded(rows)
    assert all(len(g) == len(r.options) for g, r in zip(got, reqs))


def test_engine_logits_on_text_pipelined_chunks(engine, tmp_path):
    """With more rows than one pipeline chunk (four engine micro-batches: 256 rows here),
    text encoding of chunk k + 1 overlaps the forward of chunk k; the logits equal the
    encode-everything-then-score result bitwise, and an encoding error in a later chunk is
    reported with its own line number (Engine::encode's order) before any forward error."""
    import json
    import os
    golden = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    with open(os.path.join(golden, "tokenizer_nfc.json"), encoding="utf-8") as f:
        (tmp_path / "tokenizer.json").write_text(f.read(), encoding="utf-8")
    (tmp_path / "tokenizer_config.json").write_text(json.dumps(
        {"mask_token": "[MASK]", "cls_token": "[CLS]", "sep_token": "[SEP]", "pad_token": "[PAD]"}))
    rng = np.random.default_rng(9)
    words = ["north", "south", "gold", "wood", "attack", "defend", "trade", "café", "Ελλάδα", "日本語"]
    reqs = [j1.Request(" ".join(rng.choice(words, size=int(rng.integers(5, 400)))), "which move %d?" % i,
                       [" ".join(rng.choice(words, size=int(rng.integers(1, 4)))) for _ in range(int(n))],
                       qtype=("score" if i % 3 == 1 else "choice"))
            for i, n in enumerate(rng.integers(2, 21, size=700))]
    tenc = j1.TextEncoder.load(str(tmp_path), max_length=512)
    got = engine.logits(reqs, tenc)
    encoded = [e for e, _ in tenc.encode_batch(reqs, threads=4)]
    assert got == engine.logits_encoded(encoded)
    tb = j1.TextBatch(reqs)  # the flat paths: same bits
    flat = engine.logits(tb, tenc, flat=True)
    assert flat.tolist() == [v for row in got for v in row]
    assert np.array_equal(engine.logits_flat(tenc.encode_batch(tb, threads=4, flat=True)), flat)
    strict = j1.TextEncoder.load(str(tmp_path), max_length=512, strict=True)
    bad = [j1.Request(" ".join(rng.choice(words, size=int(rng.integers(5, 30)))), "which move?",
                      [str(rng.choice(words)) for _ in range(int(rng.integers(2, 6)))]) for _ in range(700)]
    assert len(engine.logits(bad, strict)) == 700  # small rows: strict mode accepts all of them
    bad[600] = j1.Request("a state with [MASK] in it", "which?", ["left", "right"])
    with pytest.raises(j1.J1Error, match="JSONL line 601: Reserved model marker in request"):
        engine.logits(bad, strict)
