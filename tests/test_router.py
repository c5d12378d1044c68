"""Requests below the tokenizer and the hierarchical router (no GPU needed).

* j1_encode_sequence == Encoder::sequence (src/encode.rs:138-195), restated in
  oracle/router_ref.py: ids, marker positions and the truncation flag on seeded random
  requests covering every branch (48-token option cap, per-option truncation when the head
  budget falls under 16, head clipped to max(budget, 8), state cut to the room left), and
  the strict-mode refusals with the reference's messages.
* j1_router_route_many == Router::route_many (src/router.rs:143-210) over a deterministic
  scorer: chosen index, final candidates (in scoring order), display probabilities, rounds,
  model rows and cache hits, with de-duplication inside a call and the LRU cache across
  calls; Router::new / validate refusals.
"""
import math
import struct

import numpy as np
import pytest

import julia1 as j1
from oracle import router_ref as R

CLS, SEP, MASK = 1, 2, 4


def to_ref(r: j1.TokenizedRequest):
    return R.Req(list(map(int, r.head)), [list(map(int, x)) for x in r.options], list(map(int, r.state)),
                 int(r.qtype))


def rand_tokens(rng, n):
    return rng.integers(5, 50000, size=n).tolist()


def rand_request(rng, n_opt, head=(0, 80), opt=(1, 60), state=(0, 700), qtype=0):
    return j1.TokenizedRequest(rand_tokens(rng, int(rng.integers(*head))),
                               [rand_tokens(rng, int(rng.integers(*opt))) for _ in range(n_opt)],
                               rand_tokens(rng, int(rng.integers(*state))), qtype)


def ref_encode_or_error(o, r):
    try:
        return R.encode_sequence(R.EncOpts(CLS, SEP, MASK, o.max_length, o.head_length, o.strict), to_ref(r)), None
    except R.RefError as e:
        return None, str(e)


def lib_encode_or_error(o, r):
    try:
        e, tr = j1.encode_sequence(r, o)
        return (e.ids.tolist(), e.markers.tolist(), tr), None
    except j1.J1Error as e:
        return None, str(e)


@pytest.mark.parametrize("strict", [False, True])
def test_encode_sequence_matches_reference(strict):
    rng = np.random.default_rng(7 + strict)
    n_cases = 0
    branches = {"cap48": 0, "per_option": 0, "head_cut": 0, "state_cut": 0, "error": 0}
    for case in range(600):
        max_length = int(rng.choice([64, 128, 512, 1024]))
        head_length = int(rng.integers(4, max_length - 4))
        o = j1.EncoderOptions(CLS, SEP, MASK, max_length=max_length, head_length=head_length, strict=strict)
        if case % 2:  # small requests: strict mode accepts most of them
            r = rand_request(rng, int(rng.integers(1, 8)), head=(0, 20), opt=(1, 12), state=(0, 40))
        else:
            r = rand_request(rng, int(rng.integers(1, 21)), head=(0, 120), opt=(1, 70), state=(0, 900))
        want, werr = ref_encode_or_error(o, r)
        got, gerr = lib_encode_or_error(o, r)
        if werr is not None:
            branches["error"] += 1
            assert gerr is not None and gerr.endswith(werr), (case, werr, gerr)
            continue
        assert gerr is None, (case, gerr)
        assert got == (list(want[0]), list(want[1]), bool(want[2])), case
        n_cases += 1
        branches["cap48"] += any(len(x) > 48 for x in r.options)
        branches["per_option"] += head_length - sum(min(len(x), 48) + 1 for x in r.options) < 16
        branches["state_cut"] += bool(want[2])
        branches["head_cut"] += len(want[0]) < 3 + len(r.head) + len(r.state) + sum(len(x) + 1 for x in r.options)
    assert n_cases > 100
    if not strict:  # every truncation path was exercised
        assert all(v > 0 for v in branches.values()), branches
    else:
        assert branches["error"] > 0


def test_encode_sequence_layout_and_refusals():
    o = j1.EncoderOptions(CLS, SEP, MASK, max_length=32, head_length=20)
    r = j1.TokenizedRequest([10, 11], [[20, 21], [22]], [30, 31, 32])
    e, tr = j1.encode_sequence(r, o)
    assert e.ids.tolist() == [CLS, 10, 11, SEP, MASK, 20, 21, MASK, 22, SEP, 30, 31, 32, SEP]
    assert e.markers.tolist() == [4, 7] and not tr
    # the mask id cannot come from cleaned text
    bad = j1.TokenizedRequest([10, MASK], [[20], [21]], [])
    with pytest.raises(j1.J1Error, match="mask token id"):
        j1.encode_sequence(bad, o)
    with pytest.raises(j1.J1Error, match="Reserved model marker in request"):
        j1.encode_sequence(bad, j1.EncoderOptions(CLS, SEP, MASK, max_length=32, head_length=20, strict=True))
    with pytest.raises(j1.J1Error, match="max_length must leave room beyond the question head"):
        j1.encode_sequence(r, j1.EncoderOptions(CLS, SEP, MASK, max_length=24, head_length=20))
    long_opt = j1.TokenizedRequest([10], [list(range(100, 150)), [22]], [])
    with pytest.raises(j1.J1Error, match="Option exceeds 48-token model contract"):
        j1.encode_sequence(long_opt, j1.EncoderOptions(CLS, SEP, MASK, max_length=512, head_length=256, strict=True))
    e, _ = j1.encode_sequence(long_opt, j1.EncoderOptions(CLS, SEP, MASK, max_length=512, head_length=256))
    assert e.markers.tolist() == [3, 52]  # the 50-token option keeps [MASK] + 48


# ------------------------------------------------------------------ router
def fake_logits(ids, markers):
    """Deterministic logits of an encoded row: a hash of the whole row and of the option,
    so that the same option scores differently in different groups; options whose first
    token is a multiple of 11 get a large margin (exercises the confident-winner path)."""
    row = 1469598103934665603
    for t in ids:
        row = ((row ^ int(t)) * 1099511628211) & (2 ** 64 - 1)
    out = []
    for k, m in enumerate(markers):
        h = ((row ^ (k * 0x9E3779B97F4A7C15)) * 1099511628211) & (2 ** 64 - 1)
        v = ((h >> 11) / float(1 << 53)) * 6.0 - 3.0
        if int(ids[m + 1]) % 11 == 0:
            v += 9.0
        out.append(struct.unpack("f", struct.pack("f", v))[0])
    return out


def lib_scorer(rows):
    return [fake_logits(r.ids.tolist(), r.markers.tolist()) for r in rows]


def ref_scorer(enc):
    def score(reqs):
        out = []
        for q in reqs:
            ids, markers, _ = R.encode_sequence(enc, q)
            out.append(fake_logits(ids, markers))
        return out
    return score


ENC = dict(cls_id=CLS, sep_id=SEP, mask_id=MASK, max_length=512, head_length=256)


def make_pair(width=20, survivors=2, batch_size=16, cache_size=0, max_options=4096):
    lr = j1.Router(encoder=j1.EncoderOptions(**ENC), scorer=lib_scorer, width=width, survivors=survivors,
                   batch_size=batch_size, cache_size=cache_size, max_options=max_options)
    rr = R.Router(ref_scorer(R.EncOpts(CLS, SEP, MASK, 512, 256)), width=width, survivors=survivors,
                  batch_size=batch_size, cache_size=cache_size, max_options=max_options)
    return lr, rr


def check_same(got, want, mr, hits):
    res, want_mr, want_hits = want
    assert len(got) == len(res)
    for g, w in zip(got, res):
        assert g.index == w.index
        assert g.candidates == w.candidates
        assert g.rounds == w.rounds and g.hierarchical == w.hierarchical
        assert g.probability_scope == ("final_candidates" if w.hierarchical else "all_options")
        np.testing.assert_allclose(g.probabilities, w.probabilities, rtol=0, atol=1e-12)
        assert abs(sum(g.probabilities) - 1.0) < 1e-9
        assert (g.model_rows, g.cache_hits) == (want_mr, want_hits)


@pytest.mark.parametrize("width,survivors", [(20, 2), (5, 2), (4, 3), (3, 1)])
def test_router_matches_reference(width, survivors):
    rng = np.random.default_rng(100 + width)
    lr, rr = make_pair(width=width, survivors=survivors)
    rows = []
    for i in range(40):
        n = int(rng.choice([2, 3, width, width + 1, 2 * width + 1, 45, 100]))
        rows.append(rand_request(rng, n, head=(3, 20), opt=(1, 6), state=(0, 60)))
    rows.append(rows[3])  # a repeated request: its jobs are scored once
    got = lr.route_many(rows)
    want = rr.route_many([to_ref(r) for r in rows])
    check_same(got, want, None, None)
    assert got[0].hierarchical == (len(rows[0].options) > width)
    assert max(g.rounds for g in got) >= (3 if width <= 5 else 2) and any(g.rounds == 1 for g in got)
    assert got[-1].cache_hits > 0


def test_router_small_types_and_single_request():
    lr, rr = make_pair()
    rng = np.random.default_rng(3)
    rows = [rand_request(rng, 2, qtype=2), rand_request(rng, 5, qtype=1), rand_request(rng, 20)]
    check_same(lr.route_many(rows), rr.route_many([to_ref(r) for r in rows]), None, None)
    one = lr.route(rows[2])
    assert one.rounds == 1 and not one.hierarchical and one.probability_scope == "all_options"


def test_router_cache_and_lru():
    rng = np.random.default_rng(11)
    rows = [rand_request(rng, int(n), head=(3, 10), opt=(1, 4), state=(0, 20)) for n in (30, 7, 45, 2)]
    lr, rr = make_pair(cache_size=4)
    for _ in range(3):  # the second and third calls hit the (small) LRU cache like LruCache does
        check_same(lr.route_many(rows), rr.route_many([to_ref(r) for r in rows]), None, None)
    lr.clear_cache()
    rr.clear_cache()
    check_same(lr.route_many(rows), rr.route_many([to_ref(r) for r in rows]), None, None)
    big, big_ref = make_pair(cache_size=1000)
    first = big.route_many(rows)
    second = big.route_many(rows)
    assert second[0].model_rows == 0 and second[0].cache_hits >= first[0].model_rows
    assert [g.index for g in first] == [g.index for g in second]


def test_router_refusals():
    enc = j1.EncoderOptions(**ENC)
    for kw, msg in [(dict(width=21), "Require 2 <= width <= 20"), (dict(survivors=20), "Require 2 <= width"),
                    (dict(batch_size=0), "Invalid batch/cache/capacity limit"),
                    (dict(max_options=10), "Invalid batch/cache/capacity limit")]:
        with pytest.raises(j1.J1Error, match=msg):
            j1.Router(encoder=enc, scorer=lib_scorer, **kw)
    lr = j1.Router(encoder=enc, scorer=lib_scorer, max_options=50)
    rng = np.random.default_rng(5)
    for r, msg in [(rand_request(rng, 1), "Expected 2–50 options"), (rand_request(rng, 51), "Expected 2–50 options"),
                   (rand_request(rng, 3, qtype=2), "noul requires"),
                   (rand_request(rng, 21, qtype=1), "Hierarchical routing supports choice decisions only"),
                   (j1.TokenizedRequest([5], [[6], []], []), "Options must be nonempty")]:
        with pytest.raises(j1.J1Error, match=msg):
            lr.route_many([r])
    # a failing scorer surfaces as an error, not a crash
    bad = j1.Router(encoder=enc, scorer=lambda rows: [[0.0]] * len(rows))
    with pytest.raises(j1.J1Error, match="scorer callback failed"):
        bad.route_many([rand_request(rng, 3)])
    nan = j1.Router(encoder=enc, scorer=lambda rows: [[math.nan] * len(r.markers) for r in rows])
    with pytest.raises(j1.J1Error, match="finite"):
        nan.route_many([rand_request(rng, 3)])
