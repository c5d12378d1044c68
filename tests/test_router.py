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


# ------------------------------------------------------------------ known answers of the reference's tests
# tests/api.rs:139-215: the "Numeric" engine scores an option by its numeric label; here
# option i is the single token LABEL0 + i and the scorer reads it back after each marker.
LABEL0 = 1000


def numeric_request(n, qtype=0):
    return j1.TokenizedRequest([11, 12, 13], [[LABEL0 + i] for i in range(n)], [21, 22], qtype)


class Numeric:
    def __init__(self, scale):
        self.scale, self.calls = scale, []

    def lib(self, rows):  # encoded rows (library scorer callback)
        self.calls.append([len(r.markers) for r in rows])
        return [[np.float32(self.scale * float(int(r.ids[m + 1]) - LABEL0)) for m in r.markers] for r in rows]

    def ref(self, reqs):  # requests (oracle router)
        self.calls.append([len(q.options) for q in reqs])
        return [[float(np.float32(self.scale * float(o[0] - LABEL0))) for o in q.options] for q in reqs]


def both(scale, **kw):
    a, b = Numeric(scale), Numeric(scale)
    return (j1.Router(encoder=j1.EncoderOptions(**ENC), scorer=a.lib, **kw), a), (R.Router(b.ref, **kw), b)


def test_reference_router_direct_and_hierarchical():
    (lr, la), (rr, ra) = both(1.0, width=20, survivors=2, batch_size=3, cache_size=0, max_options=4096)
    sizes = [2, 20, 21, 77, 4096]
    got = lr.route_many([numeric_request(n) for n in sizes])
    want, _, _ = rr.route_many([to_ref(numeric_request(n)) for n in sizes])
    for res in (got, want):
        assert [r.index for r in res] == [1, 19, 20, 76, 4095]
        for r in res:
            assert abs(sum(r.probabilities) - 1.0) < 1e-9 and r.index in r.candidates
    assert got[0].probability_scope == "all_options" and got[4].probability_scope == "final_candidates"
    for calls in (la.calls, ra.calls):  # every engine call holds at most batch_size rows of 2..20 options
        assert all(len(c) <= 3 for c in calls) and all(2 <= n <= 20 for c in calls for n in c)
    assert la.calls == ra.calls
    assert lr.route_many([]) == []


def test_reference_router_confident_group_shortcut():
    for cw in (j1.Router.confident_winner, R.confident_winner):
        assert cw([0.0, 4.0, -3.0], 1)
        assert not cw([0.0, 3.0, -3.0], 1)
    (lr, _), (rr, _) = both(10.0)
    r = lr.route(numeric_request(2001))
    assert (r.index, r.rounds, r.model_rows) == (2000, 3, 106)
    w, rows, _ = rr.route_many([to_ref(numeric_request(2001))])
    assert (w[0].index, w[0].rounds, rows) == (2000, 3, 106)


def test_reference_router_cache_and_dedup():
    (lr, _), (rr, _) = both(1.0, width=20, survivors=2, batch_size=16, cache_size=1, max_options=4096)
    got = lr.route_many([numeric_request(5), numeric_request(5)])
    assert (got[0].model_rows, got[0].cache_hits) == (1, 1)
    assert lr.route(numeric_request(5)).model_rows == 0
    lr.clear_cache()
    assert lr.route(numeric_request(5)).model_rows == 1
    lr.route(numeric_request(6))
    assert lr.route(numeric_request(5)).model_rows == 1
    # the restated router, same sequence
    assert rr.route_many([to_ref(numeric_request(5))] * 2)[1:] == (1, 1)
    assert rr.route_many([to_ref(numeric_request(5))])[1] == 0
    rr.clear_cache()
    assert rr.route_many([to_ref(numeric_request(5))])[1] == 1
    rr.route_many([to_ref(numeric_request(6))])
    assert rr.route_many([to_ref(numeric_request(5))])[1] == 1


def test_reference_router_rejects_invalid_and_bad_engines():
    (lr, _), (rr, _) = both(1.0)
    for row in (numeric_request(1), numeric_request(30, qtype=1), numeric_request(3, qtype=2)):
        with pytest.raises(j1.J1Error):
            lr.route(row)
        with pytest.raises(R.RefError):
            rr.route_many([to_ref(row)])
    fixed = j1.Router(encoder=j1.EncoderOptions(**ENC), scorer=lambda rows: [[0.0]] * len(rows))
    with pytest.raises(j1.J1Error):
        fixed.route(numeric_request(4))
    assert R.argmax([3, 3, -1]) == 0


def test_reference_display_probabilities():
    for dp in (j1.display_probabilities, R.display_probabilities):
        assert dp([0.955, 0.044, 0.001]) == [1.0, 0.0, 0.0]
        assert dp([0.951, 0.049]) != [1.0, 0.0]
        r = dp([0.6, 0.395, 0.005])
        assert r[2] == 0.0 and abs(sum(r) - 1.0) < 1e-12 and abs(r[0] / r[1] - 0.6 / 0.395) < 1e-12
        assert dp([]) == []
