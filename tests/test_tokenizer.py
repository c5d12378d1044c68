"""Text -> token ids (no GPU needed).

* libj1's tokenizer reproduces the reference's tokenizer library (HF `tokenizers` 0.22.2,
  pinned in the reference's Cargo.lock; Tokenizer::encode_fast(text, false),
  src/encode.rs:114-129) on the committed golden encodings of two byte-level BPE
  tokenizers (tests/golden/make_tokenizer_golden.py made them with that library), and,
  where the library is importable, on freshly generated random text.
* Batch encoding on several threads equals encoding one text at a time.
* Configurations outside the supported family are refused at load time.
* The text Encoder (src/encode.rs:25-195) builds the same rows as the restated
  Encoder::sequence (oracle/router_ref.py) over the same tokenizer, with the strict-mode
  refusal of the mask token's text and its caches.
"""
import json
import os
import random

import pytest

import julia1 as j1
from conftest import ROOT
from oracle import router_ref as R

GOLDEN = os.path.join(ROOT, "tests", "golden")
KINDS = ["nfc", "prefix"]


def load(kind):
    return j1.Tokenizer.from_file(os.path.join(GOLDEN, "tokenizer_%s.json" % kind))


@pytest.mark.parametrize("kind", KINDS)
def test_golden_encodings(kind):
    tok = load(kind)
    data = json.load(open(os.path.join(GOLDEN, "tokenizer_%s_cases.json" % kind), encoding="utf-8"))
    assert data["generator"].startswith("tokenizers 0.22")
    for text, ids in data["cases"]:
        assert tok.encode(text) == ids, repr(text)


def random_text(rng):
    blocks = [(0x20, 0x7E)] * 6 + [(0xA0, 0x17F), (0x300, 0x36F), (0x370, 0x3FF), (0x400, 0x4FF), (0x590, 0x6FF),
                                   (0x900, 0x97F), (0x1100, 0x11FF), (0x2000, 0x206F), (0x3000, 0x30FF),
                                   (0x4E00, 0x4E80), (0xAC00, 0xAC40), (0xFF00, 0xFF5E), (0x1F300, 0x1F64F)]
    extras = ["[MASK]", " [MASK] ", "[CLS]", "|||IP_ADDRESS|||", "<br>", "lol", " lol ", "'s", "'LL", "\n", "\t",
              "   ", "\r\n", "é", "각", "Å", " ", "　"]
    out = []
    for _ in range(rng.randint(0, 30)):
        if rng.random() < 0.2:
            out.append(rng.choice(extras))
        else:
            a, b = rng.choice(blocks)
            out.append(chr(rng.randint(a, b)))
    return "".join(out)


@pytest.mark.parametrize("kind", KINDS)
def test_random_text_matches_tokenizers_library(kind):
    tokenizers = pytest.importorskip("tokenizers")
    path = os.path.join(GOLDEN, "tokenizer_%s.json" % kind)
    ref = tokenizers.Tokenizer.from_file(path)
    tok = load(kind)
    rng = random.Random(1234 + len(kind))
    texts = [random_text(rng) for _ in range(3000)]
    for t in texts:
        t = t.encode("utf-8", "surrogatepass").decode("utf-8", "ignore")
        assert tok.encode(t) == ref.encode(t, add_special_tokens=False).ids, repr(t)


def test_batch_threads_and_lookup():
    tok = load("nfc")
    data = json.load(open(os.path.join(GOLDEN, "tokenizer_nfc_cases.json"), encoding="utf-8"))
    texts = [t for t, _ in data["cases"]]
    one = [tok.encode(t) for t in texts]
    assert tok.encode_batch(texts, threads=1) == one
    assert tok.encode_batch(texts, threads=4) == one
    assert tok.encode_batch([]) == []
    assert tok.token_to_id("[MASK]") == 977 and tok.token_to_id("no such token") is None
    assert tok.token_to_id("the") is not None


def test_refusals(tmp_path):
    base = json.load(open(os.path.join(GOLDEN, "tokenizer_nfc.json"), encoding="utf-8"))
    for patch, msg in [(("normalizer", {"type": "Lowercase"}), "only the NFC normalizer"),
                       (("pre_tokenizer", {"type": "Whitespace"}), "only the ByteLevel pre-tokenizer"),
                       (("model", {"type": "WordPiece", "vocab": {}}), "only BPE models")]:
        d = dict(base)
        d[patch[0]] = patch[1]
        with pytest.raises(j1.J1Error, match=msg):
            j1.Tokenizer.from_str(json.dumps(d))
    d = json.loads(json.dumps(base))
    d["model"]["unk_token"] = "[UNK]"
    with pytest.raises(j1.J1Error, match="unk_token"):
        j1.Tokenizer.from_str(json.dumps(d))
    with pytest.raises(j1.J1Error, match="cannot read"):
        j1.Tokenizer.from_file(str(tmp_path / "missing.json"))
    tok = load("nfc")
    L = j1.lib()
    import ctypes as C
    n = C.c_size_t()
    buf = (C.c_uint32 * 16)()
    for bad in (b"\xff\xfe", b"\xc0\xaf", b"\xed\xa0\x80", b"\xf4\x90\x80\x80", b"ab\xe2\x82"):
        assert L.j1_tokenizer_encode(tok._h, bad, len(bad), buf, 16, C.byref(n)) == j1.INVALID_ARG, bad
    assert tok.encode("\U0010FFFF x") == tok.encode("\U0010FFFF x")


# ------------------------------------------------------------------ text encoder
@pytest.fixture(scope="module")
def enc_dir(tmp_path_factory):
    d = tmp_path_factory.mktemp("enc")
    with open(os.path.join(GOLDEN, "tokenizer_nfc.json"), encoding="utf-8") as f:
        (d / "tokenizer.json").write_text(f.read(), encoding="utf-8")
    (d / "tokenizer_config.json").write_text(json.dumps(
        {"mask_token": "[MASK]", "cls_token": "[CLS]", "sep_token": "[SEP]", "pad_token": "[PAD]"}))
    return str(d)


def test_text_encoder_matches_reference(enc_dir):
    tok = load("nfc")
    rng = random.Random(5)
    words = ["win", "lose", "draw", "attack the left flank", "café au lait", "naïve", "日本語", "don't", "[MASK] x",
             "Ελλάδα", "été", "12 345", "lol"]
    for strict in (False, True):
        enc = j1.TextEncoder.load(enc_dir, max_length=128, head_length=48, strict=strict)
        o = enc.options()
        assert (o.cls_id, o.sep_id, o.mask_id) == (974, 975, 977)
        ro = R.EncOpts(o.cls_id, o.sep_id, o.mask_id, 128, 48, strict)
        n_ok = n_err = 0
        for _ in range(300):
            k = 1 if strict else 3  # smaller requests in strict mode, which refuses large ones
            opts = [" ".join(rng.choice(words) for _ in range(rng.randint(1, k + 1))) for _ in range(rng.randint(2, 3 * k))]
            question = " ".join(rng.choice(words) for _ in range(rng.randint(1, 4 * k)))
            state = " ".join(rng.choice(words) for _ in range(rng.randint(0, 20 * k)))
            qtype = rng.choice([0, 0, 1])
            try:
                want = R.encode_text(tok.encode, "[MASK]", ro, state, question, opts, qtype)
            except R.RefError as e:
                with pytest.raises(j1.J1Error, match=str(e).split(";")[0]):
                    enc.encode(state, question, opts, qtype)
                n_err += 1
                continue
            got, tr = enc.encode(state, question, opts, qtype)
            assert (got.ids.tolist(), got.markers.tolist(), tr) == (want[0], want[1], want[2])
            n_ok += 1
            again, _ = enc.encode(state, question, opts, qtype)  # from the encoding cache
            assert again.ids.tolist() == want[0]
        assert n_ok > 50 and (n_err > 20 or not strict)
        enc.clear_cache()
        assert enc.tokenize("the game") == tok.encode("the game")
    with pytest.raises(j1.J1Error, match="max_length must leave room"):
        j1.TextEncoder.load(enc_dir, max_length=40, head_length=48)


def test_text_requests_through_router(enc_dir):
    """Text requests: TextEncoder.tokenize_request + the router give the routes of the
    restated reference over the same tokenizer (scorer double: logits from the row ids)."""
    from test_router import lib_scorer, ref_scorer  # noqa: E402
    tok = load("nfc")
    enc = j1.TextEncoder.load(enc_dir, max_length=256, head_length=96)
    o = enc.options()
    rng = random.Random(9)
    words = ["north", "south", "gold", "wood", "attack", "defend", "trade", "café", "Ελλάδα", "[MASK]", "lol"]
    reqs = [j1.Request(" ".join(rng.choice(words) for _ in range(30)), "what next?",
                       [" ".join(rng.choice(words) for _ in range(rng.randint(1, 3))) for _ in range(n)])
            for n in (2, 5, 20, 21, 45)]
    router = j1.Router(text_encoder=enc, scorer=lib_scorer)
    got = router.route_many(reqs)
    ro = R.EncOpts(o.cls_id, o.sep_id, o.mask_id, 256, 96)
    ref = R.Router(ref_scorer(ro))

    def ref_req(r):
        clean = lambda t: t.replace("[MASK]", " ")  # noqa: E731
        return R.Req(tok.encode("choice question: " + clean(r.question)), [tok.encode(" " + clean(x)) for x in r.options],
                     tok.encode(clean(r.state)), 0)

    want, _, _ = ref.route_many([ref_req(r) for r in reqs])
    assert [g.index for g in got] == [w.index for w in want]
    assert [g.candidates for g in got] == [w.candidates for w in want]
    with pytest.raises(j1.J1Error, match="Options must be nonempty strings"):
        router.route_many([j1.Request("s", "q", ["a", ""])])


def test_text_encoder_batch_equals_single(enc_dir):
    """Engine::encode's parallel encode: the batch on 4 threads gives each row's Encoder::encode."""
    enc = j1.TextEncoder.load(enc_dir, max_length=128, head_length=48)
    rng = random.Random(12)
    words = ["win", "lose", "gold", "wood", "café", "Ελλάδα", "日本語", "[MASK]", "lol", "don't"]
    rows = [j1.Request(" ".join(rng.choice(words) for _ in range(rng.randint(0, 80))),
                       " ".join(rng.choice(words) for _ in range(rng.randint(1, 6))),
                       [" ".join(rng.choice(words) for _ in range(rng.randint(1, 3))) for _ in range(rng.randint(2, 8))],
                       qtype=rng.choice(["choice", "score"]))
            for _ in range(200)]
    got = enc.encode_batch(rows, threads=4)
    enc.clear_cache()
    for (e, tr), r in zip(got, rows):
        want, wtr = enc.encode(r.state, r.question, r.options, r.qtype)
        assert e.ids.tolist() == want.ids.tolist() and e.markers.tolist() == want.markers.tolist() and tr == wtr
    strict = j1.TextEncoder.load(enc_dir, max_length=128, head_length=48, strict=True)
    with pytest.raises(j1.J1Error, match="JSONL line 2: Reserved model marker in request"):
        strict.encode_batch([j1.Request("s", "q", ["a", "b"]), j1.Request("s [MASK]", "q", ["a", "b"])], threads=2)


def test_tokenizer_and_encoder_shared_by_threads(enc_dir):
    """One tokenizer / text encoder used from several host threads at once (per-thread BPE
    caches, mutex-guarded LRU caches) gives the single-threaded results."""
    import threading
    tok = load("nfc")
    enc = j1.TextEncoder.load(enc_dir, max_length=128, head_length=48)
    data = json.load(open(os.path.join(GOLDEN, "tokenizer_nfc_cases.json"), encoding="utf-8"))
    texts = [t for t, _ in data["cases"]]
    want = [ids for _, ids in data["cases"]]
    reqs = [j1.Request(t[:200], "which?", ["a b", "c d", "e"]) for t in texts[:100]]
    want_rows = [enc.encode(r.state, r.question, r.options)[0].ids.tolist() for r in reqs]
    enc.clear_cache()
    errs = []

    def work(k):
        try:
            order = list(range(len(texts)))
            random.Random(k).shuffle(order)
            for i in order:
                assert tok.encode(texts[i]) == want[i]
            rorder = list(range(len(reqs)))
            random.Random(k + 100).shuffle(rorder)
            for i in rorder:
                assert enc.encode(reqs[i].state, reqs[i].question, reqs[i].options)[0].ids.tolist() == want_rows[i]
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    ts = [threading.Thread(target=work, args=(k,)) for k in range(6)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs, errs[:1]


def test_text_encoder_flat_batch_equals_rows(enc_dir):
    """TextBatch + encode_batch(flat=True) gives the per-row results as flat arrays."""
    enc = j1.TextEncoder.load(enc_dir, max_length=128, head_length=48)
    rng = random.Random(12)
    words = ["win", "lose", "draw", "café", "日本語", "[MASK]", "don't", "12 345"]
    rows = [j1.Request(" ".join(rng.choice(words) for _ in range(rng.randint(0, 60))), "which %d?" % i,
                       [" ".join(rng.choice(words) for _ in range(rng.randint(1, 3))) for _ in range(rng.randint(2, 20))],
                       rng.choice(["choice", "score"])) for i in range(97)]
    want = enc.encode_batch(rows, threads=3)
    tb = j1.TextBatch(rows)
    flat = enc.encode_batch(tb, threads=3, flat=True)
    got = flat.rows()
    assert [(e.ids.tolist(), e.markers.tolist(), e.qtype) for e, _ in want] == \
        [(e.ids.tolist(), e.markers.tolist(), e.qtype) for e in got]
    assert flat.truncated.tolist() == [t for _, t in want]
    assert enc.encode_batch([], flat=True).ids.size == 0


def test_nfc_quick_check_every_bmp_code_point():
    """The NFC normaliser skips texts whose code points all pass the UAX #15 quick check
    (NFC_QC = Yes), and its tables follow the library's Unicode version. For every BMP code
    point and every other one with a combining class or a canonical decomposition, alone,
    after a letter, after a Hangul leading consonant and before a combining mark, the ids
    equal the reference's tokenizer library's."""
    tokenizers = pytest.importorskip("tokenizers")
    path = os.path.join(GOLDEN, "tokenizer_nfc.json")
    ref = tokenizers.Tokenizer.from_file(path)
    tok = load("nfc")
    import unicodedata
    cps = [c for c in range(0x80, 0x10000) if not 0xD800 <= c <= 0xDFFF]
    # beyond the BMP: every code point with a combining class or a canonical decomposition
    cps += [c for c in range(0x10000, 0x110000) if unicodedata.combining(chr(c)) or
            (unicodedata.decomposition(chr(c)) and not unicodedata.decomposition(chr(c)).startswith("<"))]
    texts = []
    for c in cps:
        ch = chr(c)
        texts += [ch, "e" + ch, ch + "́", "ᄀ" + ch]
    want = [e.ids for e in ref.encode_batch(texts, add_special_tokens=False)]
    got = tok.encode_batch(texts, threads=4)
    bad = [(hex(ord(t[-1]) if len(t) > 1 and t[0] in "eᄀ" else ord(t[0])), t) for t, g, w in zip(texts, got, want)
           if g != w]
    assert not bad, bad[:10]


def test_unicode_tables_match_their_generator(tmp_path):
    """csrc/unicode_tables.h is what gen_unicode_tables.py writes from this Python's
    unicodedata, pinned to the tokenizer library's normalisation (skipped when the Unicode
    version or the library differs from the ones the header was made with)."""
    import importlib.util
    import unicodedata
    tokenizers = pytest.importorskip("tokenizers")
    header = os.path.join(ROOT, "julia1-rs_b200", "csrc", "unicode_tables.h")
    first = open(header, encoding="utf-8").read().split("\n")[:2]
    if unicodedata.unidata_version not in first[0] or tokenizers.__version__ not in first[1]:
        pytest.skip("header made with another Unicode version or tokenizer library")
    spec = importlib.util.spec_from_file_location("gen_unicode_tables",
                                                  os.path.join(ROOT, "julia1-rs_b200", "gen_unicode_tables.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    out = tmp_path / "unicode_tables.h"
    gen.main(str(out))
    got = out.read_text(encoding="utf-8").split("\n")
    want = open(header, encoding="utf-8").read().split("\n")
    assert got[2:] == want[2:]  # line 1 names the Python version that ran the generator
