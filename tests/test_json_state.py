"""State::render of JSON states (src/pyjson.rs, src/request.rs:49-54), no GPU needed.

The reference renders a JSON game state with Python's json.dumps(value, ensure_ascii=False)
byte for byte before tokenizing it. j1_json_dumps must give the same text: the known answers
of the reference's own tests (pyjson.rs:123-156), and Python's json module itself (the ground
truth pyjson.rs reproduces) on seeded random values. The text encoder renders a JSON state
before tokenizing it and refuses states that are not an object or an array.
"""
import json
import math
import os
import random
import struct

import pytest

import julia1 as j1
from conftest import ROOT


def test_reference_known_answers():
    for v, s in [(1e16, "1e+16"), (1e15, "1000000000000000.0"), (1e-5, "1e-05"), (1.5e-5, "1.5e-05"),
                 (0.0001, "0.0001"), (32.5, "32.5"), (0.1, "0.1"), (-2.0, "-2.0"),
                 (123456789012345678.0, "1.2345678901234568e+17"),
                 (1.7976931348623157e308, "1.7976931348623157e+308"), (5e-324, "5e-324")]:
        assert j1.json_dumps("[%r]" % v) == "[%s]" % s
    src = '{"b": [1, 2.50, -0, 1E5, "é\\n\\u0001\\"\\\\"], "a": {}, "c": [], "d": null, "e": true}'
    assert j1.json_dumps(src) == '{"b": [1, 2.5, 0, 100000.0, "é\\n\\u0001\\"\\\\"], "a": {}, "c": [], "d": null, "e": true}'


def rand_value(rng, depth=0):
    r = rng.random()
    if depth > 3 or r < 0.45:
        k = rng.randrange(9)
        if k == 0:
            return None
        if k == 1:
            return rng.random() < 0.5
        if k == 2:
            return rng.randint(-10 ** 6, 10 ** 6)
        if k == 3:
            return rng.randint(-10 ** 30, 10 ** 30)  # beyond double precision: kept as written
        if k == 4:  # any finite double
            while True:
                v = struct.unpack("d", struct.pack("Q", rng.getrandbits(64)))[0]
                if math.isfinite(v):
                    return v
        if k == 5:
            return rng.choice([0.0, -0.0, 0.1, 1e16, 1e15, 1e-5, 123.456, -2.5e-7, 1.0, 3.0e21])
        pool = "abcXYZ 09_-\"\\\n\r\t\b\f\x01\x1f/éß日本😀 "
        return "".join(rng.choice(pool) for _ in range(rng.randint(0, 12)))
    if r < 0.75:
        return [rand_value(rng, depth + 1) for _ in range(rng.randint(0, 5))]
    return {("k%d" % rng.randint(0, 99)) + rng.choice(["", "é", "\"", "\\"]): rand_value(rng, depth + 1)
            for _ in range(rng.randint(0, 5))}


def test_matches_python_json_module():
    rng = random.Random(31)
    for i in range(2000):
        v = [rand_value(rng)] if rng.random() < 0.5 else {"s": rand_value(rng)}
        style = i % 3
        text = json.dumps(v) if style == 0 else json.dumps(v, ensure_ascii=False, indent=1) if style == 1 \
            else json.dumps(v, separators=(",", ":"))
        assert j1.json_dumps(text) == json.dumps(json.loads(text), ensure_ascii=False), text
    # literals as written: int vs float, -0
    for text in ["[1, 1.0, 1e0, 1E+2, -0, -0.0, 10000000000000000000001, 0.30000000000000004]"]:
        assert j1.json_dumps(text) == json.dumps(json.loads(text), ensure_ascii=False)


@pytest.fixture(scope="module")
def enc_dir(tmp_path_factory):
    d = tmp_path_factory.mktemp("encj")
    with open(os.path.join(ROOT, "tests", "golden", "tokenizer_nfc.json"), encoding="utf-8") as f:
        (d / "tokenizer.json").write_text(f.read(), encoding="utf-8")
    (d / "tokenizer_config.json").write_text(json.dumps(
        {"mask_token": "[MASK]", "cls_token": "[CLS]", "sep_token": "[SEP]", "pad_token": "[PAD]"}))
    return str(d)


def test_text_encoder_renders_json_states(enc_dir):
    enc = j1.TextEncoder.load(enc_dir, max_length=256, head_length=96)
    state = {"turn": 7, "board": [[1, 0.50], [2, 1E3]], "player": "café", "hp": -0}
    text = json.dumps(state, indent=2)
    got, _ = enc.encode(text, "next move?", ["attack", "defend"], state_is_json=True)
    want, _ = enc.encode(json.dumps(json.loads(text), ensure_ascii=False), "next move?", ["attack", "defend"])
    assert got.ids.tolist() == want.ids.tolist()
    rows = enc.encode_batch([j1.Request(text, "next move?", ["attack", "defend"], state_is_json=True)], threads=2)
    assert rows[0][0].ids.tolist() == want.ids.tolist()
    for bad in ('"just a string"', "42", "{not json"):
        with pytest.raises(j1.J1Error, match="state must be text/JSON|not valid JSON"):
            enc.encode(bad, "q", ["a", "b"], state_is_json=True)
