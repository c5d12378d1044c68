"""Generate the tokenizer fixtures and golden encodings used by tests/test_tokenizer.py.

The reference tokenizes with the HF `tokenizers` crate 0.22.2 (Cargo.lock; called as
`Tokenizer::encode_fast(text, false)`, src/encode.rs:114-129). This script uses the Python
binding of the same library version (tokenizers 0.22.2) to
  1. train two small byte-level BPE tokenizers on a synthetic corpus (no real checkpoint
     exists here), in the configuration family of ModernBERT's tokenizer.json: BPE model
     without unk token, ByteLevel pre-tokenizer with the GPT-2 split, NFC normaliser,
     special tokens [UNK] [CLS] [SEP] [PAD] [MASK] ([MASK] strips the space on its left),
     plus added tokens with the other flags (rstrip, single_word, normalized) and a variant
     with add_prefix_space and ignore_merges;
  2. encode seeded test strings (`encode(text, add_special_tokens=False)`, the ids
     encode_fast returns) and store them as golden vectors.

Usage: python tests/golden/make_tokenizer_golden.py   (needs `tokenizers`; writes tests/golden/)
"""
import json
import os
import random

from tokenizers import AddedToken, Tokenizer, decoders, models, normalizers, pre_tokenizers, trainers

HERE = os.path.dirname(os.path.abspath(__file__))

WORDS = ["the", "game", "state", "player", "move", "option", "score", "choice", "route", "token", "marker",
         "question", "answer", "board", "turn", "win", "lose", "draw", "attack", "defend", "build", "trade"]
SCRIPTS = ["café", "naïve", "Über", "straße", "Ελλάδα", "привет", "мир", "日本語", "中文字", "한국어", "안녕하세요",
           "العربية", "हिन्दी", "१२३", "٣٤٥", "ⅫⅣ", "１２３", "½¾", "😀", "👍🏽", "🧑‍🚀", "ß", "ǅ", "ﬁ", "Ω", "Å"]
PUNCT = [".", ",", "!", "?", "...", "—", "-", "(", ")", "[", "]", "{", "}", "\"", "'", ":", ";", "/", "#", "$",
         "%", "&", "*", "+", "=", "<", ">", "@", "^", "_", "`", "|", "~", "«", "»", "¿", "¡", "•"]
CONTRACTIONS = ["don't", "it's", "I'M", "we're", "you've", "they'll", "I'd", "can'T", "'s", "o'clock", "rock'n'roll"]
SPACES = [" ", " ", " ", "  ", "   ", "\t", "\n", "\n\n", " \n ", " ", "　", " ", "\r\n"]
DECOMPOSED = ["e\u0301", "a\u0308", "n\u0303", "A\u030a", "\u1100\u1161\u11a8", "\u1112\u1161\u11ab",
              "o\u0323\u0302", "q\u0307\u0323", "\u0391\u0301", "c\u0327\u0306", "\u212b", "\u2126",
              "e\u0301\u0301", "\u0958", "\u1e9b\u0323"]
ADDED = ["[MASK]", " [MASK]", "[MASK] ", "x[MASK]y", "  [MASK]  ", "[CLS]", "[SEP]", "[PAD]", "[UNK]",
         "|||IP_ADDRESS|||", "<br>", "<br>   next", "lol", " lol ", "lolx", "xlol", "a lol b"]


def corpus(seed, n):
    rng = random.Random(seed)
    pool = WORDS * 6 + SCRIPTS + CONTRACTIONS + [str(rng.randint(0, 99999)) for _ in range(50)]
    for _ in range(n):
        parts = []
        for _ in range(rng.randint(5, 40)):
            parts.append(rng.choice(pool))
            parts.append(rng.choice([" "] * 8 + PUNCT[:8] + ["\n"]))
        yield "".join(parts)


def test_strings(seed, n):
    rng = random.Random(seed)
    fixed = ["", " ", "  ", "\n", "\t \t", "hello", " hello", "hello ", "hello  world", "hello   world  ",
             "Hello, World!", "don't stop", "IT'S", "123 4567 89", "a1b2c3", "x.y.z", "...!!!", "  leading",
             "trailing  ", "tab\tsep", "new\nline", "mixed \t\n spaces", "ünïcödé", "été", "한국어 텍스트",
             "각가", "emoji 😀 and 👍🏽 done", "日本語のテキスト", "١٢٣ ٤٥", "x y",
             "a　b", "The [MASK] is here", "[MASK][MASK]", "a [MASK]b", "\t[MASK]", "ip |||IP_ADDRESS||| end",
             "line<br>  break", "lol", "say lol now", "lolz", "(lol)", "_lol_", "state: {\"a\": [1, 2.5]}"]
    pieces = WORDS + SCRIPTS + PUNCT + CONTRACTIONS + DECOMPOSED + ADDED + [str(rng.randint(0, 10 ** 6))]
    out = list(fixed)
    for _ in range(n):
        s = []
        for _ in range(rng.randint(1, 14)):
            s.append(rng.choice(pieces))
            if rng.random() < 0.7:
                s.append(rng.choice(SPACES))
        out.append("".join(s))
    return out


def train(vocab_size, seed):
    tok = Tokenizer(models.BPE(unk_token=None, fuse_unk=False))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=True)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=vocab_size, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  special_tokens=[], show_progress=False)
    tok.train_from_iterator(corpus(seed, 3000), trainer)
    return tok


def kind_nfc():
    tok = train(1500, 1)
    tok.normalizer = normalizers.NFC()
    tok.add_tokens([AddedToken("|||IP_ADDRESS|||", normalized=True), AddedToken("<br>", rstrip=True, normalized=False)])
    tok.add_special_tokens([AddedToken("[UNK]", special=True), AddedToken("[CLS]", special=True),
                            AddedToken("[SEP]", special=True), AddedToken("[PAD]", special=True),
                            AddedToken("[MASK]", lstrip=True, special=True)])
    return tok


def kind_prefix():
    tok = train(900, 2)
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=True, use_regex=True)
    tok.add_tokens([AddedToken("lol", single_word=True, normalized=False)])
    tok.add_special_tokens([AddedToken("[CLS]", special=True), AddedToken("[SEP]", special=True),
                            AddedToken("[MASK]", special=True)])
    d = json.loads(tok.to_str())
    d["model"]["ignore_merges"] = True
    return Tokenizer.from_str(json.dumps(d))


def main():
    import tokenizers
    for name, build, seed in [("nfc", kind_nfc, 10), ("prefix", kind_prefix, 11)]:
        tok = build()
        path = os.path.join(HERE, "tokenizer_%s.json" % name)
        tok.save(path)
        cases = [[s, tok.encode(s, add_special_tokens=False).ids] for s in test_strings(seed, 260)]
        with open(os.path.join(HERE, "tokenizer_%s_cases.json" % name), "w") as f:
            json.dump({"generator": "tokenizers %s" % tokenizers.__version__, "tokenizer": os.path.basename(path),
                       "cases": cases}, f, ensure_ascii=False)
        print(name, os.path.getsize(path), "bytes,", len(cases), "cases")


if __name__ == "__main__":
    main()
