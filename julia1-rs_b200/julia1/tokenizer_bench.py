"""Host throughput of text -> ids: libj1's tokenizer against the reference's tokenizer
library (HF `tokenizers`, the version pinned in the reference's Cargo.lock, through its
Python binding), on the same tokenizer.json and the same synthetic texts.

Texts are router-scale request pieces: a rendered game state of ~`--words` words plus
a question and short options, mixing ASCII and other scripts. Reports tokens/s at one
thread and at `--threads` threads (the library's encode_batch runs on its own thread
pool). All outputs are compared id for id.

Usage: cd julia1-rs_b200 && python -m julia1.tokenizer_bench [--tokenizer PATH] [--texts 20000]
       [--threads N]
"""
import argparse
import json
import os
import random
import time

import julia1 as j1

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_TOK = os.path.join(HERE, "..", "..", "tests", "golden", "tokenizer_nfc.json")
WORDS = ["the", "game", "state", "player", "move", "option", "score", "choice", "route", "token", "board", "turn",
         "win", "lose", "draw", "attack", "defend", "build", "trade", "gold", "wood", "stone", "army", "north",
         "south", "café", "naïve", "Ελλάδα", "привет", "日本語", "한국어", "don't", "it's", "42", "3.14", "(x, y)",
         "{\"hp\": 17}", "—", "😀"]


def texts(n, words, seed):
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        out.append(" ".join(rng.choice(WORDS) for _ in range(rng.randint(words // 2, words))))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokenizer", default=DEFAULT_TOK)
    ap.add_argument("--texts", type=int, default=20000)
    ap.add_argument("--words", type=int, default=300)
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    a = ap.parse_args()
    corpus = texts(a.texts, a.words, 7)
    ours = j1.Tokenizer.from_file(a.tokenizer)
    line = {"tool": "tokenizer_bench", "texts": a.texts, "bytes": sum(len(t.encode()) for t in corpus),
            "host_threads": a.threads}
    ours.encode_batch(corpus[:200], threads=1)  # warm the word cache the same way for both timings
    t0 = time.perf_counter()
    flat1, offs1 = ours.encode_batch(corpus, threads=1, flat=True)
    line["libj1_1_thread_tokens_per_s"] = round(flat1.size / (time.perf_counter() - t0))
    t0 = time.perf_counter()
    flatn, offsn = ours.encode_batch(corpus, threads=a.threads, flat=True)
    line["libj1_threads_tokens_per_s"] = round(flatn.size / (time.perf_counter() - t0))
    line["tokens"] = int(flat1.size)
    ids1 = [flat1[int(offs1[i]):int(offs1[i + 1])].tolist() for i in range(len(corpus))]
    idsn = [flatn[int(offsn[i]):int(offsn[i + 1])].tolist() for i in range(len(corpus))]
    try:
        import tokenizers
    except ImportError:
        tokenizers = None
    if tokenizers is not None:
        ref = tokenizers.Tokenizer.from_file(a.tokenizer)
        ref.encode_batch(corpus[:200], add_special_tokens=False)
        t0 = time.perf_counter()
        r1 = [ref.encode(t, add_special_tokens=False).ids for t in corpus]
        line["reference_1_thread_tokens_per_s"] = round(sum(map(len, r1)) / (time.perf_counter() - t0))
        t0 = time.perf_counter()
        rn = [e.ids for e in ref.encode_batch(corpus, add_special_tokens=False)]
        line["reference_batch_tokens_per_s"] = round(sum(map(len, rn)) / (time.perf_counter() - t0))
        line["reference_version"] = tokenizers.__version__
        line["same_ids"] = ids1 == r1 == rn == idsn
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
