"""Throughput of the callers on either side of the encoder forward (measurement tools;
the forward itself is measured by bench.py).

  python bench_callers.py router    [...]   hierarchical routing over the CUDA engine
  python bench_callers.py tokenizer [...]   text -> ids against the reference's tokenizer library
  python bench_callers.py split     [...]   encode vs forward split (examples/split_timing.rs)

Each prints one JSON line per measurement. Inputs are synthetic; the model is a seeded
synthetic checkpoint of the base shape.
"""
import argparse
import json
import os
import random
import shutil
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "julia1-rs_b200"))

import numpy as np  # noqa: E402

import julia1 as j1  # noqa: E402
from julia1 import synthetic  # noqa: E402


# ---------------------------------------------------------------------------- router
# Throughput of hierarchical routing (Router::route_many, src/router.rs:143-210) over
# the CUDA engine, on a synthetic checkpoint and synthetic tokenized requests.
#
# Each request has `--options` options of ~11 tokens, a ~16-token head and a 256-token
# state: the router-scale layout of src/encode.rs:167-187 ([CLS] head [SEP]
# 20 x ([MASK] + option) [SEP] state [SEP]) for every group of 20. Reports requests/s and
# scored model rows/s (host wall clock around route_many: encoding, engine forwards and
# routing) for each router batch_size in --router-batch: 16 is the reference's default
# (Router::score sends 16 jobs per engine call, src/router.rs:111); a larger one lets the
# engine cut full micro-batches. The routes are the same for every batch_size.
#
# Usage (one B200): python bench_callers.py router [--requests 512]
#        [--options 100] [--devices 0,1] [--router-batch 16,4096]

CLS, SEP, MASK = 1, 2, 4


def router_requests(n, n_options, seed):
    rng = np.random.default_rng(seed)
    tok = lambda k: rng.integers(5, 50000, size=int(k)).tolist()  # noqa: E731
    return [j1.TokenizedRequest(tok(rng.integers(12, 20)), [tok(rng.integers(8, 14)) for _ in range(n_options)],
                                tok(256)) for _ in range(n)]


def router_main(argv):
    ap = argparse.ArgumentParser(prog="bench_callers.py router")
    ap.add_argument("--requests", type=int, default=512)
    ap.add_argument("--options", type=int, default=100)
    ap.add_argument("--devices", default="0")
    ap.add_argument("--batch-size", type=int, default=256, help="engine rows per forward")
    ap.add_argument("--router-batch", default="16,4096", help="router batch_size values (jobs per engine call)")
    a = ap.parse_args(argv)
    devs = [int(d) for d in a.devices.split(",")]
    ck = synthetic.cached_checkpoint(seed=0, perturb=True)
    opts = j1.EngineOptions(device="cuda", batch_size=a.batch_size, max_batch_tokens=131072, max_length=512)
    eng = j1.Engine.load(ck, opts, devices=devs if len(devs) > 1 else None)
    enc = j1.EncoderOptions(CLS, SEP, MASK, max_length=512, head_length=256)
    warm = router_requests(32, a.options, 1)
    rows = router_requests(a.requests, a.options, 2)
    line = {"tool": "router_bench", "requests": a.requests, "options": a.options, "devices": devs,
            "engine_batch_size": a.batch_size}
    first = None
    for rb in [int(x) for x in a.router_batch.split(",")]:
        router = j1.Router(engine=eng, encoder=enc, batch_size=rb)
        router.route_many(warm)
        t0 = time.perf_counter()
        res = router.route_many(rows)
        dt = time.perf_counter() - t0
        router.close()
        line["router_batch_%d" % rb] = {"seconds": round(dt, 4), "requests_per_s": round(a.requests / dt, 1),
                                         "model_rows": res[0].model_rows,
                                         "model_rows_per_s": round(res[0].model_rows / dt, 1),
                                         "rounds_max": max(r.rounds for r in res)}
        choice = [r.index for r in res]
        first = first or choice
        line["same_choices"] = choice == first
    print(json.dumps(line), flush=True)
    eng.close()


# ---------------------------------------------------------------------------- tokenizer
# Host throughput of text -> ids: libj1's tokenizer against the reference's tokenizer
# library (HF `tokenizers`, the version pinned in the reference's Cargo.lock, through its
# Python binding), on the same tokenizer.json and the same synthetic texts.
#
# Texts are router-scale request pieces: a rendered game state of ~`--words` words plus
# a question and short options, mixing ASCII and other scripts. Reports tokens/s at one
# thread and at `--threads` threads (the library's encode_batch runs on its own thread
# pool). All outputs are compared id for id.
#
# Usage: python bench_callers.py tokenizer [--tokenizer PATH] [--texts 20000]
#        [--threads N]

DEFAULT_TOK = os.path.join(ROOT, "tests", "golden", "tokenizer_nfc.json")
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


def tokenizer_main(argv):
    ap = argparse.ArgumentParser(prog="bench_callers.py tokenizer")
    ap.add_argument("--tokenizer", default=DEFAULT_TOK)
    ap.add_argument("--texts", type=int, default=20000)
    ap.add_argument("--words", type=int, default=300)
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    a = ap.parse_args(argv)
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


# ---------------------------------------------------------------------------- split
# Time text encoding against the model forward for the same rows: the split that the
# reference's examples/split_timing.rs prints ("batch B: encode X ms, forward Y ms").
#
# Protocol as there: one untimed pass over all rows, then per repetition the text encoder's
# caches are cleared, the rows are encoded in parallel (Engine::encode, src/engine.rs:183-188;
# here j1_text_encoder_encode_batch on `--threads` host threads) and the encoded rows are
# scored (Engine::logits_encoded, src/engine.rs:190-235; here j1_engine_logits_encoded on
# the CUDA engine with micro-batches of `--batch-size` rows), each timed on the host clock.
# A third timing is the whole text path as one call (Engine::logits, src/engine.rs:236-243;
# here j1_engine_logits_text, which encodes the next chunk of rows while the engine scores
# the current one), also with cleared caches.
#
# The rows are marshalled for the C ABI once (a TextBatch) and results are kept as flat
# arrays, so the timings are the library's (the reference's are of Rust calls); building
# per-row Python objects would add a serial cost of the Python binding to every number.
#
# Inputs are synthetic: the reference reads a public dataset of typed rows, which is not
# used here. Each row has a game-state text of about `--words` words, a question and 2 to
# 20 short options, mixing ASCII and other scripts; the tokenizer is a checkpoint
# tokenizer.json (default: the test tokenizer) and the model a seeded synthetic checkpoint
# of the base shape.
#
# Usage (one B200): python bench_callers.py split [--rows 1024]
#        [--batch-size 16,256] [--threads N] [--tokenizer-dir DIR] [--reps 3]

def split_rows(n, words, seed):
    rng = random.Random(seed)
    say = lambda k: " ".join(rng.choice(WORDS) for _ in range(k))  # noqa: E731
    rows = []
    for _ in range(n):
        state = say(rng.randint(words // 2, words))
        question = say(rng.randint(4, 12))
        options = [say(rng.randint(1, 4)) for _ in range(rng.randint(2, 20))]
        rows.append(j1.Request(state, question, options, rng.choice(["choice", "choice", "score"])))
    return rows


def tokenizer_dir(path):
    """A directory with tokenizer.json and tokenizer_config.json: `path` itself when it has
    them, else a temporary one around the default test tokenizer."""
    if path:
        return path, None
    d = tempfile.mkdtemp(prefix="j1_split_")
    shutil.copyfile(DEFAULT_TOK, os.path.join(d, "tokenizer.json"))
    with open(os.path.join(d, "tokenizer_config.json"), "w") as f:
        json.dump({"mask_token": "[MASK]", "cls_token": "[CLS]", "sep_token": "[SEP]", "pad_token": "[PAD]"}, f)
    return d, d


def split_main(argv):
    ap = argparse.ArgumentParser(prog="bench_callers.py split")
    ap.add_argument("--rows", type=int, default=1024)
    ap.add_argument("--words", type=int, default=300)
    ap.add_argument("--batch-size", default="16,256", help="engine rows per forward (comma list)")
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    ap.add_argument("--tokenizer-dir", default="")
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args(argv)
    tdir, tmp = tokenizer_dir(a.tokenizer_dir)
    try:
        enc = j1.TextEncoder.load(tdir, max_length=512, head_length=256)
        ck = synthetic.cached_checkpoint(seed=0, perturb=True)
        rows = j1.TextBatch(split_rows(a.rows, a.words, 11))
        for bs in [int(x) for x in a.batch_size.split(",")]:
            eng = j1.Engine.load(ck, j1.EngineOptions(device="cuda", batch_size=bs, max_batch_tokens=131072,
                                                      max_length=512))
            encoded = enc.encode_batch(rows, threads=a.threads, flat=True)
            eng.logits_flat(encoded)  # untimed pass, as the reference's first engine.logits
            tokens = int(encoded.ids.size)
            reps = []
            for _ in range(a.reps):
                enc.clear_cache()
                t0 = time.perf_counter()
                encoded = enc.encode_batch(rows, threads=a.threads, flat=True)
                te = time.perf_counter() - t0
                t0 = time.perf_counter()
                eng.logits_flat(encoded)
                tf = time.perf_counter() - t0
                enc.clear_cache()
                t0 = time.perf_counter()
                eng.logits(rows, enc, threads=a.threads, flat=True)
                tl = time.perf_counter() - t0
                print("batch %d: encode %.1f ms, forward %.1f ms, text -> logits in one call %.1f ms"
                      % (bs, te * 1e3, tf * 1e3, tl * 1e3), flush=True)
                reps.append((te, tf, tl))
            te, tf, tl = (min(r[k] for r in reps) for k in range(3))
            print(json.dumps({"tool": "split_timing", "rows": rows.n, "tokens": tokens, "batch_size": bs,
                              "host_threads": a.threads, "encode_ms": round(te * 1e3, 2),
                              "forward_ms": round(tf * 1e3, 2), "encode_tokens_per_s": round(tokens / te),
                              "forward_tokens_per_s": round(tokens / tf),
                              "encode_share": round(te / (te + tf), 3), "text_to_logits_ms": round(tl * 1e3, 2),
                              "text_to_logits_tokens_per_s": round(tokens / tl)}), flush=True)
            eng.close()
        enc.close()
    finally:
        if tmp:
            shutil.rmtree(tmp, ignore_errors=True)


def main():
    tools = {"router": router_main, "tokenizer": tokenizer_main, "split": split_main}
    if len(sys.argv) < 2 or sys.argv[1] not in tools:
        sys.exit("usage: python bench_callers.py {router|tokenizer|split} [options]")
    tools[sys.argv[1]](sys.argv[2:])


if __name__ == "__main__":
    main()
