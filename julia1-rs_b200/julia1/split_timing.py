"""Time text encoding against the model forward for the same rows: the split that the
reference's examples/split_timing.rs prints ("batch B: encode X ms, forward Y ms").

Protocol as there: one untimed pass over all rows, then per repetition the text encoder's
caches are cleared, the rows are encoded in parallel (Engine::encode, src/engine.rs:183-188;
here j1_text_encoder_encode_batch on `--threads` host threads) and the encoded rows are
scored (Engine::logits_encoded, src/engine.rs:190-235; here j1_engine_logits_encoded on
the CUDA engine with micro-batches of `--batch-size` rows), each timed on the host clock.
A third timing is the whole text path as one call (Engine::logits, src/engine.rs:236-243;
here j1_engine_logits_text, which encodes the next chunk of rows while the engine scores
the current one), also with cleared caches.

The rows are marshalled for the C ABI once (a TextBatch) and results are kept as flat
arrays, so the timings are the library's (the reference's are of Rust calls); building
per-row Python objects would add a serial cost of the Python binding to every number.

Inputs are synthetic: the reference reads a public dataset of typed rows, which is not
used here. Each row has a game-state text of about `--words` words, a question and 2 to
20 short options, mixing ASCII and other scripts; the tokenizer is a checkpoint
tokenizer.json (default: the test tokenizer) and the model a seeded synthetic checkpoint
of the base shape.

Usage (one B200): cd julia1-rs_b200 && python -m julia1.split_timing [--rows 1024]
       [--batch-size 16,256] [--threads N] [--tokenizer-dir DIR] [--reps 3]
"""
import argparse
import json
import os
import random
import shutil
import tempfile
import time

import julia1 as j1
from julia1 import synthetic
from julia1.tokenizer_bench import DEFAULT_TOK, WORDS


def make_rows(n, words, seed):
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=1024)
    ap.add_argument("--words", type=int, default=300)
    ap.add_argument("--batch-size", default="16,256", help="engine rows per forward (comma list)")
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    ap.add_argument("--tokenizer-dir", default="")
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args()
    tdir, tmp = tokenizer_dir(a.tokenizer_dir)
    try:
        enc = j1.TextEncoder.load(tdir, max_length=512, head_length=256)
        ck = synthetic.cached_checkpoint(seed=0, perturb=True)
        rows = j1.TextBatch(make_rows(a.rows, a.words, 11))
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


if __name__ == "__main__":
    main()
