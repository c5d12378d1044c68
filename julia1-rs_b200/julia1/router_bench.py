"""Throughput of hierarchical routing (Router::route_many, src/router.rs:143-210) over
the CUDA engine, on a synthetic checkpoint and synthetic tokenized requests.

Each request has `--options` options of ~11 tokens, a ~16-token head and a 256-token
state: the router-scale layout of src/encode.rs:167-187 ([CLS] head [SEP]
20 x ([MASK] + option) [SEP] state [SEP]) for every group of 20. Reports requests/s and
scored model rows/s (host wall clock around route_many: encoding, engine forwards and
routing), for the library's router (one engine call per round) and, with
--compare, for the same routing issuing engine calls 16 jobs at a time as the
reference does (Router::score, src/router.rs:111).

Usage (one B200): cd julia1-rs_b200 && python -m julia1.router_bench [--requests 512]
       [--options 100] [--devices 0,1] [--compare]
"""
import argparse
import json
import time

import numpy as np

import julia1 as j1
from julia1 import synthetic

CLS, SEP, MASK = 1, 2, 4


def requests(n, n_options, seed):
    rng = np.random.default_rng(seed)
    tok = lambda k: rng.integers(5, 50000, size=int(k)).tolist()  # noqa: E731
    return [j1.TokenizedRequest(tok(rng.integers(12, 20)), [tok(rng.integers(8, 14)) for _ in range(n_options)],
                                tok(256)) for _ in range(n)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=512)
    ap.add_argument("--options", type=int, default=100)
    ap.add_argument("--devices", default="0")
    ap.add_argument("--batch-size", type=int, default=256, help="engine rows per forward")
    ap.add_argument("--compare", action="store_true", help="also time engine calls of 16 jobs (reference-style)")
    a = ap.parse_args()
    devs = [int(d) for d in a.devices.split(",")]
    ck = synthetic.cached_checkpoint(seed=0, perturb=True)
    opts = j1.EngineOptions(device="cuda", batch_size=a.batch_size, max_batch_tokens=131072, max_length=512)
    eng = j1.Engine.load(ck, opts, devices=devs if len(devs) > 1 else None)
    enc = j1.EncoderOptions(CLS, SEP, MASK, max_length=512, head_length=256)
    router = j1.Router(engine=eng, encoder=enc)
    warm = requests(32, a.options, 1)
    router.route_many(warm)
    rows = requests(a.requests, a.options, 2)
    t0 = time.perf_counter()
    res = router.route_many(rows)
    dt = time.perf_counter() - t0
    line = {"tool": "router_bench", "requests": a.requests, "options": a.options, "devices": devs,
            "engine_batch_size": a.batch_size, "seconds": round(dt, 4),
            "requests_per_s": round(a.requests / dt, 1), "model_rows": res[0].model_rows,
            "model_rows_per_s": round(res[0].model_rows / dt, 1), "rounds_max": max(r.rounds for r in res)}
    if a.compare:
        # the same routing, but the engine is called 16 jobs at a time (Router::score's
        # chunks in the reference) through a scorer callback
        def chunked(enc_rows):
            out = []
            for c0 in range(0, len(enc_rows), 16):
                out.extend(eng.logits_encoded(enc_rows[c0:c0 + 16]))
            return out

        ref_style = j1.Router(encoder=enc, scorer=chunked)
        ref_style.route_many(warm)
        t0 = time.perf_counter()
        want = ref_style.route_many(rows)
        dt_ref = time.perf_counter() - t0
        line["chunks_of_16_requests_per_s"] = round(a.requests / dt_ref, 1)
        line["same_choices"] = all(g.index == w.index for g, w in zip(res, want))
        ref_style.close()
    print(json.dumps(line), flush=True)
    router.close()
    eng.close()


if __name__ == "__main__":
    main()
