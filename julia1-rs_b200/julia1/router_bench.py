"""Throughput of hierarchical routing (Router::route_many, src/router.rs:143-210) over
the CUDA engine, on a synthetic checkpoint and synthetic tokenized requests.

Each request has `--options` options of ~11 tokens, a ~16-token head and a 256-token
state: the router-scale layout of src/encode.rs:167-187 ([CLS] head [SEP]
20 x ([MASK] + option) [SEP] state [SEP]) for every group of 20. Reports requests/s and
scored model rows/s (host wall clock around route_many: encoding, engine forwards and
routing) for each router batch_size in --router-batch: 16 is the reference's default
(Router::score sends 16 jobs per engine call, src/router.rs:111); a larger one lets the
engine cut full micro-batches. The routes are the same for every batch_size.

Usage (one B200): cd julia1-rs_b200 && python -m julia1.router_bench [--requests 512]
       [--options 100] [--devices 0,1] [--router-batch 16,4096]
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
    ap.add_argument("--router-batch", default="16,4096", help="router batch_size values (jobs per engine call)")
    a = ap.parse_args()
    devs = [int(d) for d in a.devices.split(",")]
    ck = synthetic.cached_checkpoint(seed=0, perturb=True)
    opts = j1.EngineOptions(device="cuda", batch_size=a.batch_size, max_batch_tokens=131072, max_length=512)
    eng = j1.Engine.load(ck, opts, devices=devs if len(devs) > 1 else None)
    enc = j1.EncoderOptions(CLS, SEP, MASK, max_length=512, head_length=256)
    warm = requests(32, a.options, 1)
    rows = requests(a.requests, a.options, 2)
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


if __name__ == "__main__":
    main()
