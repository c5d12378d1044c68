"""Run a few forwards of the router-scale row layout for external profilers (ncu).

  python -m julia1.profile_forward [--rows R] [--seq S] [--forwards F]

Creates a seeded synthetic checkpoint (ModernBERT-base shape), stages one batch of
R rows x S tokens (20 options per row, as in bench.py) and runs F forwards through
the C ABI. Kernel launches per forward: 126 for the default 2-layer head. Weight
conversion at load issues 97 launches before the first forward.
"""
import argparse
import os
import sys

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if HERE not in sys.path:
    sys.path.insert(0, HERE)

import julia1 as j1  # noqa: E402
from julia1 import synthetic  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=32)
    ap.add_argument("--seq", type=int, default=512)
    ap.add_argument("--forwards", type=int, default=2)
    a = ap.parse_args()
    ck = synthetic.cached_checkpoint(seed=0)
    m = j1.CudaModel(ck, 0)
    rows = synthetic.synthetic_batch([a.seq] * a.rows, seed=5, option_block=(20, 11, 12))
    b = j1.Batch.new([j1.Encoded(*r) for r in rows])
    m.stage(b)
    for _ in range(a.forwards):
        m.launch()
    s = m.finish(b.marker_rows.size)
    print("ok: %d forwards of %d tokens, %d launches each, %d logits" % (a.forwards, b.tokens(), m.launch_count(),
                                                                         s.size))
    m.close()


if __name__ == "__main__":
    main()
