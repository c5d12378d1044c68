"""Benchmark: encoder tokens/s on B200 for the router-scale job.

One step = the whole router-scale job: 4096 rows x 512 tokens (a ~12-token question head,
20 options of [MASK] + 11 tokens, a 256-token state; ids uniform), cut into 16 micro-batches
of 256 rows (131,072 tokens) by the engine's plan (Engine::batches, src/engine.rs:191-210)
and dealt to the ranks by greedy token balance (strong scaling: the job is fixed, N GPUs
share it; sequences are independent, so the ranks share nothing on the data path --
replicas only, no collective on the forward). Weights are seeded N(0, 0.02) in the
reference's checkpoint layout with LayerNorm gamma=1 / beta=0 (ModernBERT-base shape,
22 layers, 2 head layers).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                  [--config c5|c2] [--rows R] [--no-cpu-baseline] [--no-extras]

  value     4096*512 tokens per step / the slowest rank's device time for its share of the
            step's forwards (CUDA events on the model's stream, per-launch profiling off);
            each rank's inputs (one staged 256-row micro-batch, replayed for each of its
            forwards: every micro-batch of the job has the same shape) are resident in HBM
  e2e       the same job through the public engine API (j1_engine_logits_encoded) with host
            buffers: each rank plans, packs, stages (pinned H2D), runs and reads back its
            rows' logits, then rank 0 gathers every rank's logits over a CPU gloo group and
            puts all 81,920 of them in row order; host wall clock on rank 0 from a barrier
  roofline  the dominant kernel family, from a second, separately timed pass with per-family
            CUDA events (kernel_breakdown); fraction of the measured burst peak
  configs   C1 (4 x 512), C3 (64 ragged rows, U[16, 1024]) and C4 (2 x 8192) forwards:
            tokens/s and encoder TFLOP/s, device-timed with the batch resident
  --config c2   the isolated fused-epilogue GEMM sweep (M in {512, 4096, 32768, 131072})
  --rows R      profiling captures: one R-row micro-batch per forward, --steps forwards

The working set per forward (~2.2 GB of activations, 220 MB of BF16 weights) is far larger
than the 126 MB L2, so no L2 flush is inserted between steps.

`--impl reference` times the reference's own CPU path (its FP32 forward,
src/cpu/mod.rs:201-340, restated in C++ as oracle/j1_oracle.cpp because the Rust crate
cannot be built here) on this host's cores, on a bounded sample of the job per step.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "julia1-rs_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

METRIC = "encoder tokens/s per B200 (256x512 BF16) at 1/2/4/8 GPUs; GEMM % tensor peak"
JOB_ROWS, BATCH_ROWS, SEQ = 4096, 256, 512
MAX_BATCH_TOKENS = BATCH_ROWS * SEQ
OPTION_BLOCK = (20, 11, 12)  # 20 options x ([MASK] + 11 tokens), 12-token question head
H, I, L, HEADS = 768, 1152, 22, 12
N_GLOBAL = 8  # layers i % 3 == 0
WINDOW = 64   # local_attention / 2
NOMINAL_TFLOPS, NOMINAL_GBS = 2250.0, 8000.0


def workload_config(world=1, rows_override=None):
    c = {"workload": "router-scale job: 4096 rows x 512 tokens, 16 micro-batches of 256 rows (BASELINE configs[4]), "
                     "split over the GPUs",
         "job_rows": JOB_ROWS, "batch_rows": BATCH_ROWS, "seq_len": SEQ, "tokens_per_step": JOB_ROWS * SEQ,
         "forwards_per_step": JOB_ROWS // BATCH_ROWS, "options_per_row": OPTION_BLOCK[0],
         "model": "ModernBERT-base shape (H768, 22 layers, 12 heads, GEGLU 1152) + 2 head layers + scorer, "
                  "random N(0,0.02)",
         "l2": "inputs larger than L2 (no flush)",
         "parallelism": "replicas x%d (micro-batches dealt by token balance, no collective on the forward; "
                        "logits gathered on rank 0 over gloo in e2e)" % world}
    if rows_override:
        c["workload"] = "profiling case: one %d-row x 512-token micro-batch per forward" % rows_override
    return c


def make_rows(seed, n=JOB_ROWS):
    from julia1 import synthetic
    return synthetic.synthetic_batch([SEQ] * n, markers_per_seq=0, seed=seed, option_block=OPTION_BLOCK)


def local_pairs(S, w=WINDOW):
    i = np.arange(S)
    return int((np.minimum(i + w, S - 1) - np.maximum(i - w, 0) + 1).sum())


def family_model(t, seqs, m):
    """Algorithmic FLOPs and HBM bytes per launch of each kernel family (one forward)."""
    pg = sum(s * s for s in seqs)
    pl = sum(local_pairs(s) for s in seqs)
    gemm = lambda M, N, K: 2.0 * M * N * K  # noqa: E731
    return {
        "gemm_qkv_rope": dict(flops=gemm(t, 3 * H, H), bytes=t * H * 2 + 3 * H * H * 2 + t * 3 * H * 2, bound="tensor"),
        "gemm_wi_geglu": dict(flops=gemm(t, 2 * I, H), bytes=t * H * 2 + 2 * I * H * 2 + t * I * 2, bound="tensor"),
        "gemm_wo_resid_ln": dict(flops=gemm(t, H, H), bytes=t * H * 2 + H * H * 2 + t * H * 8 + t * H * 2, bound="hbm"),
        "gemm_wo2_resid_ln": dict(flops=gemm(t, H, I), bytes=t * I * 2 + H * I * 2 + t * H * 8 + t * H * 2,
                                  bound="hbm"),
        "attn_global": dict(flops=4.0 * H * pg, bytes=t * 3 * H * 2 + t * H * 2, bound="tensor"),
        "attn_local": dict(flops=4.0 * H * pl, bytes=t * 3 * H * 2 + t * H * 2, bound="tensor"),
        # two head layers: full attention over every row, then marker queries only (per-launch mean)
        "head_attn": dict(flops=4.0 * H * (pg + m * SEQ) / 2, bytes=(t * 3 * H * 2 + t * H * 2 + t * 2 * H * 2 +
                                                                     m * H * 4) / 2, bound="tensor"),
        # rows kernels: embedding gather + LN (table row read, x write, xn write), final norm
        # (x read and write, xn write, type-embedding rows cached)
        "embed_ln": dict(flops=0.0, bytes=t * H * 4 + t * H * 4 + t * H * 2 + t * 4, bound="hbm"),
        "final_norm": dict(flops=0.0, bytes=t * H * 8 + t * H * 2 + t * 4, bound="hbm"),
    }


def gemm_peak_share(timed, model_f, peak, nominal=NOMINAL_TFLOPS):
    """The metric's "GEMM % tensor peak": the four encoder GEMM families' FLOPs over their
    summed device time, against a measured peak and the nominal dense bf16 peak."""
    fams = ["gemm_qkv_rope", "gemm_wo_resid_ln", "gemm_wi_geglu", "gemm_wo2_resid_ln"]
    flops = sum(model_f[f]["flops"] * timed[f][1] for f in fams if f in timed)
    ms = sum(timed[f][0] for f in fams if f in timed)
    if ms <= 0:
        return None
    tf = flops / (ms / 1e3) / 1e12
    return {"tflops": round(tf, 1), "frac_of_measured_burst": round(tf / peak, 4),
            "frac_of_nominal": round(tf / nominal, 4)}


def encoder_flops(lens):
    """Algorithmic encoder FLOPs of one forward over sequences of these lengths: the four GEMMs
    (2 M N K each, 22 layers) plus 4 H per unmasked (query, key) pair (8 global, 14 local layers)."""
    t = float(sum(lens))
    gemm = 2.0 * L * (H * 3 * H + H * H + H * 2 * I + I * H) * t
    attn = 4.0 * H * (N_GLOBAL * sum(s * s for s in lens) + (L - N_GLOBAL) * sum(local_pairs(s) for s in lens))
    return gemm + attn


def encoder_flops_per_token(S):
    return encoder_flops([S]) / S


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def traffic_table():
    """Per-launch DRAM bytes (dram__bytes_read + write) from the committed ncu summary."""
    out = {}
    p = os.path.join(ROOT, "profiles", "dram_traffic_per_launch.txt")
    if os.path.exists(p):
        for line in open(p):
            parts = line.split()
            if len(parts) >= 2 and parts[0].endswith(":") and not line.startswith("#"):
                try:
                    out[parts[0][:-1]] = float(parts[1])
                except ValueError:
                    pass
    return out


def roofline_entry(fam, fm, avg_ms, share, hbm, tf_burst, tf_sust, kind):
    """roofline object for one kernel family: algorithmic FLOPs (tensor) or bytes (HBM) per
    launch over its mean launch time, against the measured burst peak (the kernels run a few
    tenths of a millisecond at a time) with the sustained and nominal fractions beside it."""
    if fm["bound"] == "tensor":
        ach = fm["flops"] / (avg_ms / 1e3) / 1e12
        r = {"kernel": fam, "bound": "tensor", "achieved": round(ach, 1), "peak": tf_burst, "unit": "TFLOP/s",
             "frac": round(ach / tf_burst, 4), "peak_kind": "%s burst bf16 (of %s)" % (kind, kind),
             "frac_of_sustained": round(ach / tf_sust, 4), "frac_of_nominal": round(ach / NOMINAL_TFLOPS, 4),
             "algorithmic_per_launch": fm["flops"]}
    else:
        ach = fm["bytes"] / (avg_ms / 1e3) / 1e9
        r = {"kernel": fam, "bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
             "frac": round(ach / hbm, 4), "peak_kind": "%s HBM copy (of %s)" % (kind, kind),
             "frac_of_nominal": round(ach / NOMINAL_GBS, 4), "algorithmic_per_launch": fm["bytes"]}
    tr = traffic_table().get(fam)
    r["traffic"] = tr
    if tr:
        r["traffic_note"] = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one full-size launch "
                             "(profiles/dram_traffic_per_launch.txt); writes still dirty in L2 when the "
                             "kernel ends are not counted")
    r["avg_launch_ms"] = round(avg_ms, 4)
    r["share_of_step"] = round(share, 4)
    return r


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", ",".join(map(str, gpus)), "--query-gpu=" + self.FIELDS,
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f:
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9:
                continue
            try:
                sm.append(float(c[1]))
                mx.append(float(c[2]))
            except ValueError:
                continue
            for n, v in zip(names, c[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_sample(ckpt, target_s=12.0, max_rows=64, threads=None):
    """Time the reference CPU path (FP32 restatement) on a bounded sample of the same workload."""
    from oracle import oracle as orc
    import julia1 as j1
    threads = threads or len(os.sched_getaffinity(0))
    o = orc.Oracle(ckpt)
    rows = make_rows(seed=77, n=max_rows)
    b = j1.Batch.new([j1.Encoded(*r) for r in rows[:1]])
    o.forward_flat(b, mode="fp32", threads=threads)  # warm (weight packing)
    t0 = time.perf_counter()
    o.forward_flat(b, mode="fp32", threads=threads)
    per_row = time.perf_counter() - t0
    n = int(max(1, min(max_rows, target_s / max(per_row, 1e-3))))
    b = j1.Batch.new([j1.Encoded(*r) for r in rows[:n]])
    t0 = time.perf_counter()
    o.forward_flat(b, mode="fp32", threads=threads)
    dt = time.perf_counter() - t0
    return {"value": round(n * SEQ / dt, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": "%d rows x %d tokens of the same workload, FP32 CPU path (oracle/j1_oracle.cpp), %.1f s" %
                      (n, SEQ, dt)}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    from julia1 import synthetic
    from oracle import oracle as orc
    import julia1 as j1
    ckpt = synthetic.cached_checkpoint(seed=0)
    threads = len(os.sched_getaffinity(0))
    o = orc.Oracle(ckpt)
    rows = make_rows(seed=91, n=BATCH_ROWS)
    # size one step to ~5 s of CPU work so that warmup + steps stay within a few minutes
    one = j1.Batch.new([j1.Encoded(*r) for r in rows[:1]])
    o.forward_flat(one, mode="fp32", threads=threads)
    t0 = time.perf_counter()
    o.forward_flat(one, mode="fp32", threads=threads)
    per_row = time.perf_counter() - t0
    n = int(max(1, min(BATCH_ROWS, 5.0 / max(per_row, 1e-3))))
    b = j1.Batch.new([j1.Encoded(*r) for r in rows[:n]])
    for _ in range(args.warmup):
        o.forward_flat(b, mode="fp32", threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        o.forward_flat(b, mode="fp32", threads=threads)
    dt = time.perf_counter() - t0
    tok_s = n * SEQ * args.steps / dt
    sample = "%d rows x %d tokens per step (bounded sample of the 4096-row job), FP32 CPU path restated from " \
             "src/cpu (oracle/j1_oracle.cpp; the Rust crate cannot be built here)" % (n, SEQ)
    line = {"impl": "reference", "metric": METRIC, "value": round(tok_s, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(world),
            "cpu_baseline": {"value": round(tok_s, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(tok_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GEMM sweep
def run_gemm_sweep(args):
    """Isolated fused-epilogue GEMMs at hidden 768 through j1_op_gemm: QKV 768->2304 (+RoPE),
    Wo 768->768 (+FP32 residual + LayerNorm), Wi 768->2304 (+GEGLU -> 1152), Wo2 1152->768
    (+residual + LayerNorm). A ~ N(0,1) BF16, W ~ N(0,0.02). CUDA events over `--steps`
    back-to-back launches after `--warmup`; one JSON line per (GEMM, M)."""
    import torch
    import julia1 as j1
    hbm, tf_burst, _, kind = peaks()
    g = torch.Generator(device="cuda").manual_seed(0)
    cos = torch.rand((8192, 32), generator=g, device="cuda")
    sin = torch.rand((8192, 32), generator=g, device="cuda")
    shapes = [("qkv_rope", j1.EPI_QKV_ROPE, 3 * H, H), ("wo_resid_ln", j1.EPI_RESID_LN, H, H),
              ("wi_geglu", j1.EPI_GEGLU, 2 * I, H), ("wo2_resid_ln", j1.EPI_RESID_LN, H, I)]
    for M in [int(x) for x in args.m.split(",")]:
        for name, epi, N, K in shapes:
            A = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
            W = (torch.randn((N, K), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
            if epi == j1.EPI_QKV_ROPE:
                kw = dict(out=torch.empty((M, N), device="cuda", dtype=torch.bfloat16),
                          pos=torch.arange(M, device="cuda", dtype=torch.int32) % 512, rope_cos=cos, rope_sin=sin,
                          rope_cols=2 * H)
            elif epi == j1.EPI_GEGLU:
                kw = dict(out=torch.empty((M, N // 2), device="cuda", dtype=torch.bfloat16))
            else:
                kw = dict(x=torch.randn((M, N), generator=g, device="cuda"), ln_w=torch.ones(N, device="cuda"),
                          xn=torch.empty((M, N), device="cuda", dtype=torch.bfloat16))
            for _ in range(args.warmup):
                j1.op_gemm(epi, A, W, sync=False, **kw)
            torch.cuda.synchronize()
            clocks = ClockSampler([torch.cuda.current_device()])
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                j1.op_gemm(epi, A, W, sync=False, **kw)
            e1.record()
            torch.cuda.synchronize()
            clk = clocks.stop()
            ms = e0.elapsed_time(e1) / args.steps
            flops = 2.0 * M * N * K
            if epi == j1.EPI_RESID_LN:
                nbytes = M * K * 2 + N * K * 2 + M * N * 8 + M * N * 2
                frac = nbytes / ms / 1e6 / hbm
            else:
                nbytes = M * K * 2 + N * K * 2 + M * (N // 2 if epi == j1.EPI_GEGLU else N) * 2
                frac = flops / ms / 1e9 / tf_burst
            print(json.dumps({"config": "c2 GEMM sweep", "gemm": name, "M": M, "N": N, "K": K, "ms": round(ms, 4),
                              "tflops": round(flops / ms / 1e9, 1), "gbs": round(nbytes / ms / 1e6, 1),
                              "frac_of_%s_%s" % (kind, "hbm" if epi == j1.EPI_RESID_LN else "burst_bf16"):
                                  round(frac, 4), "clocks": clk}), flush=True)
            del A, W, kw


# ------------------------------------------------------------------ forward of one config
def time_resident(model, batch, steps, warmup):
    """Device time (ms) of `steps` forwards of a staged batch (CUDA events on the model's
    stream, profiling off)."""
    import torch
    stream = torch.cuda.ExternalStream(model.stream())
    model.stage(batch)
    for _ in range(warmup):
        model.launch()
    model.finish(int(batch.marker_rows.size))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        model.launch()
    e1.record(stream)
    scores = model.finish(int(batch.marker_rows.size))
    assert np.isfinite(scores).all()
    return e0.elapsed_time(e1)


def config_extras(model, steps, tf_burst):
    """C1 (4 x 512), C3 (64 ragged rows, U[16, 1024]) and C4 (2 x 8192): tokens/s and encoder
    TFLOP/s of the whole forward (head and scorer included in the time, not in the FLOPs)."""
    import julia1 as j1
    from julia1 import synthetic
    rng = np.random.default_rng(2024)
    cases = {"c1_4x512": [512] * 4, "c3_ragged64": rng.integers(16, 1025, size=64).tolist(),
             "c4_2x8192": [8192] * 2}
    out = {}
    for name, lens in cases.items():
        rows = synthetic.synthetic_batch(lens, markers_per_seq=4, seed=31, mask_markers=False)
        b = j1.Batch.new([j1.Encoded(*r) for r in rows])
        n = max(3, min(steps, 20))
        ms = time_resident(model, b, n, 3) / n
        t = b.tokens()
        tf = encoder_flops(lens) / (ms / 1e3) / 1e12
        out[name] = {"tokens": t, "sequences": len(lens), "ms_per_forward": round(ms, 3),
                     "tokens_per_s": round(t / (ms / 1e3), 1), "encoder_tflops": round(tf, 1),
                     "frac_of_measured_burst": round(tf / tf_burst, 4), "frac_of_nominal": round(tf / NOMINAL_TFLOPS, 4)}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c5", choices=["c5", "c2"])
    ap.add_argument("--m", default="512,4096,32768,131072", help="GEMM sweep M values (--config c2)")
    ap.add_argument("--rows", type=int, default=0, help="profiling case: rows per forward (one forward per step)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    import julia1 as j1
    from julia1 import synthetic
    from julia1.replicas import max_over_ranks, rank_share

    torch.cuda.set_device(local)
    if args.config == "c2":
        if rank == 0:
            run_gemm_sweep(args)
        return
    gloo = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        gloo = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=300))

    ckpt = synthetic.cached_checkpoint(seed=0, base_dir=os.environ.get("J1_CKPT_CACHE", "/tmp/j1_ckpt_r%d" % local))
    model = j1.CudaModel(ckpt, local)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    if args.rows:  # profiling case for external profilers: one forward of R rows per step
        rows = make_rows(seed=5, n=args.rows)
        b = j1.Batch.new([j1.Encoded(*r) for r in rows])
        ms = time_resident(model, b, args.steps, args.warmup)
        if rank == 0:
            print(json.dumps({"profiling_case": workload_config(world, args.rows), "forwards": args.steps,
                              "ms_per_forward": round(ms / args.steps, 3),
                              "launches_per_forward": model.launch_count()}), flush=True)
        model.close()
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    # ---------------- the job: 4096 rows, the engine's micro-batches, this rank's share
    rows = make_rows(seed=1000)
    lens = [SEQ] * JOB_ROWS
    share = rank_share(lens, BATCH_ROWS, MAX_BATCH_TOKENS, rank, world)
    n_fwd = len(share)  # forwards of this rank per step
    first = j1.Batch.new([j1.Encoded(*rows[i]) for i in share[0]])
    t_fwd, m_fwd = first.tokens(), int(first.marker_rows.size)

    # ---------------- value: inputs resident in HBM, device-timed, profiling off
    model.stage(first)
    for _ in range(args.warmup):
        model.launch()
    model.finish(m_fwd)
    launches_per_fwd = model.launch_count()
    stream = torch.cuda.ExternalStream(model.stream())
    clocks = ClockSampler([local]) if rank == 0 else None
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps * n_fwd):
        model.launch()
    e1.record(stream)
    scores = model.finish(m_fwd)
    barrier()
    clk = clocks.stop() if clocks else None
    assert np.isfinite(scores).all()
    dev_ms = max_over_ranks(e0.elapsed_time(e1), device="cuda")
    value = JOB_ROWS * SEQ * args.steps / (dev_ms / 1e3)

    # ---------------- kernel breakdown: a second pass with per-family CUDA events
    model.profile(True)
    for _ in range(n_fwd):
        model.launch()
    model.finish(m_fwd)
    fam = model.profile_read()
    model.profile(False)

    # ---------------- e2e: the job through the engine API, logits gathered on rank 0
    eng = j1.Engine.load(ckpt, j1.EngineOptions(device="cuda:%d" % local, batch_size=BATCH_ROWS,
                                                max_batch_tokens=MAX_BATCH_TOKENS, max_length=SEQ))
    mine = [i for bt in share for i in bt]
    enc = j1.EncodedBatch(np.concatenate([rows[i][0] for i in mine]).astype(np.uint32),
                          np.array([len(rows[i][0]) for i in mine], np.uint32),
                          np.concatenate([rows[i][1] for i in mine]).astype(np.uint32),
                          np.array([len(rows[i][1]) for i in mine], np.uint32),
                          np.array([rows[i][2] for i in mine], np.uint8), np.zeros(len(mine), bool))
    nmark = OPTION_BLOCK[0]
    shares_all = [rank_share(lens, BATCH_ROWS, MAX_BATCH_TOKENS, r, world) for r in range(world)]
    rows_of = [[i for bt in s for i in bt] for s in shares_all]

    def job():
        out = eng.logits_flat(enc)  # this rank's rows' logits, row after row
        if world == 1:
            full = np.empty(JOB_ROWS * nmark, np.float32)
            full.reshape(JOB_ROWS, nmark)[mine] = out.reshape(-1, nmark)
            return full
        t = torch.from_numpy(out)
        if rank == 0:
            parts = [torch.empty(len(rows_of[r]) * nmark, dtype=torch.float32) for r in range(world)]
            dist.gather(t, parts, dst=0, group=gloo)
            full = np.empty(JOB_ROWS * nmark, np.float32)
            fv = full.reshape(JOB_ROWS, nmark)
            for r in range(world):
                fv[rows_of[r]] = parts[r].numpy().reshape(-1, nmark)
            return full
        dist.gather(t, None, dst=0, group=gloo)
        return None

    for _ in range(max(1, args.warmup // 3)):
        ref_logits = job()
    barrier()
    h0 = time.perf_counter()
    for _ in range(args.steps):
        logits = job()
    h1 = time.perf_counter()
    e2e_s = max_over_ranks(h1 - h0, device="cuda")
    barrier()
    e2e = JOB_ROWS * SEQ * args.steps / e2e_s
    if rank == 0:
        assert np.isfinite(logits).all() and np.array_equal(logits, ref_logits)
    eng.close()
    ntiles = sum((n + 127) // 128 for n in first.lens.tolist())  # 128-query attention tiles
    h2d = ((3 * t_fwd + m_fwd + 7) // 8 * 8 + 8 * ntiles) * 4 * (JOB_ROWS // BATCH_ROWS)
    d2h = (m_fwd * 4 + 4) * (JOB_ROWS // BATCH_ROWS)

    # ---------------- in-process pool over all N devices (rank 0), same job
    pool = None
    if world > 1:
        barrier()
        if rank == 0:
            model.close()
            allrows = j1.EncodedBatch(np.concatenate([r[0] for r in rows]).astype(np.uint32),
                                      np.array([len(r[0]) for r in rows], np.uint32),
                                      np.concatenate([r[1] for r in rows]).astype(np.uint32),
                                      np.array([len(r[1]) for r in rows], np.uint32),
                                      np.array([r[2] for r in rows], np.uint8), np.zeros(JOB_ROWS, bool))
            peng = j1.Engine.load(ckpt, j1.EngineOptions(device="cuda", batch_size=BATCH_ROWS,
                                                         max_batch_tokens=MAX_BATCH_TOKENS, max_length=SEQ),
                                  devices=list(range(world)))
            peng.logits_flat(allrows)
            p0 = time.perf_counter()
            for _ in range(args.steps):
                pl = peng.logits_flat(allrows)
            p1 = time.perf_counter()
            peng.close()
            pool = {"value": round(JOB_ROWS * SEQ * args.steps / (p1 - p0), 1), "unit": "tokens/s",
                    "devices": world, "api": "j1_engine_create_pool + j1_engine_logits_encoded (one process)",
                    "same_logits_as_e2e": bool(np.array_equal(pl, logits))}
        # the other ranks wait on the host (gloo): an NCCL barrier would keep a kernel
        # spinning on their GPUs, which the pool is using
        dist.barrier(group=gloo)

    if rank == 0:
        hbm, tf_burst, tf_sust, kind = peaks()
        model_f = family_model(t_fwd, first.lens.tolist(), m_fwd)
        timed = {k: v for k, v in fam.items() if v[1] > 0}
        total = sum(v[0] for v in timed.values())
        dom = max(timed, key=lambda k: timed[k][0])
        roof = None
        if dom in model_f:
            roof = roofline_entry(dom, model_f[dom], timed[dom][0] / timed[dom][1], timed[dom][0] / total, hbm,
                                  tf_burst, tf_sust, kind)
        breakdown = {}
        for k, (ms, n) in sorted(timed.items(), key=lambda kv: -kv[1][0]):
            d = {"ms_per_forward": round(ms / n_fwd, 3), "launches_per_forward": n // n_fwd,
                 "share": round(ms / total, 4)}
            if k in model_f:
                if model_f[k]["flops"]:
                    d["tflops"] = round(model_f[k]["flops"] / (ms / n / 1e3) / 1e12, 1)
                d["gbs"] = round(model_f[k]["bytes"] / (ms / n / 1e3) / 1e9, 1)
                d["frac"] = round((d["tflops"] / tf_burst) if model_f[k]["bound"] == "tensor" and "tflops" in d
                                  else d["gbs"] / hbm, 4)
            breakdown[k] = d
        fpt = encoder_flops_per_token(SEQ)
        line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 3),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded ids, random-init weights)", "config": workload_config(world),
                "roofline": roof,
                "encoder_tflops": round(value * fpt / 1e12, 1),
                "encoder_tflops_per_gpu": round(value / world * fpt / 1e12, 1),
                "gemm_tensor_peak": gemm_peak_share(timed, model_f, tf_burst),
                "kernel_breakdown": breakdown,
                "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h,
                        "api": "j1_engine_logits_encoded per rank + gloo gather of the logits to rank 0 in row order"},
                "gpu_launches": int(launches_per_fwd * n_fwd * args.steps),
                "clocks": clk}
        if pool:
            line["pool_e2e"] = pool
        if world == 1 and not args.no_extras:
            line["configs"] = config_extras(model, args.steps, tf_burst)
        if world == 1 and not args.no_cpu_baseline:
            model.close()
            line["cpu_baseline"] = cpu_sample(ckpt)
            # the reference engine's default CPU thread count (src/engine.rs:160-162)
            line["cpu_baseline_4_threads"] = cpu_sample(ckpt, target_s=8.0, max_rows=16, threads=4)
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
