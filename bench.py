"""Benchmark: encoder tokens/s per B200 on the router-scale workload.

One step = one forward of a 256-row x 512-token packed batch (131,072 tokens; the
reference's "Router-scale throughput" configuration: a 256-token state plus a
20-option question block of ~12 tokens/option, ids uniform) through libj1 on this
rank's GPU. Weights are seeded N(0, 0.02) in the reference's checkpoint layout with
LayerNorm gamma=1 / beta=0 (ModernBERT-base shape, 22 layers, 2 head layers).
Every rank runs the same per-GPU batch (weak scaling; sequences are independent, so
the ranks share nothing on the data path -- replicas only, no collective).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

  value  device time over K forwards with the batch resident in HBM (CUDA events on
         the model's stream, max over ranks)
  e2e    the same metric through the public C ABI (j1_model_forward) with host
         buffers: pack + pinned staging + H2D + kernels + D2H + sync every step
The working set per step (~2.2 GB of activations, 220 MB of BF16 weights) is far
larger than the 126 MB L2, so no L2 flush is inserted between steps.

`--impl reference` times the reference's own CPU path (its FP32 forward,
src/cpu/mod.rs:201-340, restated in C++ as oracle/j1_oracle.cpp because the Rust
crate cannot be built here) on this host's cores, on a bounded sample per step.
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
ROWS, SEQ = 256, 512
OPTION_BLOCK = (20, 11, 12)  # 20 options x ([MASK] + 11 tokens), 12-token question head
H, I, L, HEADS = 768, 1152, 22, 12
N_GLOBAL = 8  # layers i % 3 == 0
WINDOW = 64   # local_attention / 2


def workload_config():
    return {"workload": "router-scale: 256 rows x 512 tokens per forward per GPU (BASELINE configs[4])",
            "rows_per_step": ROWS, "seq_len": SEQ, "tokens_per_step_per_gpu": ROWS * SEQ,
            "options_per_row": OPTION_BLOCK[0], "model": "ModernBERT-base shape (H768, 22 layers, 12 heads, GEGLU 1152)"
            " + 2 head layers + scorer, random N(0,0.02)", "l2": "inputs larger than L2 (no flush)",
            "parallelism": "replicas (data-parallel by row batch, no collective)"}


def make_rows(seed):
    from julia1 import synthetic
    return synthetic.synthetic_batch([SEQ] * ROWS, markers_per_seq=0, seed=seed, option_block=OPTION_BLOCK)


def local_pairs(S, w=WINDOW):
    i = np.arange(S)
    return int((np.minimum(i + w, S - 1) - np.maximum(i - w, 0) + 1).sum())


def family_model(t, seqs, m):
    """Algorithmic FLOPs and HBM bytes per launch of each kernel family (one forward)."""
    FF = 4 * H
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
    }


def gemm_peak_share(timed, model_f, sustained):
    """The metric's "GEMM % tensor peak": the four encoder GEMM families' FLOPs over their
    summed device time, against the measured sustained and the nominal dense bf16 peak."""
    fams = ["gemm_qkv_rope", "gemm_wo_resid_ln", "gemm_wi_geglu", "gemm_wo2_resid_ln"]
    flops = sum(model_f[f]["flops"] * timed[f][1] for f in fams if f in timed)
    ms = sum(timed[f][0] for f in fams if f in timed)
    if ms <= 0:
        return None
    tf = flops / (ms / 1e3) / 1e12
    return {"tflops": round(tf, 1), "frac_of_measured_sustained": round(tf / sustained, 4),
            "frac_of_nominal": round(tf / 2250.0, 4)}


def encoder_flops_per_token(S):
    return 2.0 * L * (H * 3 * H + H * H + H * 2 * I + I * H) + 4.0 * H * (N_GLOBAL * S + (L - N_GLOBAL) *
                                                                          local_pairs(S) / S)


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
    rows = make_rows(seed=77)
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
                      (n, SEQ, dt)}, o, n


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
    rows = make_rows(seed=91)
    # size one step to ~5 s of CPU work so that warmup + steps stay within a few minutes
    one = j1.Batch.new([j1.Encoded(*r) for r in rows[:1]])
    o.forward_flat(one, mode="fp32", threads=threads)
    t0 = time.perf_counter()
    o.forward_flat(one, mode="fp32", threads=threads)
    per_row = time.perf_counter() - t0
    n = int(max(1, min(ROWS, 5.0 / max(per_row, 1e-3))))
    b = j1.Batch.new([j1.Encoded(*r) for r in rows[:n]])
    for _ in range(args.warmup):
        o.forward_flat(b, mode="fp32", threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        o.forward_flat(b, mode="fp32", threads=threads)
    dt = time.perf_counter() - t0
    tok_s = n * SEQ * args.steps / dt
    sample = "%d rows x %d tokens per step (bounded sample of the 256-row batch), FP32 CPU path restated from " \
             "src/cpu (oracle/j1_oracle.cpp; the Rust crate cannot be built here)" % (n, SEQ)
    line = {"impl": "reference", "metric": METRIC, "value": round(tok_s, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(),
            "cpu_baseline": {"value": round(tok_s, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(tok_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    from julia1.replicas import aggregate_rate, max_over_ranks

    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    ckpt = synthetic.cached_checkpoint(seed=0, base_dir=os.environ.get("J1_CKPT_CACHE", "/tmp/j1_ckpt_r%d" % local))
    model = j1.CudaModel(ckpt, local)
    rows = make_rows(seed=1000 + rank)
    batch = j1.Batch.new([j1.Encoded(*r) for r in rows])
    t, m = batch.tokens(), int(batch.marker_rows.size)
    stream = torch.cuda.ExternalStream(model.stream())

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---------------- value: batch resident in HBM, device-timed
    model.stage(batch)
    for _ in range(args.warmup):
        model.launch()
    model.finish(m)
    launches_per_step = model.launch_count()
    model.profile(True)
    clocks = ClockSampler([local]) if rank == 0 else None
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        model.launch()
    e1.record(stream)
    scores = model.finish(m)
    barrier()
    clk = clocks.stop() if clocks else None
    dev_ms = max_over_ranks(e0.elapsed_time(e1), device="cuda")
    value = aggregate_rate(t * args.steps, e0.elapsed_time(e1) / 1e3, device="cuda")
    fam = model.profile_read()
    model.profile(False)
    assert np.isfinite(scores).all()

    # ---------------- e2e: public C ABI with host buffers (pack + H2D + kernels + D2H + sync)
    for _ in range(2):
        model.forward_flat(batch)
    barrier()
    h0 = time.perf_counter()
    for _ in range(args.steps):
        model.forward_flat(batch)
    h1 = time.perf_counter()
    barrier()
    e2e = aggregate_rate(t * args.steps, h1 - h0, device="cuda")
    ntiles = sum((n + 127) // 128 for n in batch.lens.tolist())  # 128-query attention tiles
    h2d = ((3 * t + m + 7) // 8 * 8 + 8 * ntiles) * 4
    d2h = m * 4 + 4

    if rank == 0:
        hbm, tf_burst, tf_sust, kind = peaks()
        model_f = family_model(t, batch.lens.tolist(), m)
        timed = {k: v for k, v in fam.items() if v[1] > 0}
        total = sum(v[0] for v in timed.values())
        dom = max(timed, key=lambda k: timed[k][0])
        avg_ms = timed[dom][0] / timed[dom][1]
        fm = model_f.get(dom)
        roof = None
        if fm:
            traffic = traffic_table().get(dom)
            if fm["bound"] == "tensor":
                ach = fm["flops"] / (avg_ms / 1e3) / 1e12
                roof = {"kernel": dom, "bound": "tensor", "achieved": round(ach, 1), "peak": tf_sust,
                        "unit": "TFLOP/s", "frac": round(ach / tf_sust, 4),
                        "traffic": traffic, "peak_kind": "%s sustained bf16 (of %s)" % (kind, kind)}
            else:
                ach = fm["bytes"] / (avg_ms / 1e3) / 1e9
                roof = {"kernel": dom, "bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(ach / hbm, 4), "traffic": traffic, "peak_kind": "%s HBM copy" % kind}
            roof["algorithmic_per_launch"] = fm["flops"] if fm["bound"] == "tensor" else fm["bytes"]
            # against the nominal B200 figures as well (2.25 PF/s dense bf16, 8 TB/s HBM3e)
            roof["frac_of_nominal"] = round(ach / (2250.0 if fm["bound"] == "tensor" else 8000.0), 4)
            roof["avg_launch_ms"] = round(avg_ms, 4)
            roof["share_of_step"] = round(timed[dom][0] / total, 4)
        breakdown = {}
        for k, (ms, n) in sorted(timed.items(), key=lambda kv: -kv[1][0]):
            d = {"ms_per_step": round(ms / args.steps, 3), "share": round(ms / total, 4)}
            if k in model_f:
                d["tflops"] = round(model_f[k]["flops"] / (ms / n / 1e3) / 1e12, 1)
                d["gbs"] = round(model_f[k]["bytes"] / (ms / n / 1e3) / 1e9, 1)
            breakdown[k] = d
        fpt = encoder_flops_per_token(SEQ)
        line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded ids, random-init weights)", "config": workload_config(),
                "roofline": roof,
                "encoder_tflops": round(value / world * fpt / 1e12, 1),
                "gemm_tensor_peak": gemm_peak_share(timed, model_f, tf_sust),
                "kernel_breakdown": breakdown,
                "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h},
                "gpu_launches": int(launches_per_step * args.steps),
                "clocks": clk}
        if world == 1 and not args.no_cpu_baseline:
            model.close()
            cb, _, _ = cpu_sample(ckpt)
            line["cpu_baseline"] = cb
            # the reference engine's default CPU thread count (src/engine.rs:160-162)
            cb4, _, _ = cpu_sample(ckpt, target_s=8.0, max_rows=16, threads=4)
            line["cpu_baseline_4_threads"] = cb4
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
