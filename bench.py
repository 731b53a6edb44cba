#!/usr/bin/env python
"""Decode benchmark: tokens/s of the B200 decode path (default: Llama-2-7B shape,
Q4_0, batch 1, KV cache prefilled to 512 positions) on N GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload NAME] [--ctx C]

N > 1 runs under torchrun, one rank per GPU, tensor parallel over NCCL. Prints
one JSON line (rank 0). The reference arm (--impl reference) times the
reference's own CPU ForwardToken (oracle/_ref, built from the reference's
sources) on the same synthetic model.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from mini_llama_b200 import configs as C  # noqa: E402

SEED = 20261201
# dram__bytes_read.sum + dram__bytes_write.sum of one gate/up GEMV launch
# (22016 x 4096 Q4_0), from the ncu capture summarised in
# profiles/gemv_q4_0_gateup_22016x4096.md.
GEMV_TRAFFIC_BYTES = 50.79e6
# The same counters for one launch of the persistent decode-step kernel on the
# Llama-2-7B Q4_0 shape, from the 2- and 4-layer captures in
# profiles/decode_step_kernel_llama2-7b-q4_0.md: 77.6 MB fixed (lm_head,
# embedding row, activations) plus, per layer, 114.1 MB of weights and small
# terms and the fp32 K and V rows at the context (17.0 MB at context 520).
def step_traffic_7b(layers, ctx):
    return 77.6e6 + layers * (114.08e6 + 2 * 4 * 128 * 32 * ctx)



def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=64)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--workload", choices=sorted(C.WORKLOADS) + ["gemv-sweep"],
                   default="llama2-7b-q4_0")
    p.add_argument("--sweep-n", type=str, default="4096,11008,14336")
    p.add_argument("--sweep-m", type=str, default="1,4,16,64")
    p.add_argument("--sweep-q", type=str, default="q4_0,q4_1,q8_0")
    p.add_argument("--ctx", type=int, default=512, help="KV positions filled before timing")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--layers", type=int, default=0,
                   help="override the layer count (small profiling cases only; not a bench line)")
    p.add_argument("--per-op", action="store_true",
                   help="run the step as one kernel per op instead of the persistent kernel")
    return p.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ----------------------------------------------------------------- clocks

class Clocks:
    """nvidia-smi samples during the timed region."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-i", ",".join(str(g) for g in self.gpus), "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, windows=None):
        """Median SM clock, max clock and throttle reasons over the samples;
        with windows (host (start, end) times), only samples taken inside one."""
        import datetime

        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            if windows is not None:
                try:
                    t = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    continue
                if not any(a <= t <= b for a, b in windows):
                    continue
            parts = parts[1:]
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.f.name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# -------------------------------------------------------------- CPU legs

def cpu_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def build_cpu_model(cfg, qtype, bias):
    """The reference's own CPU implementation when built (oracle/_ref), else the
    C restatement; both get the generator's exact bytes."""
    import oracle

    if oracle.ref_available():
        r = oracle.ref()
        r.set_threads(cpu_threads())
        kind, lib, threads = "reference", r, r.threads()
    else:
        kind, lib, threads = "port", oracle.port(), 1
    m = lib.model(cfg)
    for k, layer, qt, rows, cols, arr in C.host_weights(cfg, qtype, SEED, bias,
                                                        threads=cpu_threads()):
        m.set_weight(k, layer, qt, rows, cols, arr)
    return m, kind, threads


def time_cpu_tokens(m, cfg, n_warm, n_max, budget_s):
    """Greedy CPU decode from position 0: n_warm untimed, then up to n_max timed
    tokens or until budget_s of CPU time."""
    tok = C.prompt_ids(SEED, 1, cfg["vocab_size"])[0]
    pos = 0
    for _ in range(n_warm):
        tok = int(np.argmax(m.forward_token(tok, pos)))
        pos += 1
    t0 = time.perf_counter()
    n = 0
    while n < n_max:
        tok = int(np.argmax(m.forward_token(tok, pos)))
        pos += 1
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    return n, time.perf_counter() - t0


def run_reference(args, cfg, qtype, bias, world, rank):
    if rank != 0:
        return
    metric = "decode tok/s"
    try:
        m, kind, threads = build_cpu_model(cfg, qtype, bias)
    except Exception as e:  # pragma: no cover
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU build failed: {e}"}))
        return
    t_first = time.perf_counter()
    n_w, _ = time_cpu_tokens(m, cfg, 0, 1, 1e9)
    per_tok = time.perf_counter() - t_first
    budget = 150.0
    steps = max(1, min(args.steps, int(budget / max(per_tok, 1e-3))))
    warm = max(0, min(args.warmup - 1, 2))
    n, secs = time_cpu_tokens(m, cfg, warm, steps, budget)
    v = n / secs
    sample = (f"{n} greedy decode tokens of the full model from position {warm + 1} "
              f"(bounded to ~{int(budget)} s), {threads} threads")
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": v, "unit": "tok/s", "n_gpus": world,
        "steps": n, "warmup": warm + 1, "ms_per_step": 1000.0 * secs / n,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": C.QTYPE_NAMES[qtype] + "/fp32", "data": "synthetic (seeded N(0,0.02) weights)",
        "config": {"workload": args.workload, "batch": 1, "ctx": "0..%d" % (warm + n),
                   "parallelism": "cpu threads"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ---------------------------------------------------------------- GPU arm

def time_launches(torch, launch, n, min_seconds=0.0):
    """Average device time of one launch: n launches captured in a CUDA graph
    (no host launch latency between them), replayed and timed with events;
    the graph is replayed until the timed region lasts min_seconds (so clock
    samples can land in it)."""
    launch(0)  # first call outside capture: one-time kernel attributes
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(n):
                launch(i)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    reps = 1
    if min_seconds > 0:  # one replay's duration sets the count
        a.record(cur)
        g.replay()
        b.record(cur)
        torch.cuda.synchronize()
        reps = max(1, int(min_seconds * 1e3 / max(a.elapsed_time(b), 1e-3)) + 1)
    a.record(cur)
    for _ in range(reps):
        g.replay()
    b.record(cur)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / (n * reps)


def gemv_roofline(torch, mlb, cfg, qtype, world, peak):
    """Live per-launch timing of the dominant kernel: the fused gate/up GEMV of
    this rank's shard, rotating over copies that together exceed L2."""
    F = cfg["hidden_dim"] // world
    n, k = 2 * F, cfg["dim"]
    nbytes = n * ((k + 31) // 32) * C.BLOCK_BYTES[qtype] + k * 4 + (n // 2) * 4
    copies = max(2, int(np.ceil(400e6 / nbytes)))
    mats = [mlb.QMatrix.synthesize(qtype, n, k, SEED, 900 + i, raw=False) for i in range(copies)]
    x = torch.randn(1, k, device="cuda")
    y = torch.empty(1, n, device="cuda")
    ms = time_launches(torch, lambda i: mats[i % copies].gemv(x, y), 8 * copies)
    achieved = nbytes / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peak[0], "unit": "GB/s",
            "frac": achieved / peak[0],
            # the captured traffic is for the single-GPU shape (22016 x 4096)
            "traffic": GEMV_TRAFFIC_BYTES if world == 1 else None,
            "kernel": f"gemv_sb_kernel<{C.QTYPE_NAMES[qtype]}> {n}x{k}",
            "bytes_per_launch": nbytes, "us_per_launch": ms * 1e3,
            "peak_source": peak[1] + " (MEASURED_PEAKS.json hbm_gbs, burst)"}


def run_gpu(args, cfg, qtype, bias, rank, world, local):
    import torch

    import mini_llama_b200 as mlb

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
    nccl_id = None
    if world > 1:
        obj = [mlb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    model = mlb.CudaModel(cfg, device_id=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    model.synthesize(qtype, SEED, with_bias=bias)
    resident, step_weights = model.bytes()
    ctx = model.context(mlb.ATTN_CPU_COMPAT, step_kernel=False if args.per_op else None)
    step_kernel = ctx.step_kernel()
    stream = torch.cuda.ExternalStream(ctx.stream())
    tok0 = C.prompt_ids(SEED, 1, cfg["vocab_size"])[0]
    if args.ctx + args.warmup + 2 * args.steps + 2 > cfg["max_seq_len"]:
        raise SystemExit("context too long for max_seq_len")

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # fill the KV cache to ctx positions (greedy decode from position 0)
    pos = 0
    toks = ctx.decode_greedy(tok0, pos, args.ctx) if args.ctx else [tok0]
    pos += args.ctx
    tok = toks[-1]
    # warm-up
    toks = ctx.decode_greedy(tok, pos, args.warmup)
    pos += args.warmup
    tok = toks[-1] if toks else tok
    barrier()

    # timed: device-resident greedy decode, one graph launch per token
    with Clocks([local]) as clk:
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.profiler.start()
        ev0.record(stream)
        toks = ctx.decode_greedy(tok, pos, args.steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ctx_end = pos + args.steps
    pos += args.steps
    tok = toks[-1]
    clocks = clk.summary()

    # e2e: ForwardToken through the C ABI, host logits every step
    for _ in range(2):
        tok = int(np.argmax(ctx.forward_token(tok, pos)))
        pos += 1
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        lg = ctx.forward_token(tok, pos)
        tok = int(np.argmax(lg))
        pos += 1
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))

    peak = measured_peaks()
    gemv_roof = gemv_roofline(torch, mlb, cfg, qtype, world, peak)
    # whole-step HBM roofline: weights + fp32 KV read at the timed context
    kv_per_pos = 2 * cfg["n_layers"] * (cfg["n_kv_heads"] // world) * cfg["head_dim"] * 4
    mid_ctx = (args.ctx + args.warmup + ctx_end) / 2
    step_bytes = step_weights + kv_per_pos * mid_ctx
    step_s = ms / 1e3 / args.steps
    kpl = ctx.kernels_per_step()
    step_roof = {"bound": "hbm", "achieved": step_bytes / step_s / 1e9, "peak": peak[0],
                 "unit": "GB/s", "frac": step_bytes / step_s / 1e9 / peak[0],
                 "bytes_per_launch": step_bytes, "us_per_launch": step_s * 1e6,
                 "note": "algorithmic bytes: GGUF weight bytes of this rank + fp32 K and V "
                         "read per token at the mean timed context; time: CUDA events on "
                         "the context stream around the timed greedy steps",
                 "peak_source": peak[1] + " (MEASURED_PEAKS.json hbm_gbs, burst)"}
    if step_kernel:
        # one launch per step: the persistent kernel is the dominant (only) kernel
        roof = dict(step_roof, kernel=f"decode_step_kernel<{C.QTYPE_NAMES[qtype]}>",
                    traffic=(step_traffic_7b(cfg["n_layers"], mid_ctx)
                             if args.workload == "llama2-7b-q4_0" and world == 1 else None))
    else:
        roof = gemv_roof

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        try:
            m, kind, threads = build_cpu_model(cfg, qtype, bias)
            n, secs = time_cpu_tokens(m, cfg, 1, 64, 20.0)
            cpu = {"value": n / secs, "unit": "tok/s", "cores": threads, "kind": kind,
                   "sample": f"{n} greedy decode tokens of the full model at positions 1..{n} "
                             f"(~20 s of CPU time); the timed GPU run is at context "
                             f"{args.ctx}..{ctx_end}, where attention adds "
                             f"{kv_per_pos * mid_ctx / 1e9:.2f} GB/token on top of "
                             f"{step_weights / 1e9:.2f} GB of weights"}
            del m
        except Exception as e:
            cpu = {"value": None, "unit": "tok/s", "cores": 0, "kind": "unavailable",
                   "sample": str(e)[:200]}

    if rank == 0:
        value = args.steps / (ms / 1e3)
        line = {
            "metric": "decode tok/s", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": C.QTYPE_NAMES[qtype] + "/fp32",
            "data": "synthetic (seeded N(0,0.02) weights quantised like the reference; "
                    "random prompt id)",
            "config": {"workload": args.workload + (f" ({args.layers} layers)" if args.layers else ""),
                       "batch": 1, "ctx": args.ctx,
                       "ctx_end": ctx_end,
                       "parallelism": f"tp{world}" if world > 1 else "single gpu",
                       "l2": "no flush: each step streams %.2f GB of weights (> 126 MB L2)"
                             % (step_weights / 1e9),
                       "attention": "cpu-compat (reference CPU path V sum)",
                       "step": "persistent kernel" if step_kernel else "one kernel per op"},
            "e2e": {"value": args.steps / (e2e_ms / 1e3), "unit": "tok/s",
                    "h2d_bytes_per_step": 12, "d2h_bytes_per_step": cfg["vocab_size"] * 4,
                    "api": "mlb_forward_token (host logits)"},
            "roofline": roof,
            "step_roofline": step_roof,
            "gemv_roofline": gemv_roof,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": kpl * args.steps,
            "kernels_per_step": kpl,
            "resident_bytes": resident,
        }
        print(json.dumps(line))
    ctx.close()
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_gemv_sweep(args):
    """Standalone quantised GEMV/GEMM sweep: K = 4096, N x M over the formats,
    raw random GGUF blocks (fp16 scale |N(0,1)|*0.01, uniform codes), x ~ N(0,1).
    Each launch reads a different copy of the weights (copies > 2x L2)."""
    import torch

    import mini_llama_b200 as mlb

    peak = measured_peaks()
    qnames = {v: k for k, v in C.QTYPE_NAMES.items()}
    k = 4096
    rows = []
    windows = []  # host times of the timed loops (clock samples are kept from these)
    with Clocks([0]) as clk:
        for qn in args.sweep_q.split(","):
            qtype = qnames[qn]
            for n in [int(v) for v in args.sweep_n.split(",")]:
                wbytes = n * (k // 32) * C.BLOCK_BYTES[qtype]
                copies = max(2, int(np.ceil(260e6 / wbytes)))
                mats = [mlb.QMatrix.synthesize(qtype, n, k, SEED, 7000 + i, raw=True)
                        for i in range(copies)]
                for m in [int(v) for v in args.sweep_m.split(",")]:
                    x = torch.randn(m, k, device="cuda")
                    y = torch.empty(m, n, device="cuda")
                    for i in range(args.warmup):
                        mats[i % copies].gemv(x, y)
                    torch.cuda.synchronize()
                    torch.cuda.profiler.start()
                    t0 = time.time()
                    us = 1e3 * time_launches(torch, lambda i: mats[i % copies].gemv(x, y),
                                             args.steps, min_seconds=0.4)
                    windows.append((t0, time.time()))
                    torch.cuda.profiler.stop()
                    nbytes = wbytes + m * k * 4 + m * n * 4
                    rows.append({"q": qn, "n": n, "k": k, "m": m, "us": us,
                                 "gbs": nbytes / (us * 1e-6) / 1e9,
                                 "frac": nbytes / (us * 1e-6) / 1e9 / peak[0]})
                del mats
    head = next((r for r in rows if r["q"] == "q4_0" and r["m"] == 1 and r["n"] == 11008), rows[0])
    cpu = None
    if not args.no_cpu_baseline:
        import oracle

        if oracle.ref_available():
            r = oracle.ref()
            r.set_threads(cpu_threads())
            kind, lib, threads = "reference", r, r.threads()
        else:
            kind, lib, threads = "port", oracle.port(), 1
        # every (format, N) of the sweep at M = 1, ~2 s each; a batch of M rows is
        # M calls on the reference's CPU path (its batch loop is sequential)
        x = np.random.default_rng(0).normal(0, 1, k).astype(np.float32)
        single = {}
        for qn in args.sweep_q.split(","):
            qtype = qnames[qn]
            for n in [int(v) for v in args.sweep_n.split(",")]:
                w = C.synth_tensor(SEED, C.W_WQ, 0, qtype, n, k, threads=cpu_threads())
                lib.linear(qtype, x, w, n)  # warm
                t0 = time.perf_counter()
                reps = 0
                while time.perf_counter() - t0 < 2.0:
                    lib.linear(qtype, x, w, n)
                    reps += 1
                single[(qn, n)] = ((time.perf_counter() - t0) / reps, reps, w.nbytes)
        for r in rows:
            secs, _, wb = single[(r["q"], r["n"])]
            r["cpu_us"] = r["m"] * secs * 1e6
            r["cpu_gbs"] = (wb + k * 4 + r["n"] * 4) / secs / 1e9
        secs, reps, wb = single[(head["q"], head["n"])]
        cpu = {"value": (wb + k * 4 + head["n"] * 4) / secs / 1e9, "unit": "GB/s",
               "cores": threads, "kind": kind,
               "sample": f"{reps} linear calls of {head['q']} {head['n']}x{k} M=1 (~2 s); "
                         "every sweep row carries cpu_us / cpu_gbs from the same ~2 s timing "
                         "of its (format, N) at M=1, times M rows"}
    print(json.dumps({
        "metric": "quant GEMV achieved HBM GB/s", "value": head["gbs"], "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["us"] / 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": head["q"] + "/fp32", "data": "synthetic raw GGUF blocks",
        "config": {"workload": "gemv-sweep", "headline": f"{head['q']} {head['n']}x{k} M=1",
                   "l2": "rotating weight copies > 2x L2"},
        "roofline": {"bound": "hbm", "achieved": head["gbs"], "peak": peak[0], "unit": "GB/s",
                     "frac": head["frac"], "traffic": None},
        "sweep": rows, "cpu_baseline": cpu, "clocks": clk.summary(windows),
        "gpu_launches": args.steps * len(rows)}))


def main():
    args = parse_args()
    if args.workload == "gemv-sweep":
        run_gemv_sweep(args)
        return
    rank, world, local = dist_env()
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    cfg, qtype, bias = C.WORKLOADS[args.workload]
    if args.layers:
        cfg = dict(cfg, n_layers=args.layers)
    if args.impl == "reference":
        run_reference(args, cfg, qtype, bias, world, rank)
        return
    run_gpu(args, cfg, qtype, bias, rank, world, local)


if __name__ == "__main__":
    main()
