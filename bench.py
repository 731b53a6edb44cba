#!/usr/bin/env python
"""Decode benchmark: tokens/s of the B200 decode path (default: Llama-2-7B shape,
Q4_0, batch 1, KV cache at depth 512) on N GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload NAME] [--ctx C]

N > 1 runs under torchrun, one rank per GPU, tensor parallel. Prints one JSON
line (rank 0). The decode state at depth C is the seeded K/V fill
(mlb_context_fill_kv on the GPU; the same values written through the
reference's KvCache::Write on the CPU), so both arms decode from identical
states and their greedy ids are compared. The reference arm (--impl
reference) times the reference's own CPU ForwardToken (oracle/_ref, built from
the reference's sources; its model is generated and quantised inside that
library, so no library of this project is loaded in that arm).
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

from mini_llama_b200 import configs as C  # noqa: E402  (shapes only: loads no library)

SEED = 20261201
KV_SEED = SEED + 1   # seeded K/V rows of the prefilled context
KV_SCALE = 1.25      # their scale (the K/V rows of these models are ~N(0, 1.28^2))
N_CHECK = 16         # greedy ids compared against the single-GPU / CPU reference run

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# the standalone gate/up GEMV 22016 x 4096 Q4_0, from an ncu capture of that
# launch: it equals the algorithmic bytes (weights + x + y) to 0.01%.
GEMV_TRAFFIC_BYTES = 50.79e6


def step_traffic_7b(layers, ctx):
    """DRAM bytes of one decode-step launch on the Llama-2-7B Q4_0 shape,
    modelled from ncu captures of the step kernel on 2- and 4-layer cases:
    77.6 MB fixed (lm_head, embedding row, activations) plus, per layer,
    114.1 MB of weights and small terms and the fp32 K and V rows read at the
    context (2 * 4 * 128 * 32 bytes per position)."""
    return 77.6e6 + layers * (114.08e6 + 2 * 4 * 128 * 32 * ctx)


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=64)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--workload", choices=sorted(C.WORKLOADS) + ["gemv-sweep"],
                   default="llama2-7b-q4_0")
    p.add_argument("--also", type=str,
                   default="llama3-8b-q8_0@32,qwen2-72b-q4_1@32,qwen2-72b-q4_1@32:bf16",
                   help="more workloads timed in the same run: NAME, NAME@BATCH or "
                        "NAME@BATCH:bf16 (bf16 KV cache), comma separated ('none' for none)")
    p.add_argument("--batch-ctx", type=int, default=4096,
                   help="K/V depth of every sequence of the batched workloads")
    p.add_argument("--batch-kv", choices=["f32", "bf16"], default="f32",
                   help="KV cache element type of the --batch line")
    p.add_argument("--batch", type=int, default=1,
                   help="B > 1: the line is --workload decoded as B sequences in lockstep "
                        "(the batched engine) at depth --batch-ctx, nothing else")
    p.add_argument("--sweep-n", type=str, default="4096,11008,14336")
    p.add_argument("--sweep-m", type=str, default="1,4,16,64")
    p.add_argument("--sweep-q", type=str, default="q4_0,q4_1,q8_0")
    p.add_argument("--no-sweep", action="store_true", help="skip the GEMV sweep of the N=1 line")
    p.add_argument("--ctx", type=int, default=512, help="KV positions filled before timing")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-gguf-load", action="store_true",
                   help="skip the GGUF load measurement of the N=1 line")
    p.add_argument("--layers", type=int, default=0,
                   help="override the layer count (small profiling cases only; not a bench line)")
    p.add_argument("--kv", choices=["f32", "bf16"], default="f32",
                   help="KV cache element type of the head workload's context (bf16: not the "
                        "reference's parity mode; its ids are not compared with the CPU path)")
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
    """nvidia-smi samples (read-only query) during the timed region."""

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
                 "-i", ",".join(str(g) for g in self.gpus), "-lms", "50"],
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


# ----------------------------------------------------- reference CPU path

def cpu_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def cpu_decode(cfg, qtype, bias, ctx0, n_max, budget_s, warm=1):
    """The reference's own CPU ForwardToken (oracle/_ref) on the seeded model,
    decoding greedily from the seeded K/V state at depth ctx0: `warm` untimed
    tokens, then up to n_max timed tokens or budget_s seconds. The model is
    generated and quantised inside oracle/_ref (the reference's quantisers), so
    this loads no library of this project."""
    import oracle

    tok = C.prompt_ids(SEED, 1, cfg["vocab_size"])[0]
    if oracle.ref_available():
        r = oracle.ref()
        r.set_threads(cpu_threads())
        kind, threads = "reference", r.threads()
        m = r.model(cfg).synthesize(qtype, SEED, bias, threads=cpu_threads())
        m.fill_kv(ctx0, KV_SEED, KV_SCALE)
    else:  # pragma: no cover - the reference tree was absent at build time
        raise RuntimeError("oracle/_ref (the reference's CPU build) is missing")
    ids, per_tok = [], []
    pos = ctx0
    for _ in range(warm):
        tok = int(np.argmax(m.forward_token(tok, pos)))
        ids.append(tok)
        pos += 1
    t0 = time.perf_counter()
    n = 0
    while n < n_max:
        t1 = time.perf_counter()
        tok = int(np.argmax(m.forward_token(tok, pos)))
        per_tok.append(time.perf_counter() - t1)
        ids.append(tok)
        pos += 1
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    secs = time.perf_counter() - t0
    del m
    return {"ids": ids, "n": n, "secs": secs, "per_tok_median_s": statistics.median(per_tok),
            "kind": kind, "threads": threads, "pos0": ctx0 + warm, "pos1": pos}


def run_reference(args, cfg, qtype, bias, world, rank):
    if rank != 0:
        return
    try:
        r = cpu_decode(cfg, qtype, bias, args.ctx, args.steps, 150.0, warm=max(1, min(args.warmup, 2)))
    except Exception as e:  # pragma: no cover
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU build failed: {e}"}))
        return
    v = r["n"] / r["secs"]
    sample = (f"{r['n']} greedy decode tokens of the full model at positions "
              f"{r['pos0']}..{r['pos1'] - 1} after the seeded K/V fill to depth {args.ctx} "
              f"(bounded to ~150 s), {r['threads']} threads; median per token "
              f"{r['per_tok_median_s'] * 1e3:.0f} ms")
    print(json.dumps({
        "impl": "reference", "metric": "decode tok/s", "value": v, "unit": "tok/s",
        "n_gpus": world, "steps": r["n"], "warmup": max(1, min(args.warmup, 2)),
        "ms_per_step": 1000.0 * r["secs"] / r["n"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": C.QTYPE_NAMES[qtype] + "/fp32",
        "data": "synthetic (seeded N(0,0.02) weights quantised by the reference's quantisers; "
                "seeded K/V rows to the context depth)",
        "config": {"workload": args.workload, "batch": 1, "ctx": args.ctx,
                   "parallelism": "cpu threads"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": r["threads"], "kind": r["kind"],
                         "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "greedy_ids": r["ids"][:N_CHECK],
    }))


# ---------------------------------------------------------------- GPU arm

def time_launches(torch, launch, n, min_seconds=0.0):
    """Average device time of one launch: n launches captured in a CUDA graph
    (no host launch latency between them), replayed and timed with events;
    the graph is replayed until the timed region lasts min_seconds (so clock
    samples can land in it). Returns (ms per launch, host (start, end) of the
    timed replays)."""
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
    h0 = time.time()
    a.record(cur)
    for _ in range(reps):
        g.replay()
    b.record(cur)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / (n * reps), (h0, time.time())


def gemv_roofline(torch, mlb, cfg, qtype, world, peak):
    """Live per-launch timing of the standalone fused gate/up GEMV of this
    rank's shard, rotating over copies that together exceed L2."""
    F = cfg["hidden_dim"] // world
    n, k = 2 * F, cfg["dim"]
    nbytes = n * ((k + 31) // 32) * C.BLOCK_BYTES[qtype] + k * 4 + (n // 2) * 4
    copies = max(2, int(np.ceil(400e6 / nbytes)))
    mats = [mlb.QMatrix.synthesize(qtype, n, k, SEED, 900 + i, raw=False) for i in range(copies)]
    x = torch.randn(1, k, device="cuda")
    y = torch.empty(1, n, device="cuda")
    ms, _ = time_launches(torch, lambda i: mats[i % copies].gemv(x, y), 8 * copies)
    achieved = nbytes / (ms * 1e-3) / 1e9
    single = world == 1 and n == 22016 and k == 4096 and qtype == C.Q4_0
    return {"bound": "hbm", "achieved": achieved, "peak": peak[0], "unit": "GB/s",
            "frac": achieved / peak[0],
            "traffic": GEMV_TRAFFIC_BYTES if single else None,
            "traffic_source": "ncu capture of one launch of this shape" if single else None,
            "kernel": f"gemv_sb_kernel<{C.QTYPE_NAMES[qtype]}> {n}x{k}",
            "bytes_per_launch": nbytes, "us_per_launch": ms * 1e3,
            "peak_source": peak[1] + " (MEASURED_PEAKS.json hbm_gbs, burst)"}


def gemv_sweep(torch, mlb, args, peak, with_cpu=True):
    """The K = 4096 quantised GEMV/GEMM sweep: N x M over Q4_0/Q4_1/Q8_0 on raw
    random GGUF blocks (fp16 scale |N(0,1)|*0.01, uniform codes), x ~ N(0,1).
    Each launch reads another copy of the weights (copies > 2x L2). Per row:
    device time, achieved GB/s and fraction of the measured copy bandwidth, and
    (with_cpu) the reference CPU path's time for the same M rows."""
    qnames = {v: k for k, v in C.QTYPE_NAMES.items()}
    k = 4096
    rows, windows = [], []
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
                for i in range(3):
                    mats[i % copies].gemv(x, y)
                torch.cuda.synchronize()
                ms, win = time_launches(torch, lambda i: mats[i % copies].gemv(x, y),
                                        4 * copies, min_seconds=0.25)
                windows.append(win)
                nbytes = wbytes + m * k * 4 + m * n * 4
                us = ms * 1e3
                rows.append({"q": qn, "n": n, "k": k, "m": m, "us": us,
                             "gbs": nbytes / (us * 1e-6) / 1e9,
                             "frac": nbytes / (us * 1e-6) / 1e9 / peak[0]})
            del mats
    cpu = None
    if with_cpu:
        import oracle

        if oracle.ref_available():
            r = oracle.ref()
            r.set_threads(cpu_threads())
            kind, lib, threads = "reference", r, r.threads()
        else:  # pragma: no cover
            kind, lib, threads = "port", oracle.port(), 1
        # every (format, N) at M = 1 for ~1.5 s; M rows cost M calls on the
        # reference's CPU path (its batch loop is sequential)
        x = np.random.default_rng(0).normal(0, 1, k).astype(np.float32)
        single = {}
        for qn in args.sweep_q.split(","):
            qtype = qnames[qn]
            for n in [int(v) for v in args.sweep_n.split(",")]:
                w = np.random.default_rng(n).integers(0, 256, (n, (k // 32) * C.BLOCK_BYTES[qtype]),
                                                      dtype=np.uint8)
                nh = 2 if qtype == C.Q4_1 else 1
                sc = (np.abs(np.random.default_rng(n + 1).normal(0, 1, (n, k // 32, nh))) * 0.01
                      ).astype(np.float16)
                w.reshape(n, k // 32, -1)[:, :, :2 * nh] = sc.view(np.uint8).reshape(n, k // 32, 2 * nh)
                lib.linear(qtype, x, w, n)  # warm
                t0 = time.perf_counter()
                reps = 0
                while time.perf_counter() - t0 < 1.5:
                    lib.linear(qtype, x, w, n)
                    reps += 1
                single[(qn, n)] = ((time.perf_counter() - t0) / reps, reps, w.nbytes)
        for r_ in rows:
            secs, _, wb = single[(r_["q"], r_["n"])]
            r_["cpu_us"] = r_["m"] * secs * 1e6
            r_["cpu_gbs"] = (wb + k * 4 + r_["n"] * 4) / secs / 1e9
        head = next(r_ for r_ in rows if r_["q"] == "q4_0" and r_["m"] == 1)
        secs, reps, wb = single[(head["q"], head["n"])]
        cpu = {"value": (wb + k * 4 + head["n"] * 4) / secs / 1e9, "unit": "GB/s",
               "cores": threads, "kind": kind,
               "sample": f"{reps} linear calls of {head['q']} {head['n']}x{k} M=1 (~1.5 s); "
                         "every row's cpu_us is its (format, N) at M=1 times M"}
    return rows, windows, cpu


PHASE_KINDS = ("qkv", "attention", "wo", "gate_up", "down")


def step_phase_summary(ctx, tok, pos, n_layers, n=5):
    """Per-phase times of the step kernel (mlb_context_step_trace), after the
    timed region: n single steps, each read on its own, medians over steps,
    summed over layers by phase kind. span: from the latest CTA end of the
    phase before to the latest CTA end of this one (grid barriers and
    cross-rank waits count in the phase after them); work_mean / work_max:
    the mean / largest CTA time from the phase's start (after its barrier) to
    its end."""
    ctx.step_trace(True)
    spans, wmean, wmax = [], [], []
    for _ in range(n):
        tok = ctx.decode_greedy(tok, pos, 1)[-1]
        pos += 1
        st = ctx.step_trace_read().astype(np.int64)
        start, end = st[:, :, 0], st[:, :, 1]
        ends = end.max(axis=1)
        spans.append(np.diff(np.concatenate([[start[0].min()], ends])) / 1e3)
        work = (end - start) / 1e3
        wmean.append(work.mean(axis=1))
        wmax.append(work.max(axis=1))
    ctx.step_trace(False)
    out = {}
    for key, rows in (("span", spans), ("work_mean", wmean), ("work_max", wmax)):
        med = np.median(np.stack(rows), axis=0)
        d = {k: round(float(med[i:5 * n_layers:5].sum()), 1) for i, k in enumerate(PHASE_KINDS)}
        d["lm_head"] = round(float(med[5 * n_layers:].sum()), 1)
        d["total"] = round(float(med.sum()), 1)
        out[key] = d
    out["unit"] = "us per step, summed over layers (median of single traced steps, this rank)"
    return out


def measure_workload(torch, mlb, dist, args, name, cfg, qtype, bias, rank, world, local,
                     steps, warmup, peak, check_single):
    """One decode workload on this rank: seeded model and K/V state at depth
    args.ctx, `warmup` untimed greedy steps, `steps` timed ones (CUDA events
    on the context stream, max over ranks), then the e2e loop through
    mlb_forward_token with host logits. check_single: rank 0 also decodes the
    first greedy ids on one GPU (tensor-parallel runs) for the id self-check."""
    barrier = lambda: (torch.cuda.synchronize(), dist.barrier() if dist else None)  # noqa: E731

    def max_over_ranks(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    nccl_id = None
    if world > 1:
        obj = [mlb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    model = mlb.CudaModel(cfg, device_id=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    model.synthesize(qtype, SEED, with_bias=bias)
    resident, step_weights = model.bytes()
    ctx = model.context(mlb.ATTN_CPU_COMPAT, step_kernel=False if args.per_op else None,
                        kv_type=mlb.KV_BF16 if (args.kv == "bf16" and name == args.workload)
                        else mlb.KV_F32)
    step_kernel = ctx.step_kernel()
    stream = torch.cuda.ExternalStream(ctx.stream())
    tok0 = C.prompt_ids(SEED, 1, cfg["vocab_size"])[0]
    ctx0 = args.ctx
    if ctx0 + warmup + 3 * steps + 12 > cfg["max_seq_len"]:
        raise SystemExit("context too long for max_seq_len")
    ctx.fill_kv(ctx0, KV_SEED, KV_SCALE)
    ids = ctx.decode_greedy(tok0, ctx0, warmup) if warmup else []
    pos = ctx0 + warmup
    tok = ids[-1] if ids else tok0
    barrier()

    with Clocks([local]) as clk:
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0 = time.time()
        ev0.record(stream)
        ids += ctx.decode_greedy(tok, pos, steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        h1 = time.time()
        barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    clocks = clk.summary([(h0 - 0.1, h1 + 0.1)])
    pos += steps
    ctx_end = pos
    tok = ids[-1]

    # e2e: ForwardToken through the C ABI, host logits every step
    for _ in range(2):
        tok = int(np.argmax(ctx.forward_token(tok, pos)))
        pos += 1
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        lg = ctx.forward_token(tok, pos)
        tok = int(np.argmax(lg))
        pos += 1
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    # the on-device sampling loop (mlb_decode_sample, temperature 0.8, top-k
    # 40): the same step plus one sampling kernel per step, same clock rules
    sampler = mlb.Sampler(SEED, device_id=local)
    ctx.decode_sample(sampler, tok, pos, 2, 0.8, 40)
    pos += 2
    barrier()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    tok = ctx.decode_sample(sampler, tok, pos, steps, 0.8, 40)[-1]
    s1.record(stream)
    torch.cuda.synchronize()
    barrier()
    pos += steps
    sample_ms = max_over_ranks(s0.elapsed_time(s1))
    sampler.close()
    kpl = ctx.kernels_per_step()
    phases = step_phase_summary(ctx, tok, pos, cfg["n_layers"]) if step_kernel else None
    ctx.close()
    model.close()

    # the tensor-parallel ids against one GPU decoding from the same state
    tp_check = None
    if check_single and world > 1:
        if rank == 0:
            n = min(N_CHECK, len(ids))
            one = mlb.CudaModel(cfg, device_id=local).synthesize(qtype, SEED, with_bias=bias)
            c1 = one.context(mlb.ATTN_CPU_COMPAT)
            c1.fill_kv(ctx0, KV_SEED, KV_SCALE)
            ids1 = c1.decode_greedy(tok0, ctx0, n)
            c1.close()
            one.close()
            tp_check = {"tp_ids_match": ids1 == ids[:n], "n": n,
                        "against": "one GPU (step kernel) from the same seeded state"}
        barrier()

    kv_bytes = 2 if (args.kv == "bf16" and name == args.workload) else 4
    kv_per_pos = 2 * cfg["n_layers"] * (cfg["n_kv_heads"] // world) * cfg["head_dim"] * kv_bytes
    mid_ctx = (ctx0 + warmup + ctx_end) / 2
    step_bytes = step_weights + kv_per_pos * mid_ctx
    step_s = ms / 1e3 / steps
    roof = {"bound": "hbm", "achieved": step_bytes / step_s / 1e9, "peak": peak[0],
            "unit": "GB/s", "frac": step_bytes / step_s / 1e9 / peak[0],
            "bytes_per_launch": step_bytes, "us_per_launch": step_s * 1e6,
            "kernel": (f"decode_step_kernel<{C.QTYPE_NAMES[qtype]}>" if step_kernel
                       else "per-op graph"),
            "note": "algorithmic bytes: GGUF weight bytes of this rank + fp32 K and V read per "
                    "token at the mean timed context; time: CUDA events on the context stream "
                    "around the timed greedy steps (one step-kernel launch per step)",
            "peak_source": peak[1] + " (MEASURED_PEAKS.json hbm_gbs, burst)"}
    if step_kernel and name == "llama2-7b-q4_0" and world == 1 and not args.layers:
        roof["traffic"] = step_traffic_7b(cfg["n_layers"], mid_ctx)
        roof["traffic_source"] = "modelled from ncu captures of 2- and 4-layer cases"
    else:
        roof["traffic"] = None
    return {
        "name": name, "value": steps / (ms / 1e3), "ms_per_step": ms / steps, "steps": steps,
        "warmup": warmup, "ids": ids, "ctx_end": ctx_end, "clocks": clocks,
        "e2e": {"value": steps / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": 12,
                "d2h_bytes_per_step": cfg["vocab_size"] * 4,
                "api": "mlb_forward_token (host logits)"},
        "roofline": roof, "kernels_per_step": kpl, "step_kernel": step_kernel,
        "resident_bytes": resident, "step_weight_bytes": step_weights, "tp_check": tp_check,
        "gpu_launches": kpl * steps, "step_phases": phases,
        "decode_sample": {"value": steps / (sample_ms / 1e3), "unit": "tok/s",
                          "temperature": 0.8, "top_k": 40,
                          "api": "mlb_decode_sample (device sampling, ids to host at the end)"},
    }


def measure_batch(torch, mlb, dist, args, name, cfg, qtype, bias, B, ctx0, rank, world, local,
                  steps, warmup, peak, kv_bf16=False):
    """B sequences decoded in lockstep (mlb_batch_decode_greedy: the tcgen05
    GEMM for every projection, batched attention), each from its own seeded
    K/V state at depth ctx0. Time: CUDA events on the batch stream around the
    timed steps, max over ranks; tokens/s counts B tokens per step. Rank 0
    checks the greedy ids of the first and last sequence against one GPU's
    single-sequence step kernel from the same state."""
    barrier = lambda: (torch.cuda.synchronize(), dist.barrier() if dist else None)  # noqa: E731

    def max_over_ranks(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg = dict(cfg, max_seq_len=min(cfg["max_seq_len"], ctx0 + warmup + steps + 64))
    nccl_id = None
    if world > 1:
        obj = [mlb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    model = mlb.CudaModel(cfg, device_id=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    model.synthesize(qtype, SEED, with_bias=bias)
    _, step_weights = model.bytes()
    b = mlb.Batch(model, B, kv_type=mlb.KV_BF16 if kv_bf16 else mlb.KV_F32)
    for s in range(B):
        b.fill_kv(s, ctx0, KV_SEED + s, KV_SCALE)
    toks = C.prompt_ids(SEED + 7, B, cfg["vocab_size"])
    ids_w = b.decode_greedy(toks, [ctx0] * B, warmup)
    stream = torch.cuda.ExternalStream(b.stream())
    barrier()
    with Clocks([local]) as clk:
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0 = time.time()
        ev0.record(stream)
        ids_t = b.decode_greedy(ids_w[-1], [ctx0 + warmup] * B, steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        h1 = time.time()
        barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    clocks = clk.summary([(h0 - 0.1, h1 + 0.1)])
    kps = b.kernels_per_step()
    ids = np.concatenate([ids_w, ids_t])
    b.close()
    model.close()
    check = None
    if rank == 0 and kv_bf16:
        check = {"seq_ids_match": None,
                 "note": "bf16 KV cache: results follow the reference CPU path with K and V "
                         "rounded to bf16, checked against the C port in "
                         "tests/test_gpu_batch.py; the fp32 step kernel is not its comparator"}
    elif rank == 0:
        # Teacher-forced: one GPU's single-sequence step kernel is fed the
        # batch's own ids, and its argmax at every step must be the batch's
        # next id. Where it is not, the step kernel's top-2 margin there is
        # recorded (two GPU paths summing in different orders can part on a
        # near tie without either leaving the logits bar).
        n = min(N_CHECK, len(ids))
        one = (mlb.CudaModel(cfg, device_id=local).synthesize(qtype, SEED, with_bias=bias))
        c1 = one.context(mlb.ATTN_CPU_COMPAT)
        mism = []
        for s in (0, B - 1):
            c1.reset()
            c1.fill_kv(ctx0, KV_SEED + s, KV_SCALE)
            tok = toks[s]
            for t in range(n):
                lg = c1.forward_token(tok, ctx0 + t)
                top = np.argsort(lg)[-2:]
                if int(top[-1]) != int(ids[t, s]):
                    mism.append({"seq": s, "step": t, "margin": float(lg[top[-1]] - lg[top[-2]])})
                tok = int(ids[t, s])
        c1.close()
        one.close()
        check = {"seq_ids_match": not mism, "sequences": [0, B - 1], "n": n,
                 "mismatches": mism,
                 "against": "one GPU's single-sequence step kernel, teacher-forced on the "
                            "batch's ids from the same seeded state"}
    barrier()
    kv_per_pos = 2 * cfg["n_layers"] * (cfg["n_kv_heads"] // world) * cfg["head_dim"] * (
        2 if kv_bf16 else 4)
    mid_ctx = ctx0 + warmup + steps / 2
    step_bytes = step_weights + B * kv_per_pos * mid_ctx
    step_s = ms / 1e3 / steps
    return {
        "name": name, "value": B * steps / (ms / 1e3), "unit": "tok/s",
        "ms_per_step": ms / steps, "steps": steps, "warmup": warmup, "batch": B, "ctx": ctx0,
        "parallelism": f"tp{world}" if world > 1 else "single gpu",
        "roofline": {"bound": "hbm", "achieved": step_bytes / step_s / 1e9, "peak": peak[0],
                     "unit": "GB/s", "frac": step_bytes / step_s / 1e9 / peak[0],
                     "bytes_per_step": step_bytes, "weight_bytes": step_weights,
                     "kv_bytes": B * kv_per_pos * mid_ctx,
                     "note": "algorithmic bytes: GGUF weights of this rank once per step + every "
                             "sequence's K and V (%s) at the mean timed context"
                             % ("bf16" if kv_bf16 else "fp32"),
                     "peak_source": peak[1] + " (MEASURED_PEAKS.json hbm_gbs, burst)"},
        "clocks": clocks, "parity": check, "greedy_ids_seq0": [int(v) for v in ids[:N_CHECK, 0]],
        "kernels_per_step": kps, "gpu_launches": kps * steps,
        "data": "seeded weights; each sequence's K/V rows seeded to depth ctx; seeded tokens",
        "kv_cache": "bf16" if kv_bf16 else "fp32",
    }


def run_gpu(args, cfg, qtype, bias, rank, world, local):
    import torch

    import mini_llama_b200 as mlb

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    peak = measured_peaks()
    if args.batch > 1:
        run_batch_line(torch, mlb, dist, args, cfg, qtype, bias, rank, world, local, peak)
        return
    head = measure_workload(torch, mlb, dist, args, args.workload, cfg, qtype, bias, rank, world,
                            local, args.steps, args.warmup, peak, check_single=True)
    extras = []
    for spec in [] if args.also in ("", "none") or args.layers else args.also.split(","):
        name, _, bsz = spec.partition("@")
        bsz, _, kvt = bsz.partition(":")
        B = int(bsz) if bsz else 1
        if name == args.workload and B == 1:
            continue
        ecfg, eq, eb = C.WORKLOADS[name]
        try:
            if B > 1:
                r = measure_batch(torch, mlb, dist, args, name, ecfg, eq, eb, B, args.batch_ctx,
                                  rank, world, local, min(args.steps, 16),
                                  max(3, min(args.warmup, 4)), peak, kv_bf16=kvt == "bf16")
                r["name"] = f"{name}_b{B}" + ("_bf16kv" if kvt == "bf16" else "")
                extras.append(r)
            else:
                extras.append(measure_workload(torch, mlb, dist, args, name, ecfg, eq, eb, rank,
                                               world, local, min(args.steps, 24),
                                               max(3, min(args.warmup, 4)), peak,
                                               check_single=True))
        except Exception as e:  # reported, not fatal
            extras.append({"name": spec, "error": str(e)[:300]})

    gemv_roof = sweep = sweep_cpu = None
    cpu = None
    gguf = None
    if rank == 0 and world == 1:
        gemv_roof = gemv_roofline(torch, mlb, cfg, qtype, world, peak)
        if not args.no_gguf_load and not args.layers:
            try:
                gguf = gguf_load(torch, mlb, cfg, qtype, bias, local,
                                 with_ref=not args.no_cpu_baseline)
            except Exception as e:  # reported, not fatal
                gguf = {"error": str(e)[:300]}
        if not args.no_sweep and not args.layers:
            with Clocks([local]) as clk:
                sweep, windows, sweep_cpu = gemv_sweep(torch, mlb, args, peak,
                                                       with_cpu=not args.no_cpu_baseline)
            sweep_clocks = clk.summary(windows)
        if not args.no_cpu_baseline:
            try:
                r = cpu_decode(cfg, qtype, bias, args.ctx, 64, 20.0, warm=1)
                n_cmp = min(N_CHECK, len(r["ids"]), len(head["ids"]))
                cpu = {"value": r["n"] / r["secs"], "unit": "tok/s", "cores": r["threads"],
                       "kind": r["kind"],
                       "sample": f"{r['n']} greedy decode tokens of the full model at positions "
                                 f"{r['pos0']}..{r['pos1'] - 1} after the seeded K/V fill to "
                                 f"depth {args.ctx} (~20 s of CPU time); median per token "
                                 f"{r['per_tok_median_s'] * 1e3:.0f} ms",
                       "ids_match_gpu": r["ids"][:n_cmp] == head["ids"][:n_cmp],
                       "ids_compared": n_cmp}
            except Exception as e:
                cpu = {"value": None, "unit": "tok/s", "cores": 0, "kind": "unavailable",
                       "sample": str(e)[:200]}

    if rank == 0:
        value = head["value"]
        parity = {}
        if head["tp_check"]:
            parity.update(head["tp_check"])
        if cpu and "ids_match_gpu" in cpu and args.kv == "f32":
            parity["ref_ids_match"] = cpu["ids_match_gpu"]
            parity["ref_ids_compared"] = cpu["ids_compared"]
        line = {
            "metric": "decode tok/s", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": C.QTYPE_NAMES[qtype] + "/fp32",
            "data": "synthetic (seeded N(0,0.02) weights quantised like the reference; seeded "
                    "K/V rows to the context depth; seeded prompt id)",
            "config": {"workload": args.workload + (f" ({args.layers} layers)" if args.layers else ""),
                       "batch": 1, "ctx": args.ctx, "ctx_end": head["ctx_end"],
                       "parallelism": f"tp{world}" if world > 1 else "single gpu",
                       "l2": "no flush: each step streams %.2f GB of weights (> 126 MB L2)"
                             % (head["step_weight_bytes"] / 1e9),
                       "attention": "cpu-compat (reference CPU path V sum)",
                       "kv_cache": args.kv,
                       "step": "persistent kernel" if head["step_kernel"] else "one kernel per op"},
            "e2e": head["e2e"],
            "roofline": head["roofline"],
            "parity": parity,
            "greedy_ids": head["ids"][:N_CHECK],
            "cpu_baseline": cpu,
            "clocks": head["clocks"],
            "gpu_launches": head["gpu_launches"],
            "kernels_per_step": head["kernels_per_step"],
            "resident_bytes": head["resident_bytes"],
            "step_phases": head["step_phases"],
            "decode_sample": head["decode_sample"],
        }
        if gemv_roof:
            line["gemv_roofline"] = gemv_roof
        if gguf:
            line["gguf_load"] = gguf
        if sweep:
            line["gemv_sweep"] = {"rows": sweep, "cpu_baseline": sweep_cpu,
                                  "clocks": sweep_clocks,
                                  "note": "standalone gemv_sb_kernel, K = 4096, raw random GGUF "
                                          "blocks; bytes = weights + M*K*4 + M*N*4; frac of the "
                                          "measured copy bandwidth"}
        for e in extras:
            key = e["name"].replace("-", "_")
            if "error" in e:
                line[key] = {"error": e["error"]}
                continue
            if "batch" in e:
                line[key] = e
                continue
            line[key] = {"value": e["value"], "unit": "tok/s", "ms_per_step": e["ms_per_step"],
                         "steps": e["steps"], "warmup": e["warmup"], "batch": 1,
                         "ctx": args.ctx, "e2e": e["e2e"], "roofline": e["roofline"],
                         "clocks": e["clocks"], "parity": e["tp_check"],
                         "greedy_ids": e["ids"][:N_CHECK], "gpu_launches": e["gpu_launches"],
                         "parallelism": f"tp{world}" if world > 1 else "single gpu"}
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def gguf_load(torch, mlb, cfg, qtype, bias, local, with_ref):
    """The workload's model written as a GGUF v3 file (seeded weights, one
    tensor at a time) and loaded with mlb_model_load_gguf: wall time from the
    call to a finalized model (parse, pinned staged upload of every tensor,
    repack), the file then in the host page cache. Checked: the loaded model's
    logits at position 0 equal those of the same model synthesised on the
    device. with_ref: the reference's LoadGgufModel reading the same file into
    host memory (its upload to a GPU is not part of its CPU build)."""
    import shutil

    from mini_llama_b200 import gguf_writer as GW

    d = tempfile.mkdtemp(prefix="mlb_gguf_")
    path = os.path.join(d, "model.gguf")
    try:
        t0 = time.perf_counter()
        nbytes = GW.write_synthetic_model(path, cfg, qtype, SEED, bias, threads=cpu_threads())
        t_write = time.perf_counter() - t0
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        m = mlb.CudaModel.from_gguf(path, device_id=local)
        torch.cuda.synchronize()
        t_load = time.perf_counter() - t0
        tok = C.prompt_ids(SEED, 1, cfg["vocab_size"])[0]
        c = m.context(mlb.ATTN_CPU_COMPAT)
        lg = c.forward_token(tok, 0)
        c.close()
        uploaded = m.gguf_bytes
        m.close()
        s = mlb.CudaModel(cfg, device_id=local).synthesize(qtype, SEED, with_bias=bias)
        c = s.context(mlb.ATTN_CPU_COMPAT)
        same = bool(np.array_equal(lg, c.forward_token(tok, 0)))
        c.close()
        s.close()
        out = {"file_bytes": nbytes, "uploaded_bytes": uploaded, "load_s": t_load,
               "gbs": nbytes / t_load / 1e9, "write_s": t_write,
               "logits_equal_synthesized": same,
               "api": "mlb_model_load_gguf (mmap, pinned staging, repack, finalize)",
               "note": "file just written, so read from the host page cache"}
        if with_ref:
            import oracle

            if oracle.ref_available():
                t0 = time.perf_counter()
                rm = oracle.ref().load_gguf(path)
                out["reference_load_s"] = time.perf_counter() - t0
                out["reference_api"] = "LoadGgufModel into host memory (CPU build)"
                del rm
        return out
    finally:
        shutil.rmtree(d, ignore_errors=True)


def run_batch_line(torch, mlb, dist, args, cfg, qtype, bias, rank, world, local, peak):
    """--batch B: one line for --workload decoded as B sequences in lockstep."""
    r = measure_batch(torch, mlb, dist, args, args.workload, cfg, qtype, bias, args.batch,
                      args.batch_ctx, rank, world, local, args.steps, args.warmup, peak,
                      kv_bf16=args.batch_kv == "bf16")
    if rank == 0:
        print(json.dumps({
            "metric": "decode tok/s", "value": r["value"], "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": C.QTYPE_NAMES[qtype] + "/fp32", "data": r["data"],
            "config": {"workload": args.workload + (f" ({args.layers} layers)" if args.layers else ""),
                       "batch": args.batch, "ctx": args.batch_ctx, "parallelism": r["parallelism"],
                       "kv_cache": r["kv_cache"],
                       "l2": "no flush: each step streams the weights and every sequence's K/V "
                             "(> 126 MB L2)"},
            "roofline": r["roofline"], "parity": r["parity"], "clocks": r["clocks"],
            "greedy_ids_seq0": r["greedy_ids_seq0"], "gpu_launches": r["gpu_launches"],
            "kernels_per_step": r["kernels_per_step"]}))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_gemv_sweep(args):
    """The sweep alone as its own line (--workload gemv-sweep)."""
    import torch

    import mini_llama_b200 as mlb

    peak = measured_peaks()
    with Clocks([0]) as clk:
        rows, windows, cpu = gemv_sweep(torch, mlb, args, peak,
                                        with_cpu=not args.no_cpu_baseline)
    head = next((r for r in rows if r["q"] == "q4_0" and r["m"] == 1 and r["n"] == 11008), rows[0])
    print(json.dumps({
        "metric": "quant GEMV achieved HBM GB/s", "value": head["gbs"], "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["us"] / 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": head["q"] + "/fp32", "data": "synthetic raw GGUF blocks",
        "config": {"workload": "gemv-sweep", "headline": f"{head['q']} {head['n']}x4096 M=1",
                   "l2": "rotating weight copies > 2x L2"},
        "roofline": {"bound": "hbm", "achieved": head["gbs"], "peak": peak[0], "unit": "GB/s",
                     "frac": head["frac"], "traffic": None},
        "sweep": rows, "cpu_baseline": cpu, "clocks": clk.summary(windows),
        "gpu_launches": len(rows)}))


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
