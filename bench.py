#!/usr/bin/env python
"""Decode throughput of libcortex on B200: generated tokens per second.

Workload (the d=1024 configuration of the headline metric): a seeded
d=1024, 2-layer, 16-head, ctx-1024, V=16384 SNAI_V4 model (fp32 weights
N(0, 0.02), unit RMSNorm weights), 4096 independent sequences split evenly
over the ranks, prompts of 512 uniform random ids, then decode steps at
positions 512..1023 with the reference's top-k/top-p sampler (variant of
src/tensor_ffi_adapter.php:168-204: T=0.7, top_k=40, top_p=0.9, subtractive
repetition penalty 1.1 over every token fed so far) and seeded per-step
uniform draws; projections run on tcgen05 tensor cores with bf16 operands and
fp32 accumulation; the KV cache is fp32.

A step is one decode step of every local sequence (sample one id from the
current logits, feed it).  Warm-up and timed steps continue the generation;
after position 1023 the sequences are rewound to 512 (cortex_seq_rewind), so
every step attends over 513..1024 positions, like the full job.  The KV
cache (68.7 GB on one GPU) is far larger than L2, so no L2 flush is needed.

`value` is timed with CUDA events on the engine's stream over exactly
--steps steps through the device-pointer API (inputs resident in HBM);
`e2e` repeats the measurement through the host-pointer C-ABI call
(uniforms in, ids out each step).  Multi-GPU: one process per GPU under
torchrun, no collective on the data path; the max over ranks is reported.

--impl reference times the oracle port of the reference's CPU engine
(oracle/snai_oracle.c: core/cortex.nim forward + the PHP sampler, libm exp)
on all host threads over a bounded sample of the same workload.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

V, D, L, CTX, HEADS = 16384, 1024, 2, 1024, 16
PROMPT = 512
TOTAL_SEQS = 4096
T, TOP_K, TOP_P, REP = 0.7, 40, 0.9, 1.1
VARIANT = 1  # 0: src/snai_inference.php sampler, 1: src/tensor_ffi_adapter.php sampler
METRIC = "generated tokens/sec (d=1024 decode)"
UNIT = "tokens/s"
CONFIG = {
    "workload": "d=1024 L=2 heads=16 V=16384 ctx=1024, 4096 sequences, prompt 512 + decode to 1024, "
                "top-k 40 / top-p 0.9 / T 0.7 / rep 1.1 sampling",
    "model": "seeded SNAI_V4 d1024 L2 (init_base layout, N(0,0.02))",
    "global_batch": TOTAL_SEQS,
    "seq_len": CTX,
    "prompt": PROMPT,
    "gemm": "tcgen05 bf16 x bf16 -> fp32",
    "kv_cache": "fp32",
    "l2": "inputs larger than L2 (KV cache 68.7 GB / 1 GPU)",
    "parallelism": "independent sequences sharded over ranks (no collective)",
}


# Smaller configurations of the same metric (--config); the default run is c4.
CONFIGS = {
    "c2": dict(D=256, L=4, HEADS=4, PROMPT=256, TOTAL_SEQS=64, VARIANT=0, T=0.8, REP=1.15,
               workload="d=256 L=4 heads=4 V=16384 ctx=1024, 64 sequences, prompt 256 + decode, "
                        "variant-A sampling T 0.8 / rep 1.15"),
    "c3": dict(D=512, L=2, HEADS=8, PROMPT=512, TOTAL_SEQS=512, VARIANT=1, T=0.7, REP=1.1,
               workload="d=512 L=2 heads=8 V=16384 ctx=1024, 512 sequences, prompt 512 + decode to 1024, "
                        "top-k 40 / top-p 0.9 / T 0.7 / rep 1.1 sampling"),
}


def apply_config(name):
    global D, L, HEADS, PROMPT, TOTAL_SEQS, VARIANT, T, REP, METRIC
    c = CONFIGS[name]
    D, L, HEADS, PROMPT, TOTAL_SEQS = c["D"], c["L"], c["HEADS"], c["PROMPT"], c["TOTAL_SEQS"]
    VARIANT, T, REP = c["VARIANT"], c["T"], c["REP"]
    METRIC = f"generated tokens/sec (d={D} decode)"
    kv = TOTAL_SEQS * L * 2 * CTX * D * 4 / 1e9
    CONFIG.update(workload=c["workload"], model=f"seeded SNAI_V4 d{D} L{L} (init_base layout, N(0,0.02))",
                  global_batch=TOTAL_SEQS, prompt=PROMPT,
                  l2=f"KV cache {kv:.1f} GB; weights may stay L2-resident (measured as is, no flush)")


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def model_path(rank):
    d = os.environ.get("SNAI_BENCH_DIR", tempfile.gettempdir())
    return os.path.join(d, f"snai_bench_d{D}_L{L}_seed1234_r{rank}.snai")


def make_model(rank):
    from snai_b200 import modelgen
    p = model_path(rank)
    if not os.path.exists(p) or os.path.getsize(p) != modelgen.expected_size(V, D, 4 * D, L):
        modelgen.random_model(p, V, D, CTX, L, seed=1234, std=0.02)
    return p


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", ",".join(str(g) for g in self.gpus)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def visible_gpu_ids(n):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        return ids[:n]
    return [str(i) for i in range(n)]


def cpu_sample(steps_timed, nthreads, start_pos=768, nseq=None, warmup=1):
    """Times the oracle port (one thread per sequence) for a bounded sample."""
    import oracle as O
    path = make_model(0)
    o = O.Oracle(path, num_heads=HEADS)
    nseq = nseq or nthreads
    b = o.batch(nseq, start_pos, seed=99)
    for _ in range(warmup):
        b.step(VARIANT, T, REP, TOP_K, TOP_P, nthreads)
    secs = 0.0
    for _ in range(steps_timed):
        secs += b.step(VARIANT, T, REP, TOP_K, TOP_P, nthreads)
    b.close()
    o.close()
    return nseq * steps_timed / secs, secs, nseq


def reference_arm(args, rank, world):
    """The reference's CPU path (oracle port) on all host threads."""
    if rank != 0:
        return
    nthreads = os.cpu_count() or 1
    # each step: one decode step of `nthreads` sequences at positions from 768 on
    rate, secs, nseq = cpu_sample(args.steps, nthreads, warmup=args.warmup)
    sample = (f"{nseq} sequences x {args.steps} decode steps from position 768 (job mean), one thread per "
              f"sequence, after {args.warmup} warm-up steps")
    line = {"impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * secs / max(1, args.steps),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded model, random ids)", "config": CONFIG,
            "cpu_baseline": {"value": rate, "unit": UNIT, "cores": nthreads, "kind": "port", "sample": sample},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def our_arm(args, rank, world, local_rank):
    global TOTAL_SEQS
    TOTAL_SEQS = args.seqs
    import torch
    import torch.distributed as dist
    from snai_b200 import PREC_BF16, Cortex, sample_params

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if TOTAL_SEQS % world:
        raise SystemExit(f"{TOTAL_SEQS} sequences do not split over {world} ranks")
    B = TOTAL_SEQS // world
    path = make_model(rank)
    eng = Cortex(path, num_heads=HEADS, max_seqs=B, device=local_rank, precision=PREC_BF16)
    stream = torch.cuda.Stream(device=dev)
    eng.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(1234)
    prompts = rng.integers(0, V, (TOTAL_SEQS, PROMPT)).astype(np.int32)[rank * B:(rank + 1) * B]

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- prefill (reported separately) ----
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for s0 in range(0, B, 256):
            toks = torch.from_numpy(np.ascontiguousarray(prompts[s0:s0 + 256].ravel())).to(dev)
            n = min(256, B - s0)
            eng.forward_dev(toks, n, PROMPT, slots=np.arange(s0, s0 + n))
    eng.synchronize()
    prefill_s = max_over_ranks(time.perf_counter() - t0)

    prm = sample_params(VARIANT, T, REP, TOP_K, TOP_P)
    total_steps = args.warmup + args.steps
    U = torch.from_numpy(rng.random((total_steps, B), dtype=np.float32)).to(dev)
    ids = torch.zeros(B, dtype=torch.int32, device=dev)

    def step_dev(i):
        if eng.pos(0) >= CTX:
            eng.rewind(PROMPT)
        eng.decode_dev(U[i], prm, ids)

    ids_all = torch.zeros((args.steps, B), dtype=torch.int32, device=dev)

    def steps_dev(i0, n):
        # n decode steps in one call (cortex_decode_steps: one captured step
        # replayed as a CUDA graph), rewinding at the context limit
        while n > 0:
            if eng.pos(0) >= CTX:
                eng.rewind(PROMPT)
            k = min(n, CTX - eng.pos(0))
            eng.decode_steps_dev(U[i0:i0 + k], prm, ids_all[:k])
            i0 += k
            n -= k

    # ---- device-resident decode (value) ----
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step_dev(i)
    eng.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches0 = eng.launches
    # The library's CUDA-event profiler brackets every launch with events.  At
    # d=1024 (8 ms steps, the GPU never waits for the host) it runs inside the
    # timed region; the small configurations are host-launch-bound, so there
    # it runs in a separate pass after the timed region.
    prof_in_timed = args.config == "c4"
    if prof_in_timed:
        eng.profile(True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(visible_gpu_ids(world) if rank == 0 else []) as clk:
        with torch.cuda.stream(stream):
            torch.cuda.nvtx.range_push("timed")
            ev0.record(stream)
            if prof_in_timed:
                for i in range(args.steps):  # the profiler needs the per-step path
                    step_dev(args.warmup + i)
            else:
                steps_dev(args.warmup, args.steps)
            ev1.record(stream)
            torch.cuda.nvtx.range_pop()
        ev1.synchronize()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    launches = eng.launches - launches0
    barrier()
    ms_max = max_over_ranks(ms)

    if not prof_in_timed:
        eng.profile(True)
        with torch.cuda.stream(stream):
            for i in range(min(args.steps, 64)):
                step_dev(args.warmup + i)
        eng.synchronize()
    prof = eng.profile_read()
    eng.profile(False)

    # ---- end to end through the host-pointer C ABI (e2e) ----
    eng.rewind(PROMPT)
    Uh = rng.random((total_steps, B), dtype=np.float32)
    out_ids = np.zeros(B, dtype=np.int32)

    def step_host(i):
        # one call per step from host memory (uniforms in, ids out), through
        # the graph-replayed decode
        if eng.pos(0) >= CTX:
            eng.rewind(PROMPT)
        out_ids[:] = eng.decode_steps(Uh[i:i + 1], prm)[0]

    for i in range(args.warmup):
        step_host(i)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step_host(args.warmup + i)
    e1.record(stream)
    e1.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))

    tokens = TOTAL_SEQS * args.steps
    value = tokens / (ms_max / 1e3)
    e2e_value = tokens / (e2e_ms / 1e3)

    if rank == 0:
        peak, peak_kind = load_peaks()
        att_n, att_ms, att_bytes, _ = prof["attention"]
        achieved = (att_bytes / att_n) / (att_ms / att_n / 1e3) / 1e9 if att_n else None
        # DRAM traffic per launch: the ratio of ncu-measured to algorithmic
        # bytes of a smaller capture (same kernel, traffic proportional to the
        # KV positions read) times this run's algorithmic bytes per launch
        traffic = None
        tp = os.path.join(ROOT, "profiles", "attention_decode_traffic.json")
        if os.path.exists(tp) and att_n:
            try:
                traffic = json.load(open(tp))["traffic_per_algorithmic_byte"] * att_bytes / att_n
            except Exception:
                traffic = None
        total_prof_ms = sum(v[1] for v in prof.values()) or 1.0
        kernels = {k: {"launches": v[0], "ms": round(v[1], 3), "share": round(v[1] / total_prof_ms, 4),
                       "GB/s": round(v[2] / (v[1] / 1e3) / 1e9, 1) if v[1] else None,
                       "TFLOP/s": round(v[3] / (v[1] / 1e3) / 1e12, 2) if v[1] and v[3] else None}
                   for k, v in prof.items() if v[0]}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded model, random prompt ids)",
            "config": dict(CONFIG, parallelism=f"sequences sharded over {world} GPU(s)"),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 4 * B,
                    "api": "cortex_decode_steps(steps=1, SNAI_HOST_PTRS) per step"},
            "gpu_launches": int(launches),
            "roofline": {"kernel": "attention (decode, fp32 KV)", "bound": "hbm",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": (achieved / peak) if achieved else None, "traffic": traffic,
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_launch": att_bytes / att_n if att_n else None},
            "kernels": kernels,
            "prefill": {"tokens_per_s": TOTAL_SEQS * PROMPT / prefill_s, "seconds": prefill_s},
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            nthreads = os.cpu_count() or 1
            rate, secs, nseq = cpu_sample(2, nthreads)
            line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": nthreads, "kind": "port",
                                    "sample": f"{nseq} sequences x 2 decode steps from position 768, one thread "
                                              f"per sequence ({secs:.1f} s)"}
        print(json.dumps(line), flush=True)
    eng.close()


def sampler_bench(args):
    """Isolated sampler workload: fp32 logits [8192, V], V in {16384, 32000,
    131072}, N(0, 4) with 1% of entries raised by 12, a 256-id history per
    row, one uniform per row; greedy, variant A (T 0.7, rep 1.15) and variant
    B (T 0.7, top-k 50, top-p 0.95, rep 1.15).  Algorithmic bytes per row:
    4V (logits) + 4*256 (history) + 4 (uniform) + 4 (id).  Each line also
    checks 64 rows against the oracle (bit-exact ids)."""
    import torch

    import oracle as O
    from snai_b200 import VARIANT_A, VARIANT_B, sample_device, sample_params
    peak, peak_kind = load_peaks()
    rows, H = 8192, 256
    dev = torch.device("cuda")
    modes = [("greedy", sample_params(VARIANT_A, 0.01, 1.15, nan_guard=0), (VARIANT_A, 0.01, 1.15, 40, 0.9)),
             ("A_T0.7", sample_params(VARIANT_A, 0.7, 1.15, nan_guard=0), (VARIANT_A, 0.7, 1.15, 40, 0.9)),
             ("B_T0.7_k50_p0.95", sample_params(VARIANT_B, 0.7, 1.15, 50, 0.95), (VARIANT_B, 0.7, 1.15, 50, 0.95))]
    for V in (16384, 32000, 131072):
        g = torch.Generator(device=dev).manual_seed(V)
        L = torch.randn(rows, V, device=dev, generator=g) * 2.0
        L += (torch.rand(rows, V, device=dev, generator=g) < 0.01).float() * 12.0
        hist = torch.randint(0, V, (rows, H), device=dev, generator=g, dtype=torch.int32)
        U = torch.rand(rows, device=dev, generator=g)
        out = torch.zeros(rows, dtype=torch.int32, device=dev)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        for name, prm, oargs in modes:
            for _ in range(args.warmup):
                sample_device(L, U, prm, hist, None, out)
            ts = []
            for _ in range(args.steps):
                flush.zero_()  # 256 MB > L2 between timed launches
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                sample_device(L, U, prm, hist, None, out)
                e1.record()
                e1.synchronize()
                ts.append(e0.elapsed_time(e1))
            ms = float(np.median(ts))
            nbytes = rows * (4 * V + 4 * H + 8)
            gbs = nbytes / (ms / 1e3) / 1e9
            n_chk = 64
            Lh = L[:n_chk].cpu().numpy()
            Hh = hist[:n_chk].cpu().numpy()
            Uh = U[:n_chk].cpu().numpy()
            want, _ = O.sample_rows(Lh, Hh, Uh, *oargs, exp_mode=1)
            exact = bool(np.array_equal(out[:n_chk].cpu().numpy(), want))
            # CPU baseline: the oracle port on all host threads over 256 rows
            n_cpu = 256
            _, rate = O.sample_rows(L[:n_cpu].cpu().numpy(), hist[:n_cpu].cpu().numpy(), U[:n_cpu].cpu().numpy(),
                                    *oargs, exp_mode=0, nthreads=os.cpu_count() or 1)
            line = {"metric": "sampling GB/s", "value": gbs, "unit": "GB/s", "mode": name, "vocab": V,
                    "rows": rows, "ms": ms, "rows_per_s": rows / (ms / 1e3),
                    "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                                 "frac": gbs / peak, "peak_source": f"{peak_kind} hbm_gbs"},
                    "bit_exact_vs_oracle_64_rows": exact,
                    "cpu_baseline": {"value": rate, "unit": "rows/s", "cores": os.cpu_count(), "kind": "port",
                                     "sample": f"{n_cpu} rows"}}
            print(json.dumps(line), flush=True)
        del L, hist, U, out, flush
        torch.cuda.empty_cache()


def gemm_bench(args):
    """Projection micro-benchmark: the d=1024 decode step's GEMM shapes (4096
    rows; qkv N=3072, wo N=1024, up N=4096, down N=1024 with K=4096, logits
    N=16384) through decode passes of one token per slot, on the benchmark
    model's weights with a 16-position context (no 68 GB KV cache).  One
    JSON line per GEMM kind: TFLOP/s from the library's CUDA-event profiler
    against the measured bf16 peak.  With fewer than 64 rows (`--seqs`) the
    projections run as fp32 GEMVs, bound by the weight stream: the line
    then gives GB/s (weights + activations + outputs) against the measured
    copy peak; the fp32 weights (168 MB) exceed L2, so each pass streams
    most of them from HBM."""
    import torch
    from snai_b200 import PREC_BF16, Cortex, modelgen
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, peak_src = float(json.load(f)["bf16_tflops"]), "measured bf16_tflops"
    except Exception:
        peak, peak_src = 1590.0, "fallback"
    path = os.path.join(tempfile.gettempdir(), f"snai_bench_gemm_d{D}.snai")
    if not os.path.exists(path) or os.path.getsize(path) != modelgen.expected_size(V, D, 4 * D, L):
        modelgen.random_model(path, V, D, 16, L, seed=1234, std=0.02)
    B = args.seqs
    eng = Cortex(path, num_heads=HEADS, max_seqs=B, precision=PREC_BF16)
    dev = torch.device("cuda")
    rng = np.random.default_rng(7)

    stream = torch.cuda.Stream(device=dev)
    eng.set_stream(stream.cuda_stream)
    torch.cuda.set_stream(stream)

    def step():
        if eng.pos(0) >= 15:
            eng.rewind(0)
        toks = torch.from_numpy(rng.integers(0, V, B).astype(np.int32)).to(dev)
        if B < 64:
            # a pass of small GEMVs is shorter than its launches take on the
            # host: hold the stream for ~0.2 ms so that the pass is queued
            # whole and its kernels (and the profiler's events) run back to back
            torch.cuda._sleep(400000)
        eng.forward_dev(toks, B, 1)

    for _ in range(args.warmup):
        step()
    eng.synchronize()
    eng.profile(True)
    for _ in range(args.steps):
        step()
    eng.synchronize()
    prof = eng.profile_read()
    eng.profile(False)
    hbm, hbm_src = load_peaks()
    for k in ("qkv", "wo", "up", "down", "logits"):
        n, ms, nbytes, flops = prof[k]
        if not n:
            continue
        tf = flops / (ms / 1e3) / 1e12
        if B < 64:
            gbs = nbytes / (ms / 1e3) / 1e9
            print(json.dumps({"metric": "projection GB/s (fp32 GEMV)", "gemm": k, "value": gbs, "unit": "GB/s",
                              "rows": B, "launches": n, "us_per_launch": 1e3 * ms / n,
                              "bytes_per_launch": nbytes / n, "TFLOP/s": tf,
                              "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                                           "frac": gbs / hbm, "peak_source": hbm_src + " hbm_gbs"}}), flush=True)
            continue
        print(json.dumps({"metric": "projection TFLOP/s", "gemm": k, "value": tf, "unit": "TFLOP/s", "rows": B,
                          "launches": n, "us_per_launch": 1e3 * ms / n,
                          "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                                       "frac": tf / peak, "peak_source": peak_src}}), flush=True)
    if B < 64:
        # the whole decode pass of B rows (embedding, 2 layers, final norm,
        # logits), timed without the per-launch profiler so that consecutive
        # kernels overlap as they do in use: its algorithmic bytes (weights
        # once, KV cache, activations: the profiler's sums per pass) over its
        # event time
        passes = sum(prof[k][0] for k in ("logits",))
        step_bytes = sum(v[2] for v in prof.values()) / max(1, passes)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, b in ev:
            if eng.pos(0) >= 15:
                eng.rewind(0)
            toks = torch.from_numpy(rng.integers(0, V, B).astype(np.int32)).to(dev)
            torch.cuda._sleep(400000)
            a.record()
            eng.forward_dev(toks, B, 1)
            b.record()
        eng.synchronize()
        ms = sorted(a.elapsed_time(b) for a, b in ev)[len(ev) // 2]
        gbs = step_bytes / (ms / 1e3) / 1e9
        print(json.dumps({"metric": "decode pass GB/s (fp32 GEMV path)", "value": gbs, "unit": "GB/s", "rows": B,
                          "us_per_pass": 1e3 * ms, "bytes_per_pass": step_bytes, "passes": len(ev),
                          "timing": "median of per-pass CUDA events",
                          "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                                       "frac": gbs / hbm, "peak_source": hbm_src + " hbm_gbs"}}), flush=True)
    eng.close()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default: ctx - prompt - 3)")
    ap.add_argument("--config", choices=["c4", "c2", "c3"], default="c4",
                    help="c4 (default): the headline d=1024 workload; c2 / c3: the smaller configurations")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sampler", action="store_true", help="run the isolated sampling micro-benchmark")
    ap.add_argument("--gemm", action="store_true", help="run the projection GEMM micro-benchmark")
    ap.add_argument("--seqs", type=int, default=TOTAL_SEQS,
                    help="total sequences (default 4096; smaller only for profiling captures)")
    args = ap.parse_args()
    if args.config != "c4":
        apply_config(args.config)
        if args.seqs == 4096:
            args.seqs = TOTAL_SEQS
    if args.steps is None:
        args.steps = CTX - PROMPT - 3
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        print(f"note: --gpus {args.gpus} but WORLD_SIZE={world}; using {world}", file=sys.stderr)
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return
    if args.gemm:
        if rank == 0:
            gemm_bench(args)
        return
    if args.sampler:
        if rank == 0:
            sampler_bench(args)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    try:
        our_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
